// Tiled bitmask format: pack (with arena cursor), unpack, ReLU-mask and
// ReLU^2-gradient kernels (sm_100a).
//
// Reference: old/lib_sparse/sparse_pack.py:27-92 + sparse.py:154-210 (pack:
// tile kernel, torch.cumsum, compaction kernel that re-reads the tile, cursor
// index_add_), old/lib_sparse/sparse_unpack.py:5-147 (unpack / mask / grad).
// Pack here is three launches over independent tiles, none waiting on
// another: (1) each CTA reads one tile, writes its mask words and its count;
// (2) one CTA scans the counts into prefix[], reads the arena cursor and
// advances it (sffn_tile_scan_counts); (3) each CTA reads its tile again,
// ranks the set elements in registers, stages them in shared memory and
// writes them at vals[cursor + prefix[t]].  (A single pass whose tiles found
// their offsets by a decoupled look-back over their predecessors ran at a
// third of the HBM rate: every tile's store waited on that chain.)
//
// Thread layout per tile: NT = min(256, BM*BN/8) threads, U iterations, 8
// consecutive in-tile elements (one mask byte) per thread per iteration; in
// iteration `it` thread `tid` owns in-tile offsets f = 8*(it*NT + tid) + j.
#include "common.cuh"
#include "sm100.cuh"

namespace sffn {
namespace {

template <int BM, int BN>
struct TileCfg {
    static constexpr int TILE = BM * BN;
    static constexpr int TB = TILE / 8;  // mask bytes per tile
    static constexpr int NT = TILE / 8 < 256 ? TILE / 8 : 256;
    static constexpr int U = TILE / (8 * NT);
    static constexpr int NW = NT / 32;
    static constexpr int NE = U * NW;  // (iteration, warp) partial counts
    static_assert(BN % 32 == 0, "a mask word never straddles tile rows");
    static_assert(NE <= 32 || NE == 64, "scan_small handles up to 32 or exactly 64 entries");
};

// Exclusive scan, by warp 0, of NE ints in shared memory; total -> *s_total.
template <int NE>
__device__ __forceinline__ void scan_small(int* s, int* s_total, int lane) {
    if constexpr (NE <= 32) {
        int t = lane < NE ? s[lane] : 0;
        int inc = warp_incl_scan(t, lane);
        if (lane < NE) s[lane] = inc - t;
        if (lane == 31) *s_total = inc;
    } else {
        int a = s[2 * lane], b = s[2 * lane + 1];
        int inc = warp_incl_scan(a + b, lane);
        int ex = inc - a - b;
        s[2 * lane] = ex;
        s[2 * lane + 1] = ex + a;
        if (lane == 31) *s_total = inc;
    }
}

template <typename B>
__device__ __forceinline__ void load8_row(const B* __restrict__ row, long long gc, long long N,
                                          bool vec, B (&v)[8]) {
    if (vec && gc + 8 <= N) {
        if constexpr (sizeof(B) == 2) {
            uint4 q = __ldcs(reinterpret_cast<const uint4*>(row + gc));
            const B* s = reinterpret_cast<const B*>(&q);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = s[j];
        } else {
            uint4 q0 = __ldcs(reinterpret_cast<const uint4*>(row + gc));
            uint4 q1 = __ldcs(reinterpret_cast<const uint4*>(row + gc) + 1);
            v[0] = q0.x; v[1] = q0.y; v[2] = q0.z; v[3] = q0.w;
            v[4] = q1.x; v[5] = q1.y; v[6] = q1.z; v[7] = q1.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = (gc + j < N) ? row[gc + j] : B(0);
    }
}

template <typename O>
__device__ __forceinline__ void store8_row(O* __restrict__ row, long long gc, long long N, bool vec,
                                           const O (&o)[8]) {
    if (vec && gc + 8 <= N) {
        if constexpr (sizeof(O) == 2) {
            uint4 q;
            O* d = reinterpret_cast<O*>(&q);
#pragma unroll
            for (int j = 0; j < 8; ++j) d[j] = o[j];
            *reinterpret_cast<uint4*>(row + gc) = q;
        } else {
            reinterpret_cast<uint4*>(row + gc)[0] = make_uint4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<uint4*>(row + gc)[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (gc + j < N) row[gc + j] = o[j];
    }
}

// Mask byte of this thread's 8 elements, read as whole little-endian words by
// lanes 4k and shared within the group of four.
template <int TB>
__device__ __forceinline__ uint32_t mask_byte(const uint8_t* __restrict__ tile_mask, int f, int lane) {
    uint32_t w = 0;
    if ((lane & 3) == 0) w = __ldg(reinterpret_cast<const unsigned int*>(tile_mask + (f >> 3)));
    w = __shfl_sync(FULL, w, lane & ~3);
    return (w >> (8 * (lane & 3))) & 0xFFu;
}

// ----------------------------------------------------------------- pack ----
// Eight consecutive elements of a tile row held as packed 32-bit words
// (four for 16-bit types, eight for 32-bit ones), loaded with 16-byte loads
// where the row allows.
template <typename B>
struct Words8 {
    static constexpr int NW = (int)sizeof(B) * 2;
    uint32_t w[NW];
    __device__ void load(const B* __restrict__ row, long long gc, long long N, bool vec) {
        if (vec && gc + 8 <= N) {
#pragma unroll
            for (int k = 0; k < NW / 4; ++k) {
                const uint4 q = __ldcs(reinterpret_cast<const uint4*>(row + gc) + k);
                w[4 * k] = q.x;
                w[4 * k + 1] = q.y;
                w[4 * k + 2] = q.z;
                w[4 * k + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < NW; ++k) w[k] = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (gc + j < N) set(j, row[gc + j]);
        }
    }
    __device__ void zero() {
#pragma unroll
        for (int k = 0; k < NW; ++k) w[k] = 0;
    }
    __device__ void set(int j, B v) {
        if constexpr (sizeof(B) == 2) {
            const int sh = 16 * (j & 1);
            w[j >> 1] = (w[j >> 1] & ~(0xFFFFu << sh)) | ((uint32_t)v << sh);
        } else {
            w[j] = v;
        }
    }
    // bit j set iff element j > 0 (sign clear, non-zero, not NaN): x - 1 below
    // +inf as an unsigned integer of the element's width.
    __device__ uint32_t positive_byte(uint16_t inf16) const {
        uint32_t b = 0;
        if constexpr (sizeof(B) == 2) {
            const uint32_t inf2 = (uint32_t)inf16 | ((uint32_t)inf16 << 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t m = __vcmpltu2(__vsub2(w[q], 0x00010001u), inf2);
                b |= ((m & 1u) | ((m >> 15) & 2u)) << (2 * q);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) b |= (uint32_t)(w[j] - 1u < 0x7F800000u) << j;
        }
        return b;
    }
    // The set elements to consecutive shared-memory places from byte address
    // `da` (predicated stores; the address steps by each bit).
    __device__ void put_set(uint32_t bits, uint32_t da) const {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t bj = (bits >> j) & 1u;
            if constexpr (sizeof(B) == 2) {
                const uint16_t v = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
                asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q st.shared.u16 [%0], %1;\n\t}" ::"r"(da),
                             "h"(v), "r"(bj)
                             : "memory");
            } else {
                asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q st.shared.u32 [%0], %1;\n\t}" ::"r"(da),
                             "r"(w[j]), "r"(bj)
                             : "memory");
            }
            da += (uint32_t)sizeof(B) * bj;
        }
    }
};

// COUNT: mask words and counts[t].  VALUES: the set elements of tile t at
// vals[*vals_offset + prefix[t] ...] (never past cap).
template <typename B, int BM, int BN, bool VALUES>
__global__ void __launch_bounds__(TileCfg<BM, BN>::NT) tile_pack_kernel(
    const B* __restrict__ dense, long long M, long long N, long long ld, int vec, uint16_t inf16,
    uint8_t* __restrict__ bitmask, int* __restrict__ counts, const int* __restrict__ prefix,
    const int* __restrict__ vals_offset, B* __restrict__ vals, long long cap, uint32_t* __restrict__ status,
    long long gn) {
    using C = TileCfg<BM, BN>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    B* s_vals = reinterpret_cast<B*>(smem_raw);
    __shared__ int s_wx[C::NE];
    __shared__ int s_agg;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long t = blockIdx.x;
    const long long tm = t / gn, tn = t % gn;
    const long long row0 = tm * BM, col0 = tn * BN;
    uint8_t* tmask = bitmask + t * C::TB;

    Words8<B> v[C::U];
#pragma unroll
    for (int it = 0; it < C::U; ++it) {  // every load issued before any use
        const int f = 8 * (it * C::NT + tid);
        const long long gr = row0 + f / BN, gc = col0 + f % BN;
        if (gr < M) v[it].load(dense + gr * ld, gc, N, vec != 0);
        else v[it].zero();
    }
    uint32_t bits[C::U];
    int lex[C::U];
#pragma unroll
    for (int it = 0; it < C::U; ++it) {
        const int f = 8 * (it * C::NT + tid);
        const uint32_t b = v[it].positive_byte(inf16);
        bits[it] = b;
        if constexpr (!VALUES) {
            const uint32_t w = bytes_to_word(b, lane);
            if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(tmask + (f >> 3)) = w;
        }
        const int c = __popc(b);
        const int inc = warp_incl_scan(c, lane);
        lex[it] = inc - c;
        if (lane == 31) s_wx[it * C::NW + warp] = inc;
    }
    __syncthreads();
    if (warp == 0) scan_small<C::NE>(s_wx, &s_agg, lane);
    __syncthreads();
    if constexpr (!VALUES) {
        if (tid == 0) counts[t] = s_agg;
        return;
    } else {
        const uint32_t sb = smem_u32(s_vals);
#pragma unroll
        for (int it = 0; it < C::U; ++it)
            v[it].put_set(bits[it], sb + (uint32_t)((s_wx[it * C::NW + warp] + lex[it]) * (int)sizeof(B)));
        __syncthreads();
        const int agg = s_agg;
        const long long base = (long long)*vals_offset + prefix[t];
        for (int i = tid; i < agg; i += C::NT) {
            const long long p = base + i;
            if (p >= 0 && p < cap) vals[p] = s_vals[i];
        }
        if (tid == 0 && (base < 0 || base + agg > cap)) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
    }
}

// --------------------------------------------------------------- unpack ----
template <int DT, bool OUT_F32, int BM, int BN>
__global__ void __launch_bounds__(TileCfg<BM, BN>::NT) tile_unpack_kernel(
    const typename Elt<DT>::bits* __restrict__ vals, const uint8_t* __restrict__ bitmask,
    long long vals_len, const int* __restrict__ prefix, const int* __restrict__ vals_offset,
    long long M, long long N, long long gn, long long tile_row0, int square,
    typename std::conditional<OUT_F32, uint32_t, typename Elt<DT>::bits>::type* __restrict__ out,
    long long ld_out, int vec) {
    using C = TileCfg<BM, BN>;
    using B = typename Elt<DT>::bits;
    using O = typename std::conditional<OUT_F32, uint32_t, B>::type;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    B* s_vals = reinterpret_cast<B*>(smem_raw);
    __shared__ int s_wx[C::NE];
    __shared__ int s_agg;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long tl = blockIdx.x;
    const long long tm = tile_row0 + tl / gn, tn = tl % gn;
    const long long t = tm * gn + tn;
    const long long row0 = tm * BM, col0 = tn * BN;
    const long long start = (long long)*vals_offset + prefix[t];
    const int cnt = min(prefix[t + 1] - prefix[t], C::TILE);
    // The tile's values into shared memory: whole 16-byte vectors from the
    // aligned address at or below the run's start (value i then sits at
    // s_vals[sh + i]); per value where the run is not inside vals or vals is
    // not 16-byte aligned.
    constexpr int EPV = 16 / (int)sizeof(B);
    int sh = 0;
    if ((reinterpret_cast<uintptr_t>(vals) & 15u) == 0 && cnt > 0 && start >= 0 && start + cnt <= vals_len) {
        const long long a0 = start & ~(long long)(EPV - 1);
        sh = (int)(start - a0);
        const int nv = (sh + cnt + EPV - 1) / EPV;
        const uint4* v4 = reinterpret_cast<const uint4*>(vals + a0);
        uint4* s4 = reinterpret_cast<uint4*>(s_vals);
#pragma unroll 4
        for (int q = tid; q < nv; q += C::NT) {
            if (a0 + (long long)(q + 1) * EPV <= vals_len) {
                s4[q] = __ldg(v4 + q);
            } else {
#pragma unroll
                for (int e = 0; e < EPV; ++e)
                    s_vals[q * EPV + e] = a0 + q * EPV + e < vals_len ? vals[a0 + q * EPV + e] : B(0);
            }
        }
    } else {
#pragma unroll 4
        for (int i = tid; i < cnt; i += C::NT)
            s_vals[i] = (start + i >= 0 && start + i < vals_len) ? vals[start + i] : B(0);
    }

    uint32_t bits[C::U];
    int lex[C::U];
#pragma unroll
    for (int it = 0; it < C::U; ++it) {
        const int f = 8 * (it * C::NT + tid);
        const uint32_t b = mask_byte<C::TB>(bitmask + t * C::TB, f, lane);
        bits[it] = b;
        const int c = __popc(b);
        const int inc = warp_incl_scan(c, lane);
        lex[it] = inc - c;
        if (lane == 31) s_wx[it * C::NW + warp] = inc;
    }
    __syncthreads();
    if (warp == 0) scan_small<C::NE>(s_wx, &s_agg, lane);
    __syncthreads();
#pragma unroll
    for (int it = 0; it < C::U; ++it) {
        const int f = 8 * (it * C::NT + tid);
        const long long gr = row0 + f / BN, gc = col0 + f % BN;
        int r = sh + s_wx[it * C::NW + warp] + lex[it];
        O o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            B z = B(0);
            if ((bits[it] >> j) & 1u) {
                z = r < C::TILE + 2 * EPV ? s_vals[r] : B(0);
                ++r;
                if (square & 1) {
                    const float zf = Elt<DT>::to_f(z);
                    z = Elt<DT>::from_f(zf * zf);
                }
            }
            if constexpr (OUT_F32) o[j] = __float_as_uint(Elt<DT>::to_f(z));
            else o[j] = z;
            if constexpr (sizeof(O) == 4)
                if (square & 2) o[j] = tf32_round_bits(o[j]);
        }
        if (gr < M) store8_row(out + (gr - tile_row0 * BM) * ld_out, gc, N, vec != 0, o);
    }
}

// ------------------------------------------------------------ mask grad ----
template <typename B, int BM, int BN>
__global__ void __launch_bounds__(TileCfg<BM, BN>::NT) tile_mask_kernel(
    B* __restrict__ grad, long long M, long long N, long long ld, const uint8_t* __restrict__ bitmask,
    long long gn, int vec) {
    using C = TileCfg<BM, BN>;
    const int tid = threadIdx.x, lane = tid & 31;
    const long long t = blockIdx.x;
    const long long row0 = (t / gn) * BM, col0 = (t % gn) * BN;
#pragma unroll
    for (int it = 0; it < C::U; ++it) {
        const int f = 8 * (it * C::NT + tid);
        const uint32_t b = mask_byte<C::TB>(bitmask + t * C::TB, f, lane);
        const long long gr = row0 + f / BN, gc = col0 + f % BN;
        if (gr >= M) continue;
        B g[8];
        load8_row(grad + gr * ld, gc, N, vec != 0, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = ((b >> j) & 1u) ? g[j] : B(0);
        store8_row(grad + gr * ld, gc, N, vec != 0, g);
    }
}

// ----------------------------------------------------------- relu^2 grad ----
template <int DT, int BM, int BN>
__global__ void __launch_bounds__(TileCfg<BM, BN>::NT) tile_grad_relu2_kernel(
    typename Elt<DT>::bits* __restrict__ grad, long long M, long long N, long long ld,
    typename Elt<DT>::bits* __restrict__ vals, long long vals_len,
    const uint8_t* __restrict__ bitmask, const int* __restrict__ prefix,
    const int* __restrict__ vals_offset, long long gn, int square, int vec) {
    using C = TileCfg<BM, BN>;
    using B = typename Elt<DT>::bits;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    B* s_vals = reinterpret_cast<B*>(smem_raw);
    __shared__ int s_wx[C::NE];
    __shared__ int s_agg;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long t = blockIdx.x;
    const long long row0 = (t / gn) * BM, col0 = (t % gn) * BN;
    const long long start = (long long)*vals_offset + prefix[t];
    const int cnt = min(prefix[t + 1] - prefix[t], C::TILE);
    // The tile's values into shared memory: whole 16-byte vectors from the
    // aligned address at or below the run's start (value i then sits at
    // s_vals[sh + i]); per value where the run is not inside vals or vals is
    // not 16-byte aligned.
    constexpr int EPV = 16 / (int)sizeof(B);
    int sh = 0;
    if ((reinterpret_cast<uintptr_t>(vals) & 15u) == 0 && cnt > 0 && start >= 0 && start + cnt <= vals_len) {
        const long long a0 = start & ~(long long)(EPV - 1);
        sh = (int)(start - a0);
        const int nv = (sh + cnt + EPV - 1) / EPV;
        const uint4* v4 = reinterpret_cast<const uint4*>(vals + a0);
        uint4* s4 = reinterpret_cast<uint4*>(s_vals);
#pragma unroll 4
        for (int q = tid; q < nv; q += C::NT) {
            if (a0 + (long long)(q + 1) * EPV <= vals_len) {
                s4[q] = __ldg(v4 + q);
            } else {
#pragma unroll
                for (int e = 0; e < EPV; ++e)
                    s_vals[q * EPV + e] = a0 + q * EPV + e < vals_len ? vals[a0 + q * EPV + e] : B(0);
            }
        }
    } else {
#pragma unroll 4
        for (int i = tid; i < cnt; i += C::NT)
            s_vals[i] = (start + i >= 0 && start + i < vals_len) ? vals[start + i] : B(0);
    }

    uint32_t bits[C::U];
    int lex[C::U];
#pragma unroll
    for (int it = 0; it < C::U; ++it) {
        const int f = 8 * (it * C::NT + tid);
        const uint32_t b = mask_byte<C::TB>(bitmask + t * C::TB, f, lane);
        bits[it] = b;
        const int c = __popc(b);
        const int inc = warp_incl_scan(c, lane);
        lex[it] = inc - c;
        if (lane == 31) s_wx[it * C::NW + warp] = inc;
    }
    __syncthreads();
    if (warp == 0) scan_small<C::NE>(s_wx, &s_agg, lane);
    __syncthreads();
#pragma unroll
    for (int it = 0; it < C::U; ++it) {
        const int f = 8 * (it * C::NT + tid);
        const long long gr = row0 + f / BN, gc = col0 + f % BN;
        if (gr >= M) continue;
        int r = sh + s_wx[it * C::NW + warp] + lex[it];
        B g[8];
        load8_row(grad + gr * ld, gc, N, vec != 0, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float z = 0.0f;
            if ((bits[it] >> j) & 1u) {
                z = r < C::TILE + 2 * EPV ? Elt<DT>::to_f(s_vals[r]) : 0.0f;
                ++r;
            }
            // (g * 2.0) * z rounded to the storage dtype; g*2 is exact.
            g[j] = Elt<DT>::from_f((Elt<DT>::to_f(g[j]) * 2.0f) * z);
        }
        store8_row(grad + gr * ld, gc, N, vec != 0, g);
    }
    if (square) {
        for (int i = tid; i < cnt; i += C::NT) {
            if (start + i < 0 || start + i >= vals_len) continue;
            const float z = Elt<DT>::to_f(s_vals[sh + i]);
            vals[start + i] = Elt<DT>::from_f(z * z);
        }
    }
}

// ------------------------------------------------------------ dispatch ----
// Supported tile shapes.
#define SFFN_TILE_SHAPES(X) X(32, 32) X(64, 64) X(128, 128) X(64, 128) X(128, 64)

inline bool tile_shape_ok(int BM, int BN) {
#define SFFN_OK_SHAPE(a, b) if (BM == a && BN == b) return true;
    SFFN_TILE_SHAPES(SFFN_OK_SHAPE)
#undef SFFN_OK_SHAPE
    return false;
}

template <typename K>
inline cudaError_t prep_smem(K kernel, int bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

inline long long num_tiles(long long M, long long N, int BM, int BN) {
    return ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
}

template <typename B, int BM, int BN>
int launch_pack_values(const void* dense, long long M, long long N, long long ld, int vec, uint16_t inf16,
                       uint8_t* bitmask, const int* prefix, void* vals, long long cap, const int* vals_offset,
                       uint32_t* status, cudaStream_t st);

template <typename B, int BM, int BN>
int launch_pack(const void* dense, long long M, long long N, long long ld, int vec, uint16_t inf16,
                uint8_t* bitmask, int* prefix, void* vals, long long cap, int* cursor,
                int* vals_offset_out, int* counts, uint32_t* status, cudaStream_t st) {
    using C = TileCfg<BM, BN>;
    const long long gn = (N + BN - 1) / BN, nt = num_tiles(M, N, BM, BN);
    const int smem = C::TILE * (int)sizeof(B);
    auto kc = tile_pack_kernel<B, BM, BN, false>;
    kc<<<(unsigned)nt, C::NT, 0, st>>>((const B*)dense, M, N, ld, vec, inf16, bitmask, counts, nullptr, nullptr,
                                       nullptr, 0, status, gn);
    SFFN_CHECK_LAUNCH();
    if (int rc = sffn_tile_scan_counts(counts, 1, nt, prefix, cursor, vals_offset_out, status, st)) return rc;
    if (!vals) return SFFN_OK;  // counts, prefix and cursor only (sffn_tile_pack_values follows)
    return launch_pack_values<B, BM, BN>(dense, M, N, ld, vec, inf16, bitmask, prefix, vals, cap, vals_offset_out,
                                         status, st);
}

template <typename B, int BM, int BN>
int launch_pack_values(const void* dense, long long M, long long N, long long ld, int vec, uint16_t inf16,
                       uint8_t* bitmask, const int* prefix, void* vals, long long cap, const int* vals_offset,
                       uint32_t* status, cudaStream_t st) {
    using C = TileCfg<BM, BN>;
    const long long gn = (N + BN - 1) / BN, nt = num_tiles(M, N, BM, BN);
    const int smem = C::TILE * (int)sizeof(B);
    auto kv = tile_pack_kernel<B, BM, BN, true>;
    SFFN_CUDA_TRY(prep_smem(kv, smem));
    kv<<<(unsigned)nt, C::NT, smem, st>>>((const B*)dense, M, N, ld, vec, inf16, bitmask, nullptr, prefix,
                                          vals_offset, (B*)vals, cap, status, gn);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <int DT, bool OF, int BM, int BN>
int launch_unpack(const void* vals, long long vals_len, const uint8_t* bitmask, const int* prefix,
                  const int* voff, long long M, long long N, long long tr0, long long trows, int square, void* out,
                  long long ld_out, int vec, cudaStream_t st) {
    using C = TileCfg<BM, BN>;
    using B = typename Elt<DT>::bits;
    using O = typename std::conditional<OF, uint32_t, B>::type;
    const long long gn = (N + BN - 1) / BN;
    const int smem = (C::TILE + 32 / (int)sizeof(B)) * (int)sizeof(B);  // + two vectors of alignment slack
    auto k = tile_unpack_kernel<DT, OF, BM, BN>;
    SFFN_CUDA_TRY(prep_smem(k, smem));
    k<<<(unsigned)(trows * gn), C::NT, smem, st>>>((const B*)vals, bitmask, vals_len, prefix, voff,
                                                    M, N, gn, tr0, square, (O*)out, ld_out, vec);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <typename B, int BM, int BN>
int launch_mask(void* grad, long long M, long long N, long long ld, const uint8_t* bitmask, int vec,
                cudaStream_t st) {
    using C = TileCfg<BM, BN>;
    const long long gn = (N + BN - 1) / BN, nt = num_tiles(M, N, BM, BN);
    tile_mask_kernel<B, BM, BN><<<(unsigned)nt, C::NT, 0, st>>>((B*)grad, M, N, ld, bitmask, gn, vec);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <int DT, int BM, int BN>
int launch_relu2(void* grad, long long M, long long N, long long ld, void* vals, long long vals_len,
                 const uint8_t* bitmask, const int* prefix, const int* voff, int square, int vec,
                 cudaStream_t st) {
    using C = TileCfg<BM, BN>;
    using B = typename Elt<DT>::bits;
    const long long gn = (N + BN - 1) / BN, nt = num_tiles(M, N, BM, BN);
    const int smem = (C::TILE + 32 / (int)sizeof(B)) * (int)sizeof(B);  // + two vectors of alignment slack
    auto k = tile_grad_relu2_kernel<DT, BM, BN>;
    SFFN_CUDA_TRY(prep_smem(k, smem));
    k<<<(unsigned)nt, C::NT, smem, st>>>((B*)grad, M, N, ld, (B*)vals, vals_len, bitmask, prefix,
                                         voff, gn, square, vec);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

inline bool vec_ok(const void* p, long long ld, int esz) {
    return aligned16(p) && ((ld * esz) % 16 == 0);
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" size_t sffn_tile_workspace_bytes(int64_t M, int64_t N, int BM, int BN) {
    if (M < 0 || N < 0 || BM <= 0 || BN <= 0) return 0;
    return 16 + (size_t)num_tiles(M, N, BM, BN) * 8;
}

extern "C" int sffn_tile_pack(const void* dense, int dtype, int64_t M, int64_t N, int64_t ld, int BM,
                              int BN, uint8_t* bitmask, int32_t* prefix, void* vals,
                              int64_t vals_capacity, int32_t* offset_dev, int32_t* vals_offset_dev,
                              void* workspace, size_t workspace_bytes, uint32_t* status_dev,
                              void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (!tile_shape_ok(BM, BN)) return SFFN_ERR_UNSUPPORTED;
    if (M <= 0 || N <= 0 || ld < N || vals_capacity < 0) return SFFN_ERR_ARG;
    if (M * N > 0x7FFFFFFFll) return SFFN_ERR_ARG;  // int32 prefix, as in the reference
    if (!dense || !bitmask || !prefix || !offset_dev || !vals_offset_dev || !status_dev || !workspace)
        return SFFN_ERR_ARG;
    if (!vals && vals_capacity != 0) return SFFN_ERR_ARG;  // NULL vals: counts and cursor only
    if (offset_dev == vals_offset_dev) return SFFN_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(bitmask) & 3u) return SFFN_ERR_ALIGN;
    if (workspace_bytes < sffn_tile_workspace_bytes(M, N, BM, BN)) return SFFN_ERR_WORKSPACE;
    SFFN_BIND(dev_scope, dense);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int* counts = static_cast<int*>(workspace);  // one count per tile
    const int esz = esize_of(dtype);
    const int vec = vec_ok(dense, ld, esz) ? 1 : 0;
    const uint16_t inf16 = inf16_of(dtype);
#define SFFN_PACK_CASE(a, b)                                                                         \
    if (BM == a && BN == b) {                                                                        \
        if (esz == 4)                                                                                \
            return launch_pack<uint32_t, a, b>(dense, M, N, ld, vec, inf16, bitmask, prefix, vals,   \
                                               vals_capacity, offset_dev, vals_offset_dev, counts,   \
                                               status_dev, st);                                      \
        return launch_pack<uint16_t, a, b>(dense, M, N, ld, vec, inf16, bitmask, prefix, vals,       \
                                           vals_capacity, offset_dev, vals_offset_dev, counts,       \
                                           status_dev, st);                                          \
    }
    SFFN_TILE_SHAPES(SFFN_PACK_CASE)
#undef SFFN_PACK_CASE
    return SFFN_ERR_UNSUPPORTED;
}

extern "C" int sffn_tile_pack_values(const void* dense, int dtype, int64_t M, int64_t N, int64_t ld, int BM,
                                     int BN, const uint8_t* bitmask, const int32_t* prefix, void* vals,
                                     int64_t vals_capacity, const int32_t* vals_offset_dev, uint32_t* status_dev,
                                     void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (!tile_shape_ok(BM, BN)) return SFFN_ERR_UNSUPPORTED;
    if (M <= 0 || N <= 0 || ld < N || vals_capacity < 0) return SFFN_ERR_ARG;
    if (M * N > 0x7FFFFFFFll) return SFFN_ERR_ARG;
    if (!dense || !bitmask || !prefix || !vals || !vals_offset_dev || !status_dev) return SFFN_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(bitmask) & 3u) return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, dense);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int esz = esize_of(dtype);
    const int vec = vec_ok(dense, ld, esz) ? 1 : 0;
    const uint16_t inf16 = inf16_of(dtype);
    uint8_t* bm = const_cast<uint8_t*>(bitmask);
#define SFFN_PACKV_CASE(a, b)                                                                            \
    if (BM == a && BN == b) {                                                                           \
        if (esz == 4)                                                                                   \
            return launch_pack_values<uint32_t, a, b>(dense, M, N, ld, vec, inf16, bm, prefix, vals,    \
                                                      vals_capacity, vals_offset_dev, status_dev, st); \
        return launch_pack_values<uint16_t, a, b>(dense, M, N, ld, vec, inf16, bm, prefix, vals,        \
                                                  vals_capacity, vals_offset_dev, status_dev, st);     \
    }
    SFFN_TILE_SHAPES(SFFN_PACKV_CASE)
#undef SFFN_PACKV_CASE
    return SFFN_ERR_UNSUPPORTED;
}

extern "C" int sffn_tile_unpack(const void* vals, int64_t vals_len, const uint8_t* bitmask,
                                const int32_t* prefix, const int32_t* vals_offset_dev, int dtype, int64_t M, int64_t N,
                                int BM, int BN, int64_t tile_row0, int64_t tile_rows, int square,
                                void* out, int out_dtype, int64_t ld_out, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (out_dtype != dtype && out_dtype != SFFN_F32) return SFFN_ERR_DTYPE;
    if (!tile_shape_ok(BM, BN)) return SFFN_ERR_UNSUPPORTED;
    const long long gm = (M + BM - 1) / BM;
    if (M <= 0 || N <= 0 || ld_out < N || tile_row0 < 0 || tile_rows < 0 || tile_row0 + tile_rows > gm)
        return SFFN_ERR_ARG;
    if (tile_rows == 0) return SFFN_OK;
    if (!vals || !bitmask || !prefix || !vals_offset_dev || !out) return SFFN_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(bitmask) & 3u) return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, out);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool of = (out_dtype == SFFN_F32) && (dtype != SFFN_F32);
    const int vec = vec_ok(out, ld_out, esize_of(out_dtype)) ? 1 : 0;
#define SFFN_UNPACK_CASE(a, b)                                                                         \
    if (BM == a && BN == b) {                                                                          \
        if (dtype == SFFN_F32)                                                                         \
            return launch_unpack<SFFN_F32, false, a, b>(vals, vals_len, bitmask, prefix, vals_offset_dev, M, N,  \
                                                        tile_row0, tile_rows, square, out, ld_out,     \
                                                        vec, st);                                      \
        if (dtype == SFFN_BF16)                                                                        \
            return of ? launch_unpack<SFFN_BF16, true, a, b>(vals, vals_len, bitmask, prefix, vals_offset_dev,   \
                                                             M, N, tile_row0, tile_rows, square, out,  \
                                                             ld_out, vec, st)                          \
                      : launch_unpack<SFFN_BF16, false, a, b>(vals, vals_len, bitmask, prefix, vals_offset_dev,  \
                                                              M, N, tile_row0, tile_rows, square, out, \
                                                              ld_out, vec, st);                        \
        return of ? launch_unpack<SFFN_F16, true, a, b>(vals, vals_len, bitmask, prefix, vals_offset_dev, M, N,  \
                                                        tile_row0, tile_rows, square, out, ld_out,     \
                                                        vec, st)                                       \
                  : launch_unpack<SFFN_F16, false, a, b>(vals, vals_len, bitmask, prefix, vals_offset_dev, M, N, \
                                                         tile_row0, tile_rows, square, out, ld_out,    \
                                                         vec, st);                                     \
    }
    SFFN_TILE_SHAPES(SFFN_UNPACK_CASE)
#undef SFFN_UNPACK_CASE
    return SFFN_ERR_UNSUPPORTED;
}

extern "C" int sffn_tile_mask_grad(void* grad, int dtype, int64_t M, int64_t N, int64_t ld,
                                   const uint8_t* bitmask, int BM, int BN, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (!tile_shape_ok(BM, BN)) return SFFN_ERR_UNSUPPORTED;
    if (M <= 0 || N <= 0 || ld < N || !grad || !bitmask) return SFFN_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(bitmask) & 3u) return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, grad);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int esz = esize_of(dtype);
    const int vec = vec_ok(grad, ld, esz) ? 1 : 0;
#define SFFN_MASK_CASE(a, b)                                                              \
    if (BM == a && BN == b) {                                                             \
        if (esz == 4) return launch_mask<uint32_t, a, b>(grad, M, N, ld, bitmask, vec, st); \
        return launch_mask<uint16_t, a, b>(grad, M, N, ld, bitmask, vec, st);             \
    }
    SFFN_TILE_SHAPES(SFFN_MASK_CASE)
#undef SFFN_MASK_CASE
    return SFFN_ERR_UNSUPPORTED;
}

extern "C" int sffn_tile_grad_relu2(void* grad, int dtype, int64_t M, int64_t N, int64_t ld,
                                    void* vals, int64_t vals_len, const uint8_t* bitmask, const int32_t* prefix,
                                    const int32_t* vals_offset_dev, int BM, int BN, int square,
                                    void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (!tile_shape_ok(BM, BN)) return SFFN_ERR_UNSUPPORTED;
    if (M <= 0 || N <= 0 || ld < N || !grad || !vals || !bitmask || !prefix || !vals_offset_dev)
        return SFFN_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(bitmask) & 3u) return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, grad);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int vec = vec_ok(grad, ld, esize_of(dtype)) ? 1 : 0;
#define SFFN_RELU2_CASE(a, b)                                                                     \
    if (BM == a && BN == b) {                                                                     \
        if (dtype == SFFN_F32)                                                                    \
            return launch_relu2<SFFN_F32, a, b>(grad, M, N, ld, vals, vals_len, bitmask, prefix,           \
                                                vals_offset_dev, square, vec, st);               \
        if (dtype == SFFN_BF16)                                                                   \
            return launch_relu2<SFFN_BF16, a, b>(grad, M, N, ld, vals, vals_len, bitmask, prefix,          \
                                                 vals_offset_dev, square, vec, st);              \
        return launch_relu2<SFFN_F16, a, b>(grad, M, N, ld, vals, vals_len, bitmask, prefix,               \
                                            vals_offset_dev, square, vec, st);                   \
    }
    SFFN_TILE_SHAPES(SFFN_RELU2_CASE)
#undef SFFN_RELU2_CASE
    return SFFN_ERR_UNSUPPORTED;
}
