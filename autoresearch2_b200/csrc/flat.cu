// Flat bitmask format: pack and unpack (sm_100a).
//
// Reference: old/sparse_pack.py:6-106 (count/pack kernel, one-program serial
// prefix, vals kernel -- the dense tensor is read twice) and
// old/sparse_unpack.py:6-97 (popcount, one-program serial prefix, rebuild).
//
// Both directions are ONE single-pass kernel over tiles of 32 KB of dense
// data (16384 bf16/fp16 or 8192 fp32 elements), one tile per CTA of 256
// threads.  A CTA takes the next tile number from a ticket counter, so every
// tile's predecessors have started before it and the decoupled look-back that
// gives the tile its offset in `vals` always ends.  The look-back reads 512
// predecessor states per round in coalesced rows, so the resolved frontier
// moves 16 MB of dense data per L2 round trip and does not limit the
// bandwidth.  Every byte of the dense tensor, the mask and the values crosses
// HBM exactly once.
//
//   pack:   bring the tile into shared memory with one bulk copy, write the
//           mask words, scan the counts, publish the tile aggregate, look
//           back, and write each thread's set elements from the staged tile
//           to their places in `vals`.
//   unpack: load the tile's mask, scan the counts, publish, look back, load
//           the tile's values (16-byte loads where `vals` allows) into shared
//           memory, expand and write the dense tile with 16-byte streaming
//           stores.
//
// Thread layout: in group g thread `tid` owns the 8 consecutive elements
// f = 8*(tid + 256*g) .. +7 of its tile, i.e. mask byte tid + 256*g of the
// tile; lanes 4k..4k+3 form one little-endian uint32 mask word (bit f%32 of
// word f/32 == bit f%8 of byte f/8).  Values are ordered by f: group-major,
// then thread, then element -- the (group, warp) partial counts are scanned in
// that order.
#include <stdio.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace sffn {
namespace {

constexpr int FT_TILE_BYTES = 32768; // dense bytes per tile
constexpr int FT_MIN_TILE = 8192;    // elements per tile of the widest type
constexpr int FT_LBW = 16;           // look-back: 16 rows of 32 states per round

// 8 elements held as raw 16-byte (2-byte types) or 32-byte (4-byte types) vectors.
template <typename B> struct Vec8;
template <> struct Vec8<uint16_t> {
    uint4 q;
    __device__ uint16_t get(int j) const {
        const uint32_t w = j < 2 ? q.x : j < 4 ? q.y : j < 6 ? q.z : q.w;
        return (uint16_t)(w >> (16 * (j & 1)));
    }
    __device__ void set(int j, uint16_t v) {
        const int sh = 16 * (j & 1);
        const uint32_t keep = ~(0xFFFFu << sh), x = (uint32_t)v << sh;
        if (j < 2) q.x = (q.x & keep) | x;
        else if (j < 4) q.y = (q.y & keep) | x;
        else if (j < 6) q.z = (q.z & keep) | x;
        else q.w = (q.w & keep) | x;
    }
    __device__ void zero() { q = make_uint4(0, 0, 0, 0); }
    // bit j set iff element j's bit pattern (sign ignored) is nonzero.  Adding
    // 0x7FFF to a 15-bit magnitude carries into bit 15 exactly when it is > 0;
    // the carries of words 0..3 land on bits 0,16 / 2,18 / 4,20 / 6,22 of x,
    // and x | x >> 15 brings the odd elements down to bits 1, 3, 5, 7.
    __device__ uint32_t nonzero_byte() const {
        const uint32_t t0 = (q.x & 0x7FFF7FFFu) + 0x7FFF7FFFu, t1 = (q.y & 0x7FFF7FFFu) + 0x7FFF7FFFu;
        const uint32_t t2 = (q.z & 0x7FFF7FFFu) + 0x7FFF7FFFu, t3 = (q.w & 0x7FFF7FFFu) + 0x7FFF7FFFu;
        const uint32_t x = ((t0 & 0x80008000u) >> 15) | ((t1 & 0x80008000u) >> 13) |
                           ((t2 & 0x80008000u) >> 11) | ((t3 & 0x80008000u) >> 9);
        return (x | (x >> 15)) & 0xFFu;
    }
    __device__ void store_first16(uint16_t* p) const { *reinterpret_cast<uint4*>(p) = q; }
    __device__ void load_smem(const uint16_t* p) { q = *reinterpret_cast<const uint4*>(p); }
    __device__ void store_global_cs(uint16_t* p) const { __stcs(reinterpret_cast<uint4*>(p), q); }
};
template <> struct Vec8<uint32_t> {
    uint4 a, b;
    __device__ uint32_t get(int j) const {
        return j == 0 ? a.x : j == 1 ? a.y : j == 2 ? a.z : j == 3 ? a.w
             : j == 4 ? b.x : j == 5 ? b.y : j == 6 ? b.z : b.w;
    }
    __device__ void set(int j, uint32_t v) {
        if (j == 0) a.x = v; else if (j == 1) a.y = v; else if (j == 2) a.z = v;
        else if (j == 3) a.w = v; else if (j == 4) b.x = v; else if (j == 5) b.y = v;
        else if (j == 6) b.z = v; else b.w = v;
    }
    __device__ void zero() { a = make_uint4(0, 0, 0, 0); b = a; }
    __device__ uint32_t nonzero_byte() const {
        uint32_t r = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) r |= (uint32_t)nonzero_bits(get(j)) << j;
        return r;
    }
    __device__ void store_first16(uint32_t* p) const { *reinterpret_cast<uint4*>(p) = a; }
    __device__ void load_smem(const uint32_t* p) {
        a = reinterpret_cast<const uint4*>(p)[0];
        b = reinterpret_cast<const uint4*>(p)[1];
    }
    __device__ void store_global_cs(uint32_t* p) const {
        __stcs(reinterpret_cast<uint4*>(p), a);
        __stcs(reinterpret_cast<uint4*>(p) + 1, b);
    }
};

// ------------------------------------------------------------------ pack ----
// Persistent and pipelined, one CTA per SM: 16 compute warps and a look-back
// warp, a ring of five 32 KB input buffers filled by bulk copies, and a 32 KB
// ring of compacted values.  Iteration k of the compute warps:
//   1. scan tile k: mask bytes, mask words to global memory, counts, CTA scan,
//      publication of the tile aggregate for the look-back warp;
//   2. compact tile k's set elements into the value ring (writing out older
//      tiles first if the ring lacks room);
//   3. start the bulk copy of tile k+5 into the input buffer just freed;
//   4. write to `vals` every compacted tile up to k-2, at the offset the
//      look-back warp found for it meanwhile.
// So the input buffers are busy only while a tile is in flight or scanned,
// and the look-back latency stays off the compute warps' path.
// Warp w owns the contiguous chunks (8 elements each) CPW*w .. CPW*w+CPW-1 of
// the tile.  In the load layout lane l reads chunks l, l+32, ... (512
// contiguous bytes of shared memory per instruction); in the count layout
// lane l owns G consecutive chunks (one mask word) and compacts them by
// walking the word's set bits, at the warp's base + its exclusive count.
constexpr int FP_CW = 16;                 // compute warps
constexpr int FP_CT = FP_CW * 32;         // compute threads
constexpr int FP_THREADS = FP_CT + 32;    // plus the look-back warp
constexpr int FP_NB = 5;                  // input tile buffers
constexpr int FP_D = 2;                   // a tile is written out D iterations after its scan
static_assert(FP_D < FP_NB, "a tile's bookkeeping lives until its write-out");
constexpr int FP_BAR = 1;                 // named barrier of the compute warps

// OR of `p` over the `n` threads that reach named barrier `id`.
__device__ __forceinline__ bool named_bar_or(int id, int n, bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

template <typename B>
struct PackCfg {
    static constexpr int TILE = FT_TILE_BYTES / (int)sizeof(B);  // elements per tile
    static constexpr int CHUNKS = TILE / 8;                      // mask bytes per tile
    static constexpr int CPW = CHUNKS / FP_CW;                    // chunks per warp
    static constexpr int G = CPW / 32;                            // chunks per lane
    static constexpr int EPV = 16 / (int)sizeof(B);               // elements per 16 bytes
    static_assert(G == 4 || G == 2, "32- or 16-bit mask words per lane");
    static constexpr int RC = TILE;  // value ring, in elements (a power of two)
    static_assert((RC & (RC - 1)) == 0, "ring index by mask");
    static constexpr size_t SMEM = (size_t)(FP_NB * TILE + RC) * sizeof(B) + (size_t)CHUNKS;
};

// This lane's G mask bytes (count layout) from the warp's byte region.
template <int G>
__device__ __forceinline__ uint32_t lane_bits(const uint8_t* wmb, int lane) {
    if constexpr (G == 4) return *reinterpret_cast<const uint32_t*>(wmb + 4 * lane);
    else return *reinterpret_cast<const uint16_t*>(wmb + 2 * lane);
}

// VEC: `vals` is 16-byte aligned (16-byte stores for the write-out).
template <typename B, bool VEC>
__global__ void __launch_bounds__(FP_THREADS, 1) flat_pack_kernel(
    const B* __restrict__ dense, long long n, uint8_t* __restrict__ mask, B* __restrict__ vals,
    long long cap, long long* __restrict__ nnz_out, unsigned long long* __restrict__ states,
    unsigned int* __restrict__ ticket, uint32_t* __restrict__ status, long long ntiles) {
    using C = PackCfg<B>;
    constexpr int TILE = C::TILE, CPW = C::CPW, G = C::G, EPV = C::EPV, RC = C::RC;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    B* s_buf = reinterpret_cast<B*>(smem_raw);                                 // [NB][TILE]
    B* s_ring = s_buf + (size_t)FP_NB * TILE;                                  // [RC]
    uint8_t* s_mb = reinterpret_cast<uint8_t*>(s_ring + RC);                   // [CHUNKS]
    __shared__ __align__(8) uint64_t full[FP_NB], pub[FP_NB], exr[FP_NB];
    __shared__ long long s_tile[FP_NB];  // tile in each input buffer
    // per scanned tile j, in slot j % NB until its write-out: tile number,
    // offset in `vals`, value count, start in the value ring
    __shared__ long long s_wtile[FP_NB], s_ex[FP_NB], s_rst[FP_NB];
    __shared__ int s_agg[FP_NB];
    __shared__ int s_wt[FP_CW];
    __shared__ volatile int s_abort;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long nbytes = (n + 7) >> 3;
    if (tid == 0) {
        for (int j = 0; j < FP_NB; ++j) {
            mbar_init(&full[j], 1);
            mbar_init(&pub[j], 1);
            mbar_init(&exr[j], 1);
        }
        s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // ---------------------------------------------------- look-back warp ----
    // Resolves this CTA's scanned tiles in order: tile j in slot j % NB.
    if (warp == FP_CW) {
        for (int j = 0;; ++j) {
            const int b = j % FP_NB;
            const bool ok = __all_sync(FULL, mbar_wait_bounded(&pub[b], (uint32_t)(j / FP_NB) & 1u));
            if (!ok || s_abort) {
                if (!ok && lane == 0) {
                    atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                    s_abort = 1;
                }
                break;
            }
            const long long t = s_wtile[b];
            if (t >= ntiles) break;
            const unsigned long long ex =
                lookback_rows<FT_LBW>(states, t, (unsigned long long)s_agg[b], status, lane);
            if (lane == 0) {
                s_ex[b] = (long long)ex;
                mbar_arrive(&exr[b]);
            }
            __syncwarp();
        }
        return;
    }

    // ------------------------------------------------------ compute warps ----
    // thread 0: take the next tile into buffer j and start its copy
    auto acquire = [&](int j) {
        const long long t = (long long)atomicAdd(ticket, 1u);
        s_tile[j] = t;
        uint32_t bytes = 0;
        if (t < ntiles) {
            const long long nv = min((long long)TILE, n - t * TILE);
            bytes = (uint32_t)(nv * (long long)sizeof(B)) & ~15u;
        }
        if (bytes) {
            mbar_arrive_expect_tx(&full[j], bytes);
            bulk_g2s(s_buf + (size_t)j * TILE, dense + t * TILE, bytes, &full[j]);
        } else {
            mbar_arrive(&full[j]);
        }
    };
    // Give up after a wait ran out: resolve the tiles this CTA holds for the
    // successors, wait (bounded) for the `cnt` copies in flight from iteration
    // k0 on, and wake the look-back warp.
    auto abort_all = [&](int k0, int cnt) {
        if (tid == 0) {
            atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
            s_abort = 1;
            for (int j = 0; j < FP_NB; ++j) {
                if (s_tile[j] < ntiles) st_relaxed_u64(&states[s_tile[j]], LB_INCL);
                if (s_wtile[j] < ntiles) st_relaxed_u64(&states[s_wtile[j]], LB_INCL);
            }
            for (int j = 0; j < cnt; ++j)
                (void)mbar_wait_bounded(&full[(k0 + j) % FP_NB], (uint32_t)((k0 + j) / FP_NB) & 1u);
            for (int j = 0; j < FP_NB; ++j) mbar_arrive(&pub[j]);
        }
    };
    if (tid == 0)
        for (int j = 0; j < FP_NB; ++j) {
            s_wtile[j] = ntiles;
            acquire(j);
        }

    // Every compute thread keeps the same ring and write-out counters.
    long long head = 0, tail = 0;  // value ring: elements written / freed
    int wnext = 0;                 // next scanned tile to write out
    int k_end = -1;                // first iteration whose tile was past the end
    // Writes tile j's compacted values to `vals` (after its look-back); false
    // if the wait for the look-back ran out (the CTA then gives up).
    auto write_out = [&](int j) -> bool {
        const int bj = j % FP_NB;
        const bool okw = mbar_wait_bounded(&exr[bj], (uint32_t)(j / FP_NB) & 1u);
        if (named_bar_or(FP_BAR, FP_CT, !okw)) return false;
        const long long ex = s_ex[bj], rs = s_rst[bj], tw = s_wtile[bj];
        const int agg = s_agg[bj];
        // [ex, ex + agg) clipped to the capacity of `vals`
        const int lim = (int)max(0ll, min((long long)agg, cap - ex));
        int done = 0;
        if (VEC) {
            const int h = min(lim, (int)((EPV - ex % EPV) % EPV));  // to a 16-byte boundary
            if (tid < h) vals[ex + tid] = s_ring[(rs + tid) & (RC - 1)];
            const int nvec = (lim - h) / EPV;
            for (int v = tid; v < nvec; v += FP_CT) {
                const long long i0 = rs + h + v * EPV;
                Vec8<B> o;
#pragma unroll
                for (int e = 0; e < EPV; ++e) o.set(e, s_ring[(i0 + e) & (RC - 1)]);
                o.store_first16(vals + ex + h + v * EPV);
            }
            done = h + nvec * EPV;
        }
        for (int i = done + tid; i < lim; i += FP_CT) vals[ex + i] = s_ring[(rs + i) & (RC - 1)];
        if (tid == 0) {
            if (ex + agg > cap) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
            if (tw == ntiles - 1) *nnz_out = ex + agg;
        }
        tail += agg;
        return true;
    };

    for (int k = 0;; ++k) {
        const int b = k % FP_NB;
        bool have = false;
        if (k_end < 0) {
            // ---- 1. scan of tile k ----
            const bool ok = mbar_wait_bounded(&full[b], (uint32_t)(k / FP_NB) & 1u);
            if (named_bar_or(FP_BAR, FP_CT, !ok)) {
                abort_all(k, FP_NB);
                return;
            }
            have = s_tile[b] < ntiles;
            if (!have) {
                k_end = k;
                if (tid == 0) {
                    s_wtile[b] = ntiles;
                    mbar_arrive(&pub[b]);  // tells the look-back warp that the tiles ended
                }
            }
        }
        if (have) {
            const long long t = s_tile[b];
            const B* in = s_buf + (size_t)b * TILE;
            const long long base = t * TILE;
            const int nvalid = (int)min((long long)TILE, n - base);
            const int tma_elems =
                (int)(((long long)nvalid * (long long)sizeof(B)) & ~15ll) / (int)sizeof(B);
            if (tma_elems < nvalid) {  // the last tile's tail, not a multiple of 16 bytes
                for (int i = tma_elems + tid; i < nvalid; i += FP_CT)
                    const_cast<B*>(in)[i] = dense[base + i];
                named_bar_sync(FP_BAR, FP_CT);
            }
            uint8_t* wmb = s_mb + CPW * warp;
            // load layout: mask byte of chunk CPW*warp + lane + 32*g
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const int f = 8 * (CPW * warp + lane + 32 * g);
                uint32_t byte = 0;
                if (f < nvalid) {
                    Vec8<B> v;
                    v.load_smem(in + f);
                    byte = v.nonzero_byte();
                    if (f + 8 > nvalid) byte &= (1u << (nvalid - f)) - 1u;
                }
                wmb[lane + 32 * g] = (uint8_t)byte;
            }
            __syncwarp();
            // count layout: this lane's G chunks as one mask word
            uint32_t m = lane_bits<G>(wmb, lane);
            {
                const long long byte0 = (base >> 3) + (long long)CPW * warp + (long long)G * lane;
                if (byte0 + G <= nbytes) {
                    if (G == 4) *reinterpret_cast<uint32_t*>(mask + byte0) = m;
                    else *reinterpret_cast<uint16_t*>(mask + byte0) = (uint16_t)m;
                } else {
                    for (int e = 0; e < G; ++e)
                        if (byte0 + e < nbytes) mask[byte0 + e] = (uint8_t)(m >> (8 * e));
                }
            }
            const int cnt = __popc(m);
            const int inc = warp_incl_scan(cnt, lane);
            if (lane == 31) s_wt[warp] = inc;
            named_bar_sync(FP_BAR, FP_CT);
            const int wv = lane < FP_CW ? s_wt[lane] : 0;
            const int wi = warp_incl_scan(wv, lane);
            const int wbase = __shfl_sync(FULL, wi - wv, warp);
            const int agg = __shfl_sync(FULL, wi, FP_CW - 1);
            if (tid == 0) {
                s_wtile[b] = t;
                s_agg[b] = agg;
                s_rst[b] = head;
                lookback_publish_relaxed(states, t, (unsigned long long)agg);
                mbar_arrive(&pub[b]);
            }
            // ---- 2. compaction into the value ring ----
            if (RC - (head - tail) < agg) {
                while (RC - (head - tail) < agg)
                    if (!write_out(wnext++)) {
                        abort_all(k + 1, FP_NB - 1);
                        return;
                    }
                named_bar_sync(FP_BAR, FP_CT);  // freed ring slots fully read
            }
            {
                const B* src = in + 8 * (CPW * warp + G * lane);
                long long p = head + wbase + (inc - cnt);
                while (m) {
                    const int j = __ffs(m) - 1;
                    m &= m - 1;
                    s_ring[(p++) & (RC - 1)] = src[j];
                }
            }
            head += agg;
        }
        // ---- 3. the input buffer of tile k is free: tile k+NB ----
        named_bar_sync(FP_BAR, FP_CT);
        if (tid == 0 && have) {
            fence_proxy_async_smem();
            acquire(b);
        }
        // ---- 4. write-out of the tiles scanned D or more iterations ago ----
        const int upto = k_end < 0 ? k - FP_D : k_end - 1;
        while (wnext <= upto)
            if (!write_out(wnext++)) {
                abort_all(k + 1, k_end < 0 ? FP_NB : 0);
                return;
            }
        if (k_end >= 0) break;  // every scanned tile is written
        named_bar_sync(FP_BAR, FP_CT);  // ring slots written out are fully read
    }
}


// ---------------------------------------------------------------- unpack ----
constexpr int PK_CW = 8;                       // compute warps (unpack)
constexpr int PK_THREADS = (PK_CW + 1) * 32;   // plus the look-back warp
constexpr int PK_NB = 3;                       // tile buffers
constexpr int PK_BAR = 1;                      // named barrier of the compute warps
constexpr int PK_CT = PK_CW * 32;              // compute threads

// The CPT mask bytes of owner thread `o` (count layout) as one word.
template <int CPT>
__device__ __forceinline__ uint64_t owner_bits(const uint8_t* s_mb, int o) {
    if constexpr (CPT == 8) return *reinterpret_cast<const uint64_t*>(s_mb + 8 * o);
    else return *reinterpret_cast<const uint32_t*>(s_mb + 4 * o);
}

// Same pipeline as pack.  In iteration k the compute warps count tile k (its
// mask words were loaded into registers during iteration k-1) and expand tile
// k-1; the look-back warp resolves tile k and then starts the bulk copy of its
// values into the tile's buffer, so the values are in shared memory when the
// compute warps expand it in iteration k+1.  The dense tile is written with
// 16-byte streaming stores, 512 contiguous bytes per warp instruction.
template <typename B>
struct UnpackCfg {
    static constexpr int TILE = FT_TILE_BYTES / (int)sizeof(B);
    static constexpr int CHUNKS = TILE / 8;
    static constexpr int G = CHUNKS / PK_CT;
    static constexpr int EPV = 16 / (int)sizeof(B);  // elements per 16-byte vector
    static constexpr int VCAP = TILE + 2 * EPV;      // staged values, with alignment slack
    static_assert(G == 8 || G == 4, "64- or 32-bit words in the count layout");
    static constexpr size_t SMEM =
        (size_t)PK_NB * VCAP * sizeof(B) + (size_t)PK_NB * CHUNKS + (size_t)PK_NB * PK_CT * 4;
};

// VEC: `vals` is 16-byte aligned, so the look-back warp bulk-copies values.
template <typename B, bool VEC>
__global__ void __launch_bounds__(PK_THREADS, 2) flat_unpack_kernel(
    const B* __restrict__ vals, long long vals_len, const uint8_t* __restrict__ mask, long long n,
    B* __restrict__ out, unsigned long long* __restrict__ states, unsigned int* __restrict__ ticket,
    uint32_t* __restrict__ status, long long ntiles) {
    using C = UnpackCfg<B>;
    constexpr int TILE = C::TILE, CHUNKS = C::CHUNKS, G = C::G, EPV = C::EPV, VCAP = C::VCAP;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    B* s_vals = reinterpret_cast<B*>(smem_raw);                                // [NB][VCAP]
    uint8_t* s_mb = smem_raw + (size_t)PK_NB * VCAP * sizeof(B);               // [NB][CHUNKS]
    int* s_off = reinterpret_cast<int*>(s_mb + (size_t)PK_NB * CHUNKS);        // [NB][CT]
    __shared__ __align__(8) uint64_t pub[PK_NB], vfull[PK_NB];
    __shared__ long long s_tile[PK_NB], s_ex[PK_NB], s_va0[PK_NB], s_vend[PK_NB];
    __shared__ int s_wt[PK_NB][PK_CW], s_wb[PK_NB][PK_CW], s_agg[PK_NB];
    __shared__ volatile int s_abort;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long nbytes = (n + 7) >> 3;
    if (tid == 0) {
        for (int j = 0; j < PK_NB; ++j) {
            mbar_init(&pub[j], 1);
            mbar_init(&vfull[j], 1);
        }
        s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // ---------------------------------------------------- look-back warp ----
    if (warp == PK_CW) {
        for (int k = 0;; ++k) {
            const int b = k % PK_NB;
            const bool ok = __all_sync(FULL, mbar_wait_bounded(&pub[b], (uint32_t)(k / PK_NB) & 1u));
            if (!ok || s_abort) {
                if (!ok && lane == 0) {
                    atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                    s_abort = 1;
                }
                break;
            }
            const long long t = s_tile[b];
            if (t >= ntiles) break;
            const int agg = s_agg[b];
            const long long ex =
                (long long)lookback_rows<FT_LBW>(states, t, (unsigned long long)agg, status, lane);
            if (lane == 0) {
                // values [ex, ex+agg): the 16-byte-aligned part that lies inside
                // vals_len by one bulk copy, the rest by the compute warps
                long long a0 = ex, a1 = ex;
                if (VEC) {
                    a0 = ex & ~(long long)(EPV - 1);
                    a1 = min((ex + agg + EPV - 1) & ~(long long)(EPV - 1),
                             vals_len & ~(long long)(EPV - 1));
                    if (a1 < a0) a1 = a0;
                }
                s_ex[b] = ex;
                s_va0[b] = a0;
                s_vend[b] = a1;
                if (a1 > a0) {
                    fence_proxy_async_smem();
                    const uint32_t bytes = (uint32_t)((a1 - a0) * (long long)sizeof(B));
                    mbar_arrive_expect_tx(&vfull[b], bytes);
                    bulk_g2s(s_vals + (size_t)b * VCAP, vals + a0, bytes, &vfull[b]);
                } else {
                    mbar_arrive(&vfull[b]);
                }
            }
            __syncwarp();
        }
        return;
    }

    // ------------------------------------------------------ compute warps ----
    // this thread's G mask bytes (count layout) of tile t, bits past n cleared
    auto load_bits = [&](long long t) -> uint64_t {
        if (t >= ntiles) return 0;
        const long long base = t * TILE;
        const long long byte0 = (base >> 3) + (long long)G * tid;
        uint64_t m = 0;
        if (byte0 + G <= nbytes) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(mask + byte0);
            m = __ldcs(src);
            if (G == 8) m |= (uint64_t)__ldcs(src + 1) << 32;
        } else {
            for (int e = 0; e < G; ++e)
                if (byte0 + e < nbytes) m |= (uint64_t)mask[byte0 + e] << (8 * e);
        }
        const long long e0 = base + 8LL * G * tid;  // element of bit 0
        if (e0 + 8 * G > n) {
            const long long keep = n - e0;
            m = keep <= 0 ? 0 : (m & ((1ull << keep) - 1ull));
        }
        return m;
    };
    if (tid == 0) s_tile[0] = (long long)atomicAdd(ticket, 1u);
    named_bar_sync(PK_BAR, PK_CT);
    uint64_t m_cur = load_bits(s_tile[0]);

    for (int k = 0;; ++k) {
        const int b = k % PK_NB, bn = (k + 1) % PK_NB;
        if (tid == 0) s_tile[bn] = (long long)atomicAdd(ticket, 1u);
        named_bar_sync(PK_BAR, PK_CT);
        const uint64_t m_next = load_bits(s_tile[bn]);  // consumed next iteration
        // ---- counts of tile k ----
        const long long t = s_tile[b];
        const bool have = t < ntiles;
        if (have) {
            uint8_t* mb = s_mb + (size_t)b * CHUNKS;
            if (G == 8) *reinterpret_cast<uint64_t*>(mb + 8 * tid) = m_cur;
            else *reinterpret_cast<uint32_t*>(mb + 4 * tid) = (uint32_t)m_cur;
            const int cnt = __popcll(m_cur);
            const int inc = warp_incl_scan(cnt, lane);
            s_off[(size_t)b * PK_CT + tid] = inc - cnt;
            if (lane == 31) s_wt[b][warp] = inc;
            named_bar_sync(PK_BAR, PK_CT);
            if (warp == 0) {
                const int w = lane < PK_CW ? s_wt[b][lane] : 0;
                const int wi = warp_incl_scan(w, lane);
                if (lane < PK_CW) s_wb[b][lane] = wi - w;
                const int agg = __shfl_sync(FULL, wi, PK_CW - 1);
                if (lane == 0) {
                    s_agg[b] = agg;
                    lookback_publish_relaxed(states, t, (unsigned long long)agg);
                    mbar_arrive(&pub[b]);
                }
            }
        } else if (tid == 0) {
            mbar_arrive(&pub[b]);  // tells the look-back warp that the tiles ended
        }

        // ---- expansion of tile k-1 ----
        if (k >= 1) {
            const int bp = (k - 1) % PK_NB;
            const long long tp = s_tile[bp];
            if (tp < ntiles) {
                const bool okp = mbar_wait_bounded(&vfull[bp], (uint32_t)((k - 1) / PK_NB) & 1u);
                if (named_bar_or(PK_BAR, PK_CT, !okp)) {
                    if (tid == 0) {
                        atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        for (int j = 0; j < PK_NB; ++j)
                            if (s_tile[j] < ntiles) st_relaxed_u64(&states[s_tile[j]], LB_INCL);
                        (void)mbar_wait_bounded(&vfull[bp], (uint32_t)((k - 1) / PK_NB) & 1u);
                        for (int j = 0; j < PK_NB; ++j) mbar_arrive(&pub[j]);
                    }
                    return;
                }
                const long long ex = s_ex[bp], a0 = s_va0[bp], vend = s_vend[bp];
                const int agg = s_agg[bp];
                B* sv = s_vals + (size_t)bp * VCAP;
                if (tid == 0 && ex + agg > vals_len) atomicOr(status, SFFN_STATUS_VALS_SHORT);
                // values not covered by the bulk copy (none, except at the end of
                // `vals` or when `vals` is not 16-byte aligned); past vals_len -> 0
                const long long r0 = max(ex, vend), r1 = ex + agg;
                if (r0 < r1) {
                    for (long long i = r0 + tid; i < r1; i += PK_CT) sv[i - a0] = i < vals_len ? vals[i] : B(0);
                    named_bar_sync(PK_BAR, PK_CT);
                }
                const uint8_t* mbp = s_mb + (size_t)bp * CHUNKS;
                const int* offp = s_off + (size_t)bp * PK_CT;
                const long long base = tp * TILE;
                const int nvalid = (int)min((long long)TILE, n - base);
                const int shift = (int)(ex - a0);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const int c = tid + PK_CT * g, f = 8 * c;
                    if (f >= nvalid) continue;
                    const uint32_t byte = mbp[c];
                    Vec8<B> o;
                    o.zero();
                    if (byte) {
                        const int ow = c / G, sub = c % G;
                        const uint64_t mo = owner_bits<G>(mbp, ow);
                        int r = shift + s_wb[bp][ow >> 5] + offp[ow] +
                                __popcll(mo & ((1ull << (8 * sub)) - 1ull));
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if ((byte >> j) & 1u) o.set(j, sv[r++]);
                    }
                    if (f + 8 <= nvalid) {
                        o.store_global_cs(out + base + f);
                    } else {
                        for (int j = 0; j < 8; ++j)
                            if (f + j < nvalid) out[base + f + j] = o.get(j);
                    }
                }
            }
        }
        if (!have) break;
        named_bar_sync(PK_BAR, PK_CT);  // buffers of tile k-1 fully read
        m_cur = m_next;
    }
}

template <typename B>
inline long long flat_tiles(long long n) { return (n + PackCfg<B>::TILE - 1) / PackCfg<B>::TILE; }

template <typename K>
cudaError_t allow_smem(K kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// `scratch`: [0,16) tile ticket, then one 8-byte look-back state per tile;
// both are cleared on the stream before the kernel runs.
int num_sms() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

template <typename B, bool VEC>
int launch_pack_v(const B* dense, long long n, uint8_t* mask, B* vals, long long cap,
                  long long* nnz, unsigned long long* states, unsigned int* ticket,
                  uint32_t* status, long long nt, cudaStream_t st) {
    auto k = flat_pack_kernel<B, VEC>;
    const int smem = (int)PackCfg<B>::SMEM;
    SFFN_CUDA_TRY(allow_smem(k, smem));
    int per_sm = 0;
    SFFN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, FP_THREADS, smem));
    if (per_sm < 1) return SFFN_ERR_CUDA;
    const long long grid = std::min<long long>(nt, (long long)per_sm * num_sms());
    k<<<(unsigned)grid, FP_THREADS, smem, st>>>(dense, n, mask, vals, cap, nnz, states, ticket,
                                                 status, nt);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <typename B>
int launch_pack(const void* dense, long long n, uint8_t* mask, void* vals, long long cap,
                int64_t* nnz_dev, void* scratch, uint32_t* status, cudaStream_t st) {
    const long long nt = flat_tiles<B>(n);
    auto* ticket = static_cast<unsigned int*>(scratch);
    auto* states = reinterpret_cast<unsigned long long*>(static_cast<char*>(scratch) + 16);
    SFFN_CUDA_TRY(cudaMemsetAsync(scratch, 0, 16 + (size_t)nt * 8, st));
    const B* d = static_cast<const B*>(dense);
    B* v = static_cast<B*>(vals);
    long long* nz = reinterpret_cast<long long*>(nnz_dev);
    if (aligned16(vals))
        return launch_pack_v<B, true>(d, n, mask, v, cap, nz, states, ticket, status, nt, st);
    return launch_pack_v<B, false>(d, n, mask, v, cap, nz, states, ticket, status, nt, st);
}

template <typename B, bool VEC>
int launch_unpack_v(const B* vals, long long vals_len, const uint8_t* mask, long long n, B* out,
                    unsigned long long* states, unsigned int* ticket, uint32_t* status,
                    long long nt, cudaStream_t st) {
    auto k = flat_unpack_kernel<B, VEC>;
    const int smem = (int)UnpackCfg<B>::SMEM;
    SFFN_CUDA_TRY(allow_smem(k, smem));
    int per_sm = 0;
    SFFN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, PK_THREADS, smem));
    if (per_sm < 1) return SFFN_ERR_CUDA;
    const long long grid = std::min<long long>(nt, (long long)per_sm * num_sms());
    k<<<(unsigned)grid, PK_THREADS, smem, st>>>(vals, vals_len, mask, n, out, states, ticket,
                                                 status, nt);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <typename B>
int launch_unpack(const void* vals, long long vals_len, const uint8_t* mask, long long n, void* out,
                  void* scratch, uint32_t* status, cudaStream_t st) {
    const long long nt = flat_tiles<B>(n);
    auto* ticket = static_cast<unsigned int*>(scratch);
    auto* states = reinterpret_cast<unsigned long long*>(static_cast<char*>(scratch) + 16);
    SFFN_CUDA_TRY(cudaMemsetAsync(scratch, 0, 16 + (size_t)nt * 8, st));
    const B* v = static_cast<const B*>(vals);
    if (aligned16(vals))
        return launch_unpack_v<B, true>(v, vals_len, mask, n, static_cast<B*>(out), states, ticket,
                                        status, nt, st);
    return launch_unpack_v<B, false>(v, vals_len, mask, n, static_cast<B*>(out), states, ticket,
                                     status, nt, st);
}

}  // namespace
}  // namespace sffn

using namespace sffn;

// Workspace: [0,16) tile ticket, then one 8-byte look-back state per tile of
// 32 KB of dense data, counted for the widest type (8192 elements per tile).
extern "C" size_t sffn_flat_workspace_bytes(int64_t n) {
    if (n < 0) return 0;
    return 16 + (size_t)((n + FT_MIN_TILE - 1) / FT_MIN_TILE) * 8;
}

extern "C" int sffn_flat_pack(const void* dense, int dtype, int64_t n, uint8_t* packed_mask,
                              void* vals, int64_t vals_capacity, int64_t* nnz_dev, void* workspace,
                              size_t workspace_bytes, uint32_t* status_dev, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (n < 0 || vals_capacity < 0 || !nnz_dev || !status_dev) return SFFN_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        if (int rc = bind_device_of(nnz_dev)) return rc;
        SFFN_CUDA_TRY(cudaMemsetAsync(nnz_dev, 0, sizeof(int64_t), st));
        return SFFN_OK;
    }
    if (!dense || !packed_mask || (!vals && vals_capacity > 0) || !workspace) return SFFN_ERR_ARG;
    if (!aligned16(dense) || (reinterpret_cast<uintptr_t>(packed_mask) & 3u)) return SFFN_ERR_ALIGN;
    if (workspace_bytes < sffn_flat_workspace_bytes(n)) return SFFN_ERR_WORKSPACE;
    if ((n + FT_MIN_TILE - 1) / FT_MIN_TILE > 0x7FFFFFFFll) return SFFN_ERR_ARG;  // grid limit
    if (int rc = bind_device_of(dense)) return rc;
    if (esize_of(dtype) == 4)
        return launch_pack<uint32_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, workspace,
                                     status_dev, st);
    return launch_pack<uint16_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, workspace,
                                 status_dev, st);
}

extern "C" int sffn_flat_unpack(const void* vals, int64_t vals_len, const uint8_t* packed_mask,
                                int dtype, int64_t n, void* out, void* workspace,
                                size_t workspace_bytes, uint32_t* status_dev, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (n < 0 || vals_len < 0 || !status_dev) return SFFN_ERR_ARG;
    if (n == 0) return SFFN_OK;
    if (!packed_mask || !out || !workspace || (!vals && vals_len > 0)) return SFFN_ERR_ARG;
    if (!aligned16(out) || (reinterpret_cast<uintptr_t>(packed_mask) & 3u)) return SFFN_ERR_ALIGN;
    if (workspace_bytes < sffn_flat_workspace_bytes(n)) return SFFN_ERR_WORKSPACE;
    if ((n + FT_MIN_TILE - 1) / FT_MIN_TILE > 0x7FFFFFFFll) return SFFN_ERR_ARG;  // grid limit
    if (int rc = bind_device_of(out)) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (esize_of(dtype) == 4)
        return launch_unpack<uint32_t>(vals, vals_len, packed_mask, n, out, workspace, status_dev, st);
    return launch_unpack<uint16_t>(vals, vals_len, packed_mask, n, out, workspace, status_dev, st);
}

// ---------------------------------------------------------------------------
// sffn_flat_pack_noalloc: the flat pack for callers that cannot allocate.
//
// Some callers have no way to obtain device memory: plug-ins handed only their
// input and output buffers by a host application, programs whose memory
// manager owns the whole device or works to a fixed, pre-planned budget, and
// latency-critical paths that cannot afford the device-wide synchronisation a
// cudaMalloc may cause.  This entry point needs no workspace from them: the
// look-back state lives in the fixed array below, which every GPU that loads
// this library holds until the process exits.
//
// Set-up: the first call on a device looks up that device's address of the
// array with cudaGetSymbolAddress (with the device current) and caches it;
// make that first call before any stream capture.  Every call shares the
// array and finds the previous call's contents in it, so each call clears the
// part it uses before its kernel runs; calls that overlap on the GPU (other
// streams, other host threads) race on it and must be serialised by the caller.
// ---------------------------------------------------------------------------
namespace sffn {
namespace {

constexpr long long kNoAllocMaxTiles = 4096;  // 4096 tiles of 32 KB of input
static __device__ __align__(256) unsigned char g_noalloc_scratch[16 + kNoAllocMaxTiles * 8];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of the scratch array on `dev` (which must be current).
int noalloc_scratch(int dev, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return SFFN_ERR_ARG;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            set_cuda_error(e);
            return SFFN_ERR_CUDA;
        }
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return SFFN_OK;
}

}  // namespace
}  // namespace sffn

// Largest n accepted: 67,108,864 elements of 2 bytes, 33,554,432 of 4 bytes.
static long long noalloc_max_elements(int dtype) {
    return kNoAllocMaxTiles * (FT_TILE_BYTES / esize_of(dtype));
}

extern "C" int sffn_flat_pack_noalloc(const void* dense, int dtype, int64_t n, uint8_t* packed_mask,
                                      void* vals, int64_t vals_capacity, int64_t* nnz_dev,
                                      uint32_t* status_dev, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (n < 0 || vals_capacity < 0 || !nnz_dev || !status_dev) return SFFN_ERR_ARG;
    if (n > noalloc_max_elements(dtype)) {
        char msg[160];
        snprintf(msg, sizeof(msg), "sffn_flat_pack_noalloc: %lld elements exceed its fixed scratch capacity of %lld",
                 (long long)n, noalloc_max_elements(dtype));
        set_error_text(msg);
        return SFFN_ERR_TOO_LARGE;
    }
    if (n > 0 && (!dense || !packed_mask || (!vals && vals_capacity > 0))) return SFFN_ERR_ARG;
    if (n > 0 && (!aligned16(dense) || (reinterpret_cast<uintptr_t>(packed_mask) & 3u))) return SFFN_ERR_ALIGN;
    // Select the device that owns the output (cudaSetDevice initialises its
    // context); nothing on this path allocates or frees device memory.
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, nnz_dev) != cudaSuccess ||
        (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
        cudaGetLastError();
        return SFFN_ERR_ARG;
    }
    SFFN_CUDA_TRY(cudaSetDevice(attr.device));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        SFFN_CUDA_TRY(cudaMemsetAsync(nnz_dev, 0, sizeof(int64_t), st));
        return SFFN_OK;
    }
    void* scratch = nullptr;
    if (int rc = noalloc_scratch(attr.device, &scratch)) return rc;
    // launch_pack clears the ticket and the states this call uses (the
    // previous call left its own in the array) before the kernel runs.
    if (esize_of(dtype) == 4)
        return launch_pack<uint32_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, scratch,
                                     status_dev, st);
    return launch_pack<uint16_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, scratch,
                                 status_dev, st);
}
