// Flat bitmask format: pack and unpack (sm_100a).
//
// Reference: old/sparse_pack.py:6-106 (count/pack kernel, one-program serial
// prefix, vals kernel -- the dense tensor is read twice) and
// old/sparse_unpack.py:6-97 (popcount, one-program serial prefix, rebuild).
//
// Two implementations:
//   * sffn_flat_pack / sffn_flat_unpack (workspace): per-tile counts, one
//     scan block, then independent blocks that compact or expand their tile
//     at its offset -- full occupancy, no waits between blocks (see "scan-based
//     path" below).  Unpack reads the mask twice, pack the dense tensor.
//   * sffn_flat_pack_noalloc (fixed 32 KB scratch): one single-pass persistent
//     kernel over 32 KB tiles whose offsets come from a decoupled look-back
//     (see "pack" below), so the dense tensor crosses HBM once and the scratch
//     holds one state per tile.
//
// Mask layout: element f -> byte f/8, bit f%8 (a little-endian uint32 word w
// holds elements 32w .. 32w+31).  Values are in element order.
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
    __device__ void load_global(const uint16_t* p) { q = __ldg(reinterpret_cast<const uint4*>(p)); }
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
    __device__ void load_global(const uint32_t* p) {
        a = __ldg(reinterpret_cast<const uint4*>(p));
        b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
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
// Persistent and pipelined, one CTA per SM: 16 compute warps, two look-back
// warps (even and odd tiles of the CTA), and a loader warp that takes tiles
// by ticket and fills a ring of five 32 KB input buffers by bulk copies, so
// neither the ticket nor the look-back latency is on the compute warps' path.
// The loader keeps four ticket requests in flight (one thread's atomics on
// one address return in order, so its tiles still rise); one tile per ticket
// keeps the CTAs' tiles interleaved -- a CTA holding a run of consecutive
// tiles would make the next CTA's look-backs wait on its iterations, and so
// on around the grid.  A 32 KB ring holds compacted values.  Iteration k of
// the compute warps:
//   1. scan tile k from its input buffer into registers: mask bytes to global
//      memory, counts, CTA scan, publication of the tile aggregate for the
//      look-back warps;
//   2. the input buffer is free again: hand it back to the loader;
//   3. compact tile k's set elements from registers into the value ring
//      (writing out older tiles first if the ring lacks room);
//   4. write to `vals` every compacted tile up to k-2, at the offset the
//      look-back warp found for it meanwhile, in 16-byte stores realigned
//      from the ring by funnel shifts.
// Thread layout: warp w owns the chunks (8 elements, one mask byte) CPW*w ..
// CPW*w + CPW - 1 of the tile; lane l takes chunks l, l+32, ... (G of them),
// so each shared-memory load of a warp reads 512 contiguous bytes and each
// mask-byte store writes 32 contiguous bytes.  Values are ordered by chunk:
// the warp's chunks of round u (l + 32u over the lanes) follow all chunks of
// the rounds before.
constexpr int FP_CW = 16;                 // compute warps
constexpr int FP_CT = FP_CW * 32;         // compute threads
constexpr int FP_LB = FP_CW;              // first of the two look-back warps
constexpr int FP_LOADER = FP_CW + 2;      // loader warp
constexpr int FP_THREADS = FP_CT + 96;    // plus the look-back and loader warps
constexpr int FP_NB = 5;                  // input tile buffers
constexpr int FP_TQ = 4;                  // ticket requests in flight
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
    static_assert(G == 4 || G == 2, "four or two chunks per lane");
    static constexpr int RC = TILE;  // value ring, in elements (a power of two)
    static_assert((RC & (RC - 1)) == 0, "ring index by mask");
    static constexpr size_t SMEM = (size_t)(FP_NB * TILE + RC) * sizeof(B);
};

// The 16 bytes that start D elements into the 32 bytes a:b (D < EPV).
template <typename B, int D>
__device__ __forceinline__ uint4 realign(const uint4 a, const uint4 b) {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t o[4];
    if constexpr (sizeof(B) == 2) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            o[i] = (D & 1) ? __funnelshift_r(w[D / 2 + i], w[D / 2 + i + 1], 16) : w[D / 2 + i];
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = w[D + i];
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// nvec 16-byte vectors to dst (16-byte aligned) from the ring, whose element
// at ring position a0 + D begins them (a0 a multiple of EPV).
template <typename B, int D>
__device__ __forceinline__ void ring_copy_out(const B* s_ring, uint32_t a0, int nvec, B* dst, int tid) {
    using C = PackCfg<B>;
    for (int v = tid; v < nvec; v += FP_CT) {
        const uint32_t ra = (a0 + (uint32_t)(C::EPV * v)) & (uint32_t)(C::RC - 1);
        const uint4 x = *reinterpret_cast<const uint4*>(s_ring + ra);
        uint4 o = x;
        if constexpr (D != 0) {
            const uint4 y =
                *reinterpret_cast<const uint4*>(s_ring + ((ra + (uint32_t)C::EPV) & (uint32_t)(C::RC - 1)));
            o = realign<B, D>(x, y);
        }
        *reinterpret_cast<uint4*>(dst + (size_t)C::EPV * v) = o;
    }
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
    B* s_buf = reinterpret_cast<B*>(smem_raw);  // [NB][TILE]
    B* s_ring = s_buf + (size_t)FP_NB * TILE;   // [RC]
    __shared__ __align__(8) uint64_t full[FP_NB], empty[FP_NB], pub[FP_NB], exr[FP_NB];
    __shared__ long long s_tile[FP_NB];  // tile in each input buffer
    // per scanned tile j, in slot j % NB until its write-out: tile number,
    // offset in `vals`, value count, start in the value ring
    __shared__ long long s_wtile[FP_NB], s_ex[FP_NB];
    __shared__ uint32_t s_rst[FP_NB];
    __shared__ int s_agg[FP_NB];
    __shared__ int s_wt[FP_CW];
    __shared__ volatile int s_abort;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int j = 0; j < FP_NB; ++j) {
            mbar_init(&full[j], 1);
            mbar_init(&empty[j], 1);
            mbar_init(&pub[j], 1);
            mbar_init(&exr[j], 1);
            s_wtile[j] = ntiles;
        }
        s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // --------------------------------------------------- look-back warps ----
    // Warp i resolves this CTA's scanned tiles j = i, i+2, ... in order: tile
    // j in slot j % NB.  The two run side by side: a tile's look-back reads
    // its predecessor's aggregate, published at its scan, not its result.
    if (warp == FP_LB || warp == FP_LB + 1) {
        for (int j = warp - FP_LB;; j += 2) {
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

    // ------------------------------------------------------- loader warp ----
    // Fill j goes to buffer j % NB once the compute warps freed it; the
    // first past-the-end tile is the last fill (the compute warps stop there).
    if (warp == FP_LOADER) {
        if (lane == 0) {
            unsigned int q[FP_TQ];  // tickets requested, oldest first
#pragma unroll
            for (int i = 0; i < FP_TQ; ++i) q[i] = atomicAdd(ticket, 1u);
            int last[FP_NB] = {0};  // 1 + phase of each buffer's latest fill
            for (int j = 0;; ++j) {
                const int b = j % FP_NB;
                const bool ok = mbar_wait_bounded(&empty[b], ((uint32_t)(j / FP_NB) & 1u) ^ 1u);
                if (!ok || s_abort) {
                    if (!ok) {
                        atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                    }
                    // tiles taken but not handed over: resolved, so that the
                    // successors' look-backs end
#pragma unroll
                    for (int i = 0; i < FP_TQ; ++i)
                        if ((long long)q[i] < ntiles) st_relaxed_u64(&states[q[i]], LB_INCL);
                    break;
                }
                const long long t = (long long)q[0];
#pragma unroll
                for (int i = 0; i + 1 < FP_TQ; ++i) q[i] = q[i + 1];
                q[FP_TQ - 1] = atomicAdd(ticket, 1u);
                s_tile[b] = t;
                uint32_t bytes = 0;
                if (t < ntiles) {
                    const long long nv = min((long long)TILE, n - t * TILE);
                    bytes = (uint32_t)(nv * (long long)sizeof(B)) & ~15u;
                }
                if (bytes) {
                    mbar_arrive_expect_tx(&full[b], bytes);
                    bulk_g2s(s_buf + (size_t)b * TILE, dense + t * TILE, bytes, &full[b]);
                } else {
                    mbar_arrive(&full[b]);
                }
                last[b] = j / FP_NB + 1;
                if (t >= ntiles) break;  // the queued tickets are past the end too
            }
            // no copy may still be writing this CTA's shared memory when it exits
            for (int b = 0; b < FP_NB; ++b)
                if (last[b]) (void)mbar_wait_bounded(&full[b], (uint32_t)(last[b] - 1) & 1u);
        }
        __syncwarp();
        return;
    }

    // ------------------------------------------------------ compute warps ----
    // Give up after a wait ran out: resolve the tiles this CTA holds for the
    // successors and wake the look-back and loader warps.
    auto abort_all = [&]() {
        if (tid == 0) {
            atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
            s_abort = 1;
            for (int j = 0; j < FP_NB; ++j) {
                if (s_tile[j] < ntiles) st_relaxed_u64(&states[s_tile[j]], LB_INCL);
                if (s_wtile[j] < ntiles) st_relaxed_u64(&states[s_wtile[j]], LB_INCL);
            }
            for (int j = 0; j < FP_NB; ++j) {
                mbar_arrive(&pub[j]);
                mbar_arrive(&empty[j]);
            }
        }
    };

    // Every compute thread keeps the same ring and write-out counters.
    uint32_t head = 0, tail = 0;  // value ring: elements written / freed (mod 2^32)
    int wnext = 0;                // next scanned tile to write out
    int k_end = -1;               // first iteration whose tile was past the end
    // Writes tile j's compacted values to `vals` (after its look-back); false
    // if the wait for the look-back ran out (the CTA then gives up).
    auto write_out = [&](int j) -> bool {
        const int bj = j % FP_NB;
        const bool okw = mbar_wait_bounded(&exr[bj], (uint32_t)(j / FP_NB) & 1u);
        if (named_bar_or(FP_BAR, FP_CT, !okw)) return false;
        const long long ex = s_ex[bj], tw = s_wtile[bj];
        const uint32_t rs = s_rst[bj];
        const int agg = s_agg[bj];
        // [ex, ex + agg) clipped to the capacity of `vals`
        const int lim = (int)max(0ll, min((long long)agg, cap - ex));
        int done = 0;
        if (VEC) {
            const int h = min(lim, (int)((EPV - ex % EPV) % EPV));  // to a 16-byte boundary
            if (tid < h) vals[ex + tid] = s_ring[(rs + tid) & (RC - 1)];
            const int nvec = (lim - h) / EPV;
            const uint32_t r0 = rs + (uint32_t)h;
            const uint32_t a0 = r0 & ~(uint32_t)(EPV - 1);
            B* dst = vals + ex + h;
            switch ((int)(r0 & (uint32_t)(EPV - 1))) {  // uniform: one loop per tile
                case 0: ring_copy_out<B, 0>(s_ring, a0, nvec, dst, tid); break;
                case 1: ring_copy_out<B, 1>(s_ring, a0, nvec, dst, tid); break;
                case 2: ring_copy_out<B, 2>(s_ring, a0, nvec, dst, tid); break;
                case 3: ring_copy_out<B, 3>(s_ring, a0, nvec, dst, tid); break;
                case 4: if constexpr (EPV > 4) ring_copy_out<B, (EPV > 4 ? 4 : 0)>(s_ring, a0, nvec, dst, tid); break;
                case 5: if constexpr (EPV > 4) ring_copy_out<B, (EPV > 4 ? 5 : 0)>(s_ring, a0, nvec, dst, tid); break;
                case 6: if constexpr (EPV > 4) ring_copy_out<B, (EPV > 4 ? 6 : 0)>(s_ring, a0, nvec, dst, tid); break;
                default: if constexpr (EPV > 4) ring_copy_out<B, (EPV > 4 ? 7 : 0)>(s_ring, a0, nvec, dst, tid); break;
            }
            done = h + nvec * EPV;
        }
        for (int i = done + tid; i < lim; i += FP_CT) vals[ex + i] = s_ring[(rs + (uint32_t)i) & (RC - 1)];
        if (tid == 0) {
            if (ex + agg > cap) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
            if (tw == ntiles - 1) *nnz_out = ex + agg;
        }
        tail += (uint32_t)agg;
        return true;
    };

    for (int k = 0;; ++k) {
        const int b = k % FP_NB;
        bool have = false;
        if (k_end < 0) {
            // ---- 1. scan of tile k ----
            const bool ok = mbar_wait_bounded(&full[b], (uint32_t)(k / FP_NB) & 1u);
            if (named_bar_or(FP_BAR, FP_CT, !ok)) {
                abort_all();
                return;
            }
            have = s_tile[b] < ntiles;
            if (!have) {
                k_end = k;
                if (tid == 0) {
                    // tell both look-back warps that the tiles ended (slot k+1
                    // held tile k+1-NB, written out two iterations ago)
                    const int b1 = (k + 1) % FP_NB;
                    s_wtile[b] = ntiles;
                    s_wtile[b1] = ntiles;
                    mbar_arrive(&pub[b]);
                    mbar_arrive(&pub[b1]);
                }
            }
        }
        if (have) {
            const long long t = s_tile[b];
            B* in = s_buf + (size_t)b * TILE;
            const long long base = t * TILE;
            const int nvalid = (int)min((long long)TILE, n - base);
            const int tma_elems =
                (int)(((long long)nvalid * (long long)sizeof(B)) & ~15ll) / (int)sizeof(B);
            if (tma_elems < nvalid) {  // the last tile's tail, not a multiple of 16 bytes
                for (int i = tma_elems + tid; i < nvalid; i += FP_CT) in[i] = dense[base + i];
                named_bar_sync(FP_BAR, FP_CT);
            }
            // this lane's chunks l + 32u of the warp: values and mask bytes
            Vec8<B> v[G];
            uint32_t mb[G];
#pragma unroll
            for (int u = 0; u < G; ++u) {
                const int ci = CPW * warp + lane + 32 * u;  // chunk of the tile
                const int f = 8 * ci;
                mb[u] = 0;
                v[u].zero();
                if (f < nvalid) {
                    v[u].load_smem(in + f);
                    uint32_t byte = v[u].nonzero_byte();
                    if (f + 8 > nvalid) byte &= (1u << (nvalid - f)) - 1u;
                    mb[u] = byte;
                    mask[(base >> 3) + ci] = (uint8_t)byte;  // 32 contiguous bytes per warp
                }
            }
            // offsets of the chunks in the warp's value order: two counts per
            // scanned word (each at most 32 * 8 = 256 over the warp)
            int off[G], wtot;
            if constexpr (G == 4) {
                const int pa = __popc(mb[0]) | (__popc(mb[1]) << 16), pb = __popc(mb[2]) | (__popc(mb[3]) << 16);
                const int ia = warp_incl_scan(pa, lane), ib = warp_incl_scan(pb, lane);
                const int ta = __shfl_sync(FULL, ia, 31), tb = __shfl_sync(FULL, ib, 31);
                const int ea = ia - pa, eb = ib - pb;
                const int t0 = ta & 0xFFFF, t1 = ta >> 16, t2 = tb & 0xFFFF;
                off[0] = ea & 0xFFFF;
                off[1] = t0 + (ea >> 16);
                off[2] = t0 + t1 + (eb & 0xFFFF);
                off[3] = t0 + t1 + t2 + (eb >> 16);
                wtot = t0 + t1 + t2 + (tb >> 16);
            } else {
                const int pa = __popc(mb[0]) | (__popc(mb[1]) << 16);
                const int ia = warp_incl_scan(pa, lane);
                const int ta = __shfl_sync(FULL, ia, 31);
                const int ea = ia - pa;
                off[0] = ea & 0xFFFF;
                off[1] = (ta & 0xFFFF) + (ea >> 16);
                wtot = (ta & 0xFFFF) + (ta >> 16);
            }
            if (lane == 0) s_wt[warp] = wtot;
            named_bar_sync(FP_BAR, FP_CT);  // also: every lane has read buffer b
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
                // ---- 2. the input buffer is free: back to the loader ----
                fence_proxy_async_smem();
                mbar_arrive(&empty[b]);
            }
            // ---- 3. compaction into the value ring ----
            if (RC - (int)(head - tail) < agg) {
                while (RC - (int)(head - tail) < agg)
                    if (!write_out(wnext++)) {
                        abort_all();
                        return;
                    }
                named_bar_sync(FP_BAR, FP_CT);  // freed ring slots fully read
            }
            const uint32_t p0 = head + (uint32_t)wbase;
            if (4 * agg > TILE) {
                // dense tile: every element tested, predicated stores
#pragma unroll
                for (int u = 0; u < G; ++u) {
                    uint32_t p = p0 + (uint32_t)off[u];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if ((mb[u] >> j) & 1u) s_ring[(p++) & (RC - 1)] = v[u].get(j);
                }
            } else {
                // sparse tile: walk the set bits
#pragma unroll
                for (int u = 0; u < G; ++u) {
                    uint32_t p = p0 + (uint32_t)off[u], bb = mb[u];
                    while (bb) {
                        const int j = __ffs(bb) - 1;
                        bb &= bb - 1u;
                        s_ring[(p++) & (RC - 1)] = v[u].get(j);
                    }
                }
            }
            head += (uint32_t)agg;
        }
        // ---- 4. write-out of the tiles scanned D or more iterations ago ----
        const int upto = k_end < 0 ? k - FP_D : k_end - 1;
        while (wnext <= upto)
            if (!write_out(wnext++)) {
                abort_all();
                return;
            }
        if (k_end >= 0) break;  // every scanned tile is written
        named_bar_sync(FP_BAR, FP_CT);  // ring slots written out are fully read
    }
}


// ------------------------------------------------------ scan-based path ----
// The workspace entry points run two launches over tiles of FS_TILE = 8192
// elements (256 threads x 32), with no waits between blocks:
//   pack:   flat_pack_stage_kernel (one read of the dense tensor: mask bytes,
//           tile counts, and the tile's set elements compacted in shared
//           memory and written to the tile's own 16-byte aligned segment of
//           a staging area) -> flat_pack_move_kernel (each tile's values
//           from the staging area to their offset in vals);
//   unpack: flat_mask_popc_kernel (tile counts from the mask) ->
//           flat_expand_kernel (the tile's values staged by 16-byte loads,
//           expanded into 16-byte streaming stores).
// A counting block adds its tile count to the sum of its group of 256 tiles;
// a second-kernel block finds its offset from at most 255 counts and nt/256
// group sums, loaded together in one round trip (tile_offset).  Every block
// is independent, so the kernels run at full occupancy and memory latency is
// hidden by other blocks.  The pack reads the dense tensor once and moves
// the values twice (2 n + n/8 + 6 nnz bytes against the 2 n + n/8 + 2 nnz it
// must move); unpack re-reads only the mask.
// Thread layout: warp w owns chunks 128w .. 128w+127 of the tile, lane l takes
// chunks l, l+32, l+64, l+96, and values are ordered by chunk.
//
// Workspace: int32 tile counts, then the int64 sums of the 256-tile groups
// (zeroed on the stream before the counting kernel), then (pack only) the
// staging area of FS_TILE elements per tile, 16-byte aligned.
constexpr int FS_TILE = FT_MIN_TILE;  // elements per tile
constexpr int FS_T = 256;             // threads per tile
constexpr int FS_W = FS_T / 32;
static_assert(FS_TILE == FS_T * 32, "32 elements per thread");

struct TileSums {
    int* counts;              // [nt]
    unsigned long long* g1;   // [ceil(nt / 256)]
};

inline TileSums tile_sums(void* ws, long long nt) {
    char* p = static_cast<char*>(ws);
    TileSums t;
    t.counts = reinterpret_cast<int*>(p);
    t.g1 = reinterpret_cast<unsigned long long*>(p + ((nt * 4 + 7) & ~7ll));
    return t;
}
inline size_t tile_sums_zero_bytes(long long nt) { return (size_t)((nt + 255) / 256) * 8; }

// Tile t's count into the tables (one thread).
__device__ __forceinline__ void tile_sums_add(const TileSums& ts, long long t, int cnt) {
    ts.counts[t] = cnt;
    if (cnt) atomicAdd(ts.g1 + (t >> 8), (unsigned long long)cnt);
}

// Elements before tile t: the counts of the earlier tiles of its 256-group
// and the sums of the earlier 256-groups.  Block-collective (FS_T threads).
__device__ __forceinline__ long long tile_offset(const TileSums& ts, long long t, long long* s_red) {
    const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
    const long long a = t & ~255ll, b1 = t >> 8;
    long long s = 0;
    if (a + i < t) s += __ldg(ts.counts + a + i);
    for (long long k = i; k < b1; k += FS_T) s += (long long)__ldg(ts.g1 + k);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
    if (lane == 0) s_red[warp] = s;
    __syncthreads();
    long long r = 0;
#pragma unroll
    for (int w = 0; w < FS_W; ++w) r += s_red[w];
    return r;
}

// Chunk-order offsets of this lane's G chunks (l + 32u of its warp) inside
// the block, and the block total.  Two counts (each at most 8, at most 256
// over the warp) share one scanned word.
template <int G>
__device__ __forceinline__ void block_chunk_offsets(const uint32_t (&mb)[G], int (&off)[G], int& total,
                                                    int* s_wt, int warp, int lane) {
    int ex[G], tot[G];
#pragma unroll
    for (int h = 0; h < G / 2; ++h) {
        const int pv = __popc(mb[2 * h]) | (__popc(mb[2 * h + 1]) << 16);
        const int iv = warp_incl_scan(pv, lane);
        const int tv = __shfl_sync(FULL, iv, 31);
        const int ev = iv - pv;
        ex[2 * h] = ev & 0xFFFF;
        ex[2 * h + 1] = ev >> 16;
        tot[2 * h] = tv & 0xFFFF;
        tot[2 * h + 1] = tv >> 16;
    }
    int wsum = 0;
#pragma unroll
    for (int u = 0; u < G; ++u) {
        off[u] = wsum + ex[u];
        wsum += tot[u];
    }
    if (lane == 0) s_wt[warp] = wsum;
    __syncthreads();
    int wbase = 0;
    total = 0;
#pragma unroll
    for (int w = 0; w < FS_W; ++w) {
        const int x = s_wt[w];
        wbase += w < warp ? x : 0;
        total += x;
    }
#pragma unroll
    for (int u = 0; u < G; ++u) off[u] += wbase;
}

// Tiles per block of the expand kernel: two for 16-bit types (32 KB of dense
// output per block), one for 32-bit types.  The compact kernel holds its
// values in registers and keeps one tile per block (two would halve its
// occupancy).
template <typename B>
constexpr int fs_tpb() { return sizeof(B) == 2 ? 2 : 1; }

// Eight tiles per block: each warp counts one tile's 1024 mask bytes (16 B per
// lane, two rounds).
constexpr int FP_TPB = FS_W;
__global__ void __launch_bounds__(FS_T) flat_mask_popc_kernel(const uint8_t* __restrict__ mask, long long n,
                                                              long long nt, TileSums ts) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long t = (long long)blockIdx.x * FP_TPB + warp;
    if (t >= nt) return;
    const long long base = t * FS_TILE;
    int cnt = 0;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const long long f = base + 128LL * (lane + 32 * r);  // 16 mask bytes
        if (f + 128 <= n) {
            const uint8_t* m = mask + (f >> 3);
            if ((reinterpret_cast<uintptr_t>(mask) & 15u) == 0) {
                const uint4 w = __ldg(reinterpret_cast<const uint4*>(m));
                cnt += __popc(w.x) + __popc(w.y) + __popc(w.z) + __popc(w.w);
            } else {  // the mask is only 4-byte aligned
#pragma unroll
                for (int k = 0; k < 4; ++k) cnt += __popc(__ldg(reinterpret_cast<const uint32_t*>(m) + k));
            }
        } else if (f < n) {
            for (int k = 0; k < 16; ++k) {
                const long long g = f + 8 * k;
                if (g < n) {
                    uint32_t b = __ldg(mask + (g >> 3));
                    if (g + 8 > n) b &= (1u << (n - g)) - 1u;
                    cnt += __popc(b);
                }
            }
        }
    }
    cnt = __reduce_add_sync(FULL, cnt);
    if (lane == 0) tile_sums_add(ts, t, cnt);
}

// Shared-memory store of a 16- or 32-bit value under a predicate (no branch).
__device__ __forceinline__ void st_shared_if(uint32_t addr, uint16_t v, uint32_t p) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q st.shared.u16 [%0], %1;\n\t}" ::"r"(addr),
                 "h"(v), "r"(p)
                 : "memory");
}
__device__ __forceinline__ void st_shared_if(uint32_t addr, uint32_t v, uint32_t p) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q st.shared.u32 [%0], %1;\n\t}" ::"r"(addr),
                 "r"(v), "r"(p)
                 : "memory");
}

// The chunk's set elements to consecutive places from shared address `da`
// (returned advanced): predicated stores, the address stepped by each bit.
template <typename B>
__device__ __forceinline__ uint32_t put_set(const Vec8<B>& v, uint32_t bits, uint32_t da) {
    if constexpr (sizeof(B) == 2) {
        const uint32_t w[4] = {v.q.x, v.q.y, v.q.z, v.q.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t b0 = (bits >> (2 * q)) & 1u, b1 = (bits >> (2 * q + 1)) & 1u;
            st_shared_if(da, (uint16_t)w[q], b0);
            da += 2 * b0;
            st_shared_if(da, (uint16_t)(w[q] >> 16), b1);
            da += 2 * b1;
        }
    } else {
        const uint32_t w[8] = {v.a.x, v.a.y, v.a.z, v.a.w, v.b.x, v.b.y, v.b.z, v.b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t bj = (bits >> j) & 1u;
            st_shared_if(da, w[j], bj);
            da += 4 * bj;
        }
    }
    return da;
}

// The chunk rebuilt from consecutive values at `sp`: set elements take the
// next value, the others zero.  Every slot is read (the read past the last
// value stays inside the staging buffer) and masked, so there is no branch.
template <typename B>
__device__ __forceinline__ void take_set(Vec8<B>& o, uint32_t bits, const B* sp) {
    if constexpr (sizeof(B) == 2) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t b0 = (bits >> (2 * q)) & 1u, b1 = (bits >> (2 * q + 1)) & 1u;
            const uint32_t lo = (uint32_t)*sp & (0u - b0);
            sp += b0;
            const uint32_t hi = (uint32_t)*sp & (0u - b1);
            sp += b1;
            w[q] = lo | (hi << 16);
        }
        o.q = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t bj = (bits >> j) & 1u;
            w[j] = *sp & (0u - bj);
            sp += bj;
        }
        o.a = make_uint4(w[0], w[1], w[2], w[3]);
        o.b = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// Expansion of 16-bit elements, four (one mask nibble n) at a time: from the
// next four staged values packed as x (values 0, 1) and y (values 2, 3),
// output halfwords 0-1 are __byte_perm(x, 0, low half of nib_take_sel(n)) --
// bytes 4-5 of the zero word where unset -- and halfwords 2-3 are
// __byte_perm(x, y, high half) masked by nib_take_mask(n).  (A matching
// compaction by permutes needs 16 more registers in the compact kernel and
// measured slower there than the predicated stores.)
__host__ __device__ constexpr uint32_t nib_take_sel(int n) {
    uint32_t s = 0;
    int r = 0;
    for (int e = 0; e < 4; ++e) {
        uint32_t pair = e < 2 ? (4u | (5u << 4)) : (0u | (1u << 4));
        if ((n >> e) & 1) {
            pair = (uint32_t)((2 * r) | ((2 * r + 1) << 4));
            ++r;
        }
        s |= pair << (8 * e);
    }
    return s;
}
__host__ __device__ constexpr uint32_t nib_take_mask(int n) {
    return (((n >> 2) & 1) ? 0x0000FFFFu : 0u) | (((n >> 3) & 1) ? 0xFFFF0000u : 0u);
}
static_assert(nib_take_sel(0b1001) == 0x32105410u && nib_take_mask(0b1001) == 0xFFFF0000u, "take table");

// The chunk rebuilt from the consecutive staged values at `sp`.  Reads up to
// three values past the chunk's last one (inside the staging buffer).
__device__ __forceinline__ uint4 take_set16(uint32_t bits, const uint16_t* sp, const uint2* s_take) {
    uint32_t w[4];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        const uint32_t n = (bits >> (4 * g)) & 15u;
        const uint32_t x = (uint32_t)sp[0] | ((uint32_t)sp[1] << 16);
        const uint32_t y = (uint32_t)sp[2] | ((uint32_t)sp[3] << 16);
        const uint2 t = s_take[n];
        w[2 * g] = __byte_perm(x, 0u, t.x & 0xFFFFu);
        w[2 * g + 1] = __byte_perm(x, y, t.x >> 16) & t.y;
        sp += __popc(n);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Pack, first kernel: one read of the tile, its mask bytes and count, and
// its set elements compacted in shared memory and written, with 16-byte
// stores, to the tile's own segment stage[t * FS_TILE ...] (16-byte aligned:
// no realignment here).  Indices inside the tile are 32-bit.
template <typename B>
__global__ void __launch_bounds__(FS_T) flat_pack_stage_kernel(const B* __restrict__ dense, long long n,
                                                               uint8_t* __restrict__ mask, TileSums ts,
                                                               B* __restrict__ stage) {
    constexpr int EPV = 16 / (int)sizeof(B);
    constexpr int G = 4;
    __shared__ __align__(16) B s_val[FS_TILE];
    __shared__ int s_wt[FS_W];
    const long long t = (long long)blockIdx.x, base = t * FS_TILE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int rem = (int)min(n - base, (long long)FS_TILE);
    const B* db = dense + base;
    Vec8<B> v[G];
#pragma unroll
    for (int u = 0; u < G; ++u) {  // every load issued before any use
        const int f = 8 * (32 * G * warp + lane + 32 * u);
        v[u].zero();
        if (f + 8 <= rem) v[u].load_global(db + f);
        else
            for (int j = 0; j < 8; ++j)
                if (f + j < rem) v[u].set(j, db[f + j]);
    }
    uint32_t mb[G];
#pragma unroll
    for (int u = 0; u < G; ++u) {
        const int f = 8 * (32 * G * warp + lane + 32 * u);
        mb[u] = v[u].nonzero_byte();  // zero-filled past n
        if (f < rem) mask[(base + f) >> 3] = (uint8_t)mb[u];
    }
    int off[G], total;
    block_chunk_offsets<G>(mb, off, total, s_wt, warp, lane);
    const uint32_t sbase = smem_u32(s_val);
#pragma unroll
    for (int u = 0; u < G; ++u) put_set<B>(v[u], mb[u], sbase + (uint32_t)(off[u] * (int)sizeof(B)));
    if (tid == 0) tile_sums_add(ts, t, total);
    __syncthreads();
    B* so = stage + base;
    const int nvec = total / EPV;
    for (int q = tid; q < nvec; q += FS_T)
        *reinterpret_cast<uint4*>(so + EPV * q) = *reinterpret_cast<const uint4*>(s_val + EPV * q);
    for (int i = EPV * nvec + tid; i < total; i += FS_T) so[i] = s_val[i];
}

// Pack, second kernel: MV_TPB consecutive tiles per block, their values from
// the staging segments to vals[offset ...] (never past cap).  The offset of
// the block's first tile comes from the tile counts and group sums; the
// others add the block's counts before them.  The last tile writes the total.
constexpr int MV_TPB = 16;
template <typename B>
__global__ void __launch_bounds__(FS_T) flat_pack_move_kernel(const B* __restrict__ stage, TileSums ts, long long nt,
                                                              B* __restrict__ vals, long long cap,
                                                              long long* __restrict__ nnz_out,
                                                              uint32_t* __restrict__ status) {
    __shared__ long long s_red[FS_W];
    __shared__ int s_cnt[MV_TPB], s_pre[MV_TPB + 1];
    const long long t0 = (long long)blockIdx.x * MV_TPB;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ntb = (int)min((long long)MV_TPB, nt - t0);
    if (tid < MV_TPB) s_cnt[tid] = tid < ntb ? __ldg(ts.counts + t0 + tid) : 0;
    const long long ex0 = tile_offset(ts, t0, s_red);  // its barrier also publishes s_cnt
    if (warp == 0) {
        const int c = lane < MV_TPB ? s_cnt[lane] : 0;
        const int inc = warp_incl_scan(c, lane);
        if (lane < MV_TPB) s_pre[lane] = inc - c;
        if (lane == MV_TPB - 1) s_pre[MV_TPB] = inc;
    }
    __syncthreads();
    const long long total = s_pre[MV_TPB];
    if (tid == 0) {
        if (t0 + ntb >= nt) *nnz_out = ex0 + total;
        if (ex0 + total > cap) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
    }
    // warp w moves tiles w, w + 8: each tile's values are one contiguous run
    for (int k = warp; k < ntb; k += FS_W) {
        const long long ex = ex0 + s_pre[k];
        const int lim = (int)max(0ll, min((long long)s_cnt[k], cap - ex));
        const B* si = stage + (t0 + k) * FS_TILE;
        B* vo = vals + ex;
        if constexpr (sizeof(B) == 2) {
            // 16-byte stores realigned from the (16-byte aligned) staging segment
            if (lim > 0) copy_run16<32>(si, vo, lim, lane);
            continue;
        }
        int i = lane;
        for (; i + 96 < lim; i += 128) {  // four loads in flight per lane
            const B a0 = __ldcs(si + i), a1 = __ldcs(si + i + 32), a2 = __ldcs(si + i + 64), a3 = __ldcs(si + i + 96);
            vo[i] = a0;
            vo[i + 32] = a1;
            vo[i + 64] = a2;
            vo[i + 96] = a3;
        }
        for (; i < lim; i += 32) vo[i] = __ldcs(si + i);
    }
}

// The total count (sum of the group sums) into *nnz_out: one warp.
__global__ void flat_total_kernel(const unsigned long long* __restrict__ g1, long long ng,
                                  long long* __restrict__ nnz_out) {
    unsigned long long s = 0;
    for (long long i = threadIdx.x; i < ng; i += 32) s += g1[i];
    s = warp_sum_u64(s);
    if (threadIdx.x == 0) *nnz_out = (long long)s;
}

template <typename B, bool VEC>
__global__ void __launch_bounds__(FS_T) flat_expand_kernel(const B* __restrict__ vals, long long vals_len,
                                                           const uint8_t* __restrict__ mask, TileSums ts,
                                                           long long n, B* __restrict__ out,
                                                           uint32_t* __restrict__ status) {
    constexpr int EPV = 16 / (int)sizeof(B);
    constexpr int TPB = fs_tpb<B>(), G = 4 * TPB;
    __shared__ __align__(16) B s_val[TPB * FS_TILE + 2 * EPV];
    __shared__ int s_wt[FS_W];
    __shared__ long long s_red[FS_W];
    __shared__ uint2 s_take[16];
    if (threadIdx.x < 16)  // read after the next barrier
        s_take[threadIdx.x] = make_uint2(nib_take_sel((int)threadIdx.x), nib_take_mask((int)threadIdx.x));
    const long long t = (long long)blockIdx.x * TPB, base = t * FS_TILE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int rem = (int)min(n - base, (long long)(TPB * FS_TILE));
    uint32_t mb[G];
    {  // mask bytes of chunks l + 32u of the warp, bits past n clear
        const uint8_t* mbase = mask + (base >> 3);
#pragma unroll
        for (int u = 0; u < G; ++u) {
            const int f = 8 * (32 * G * warp + lane + 32 * u);
            uint32_t b = 0;
            if (f < rem) {
                b = __ldg(mbase + (f >> 3));
                if (f + 8 > rem) b &= (1u << (rem - f)) - 1u;
            }
            mb[u] = b;
        }
    }
    const long long ex = tile_offset(ts, t, s_red);  // its loads in flight with the mask's
    int off[G], total;
    block_chunk_offsets<G>(mb, off, total, s_wt, warp, lane);
    if (tid == 0 && ex + total > vals_len) atomicOr(status, SFFN_STATUS_VALS_SHORT);
    // stage vals[ex, ex + total) at staging index sh + i; past vals_len -> 0
    const int sh = (int)(ex % EPV);
    const long long a0 = ex - sh;  // 16-byte aligned in `vals` when VEC
    const int span = sh + total;
    const long long avail = vals_len - a0;  // values from a0 that exist
    const B* va = vals + a0;
    if (VEC) {
        for (int q = tid; EPV * q < span; q += FS_T) {
            if (EPV * q + EPV <= avail) {
                *reinterpret_cast<uint4*>(s_val + EPV * q) = __ldg(reinterpret_cast<const uint4*>(va + EPV * q));
            } else {
#pragma unroll
                for (int e = 0; e < EPV; ++e) s_val[EPV * q + e] = EPV * q + e < avail ? va[EPV * q + e] : B(0);
            }
        }
    } else {
        for (int i = tid; i < span; i += FS_T) s_val[i] = i < avail ? va[i] : B(0);
    }
    __syncthreads();
    B* ob = out + base;
#pragma unroll
    for (int u = 0; u < G; ++u) {
        const int f = 8 * (32 * G * warp + lane + 32 * u);
        if (f >= rem) continue;
        Vec8<B> o;
        if constexpr (sizeof(B) == 2) o.q = take_set16(mb[u], s_val + sh + off[u], s_take);
        else take_set<B>(o, mb[u], s_val + sh + off[u]);
        if (f + 8 <= rem) o.store_global_cs(ob + f);
        else
            for (int j = 0; j < 8; ++j)
                if (f + j < rem) ob[f + j] = o.get(j);
    }
}

template <typename B>
inline long long flat_tiles(long long n) { return (n + PackCfg<B>::TILE - 1) / PackCfg<B>::TILE; }

template <typename K>
cudaError_t allow_smem(K kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

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

// The single-pass look-back pack, for sffn_flat_pack_noalloc: `scratch` is
// [0, 16) the tile ticket, then one 8-byte look-back state per 32 KB tile;
// both are cleared on the stream before the kernel runs.
template <typename B>
int launch_pack_lookback(const void* dense, long long n, uint8_t* mask, void* vals, long long cap,
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

// Byte offset of the pack's staging area in the workspace (16-byte aligned).
inline size_t pack_stage_offset(long long nt) {
    return ((size_t)((nt * 4 + 7) & ~7ll) + (size_t)((nt + 255) / 256) * 8 + 15) & ~(size_t)15;
}

template <typename B>
int launch_pack_count(const void* dense, long long n, uint8_t* mask, void* ws, cudaStream_t st) {
    const long long nt = (n + FS_TILE - 1) / FS_TILE;
    const TileSums ts = tile_sums(ws, nt);
    SFFN_CUDA_TRY(cudaMemsetAsync(ts.g1, 0, tile_sums_zero_bytes(nt), st));
    B* stage = reinterpret_cast<B*>(static_cast<char*>(ws) + pack_stage_offset(nt));
    flat_pack_stage_kernel<B><<<(unsigned)nt, FS_T, 0, st>>>(static_cast<const B*>(dense), n, mask, ts, stage);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <typename B>
int launch_pack_values(long long n, void* vals, long long cap, int64_t* nnz_dev, void* ws, uint32_t* status,
                       cudaStream_t st) {
    const long long nt = (n + FS_TILE - 1) / FS_TILE;
    const TileSums ts = tile_sums(ws, nt);
    const B* stage = reinterpret_cast<const B*>(static_cast<const char*>(ws) + pack_stage_offset(nt));
    flat_pack_move_kernel<B><<<(unsigned)((nt + MV_TPB - 1) / MV_TPB), FS_T, 0, st>>>(
        stage, ts, nt, static_cast<B*>(vals), cap, reinterpret_cast<long long*>(nnz_dev), status);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <typename B>
int launch_unpack(const void* vals, long long vals_len, const uint8_t* mask, long long n, void* out,
                  void* ws, uint32_t* status, cudaStream_t st) {
    const long long nt = (n + FS_TILE - 1) / FS_TILE;
    const TileSums ts = tile_sums(ws, nt);
    SFFN_CUDA_TRY(cudaMemsetAsync(ts.g1, 0, tile_sums_zero_bytes(nt), st));
    flat_mask_popc_kernel<<<(unsigned)((nt + FP_TPB - 1) / FP_TPB), FS_T, 0, st>>>(mask, n, nt, ts);
    SFFN_CHECK_LAUNCH();
    const B* v = static_cast<const B*>(vals);
    B* o = static_cast<B*>(out);
    const unsigned nb = (unsigned)((nt + fs_tpb<B>() - 1) / fs_tpb<B>());
    if (aligned16(vals))
        flat_expand_kernel<B, true><<<nb, FS_T, 0, st>>>(v, vals_len, mask, ts, n, o, status);
    else
        flat_expand_kernel<B, false><<<nb, FS_T, 0, st>>>(v, vals_len, mask, ts, n, o, status);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

// Workspace of the unpack: 16 bytes plus 8 per tile of 8192 elements (int32
// tile counts followed by the int64 sums of 256-tile groups).  The pack needs
// the same tables plus a staging area of one 8192-element segment per tile
// (sffn_flat_pack_workspace_bytes).  The persistent look-back pack of the
// no-alloc entry point keeps a 16-byte ticket and one state word per 32 KB
// tile of dense data in its static array instead.
extern "C" size_t sffn_flat_workspace_bytes(int64_t n) {
    if (n < 0) return 0;
    return 16 + (size_t)((n + FT_MIN_TILE - 1) / FT_MIN_TILE) * 8;
}

extern "C" size_t sffn_flat_pack_workspace_bytes(int64_t n, int dtype) {
    if (n < 0 || !dtype_ok(dtype)) return 0;
    const long long nt = (n + FS_TILE - 1) / FS_TILE;
    return pack_stage_offset(nt) + (size_t)nt * FS_TILE * esize_of(dtype);
}

namespace {
// Shared checks of the pack entry points (n > 0).
int pack_args_ok(const void* dense, int dtype, int64_t n, const uint8_t* mask, size_t ws_bytes, const void* ws) {
    if (!dense || !mask || !ws) return SFFN_ERR_ARG;
    if (!aligned16(dense) || (reinterpret_cast<uintptr_t>(mask) & 3u) || !aligned16(ws)) return SFFN_ERR_ALIGN;
    if (ws_bytes < sffn_flat_pack_workspace_bytes(n, dtype)) return SFFN_ERR_WORKSPACE;
    if ((n + FT_MIN_TILE - 1) / FT_MIN_TILE > 0x7FFFFFFFll) return SFFN_ERR_ARG;  // grid limit
    return SFFN_OK;
}
}  // namespace

extern "C" int sffn_flat_pack_count(const void* dense, int dtype, int64_t n, uint8_t* packed_mask, int64_t* nnz_dev,
                                    void* workspace, size_t workspace_bytes, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (n < 0 || !nnz_dev) return SFFN_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        SFFN_BIND(dev_scope, nnz_dev);
        SFFN_CUDA_TRY(cudaMemsetAsync(nnz_dev, 0, sizeof(int64_t), st));
        return SFFN_OK;
    }
    if (int rc = pack_args_ok(dense, dtype, n, packed_mask, workspace_bytes, workspace)) return rc;
    SFFN_BIND(dev_scope, dense);
    const int rc = esize_of(dtype) == 4 ? launch_pack_count<uint32_t>(dense, n, packed_mask, workspace, st)
                                        : launch_pack_count<uint16_t>(dense, n, packed_mask, workspace, st);
    if (rc) return rc;
    const long long nt = (n + FS_TILE - 1) / FS_TILE;
    flat_total_kernel<<<1, 32, 0, st>>>(tile_sums(workspace, nt).g1, (nt + 255) / 256,
                                        reinterpret_cast<long long*>(nnz_dev));
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_flat_pack_values(int dtype, int64_t n, void* vals, int64_t vals_capacity, int64_t* nnz_dev,
                                     void* workspace, size_t workspace_bytes, uint32_t* status_dev, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (n < 0 || vals_capacity < 0 || !nnz_dev || !status_dev) return SFFN_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        SFFN_BIND(dev_scope, nnz_dev);
        SFFN_CUDA_TRY(cudaMemsetAsync(nnz_dev, 0, sizeof(int64_t), st));
        return SFFN_OK;
    }
    if ((!vals && vals_capacity > 0) || !workspace) return SFFN_ERR_ARG;
    if (!aligned16(workspace)) return SFFN_ERR_ALIGN;
    if (workspace_bytes < sffn_flat_pack_workspace_bytes(n, dtype)) return SFFN_ERR_WORKSPACE;
    SFFN_BIND(dev_scope, workspace);
    return esize_of(dtype) == 4
               ? launch_pack_values<uint32_t>(n, vals, vals_capacity, nnz_dev, workspace, status_dev, st)
               : launch_pack_values<uint16_t>(n, vals, vals_capacity, nnz_dev, workspace, status_dev, st);
}

extern "C" int sffn_flat_pack(const void* dense, int dtype, int64_t n, uint8_t* packed_mask,
                              void* vals, int64_t vals_capacity, int64_t* nnz_dev, void* workspace,
                              size_t workspace_bytes, uint32_t* status_dev, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (n < 0 || vals_capacity < 0 || !nnz_dev || !status_dev) return SFFN_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        SFFN_BIND(dev_scope, nnz_dev);
        SFFN_CUDA_TRY(cudaMemsetAsync(nnz_dev, 0, sizeof(int64_t), st));
        return SFFN_OK;
    }
    if (!vals && vals_capacity > 0) return SFFN_ERR_ARG;
    if (int rc = pack_args_ok(dense, dtype, n, packed_mask, workspace_bytes, workspace)) return rc;
    SFFN_BIND(dev_scope, dense);
    if (esize_of(dtype) == 4) {
        if (int rc = launch_pack_count<uint32_t>(dense, n, packed_mask, workspace, st)) return rc;
        return launch_pack_values<uint32_t>(n, vals, vals_capacity, nnz_dev, workspace, status_dev, st);
    }
    if (int rc = launch_pack_count<uint16_t>(dense, n, packed_mask, workspace, st)) return rc;
    return launch_pack_values<uint16_t>(n, vals, vals_capacity, nnz_dev, workspace, status_dev, st);
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
    SFFN_BIND(dev_scope, out);
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
// Set-up: the first call on a device (more precisely, in a CUDA context: a
// device reset makes a new primary context, in which the array may sit
// elsewhere) looks up that device's address of the array with
// cudaGetSymbolAddress, with the device current, and caches it keyed by the
// context's unique id; make that first call before any stream capture.  Every
// call shares the array and finds the previous call's contents in it, so each
// call clears the part it uses before its kernel runs; calls that overlap on
// the GPU (other streams, other host threads) race on it and must be
// serialised by the caller.  The call binds the device of `dense` and puts
// back the caller's current device (context) before it returns; every pointer
// argument must live on that device.
// ---------------------------------------------------------------------------
namespace sffn {
namespace {

constexpr long long kNoAllocMaxTiles = 4096;  // 4096 tiles of 32 KB of input
static __device__ __align__(256) unsigned char g_noalloc_scratch[16 + kNoAllocMaxTiles * 8];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
struct ScratchAddr {
    unsigned long long ctx_id;  // context the address belongs to (0: none cached)
    void* addr;
};
ScratchAddr g_noalloc_addr[kMaxDevices] = {};

// Device address of the scratch array on `dev`, whose context is current.
int noalloc_scratch(int dev, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return SFFN_ERR_ARG;
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    ScratchAddr& c = g_noalloc_addr[dev];
    if (ctx == 0 || c.ctx_id != ctx || !c.addr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            set_cuda_error(e);
            return SFFN_ERR_CUDA;
        }
        c.ctx_id = ctx;  // 0 (id unknown): looked up again on the next call
        c.addr = p;
    }
    *out = c.addr;
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
    // The device that owns the input (the count, for an empty input); every
    // other buffer must be on it.  Nothing on this path allocates or frees
    // device memory.
    DeviceScope dev_scope;
    if (int rc = dev_scope.bind_same(n > 0 ? dense : nnz_dev,
                                     {nnz_dev, status_dev, n > 0 ? packed_mask : nullptr,
                                      n > 0 && vals_capacity > 0 ? vals : nullptr}))
        return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        SFFN_CUDA_TRY(cudaMemsetAsync(nnz_dev, 0, sizeof(int64_t), st));
        return SFFN_OK;
    }
    void* scratch = nullptr;
    if (int rc = noalloc_scratch(dev_scope.device(), &scratch)) return rc;
    // launch_pack_lookback clears the ticket and the states this call uses
    // (the previous call left its own in the array) before the kernel runs.
    if (esize_of(dtype) == 4)
        return launch_pack_lookback<uint32_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, scratch,
                                              status_dev, st);
    return launch_pack_lookback<uint16_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, scratch,
                                          status_dev, st);
}
