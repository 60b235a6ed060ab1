// Small kernels around the fused FFN GEMMs (sm_100a).
//
//   tile_scan_kernel    per-tile counts (summed over `parts` partial counts)
//                       -> exclusive prefix[num_tiles + 1]; reads the int32
//                       arena cursor into vals_offset and advances it by the
//                       total (sparse.py:181-204 without a host round trip).
//   tile_rows_kernel    per 128x128 tile: row counts from the bitmask, a
//                       128-row scan, row_offsets[t][r] = prefix[t] + (values
//                       in rows < r); optionally moves each row's values from
//                       its fixed 128-element slot segment (written by the
//                       up-projection epilogue, which cannot know the final
//                       offsets) to vals[vals_offset + row_offsets[t][r] ...].
//   live_kblocks_kernel for each 256-row tile (two rows of 128x128 format
//                       tiles, the GEMM's CTA-pair tile) of a tiled bitmask,
//                       the ascending list of 64-column blocks holding any set
//                       bit: the down-projection skips the others.  One warp
//                       per k-block; the last CTA of a tile compacts.
#include <algorithm>

#include "common.cuh"

namespace sffn {
namespace {

constexpr int SCAN_NT = 1024;

// One CTA: thread tid owns a contiguous run of tiles; run sums are scanned
// with warp shuffles (two levels), then each thread writes its run's prefixes.
__global__ void __launch_bounds__(SCAN_NT) tile_scan_kernel(const int* __restrict__ counts, int parts,
                                                           long long ntiles, int* __restrict__ prefix,
                                                           int* __restrict__ cursor,
                                                           int* __restrict__ vals_offset_out,
                                                           uint32_t* __restrict__ status) {
    __shared__ long long s_warp[SCAN_NT / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long per = (ntiles + SCAN_NT - 1) / SCAN_NT;
    const long long lo = tid * per, hi = min(lo + per, ntiles);
    const bool vec4 = parts == 4 && (reinterpret_cast<uintptr_t>(counts) & 15u) == 0;
    auto count = [&](long long t) {
        if (vec4) {
            const int4 c = __ldg(reinterpret_cast<const int4*>(counts) + t);
            return c.x + c.y + c.z + c.w;
        }
        int c = 0;
        for (int k = 0; k < parts; ++k) c += __ldg(counts + t * parts + k);
        return c;
    };
    long long sum = 0;
    for (long long t = lo; t < hi; ++t) sum += count(t);
    long long inc = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long v = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        long long w = s_warp[lane], wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long v = __shfl_up_sync(FULL, wi, o);
            if (lane >= o) wi += v;
        }
        s_warp[lane] = wi - w;  // exclusive prefix of each warp
    }
    __syncthreads();
    long long run = s_warp[warp] + inc - sum;
    for (long long t = lo; t < hi; ++t) {
        prefix[t] = (int)run;
        run += count(t);
    }
    if (tid == SCAN_NT - 1) {
        const long long total = run;  // the last thread's run ends at the total
        prefix[ntiles] = (int)total;
        const int cur = *cursor;
        *vals_offset_out = cur;
        const long long next = (long long)cur + total;
        if (next > 0x7FFFFFFFll || total > 0x7FFFFFFFll) atomicOr(status, SFFN_STATUS_CURSOR_OVERFLOW);
        *cursor = (int)(next > 0x7FFFFFFFll ? 0x7FFFFFFFll : next);
    }
}

// One CTA (128 threads, thread = tile row) per 128x128 tile.
__global__ void __launch_bounds__(128) tile_rows_kernel(const uint8_t* __restrict__ mask,
                                                        const int* __restrict__ prefix,
                                                        int* __restrict__ row_offsets,
                                                        const uint16_t* __restrict__ slots,
                                                        const int* __restrict__ vals_offset,
                                                        uint16_t* __restrict__ vals, long long cap,
                                                        uint32_t* __restrict__ status,
                                                        uint4* __restrict__ colmask) {
    __shared__ int s_warp[4];
    __shared__ uint4 s_or[4];
    const long long t = blockIdx.x;
    const int r = threadIdx.x, lane = r & 31, warp = r >> 5;
    const uint4 mw = __ldg(reinterpret_cast<const uint4*>(mask + t * 2048 + r * 16));
    const int cnt = __popc(mw.x) + __popc(mw.y) + __popc(mw.z) + __popc(mw.w);
    const int inc = warp_incl_scan(cnt, lane);
    if (lane == 31) s_warp[warp] = inc;
    if (colmask) {
        // the tile's live columns: OR of its 128 rows' mask words
        const uint4 o = make_uint4(__reduce_or_sync(FULL, mw.x), __reduce_or_sync(FULL, mw.y),
                                   __reduce_or_sync(FULL, mw.z), __reduce_or_sync(FULL, mw.w));
        if (lane == 0) s_or[warp] = o;
    }
    __syncthreads();
    if (colmask && r == 0) {
        uint4 o = s_or[0];
#pragma unroll
        for (int w = 1; w < 4; ++w) {
            o.x |= s_or[w].x;
            o.y |= s_or[w].y;
            o.z |= s_or[w].z;
            o.w |= s_or[w].w;
        }
        colmask[t] = o;
    }
    int before = 0;
    for (int w = 0; w < warp; ++w) before += s_warp[w];
    const int roff = prefix[t] + before + inc - cnt;
    if (row_offsets) row_offsets[t * 128 + r] = roff;
    if (!slots) return;
    const long long base = (long long)*vals_offset;
    // Warp-cooperative, coalesced copy of the warp's 32 row segments (lane k
    // moves value k of a row), all 32 rows' loads issued before any store,
    // so a warp waits for one memory round trip per 32 values of its rows.
    int maxc = cnt;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) maxc = max(maxc, __shfl_xor_sync(FULL, maxc, o));
    const uint16_t* wsrc = slots + t * 16384 + warp * 32 * 128;
    for (int k0 = 0; k0 < maxc; k0 += 32) {
        const int k = k0 + lane;
        uint16_t v[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            const int c = __shfl_sync(FULL, cnt, u);
            v[u] = k < c ? __ldcs(wsrc + u * 128 + k) : (uint16_t)0;
        }
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            const int c = __shfl_sync(FULL, cnt, u);
            const long long p = base + __shfl_sync(FULL, roff, u) + k;
            if (k < c) {
                if (p >= 0 && p < cap) vals[p] = v[u];
                else atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
            }
        }
    }
}

// One CTA (128 threads) per 128x128 tile, after the up-projection wrote each
// warp's 32 rows of the tile packed in arena order at slots[t*16384 + w*4096]
// (warp w, count counts[t*4 + w]) and each row's offset in its warp's run:
// warp w moves its segment to the arena as one contiguous run, the row
// offsets gain prefix[t] and the counts of the warps before, and
// (optionally) colmask receives the tile's live columns.
constexpr int SEG = 4096;  // values of one warp's segment of a tile slot
__global__ void __launch_bounds__(128) tile_copy_kernel(const uint16_t* __restrict__ slots,
                                                        const int* __restrict__ counts,
                                                        const int* __restrict__ prefix,
                                                        const int* __restrict__ vals_offset,
                                                        uint16_t* __restrict__ vals, long long cap,
                                                        int* __restrict__ row_offsets,
                                                        const uint8_t* __restrict__ mask,
                                                        uint4* __restrict__ colmask,
                                                        uint32_t* __restrict__ status) {
    __shared__ uint4 s_or[4];
    const long long t = blockIdx.x;
    const int r = threadIdx.x, lane = r & 31, warp = r >> 5;
    const int4 cw = *reinterpret_cast<const int4*>(counts + t * 4);
    const int before = (warp > 0 ? cw.x : 0) + (warp > 1 ? cw.y : 0) + (warp > 2 ? cw.z : 0);
    const int n = warp == 0 ? cw.x : warp == 1 ? cw.y : warp == 2 ? cw.z : cw.w;
    const long long p0 = (long long)prefix[t] + before;
    if (row_offsets) row_offsets[t * 128 + r] += (int)p0;
    if (colmask) {
        const uint4 mw = __ldg(reinterpret_cast<const uint4*>(mask + t * 2048 + r * 16));
        const uint4 o = make_uint4(__reduce_or_sync(FULL, mw.x), __reduce_or_sync(FULL, mw.y),
                                   __reduce_or_sync(FULL, mw.z), __reduce_or_sync(FULL, mw.w));
        if (lane == 0) s_or[warp] = o;
        __syncthreads();
        if (r == 0)
            colmask[t] = make_uint4(s_or[0].x | s_or[1].x | s_or[2].x | s_or[3].x,
                                    s_or[0].y | s_or[1].y | s_or[2].y | s_or[3].y,
                                    s_or[0].z | s_or[1].z | s_or[2].z | s_or[3].z,
                                    s_or[0].w | s_or[1].w | s_or[2].w | s_or[3].w);
    }
    if (n <= 0) return;
    const long long base = (long long)*vals_offset + p0;
    const uint16_t* src = slots + t * 16384 + warp * SEG;
    if (base < 0 || base + n > cap || n > SEG) {
        // past the arena: the values that fit, and the overflow flag
        for (int i = lane; i < n && i < SEG; i += 32) {
            const long long p = base + i;
            if (p >= 0 && p < cap) vals[p] = src[i];
        }
        if (lane == 0) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
        return;
    }
    copy_run16<32>(src, vals + base, n, lane);
}

// Grid (pair tile, group of 8 k-blocks); warp w of a CTA tests k-block
// 8*group + w over the pair's two 128-row format tiles with all loads issued
// at once, and writes a 0/1 flag into kb_list[tile][kb].  The last CTA of a
// pair tile (counted in kb_count[tile], zeroed before the launch) compacts the
// flags in place into the ascending list of live k-blocks and stores the count.
constexpr int LIVE_WARPS = 8;
__global__ void __launch_bounds__(LIVE_WARPS * 32) live_kblocks_kernel(const uint8_t* __restrict__ mask,
                                                                      int gm_f, int gn_f, int nkb,
                                                                      int* __restrict__ kb_list,
                                                                      int* __restrict__ kb_count) {
    const int tp = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb = blockIdx.y * LIVE_WARPS + warp;
    int* flags = kb_list + (long long)tp * nkb;
    if (kb < nkb) {
        uint2 w[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int tm = 2 * tp + h;
            const long long tf = (long long)min(tm, gm_f - 1) * gn_f + kb / 2;
            const uint8_t* tmask = mask + tf * 2048 + (kb & 1) * 8;  // 2 words of each 16-byte row
#pragma unroll
            for (int q = 0; q < 4; ++q)
                w[h][q] = tm < gm_f ? *reinterpret_cast<const uint2*>(tmask + (lane + 32 * q) * 16) : make_uint2(0, 0);
        }
        uint32_t any = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int q = 0; q < 4; ++q) any |= w[h][q].x | w[h][q].y;
        any = __any_sync(FULL, any != 0);
        if (lane == 0) flags[kb] = any ? 1 : 0;
    }
    __threadfence();
    __syncthreads();
    __shared__ bool s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(&kb_count[tp], 1) == (int)gridDim.y - 1;
    __syncthreads();
    if (!s_last || warp != 0) return;
    __threadfence();
    // ordered in-place compaction: entry n <= kb is written after flag kb is read
    int n = 0;
    for (int k0 = 0; k0 < nkb; k0 += 32) {
        const int k = k0 + lane;
        const bool live = k < nkb && __ldcg(flags + k) != 0;
        const unsigned b = __ballot_sync(FULL, live);
        if (live) flags[n + __popc(b & ((1u << lane) - 1u))] = k;
        n += __popc(b);
    }
    if (lane == 0) kb_count[tp] = n;
}

// The same lists for the weight-gradient GEMMs, whose contraction runs over
// tokens: for each 256-column tile p of the activation (two columns of
// 128x128 format tiles; the M tile of dpre^T @ x and a^T @ dout), the
// ascending list of 64-row token blocks holding any set bit.  Warp w of a CTA
// tests token block 8*group + w over the two format tiles' 64 rows.
__global__ void __launch_bounds__(LIVE_WARPS * 32) live_kblocks_t_kernel(const uint8_t* __restrict__ mask,
                                                                        int gm_f, int gn_f, int nkb,
                                                                        int* __restrict__ kb_list,
                                                                        int* __restrict__ kb_count) {
    const int tp = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb = blockIdx.y * LIVE_WARPS + warp;
    int* flags = kb_list + (long long)tp * nkb;
    if (kb < nkb) {
        const int tm = kb >> 1;
        uint4 w[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int tn = 2 * tp + h;
            const bool ok = tn < gn_f && tm < gm_f;
            const uint8_t* tmask = mask + ((long long)tm * gn_f + min(tn, gn_f - 1)) * 2048 + (kb & 1) * 64 * 16;
#pragma unroll
            for (int q = 0; q < 2; ++q)
                w[h][q] = ok ? *reinterpret_cast<const uint4*>(tmask + (lane + 32 * q) * 16) : make_uint4(0, 0, 0, 0);
        }
        uint32_t any = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int q = 0; q < 2; ++q) any |= w[h][q].x | w[h][q].y | w[h][q].z | w[h][q].w;
        any = __any_sync(FULL, any != 0);
        if (lane == 0) flags[kb] = any ? 1 : 0;
    }
    __threadfence();
    __syncthreads();
    __shared__ bool s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(&kb_count[tp], 1) == (int)gridDim.y - 1;
    __syncthreads();
    if (!s_last || warp != 0) return;
    __threadfence();
    int n = 0;
    for (int k0 = 0; k0 < nkb; k0 += 32) {
        const int k = k0 + lane;
        const bool live = k < nkb && __ldcg(flags + k) != 0;
        const unsigned b = __ballot_sync(FULL, live);
        if (live) flags[n + __popc(b & ((1u << lane) - 1u))] = k;
        n += __popc(b);
    }
    if (lane == 0) kb_count[tp] = n;
}

// Three-term bf16 split of a float32 (or float16) matrix for the split-bf16
// products: x = hi + mid + lo with hi = bf16(x), mid = bf16(x - hi),
// lo = bf16(x - hi - mid) (each difference exact in float32), so the three
// pieces carry x's 24 significant bits.  Row r of dst holds six blocks of
// `cols` elements, the pieces in the order `order` gives (two bits per
// block: 0 hi, 1 mid, 2 lo); src element (r, c) is at src[r*s_row + c*s_col].
// The product of an A split in the order hi hi mid hi lo mid with a B split
// in the order hi mid hi lo hi mid, contracted over the 6*cols columns,
// sums hi*hi + hi*mid + mid*hi + hi*lo + lo*hi + mid*mid: the float32
// product up to terms of relative size 2^-24.
template <typename S>
__global__ void __launch_bounds__(256) split3_kernel(const S* __restrict__ src, long long rows, long long cols,
                                                     long long s_row, long long s_col, uint16_t* __restrict__ dst,
                                                     long long ld_dst, uint32_t order) {
    const long long n = rows * cols;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / cols, c = i - r * cols;
        float x;
        if constexpr (sizeof(S) == 4) x = __ldg(src + r * s_row + c * s_col);
        else x = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const uint16_t*>(src) + r * s_row + c * s_col)));
        const __nv_bfloat16 hi = __float2bfloat16_rn(x);
        const float r1 = x - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
        const uint16_t piece[3] = {__bfloat16_as_ushort(hi), __bfloat16_as_ushort(mid), __bfloat16_as_ushort(lo)};
        uint16_t* d = dst + r * ld_dst + c;
#pragma unroll
        for (int b = 0; b < 6; ++b) d[b * cols] = piece[(order >> (2 * b)) & 3u];
    }
}

// dst[i] = src[i] rounded to TF32 (tf32_round_bits), four at a time when
// both are 16-byte aligned (vec), else one at a time.
__global__ void __launch_bounds__(256) round_tf32_kernel(const uint32_t* src, uint32_t* dst, long long n, int vec) {
    const long long n4 = vec ? n / 4 : 0;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        uint4 v = __ldcs(reinterpret_cast<const uint4*>(src) + i);
        v = make_uint4(tf32_round_bits(v.x), tf32_round_bits(v.y), tf32_round_bits(v.z), tf32_round_bits(v.w));
        __stcs(reinterpret_cast<uint4*>(dst) + i, v);
    }
    for (long long i = 4 * n4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = tf32_round_bits(src[i]);
}

// dst[c][r] = src[r][c] for 16-bit elements: a 64 x 64 tile per CTA, read
// and written in 16-byte rows through shared memory padded to 66 elements a
// row (column reads of 2-byte elements then fall in distinct banks).
constexpr int TR_T = 64;
constexpr int TR_LD = TR_T + 2;
__global__ void __launch_bounds__(256) transpose16_kernel(const uint16_t* __restrict__ src, long long ld_src,
                                                          int rows, int cols, uint16_t* __restrict__ dst,
                                                          long long ld_dst) {
    __shared__ uint16_t tile[TR_T][TR_LD];
    const int r0 = blockIdx.y * TR_T, c0 = blockIdx.x * TR_T;
    const int t = threadIdx.x;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int idx = t + 256 * i;  // 512 16-byte pieces: 64 rows x 8
        const int rr = idx >> 3, cc = (idx & 7) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r0 + rr < rows && c0 + cc < cols)  // cols % 8 == 0: whole pieces
            v = __ldg(reinterpret_cast<const uint4*>(src + (long long)(r0 + rr) * ld_src + c0 + cc));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            tile[rr][cc + 2 * h] = (uint16_t)w[h];
            tile[rr][cc + 2 * h + 1] = (uint16_t)(w[h] >> 16);
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int idx = t + 256 * i;  // 64 output rows (source columns) x 8 pieces
        const int oc = idx >> 3, orr = (idx & 7) * 8;
        if (c0 + oc < cols && r0 + orr < rows) {  // rows % 8 == 0
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h)
                w[h] = (uint32_t)tile[orr + 2 * h][oc] | ((uint32_t)tile[orr + 2 * h + 1][oc] << 16);
            *reinterpret_cast<uint4*>(dst + (long long)(c0 + oc) * ld_dst + r0 + orr) =
                make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// ---------------------------------------------------------------------------
// Compacted-K operands of the bitmask-sparse down-projection (and dX).
//
// For each 128-row tile tm of a [T, F] activation in the 128x128 tiled
// format, the live columns are those holding a set bit in any of the tile's
// rows (the OR of the rows' mask words, `colmask`, one uint4 per format tile,
// written by tile_rows_kernel).  The contraction over F then runs over the
// tile's live columns only: the activation's live columns, compacted, times
// the rows of the other operand gathered at the same column indices.
// ---------------------------------------------------------------------------
constexpr int CK_LIST_T = 128;

// One CTA per row tile: counts per 128-column block, their exclusive prefix
// (colpref[tm][n], by warp prefix sums), the ascending live-column list
// idx[tm][0, K) and its padding up to a multiple of 64 with a dead column of
// the tile (whose entries are zero in every row of it), and kcount[tm] = K.
__global__ void __launch_bounds__(CK_LIST_T) ck_lists_kernel(const uint4* __restrict__ colmask, int gn, int F,
                                                            int* __restrict__ idx, long long ld_idx,
                                                            int* __restrict__ kcount, int* __restrict__ colpref) {
    extern __shared__ int s_cnt[];  // [gn] counts, then exclusive prefixes
    __shared__ int s_warp[CK_LIST_T / 32];
    __shared__ int s_dead;
    const int tm = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint4* cm = colmask + (long long)tm * gn;
    if (tid == 0) s_dead = 0x7FFFFFFF;
    __syncthreads();
    // per-thread run of blocks, counts and the first dead column below F
    const int per = (gn + CK_LIST_T - 1) / CK_LIST_T;
    const int lo = min(tid * per, gn), hi = min(lo + per, gn);
    int run = 0, dead = 0x7FFFFFFF;
    for (int n = lo; n < hi; ++n) {
        const uint4 L = __ldg(cm + n);
        const int c = __popc(L.x) + __popc(L.y) + __popc(L.z) + __popc(L.w);
        s_cnt[n] = c;
        run += c;
        if (dead == 0x7FFFFFFF && c < 128) {
            const uint32_t w[4] = {L.x, L.y, L.z, L.w};
            for (int q = 0; q < 4 && dead == 0x7FFFFFFF; ++q)
                if (~w[q]) {
                    const int col = n * 128 + 32 * q + __ffs(~w[q]) - 1;
                    if (col < F) dead = col;
                }
        }
    }
    if (dead != 0x7FFFFFFF) atomicMin(&s_dead, dead);
    const int inc = warp_incl_scan(run, lane);
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < CK_LIST_T / 32; ++w) {
        if (w < warp) before += s_warp[w];
        total += s_warp[w];
    }
    if (!idx) {  // counts only
        if (tid == 0) kcount[tm] = total;
        return;
    }
    int p = before + inc - run;
    for (int n = lo; n < hi; ++n) {
        const int c = s_cnt[n];
        s_cnt[n] = p;
        if (colpref) colpref[(long long)tm * gn + n] = p;
        p += c;
    }
    __syncthreads();
    int* list = idx + (long long)tm * ld_idx;
    // thread = column of a block: coalesced writes of each block's live columns
    for (int n = 0; n < gn; ++n) {
        const uint4 L = __ldg(cm + n);
        const uint32_t w[4] = {L.x, L.y, L.z, L.w};
        const int q = tid >> 5, b = tid & 31;
        if ((w[q] >> b) & 1u) {
            int rank = __popc(w[q] & ((1u << b) - 1u));
            for (int k = 0; k < q; ++k) rank += __popc(w[k]);
            list[s_cnt[n] + rank] = n * 128 + tid;
        }
    }
    const int padded = (total + 63) & ~63;
    for (int j = total + tid; j < padded; j += CK_LIST_T) list[j] = s_dead;  // total < padded <= F: a dead column exists
    if (tid == 0) kcount[tm] = total;
}

// One CTA (128 threads, thread = row) per format tile (tm, n): the tile's
// values of z from the packed form (bitmask, per-row offsets into vals),
// act(z) (z*z rounded to bf16 for ReLU^2, z for ReLU) at the tile's live
// columns, zeros where the row's bit is clear, written as row segments of
// ac[row][colpref[tm][n] ...] through shared memory.
constexpr int CK_SROW = 130;  // staged row stride in elements (65 words: conflict-free by row)
constexpr int CK_GATHER_SMEM = (16384 + 128 * CK_SROW) * 2;
__global__ void __launch_bounds__(128) ck_gather_packed_kernel(const uint16_t* __restrict__ vals, long long vals_len,
                                                               const uint8_t* __restrict__ mask,
                                                               const int* __restrict__ prefix,
                                                               const int* __restrict__ row_offsets,
                                                               const int* __restrict__ vals_offset,
                                                               const uint4* __restrict__ colmask,
                                                               const int* __restrict__ colpref,
                                                               const int* __restrict__ kcount, int gn, int act,
                                                               uint16_t* __restrict__ ac, long long ld_ac,
                                                               uint32_t* __restrict__ status) {
    // the tile's values (contiguous in vals, read coalesced), then the staged
    // output rows
    extern __shared__ __align__(16) uint16_t s_dyn[];
    uint16_t* s_vals = s_dyn;
    uint16_t* s_tile = s_dyn + 16384;
    const int tm = blockIdx.x, n = blockIdx.y;
    const long long t = (long long)tm * gn + n;
    const int r = threadIdx.x;
    if (n == 0) {
        // the list's padding columns [K, K rounded up to 64) are zero
        const int K = __ldg(kcount + tm), Kp = (K + 63) & ~63;
        uint16_t* row = ac + ((long long)tm * 128 + r) * ld_ac;
        for (int j = K; j < Kp; ++j) row[j] = 0;
    }
    const uint4 L = __ldg(colmask + t);
    const uint32_t lw[4] = {L.x, L.y, L.z, L.w};
    const int cnt = __popc(L.x) + __popc(L.y) + __popc(L.z) + __popc(L.w);
    if (cnt == 0) return;  // uniform over the CTA
    const uint4 b4 = __ldg(reinterpret_cast<const uint4*>(mask + t * 2048 + r * 16));
    const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
    const int p0 = __ldg(prefix + t), tcnt = min(__ldg(prefix + t + 1) - p0, 16384);
    const long long vb = (long long)*vals_offset + p0;
    bool short_vals = false;
    for (int i = r; i < tcnt; i += 128) {
        uint16_t v = 0;
        if (vb + i < vals_len) {
            v = __ldg(vals + vb + i);
            if (act == 1) v = __bfloat16_as_ushort(__hmul(__ushort_as_bfloat16(v), __ushort_as_bfloat16(v)));
        } else {
            short_vals = true;
        }
        s_vals[i] = v;
    }
    if (short_vals) atomicOr(status, SFFN_STATUS_VALS_SHORT);
    __syncthreads();
    int p = __ldg(row_offsets + t * 128 + r) - p0;  // this row's first value in s_vals
    uint16_t* srow = s_tile + r * CK_SROW;
    int k = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t live = lw[q];  // the same for every thread: uniform loop
        while (live) {
            const int c = __ffs(live) - 1;
            live &= live - 1u;
            const uint32_t hit = (bw[q] >> c) & 1u;
            srow[k++] = hit && p < tcnt ? s_vals[p] : (uint16_t)0;
            p += (int)hit;
        }
    }
    __syncthreads();
    // warp w writes rows w, w + 4, ...: each row's cnt values are contiguous
    const int warp = r >> 5, lane = r & 31;
    const long long col0 = __ldg(colpref + t);
    for (int rr = warp; rr < 128; rr += 4) {
        uint16_t* dst = ac + ((long long)tm * 128 + rr) * ld_ac + col0;
        const uint16_t* src = s_tile + rr * CK_SROW;
        for (int j = lane; j < cnt; j += 32) dst[j] = src[j];
    }
}

// In place, one warp per row of x [T, ld]: x[row][j] = x[row][idx[tm][j]]
// for j < K, 32 at a time in ascending j, then zeros up to the padded count.
// Since idx ascends with idx[j] >= j, a read never sees a position an earlier
// round wrote, and each round's reads finish before its writes (__syncwarp).
// Rows of tiles whose every column is live are left as they are.
__global__ void __launch_bounds__(256) ck_compact_rows_kernel(uint16_t* __restrict__ x, long long ld, int F,
                                                             long long T, const int* __restrict__ idx,
                                                             long long ld_idx, const int* __restrict__ kcount) {
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= T) return;
    const int lane = threadIdx.x & 31;
    const int tm = (int)(row >> 7);
    const int K = __ldg(kcount + tm);
    if (K >= F) return;
    const int Kp = (K + 63) & ~63;
    const int* list = idx + (long long)tm * ld_idx;
    uint16_t* xr = x + row * ld;
    for (int j0 = 0; j0 < K; j0 += 32) {
        const int j = j0 + lane;
        uint16_t v = 0;
        if (j < K) v = xr[__ldg(list + j)];
        __syncwarp();
        if (j < K) xr[j] = v;
        __syncwarp();
    }
    for (int j = K + lane; j < Kp; j += 32) xr[j] = 0;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" int sffn_transpose16(const void* src, int64_t ld_src, int64_t rows, int64_t cols, void* dst,
                                int64_t ld_dst, void* stream) {
    if (rows < 0 || cols < 0 || rows % 8 || cols % 8) return SFFN_ERR_ARG;
    if (rows == 0 || cols == 0) return SFFN_OK;
    if (!src || !dst || ld_src < cols || ld_dst < rows) return SFFN_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 16 || ld_src % 8 || ld_dst % 8)
        return SFFN_ERR_ALIGN;
    if (rows / TR_T + 1 > 65535) return SFFN_ERR_ARG;
    const dim3 grid((unsigned)((cols + TR_T - 1) / TR_T), (unsigned)((rows + TR_T - 1) / TR_T));
    transpose16_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(src), ld_src, (int)rows, (int)cols, static_cast<uint16_t*>(dst), ld_dst);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_tile_scan_counts(const int32_t* tile_counts, int parts, int64_t ntiles, int32_t* prefix,
                                     int32_t* offset_dev, int32_t* vals_offset_dev, uint32_t* status_dev,
                                     void* stream) {
    if (ntiles <= 0 || parts <= 0 || !tile_counts || !prefix || !offset_dev || !vals_offset_dev || !status_dev)
        return SFFN_ERR_ARG;
    if (offset_dev == vals_offset_dev) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, tile_counts);
    tile_scan_kernel<<<1, SCAN_NT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        tile_counts, parts, ntiles, prefix, offset_dev, vals_offset_dev, status_dev);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_tile_gather_slots(const void* slots, const uint8_t* bitmask, const int32_t* prefix,
                                      const int32_t* vals_offset_dev, int64_t ntiles, void* vals,
                                      int64_t vals_capacity, int dtype, int32_t* row_offsets,
                                      uint32_t* colmask, uint32_t* status_dev, void* stream) {
    if (dtype != SFFN_BF16 && dtype != SFFN_F16) return SFFN_ERR_DTYPE;
    if (ntiles <= 0 || !slots || !bitmask || !prefix || !vals_offset_dev || !vals || !status_dev)
        return SFFN_ERR_ARG;
    if (!aligned16(bitmask) || !aligned16(colmask)) return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, vals);
    tile_rows_kernel<<<(unsigned)ntiles, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        bitmask, prefix, row_offsets, static_cast<const uint16_t*>(slots), vals_offset_dev,
        static_cast<uint16_t*>(vals), vals_capacity, status_dev, reinterpret_cast<uint4*>(colmask));
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_tile_copy_slots(const void* slots, const int32_t* tile_counts, const int32_t* prefix,
                                    const int32_t* vals_offset_dev, int64_t ntiles, void* vals,
                                    int64_t vals_capacity, int32_t* row_offsets, const uint8_t* bitmask,
                                    uint32_t* colmask, uint32_t* status_dev, void* stream) {
    if (ntiles <= 0 || ntiles > 0x7FFFFFFF || !slots || !tile_counts || !prefix || !vals_offset_dev || !vals ||
        !status_dev)
        return SFFN_ERR_ARG;
    if (colmask && !bitmask) return SFFN_ERR_ARG;
    if (!aligned16(slots) || !aligned16(tile_counts) || !aligned16(bitmask) || !aligned16(colmask) ||
        (reinterpret_cast<uintptr_t>(vals) & 1u))
        return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, vals);
    tile_copy_kernel<<<(unsigned)ntiles, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(slots), tile_counts, prefix, vals_offset_dev, static_cast<uint16_t*>(vals),
        vals_capacity, row_offsets, bitmask, reinterpret_cast<uint4*>(colmask), status_dev);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_tile_row_offsets(const uint8_t* bitmask, const int32_t* prefix, int64_t ntiles,
                                     int32_t* row_offsets, uint32_t* colmask, void* stream) {
    if (ntiles <= 0 || !bitmask || !prefix || (!row_offsets && !colmask)) return SFFN_ERR_ARG;
    if (!aligned16(bitmask) || !aligned16(colmask)) return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, bitmask);
    tile_rows_kernel<<<(unsigned)ntiles, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        bitmask, prefix, row_offsets, nullptr, nullptr, nullptr, 0, nullptr, reinterpret_cast<uint4*>(colmask));
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_live_kblocks(const uint8_t* bitmask, int64_t M, int64_t N, int32_t* kb_list,
                                 int32_t* kb_count, void* stream) {
    if (M <= 0 || N <= 0 || !bitmask || !kb_list || !kb_count) return SFFN_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(bitmask) & 7u) return SFFN_ERR_ALIGN;
    const long long gm = (M + 127) / 128, gp = (M + 255) / 256, gn_f = (N + 127) / 128, nkb = (N + 63) / 64;
    if (gp > 0x7FFFFFFF || nkb > 0x7FFFFFFF) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, bitmask);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    SFFN_CUDA_TRY(cudaMemsetAsync(kb_count, 0, (size_t)gp * sizeof(int32_t), st));
    const dim3 grid((unsigned)gp, (unsigned)((nkb + LIVE_WARPS - 1) / LIVE_WARPS));
    live_kblocks_kernel<<<grid, LIVE_WARPS * 32, 0, st>>>(bitmask, (int)gm, (int)gn_f, (int)nkb, kb_list,
                                                         kb_count);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

// ---------------------------------------------------------------------------
// Compacted-K operands (see the kernels above).
// ---------------------------------------------------------------------------
extern "C" int sffn_ck_lists(const uint32_t* colmask, int64_t T, int64_t F, int32_t* idx, int64_t ld_idx,
                             int32_t* kcount, int32_t* colpref, void* stream) {
    if (T <= 0 || F <= 0 || T % 128 || F % 64 || !colmask || !kcount || (!idx && colpref)) return SFFN_ERR_ARG;
    if (ld_idx < F || F > 65536 || !aligned16(colmask)) return SFFN_ERR_ARG;
    const long long gm = T / 128, gn = (F + 127) / 128;
    if (gm > 0x7FFFFFFF) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, colmask);
    ck_lists_kernel<<<(unsigned)gm, CK_LIST_T, (size_t)gn * sizeof(int), reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint4*>(colmask), (int)gn, (int)F, idx, ld_idx, kcount, colpref);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_ck_gather_packed(const void* vals, int64_t vals_len, const uint8_t* bitmask,
                                     const int32_t* prefix, const int32_t* row_offsets,
                                     const int32_t* vals_offset_dev,
                                     const uint32_t* colmask, const int32_t* colpref, const int32_t* kcount,
                                     int64_t T, int64_t F, int act, void* ac, int64_t ld_ac, uint32_t* status_dev,
                                     void* stream) {
    if (T <= 0 || F <= 0 || T % 128 || F % 64 || (act != 0 && act != 1)) return SFFN_ERR_ARG;
    if (!vals || !bitmask || !prefix || !row_offsets || !vals_offset_dev || !colmask || !colpref || !kcount || !ac ||
        !status_dev)
        return SFFN_ERR_ARG;
    if (ld_ac < F || !aligned16(bitmask) || !aligned16(colmask)) return SFFN_ERR_ARG;
    const long long gm = T / 128, gn = (F + 127) / 128;
    if (gm > 0x7FFFFFFF || gn > 65535) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, ac);
    SFFN_CUDA_TRY(cudaFuncSetAttribute(ck_gather_packed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       CK_GATHER_SMEM));
    ck_gather_packed_kernel<<<dim3((unsigned)gm, (unsigned)gn), 128, CK_GATHER_SMEM,
                              reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(vals), vals_len, bitmask, prefix, row_offsets, vals_offset_dev,
        reinterpret_cast<const uint4*>(colmask), colpref, kcount, (int)gn, act, static_cast<uint16_t*>(ac), ld_ac,
        status_dev);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_ck_compact_rows(void* x, int64_t ld, int64_t T, int64_t F, const int32_t* idx, int64_t ld_idx,
                                    const int32_t* kcount, void* stream) {
    if (T <= 0 || F <= 0 || T % 128 || F % 64 || !x || !idx || !kcount || ld < F || ld_idx < F) return SFFN_ERR_ARG;
    if (F > 65536) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, x);
    ck_compact_rows_kernel<<<(unsigned)((T + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint16_t*>(x), ld, (int)F, (long long)T, idx, ld_idx, kcount);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_live_kblocks_t(const uint8_t* bitmask, int64_t M, int64_t N, int32_t* kb_list,
                                   int32_t* kb_count, void* stream) {
    if (M <= 0 || N <= 0 || !bitmask || !kb_list || !kb_count) return SFFN_ERR_ARG;
    if (!aligned16(bitmask)) return SFFN_ERR_ALIGN;
    const long long gm = (M + 127) / 128, gn_f = (N + 127) / 128, gp = (N + 255) / 256, nkb = (M + 63) / 64;
    if (gp > 0x7FFFFFFF || nkb > 0x7FFFFFFF || gm > 0x7FFFFFFF) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, bitmask);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    SFFN_CUDA_TRY(cudaMemsetAsync(kb_count, 0, (size_t)gp * sizeof(int32_t), st));
    const dim3 grid((unsigned)gp, (unsigned)((nkb + LIVE_WARPS - 1) / LIVE_WARPS));
    live_kblocks_t_kernel<<<grid, LIVE_WARPS * 32, 0, st>>>(bitmask, (int)gm, (int)gn_f, (int)nkb, kb_list, kb_count);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_round_tf32(const float* src, float* dst, int64_t n, void* stream) {
    if (n < 0 || (n > 0 && (!src || !dst))) return SFFN_ERR_ARG;
    if (n == 0) return SFFN_OK;
    DeviceScope dev_scope;
    if (int rc = dev_scope.bind_same(dst, {src})) return rc;
    const int vec = aligned16(src) && aligned16(dst);
    const unsigned grid = (unsigned)std::min<long long>((n / 4 + 255) / 256 + 1, 148ll * 16);
    round_tf32_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint32_t*>(src), reinterpret_cast<uint32_t*>(dst), n, vec);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_split_bf16x3(const void* src, int dtype, int64_t rows, int64_t cols, int64_t s_row, int64_t s_col,
                                 void* dst, int64_t ld_dst, int b_order, void* stream) {
    if (dtype != SFFN_F32 && dtype != SFFN_F16) return SFFN_ERR_DTYPE;
    if (rows <= 0 || cols <= 0 || !src || !dst || ld_dst < 6 * cols) return SFFN_ERR_ARG;
    // A: hi hi mid hi lo mid; B: hi mid hi lo hi mid (two bits per block)
    const uint32_t order = b_order ? (0u | 1u << 2 | 0u << 4 | 2u << 6 | 0u << 8 | 1u << 10)
                                   : (0u | 0u << 2 | 1u << 4 | 0u << 6 | 2u << 8 | 1u << 10);
    DeviceScope dev_scope;
    if (int rc = dev_scope.bind_same(dst, {src})) return rc;
    const long long n = rows * cols;
    const unsigned grid = (unsigned)std::min<long long>((n + 255) / 256, 148ll * 16);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == SFFN_F32)
        split3_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(src), rows, cols, s_row, s_col,
                                                   static_cast<uint16_t*>(dst), ld_dst, order);
    else
        split3_kernel<uint16_t><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(src), rows, cols, s_row, s_col,
                                                      static_cast<uint16_t*>(dst), ld_dst, order);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

