// Small kernels around the fused FFN GEMMs (sm_100a).
//
//   tile_scan_kernel    per-tile counts -> exclusive prefix[num_tiles + 1];
//                       reads the int32 arena cursor into vals_offset and
//                       advances it by the total (sparse.py:181-204 without a
//                       host round trip).
//   slot_gather_kernel  moves each tile's compacted values from its fixed slot
//                       (written by the up-projection epilogue, which cannot
//                       know the tile's final offset) to
//                       vals[vals_offset + prefix[t] ...].
//   live_kblocks_kernel for each 256-row tile (two rows of 128x128 format
//                       tiles, the GEMM's CTA-pair tile) of a tiled bitmask,
//                       the ascending list of 64-column blocks holding any set
//                       bit: the down-projection skips the others.
#include "common.cuh"

namespace sffn {
namespace {

constexpr int SCAN_NT = 1024;

__global__ void __launch_bounds__(SCAN_NT) tile_scan_kernel(const int* __restrict__ counts, long long ntiles,
                                                           int* __restrict__ prefix, int* __restrict__ cursor,
                                                           int* __restrict__ vals_offset_out,
                                                           uint32_t* __restrict__ status) {
    __shared__ long long s_part[SCAN_NT];
    const int tid = threadIdx.x;
    const long long per = (ntiles + SCAN_NT - 1) / SCAN_NT;
    const long long lo = tid * per, hi = min(lo + per, ntiles);
    long long sum = 0;
    for (long long t = lo; t < hi; ++t) sum += counts[t];
    s_part[tid] = sum;
    __syncthreads();
    // Hillis-Steele inclusive scan of the 1024 partial sums
    for (int o = 1; o < SCAN_NT; o <<= 1) {
        const long long v = tid >= o ? s_part[tid - o] : 0;
        __syncthreads();
        s_part[tid] += v;
        __syncthreads();
    }
    long long run = s_part[tid] - sum;
    for (long long t = lo; t < hi; ++t) {
        prefix[t] = (int)run;
        run += counts[t];
    }
    if (tid == SCAN_NT - 1) {
        const long long total = s_part[SCAN_NT - 1];
        prefix[ntiles] = (int)total;
        const int cur = *cursor;
        *vals_offset_out = cur;
        const long long next = (long long)cur + total;
        if (next > 0x7FFFFFFFll || total > 0x7FFFFFFFll) atomicOr(status, SFFN_STATUS_CURSOR_OVERFLOW);
        *cursor = (int)(next > 0x7FFFFFFFll ? 0x7FFFFFFFll : next);
    }
}

__global__ void __launch_bounds__(256) slot_gather_kernel(const uint16_t* __restrict__ slots, int tile_elems,
                                                          const int* __restrict__ prefix,
                                                          const int* __restrict__ vals_offset,
                                                          uint16_t* __restrict__ vals, long long cap,
                                                          uint32_t* __restrict__ status) {
    const long long t = blockIdx.x;
    const int cnt = min(prefix[t + 1] - prefix[t], tile_elems);
    const long long dst = (long long)*vals_offset + prefix[t];
    const uint16_t* src = slots + t * tile_elems;
    if (threadIdx.x == 0 && (dst < 0 || dst + cnt > cap)) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
    for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
        const long long p = dst + i;
        if (p >= 0 && p < cap) vals[p] = __ldcs(src + i);
    }
}

// One CTA per 256-row tile; one warp per 64-column block at a time.
__global__ void __launch_bounds__(256) live_kblocks_kernel(const uint8_t* __restrict__ mask, int gm_f, int gn_f,
                                                           int nkb, int* __restrict__ kb_list,
                                                           int* __restrict__ kb_count) {
    extern __shared__ int s_live[];  // [nkb]
    const int tp = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int kb = warp; kb < nkb; kb += blockDim.x / 32) {
        uint32_t any = 0;
        for (int h = 0; h < 2; ++h) {
            const int tm = 2 * tp + h;
            if (tm >= gm_f) break;
            const long long tf = (long long)tm * gn_f + kb / 2;
            const uint8_t* tmask = mask + tf * 2048 + (kb & 1) * 8;  // 2 words of each 16-byte row
#pragma unroll
            for (int r = lane; r < 128; r += 32) {
                const uint2 w = *reinterpret_cast<const uint2*>(tmask + r * 16);
                any |= w.x | w.y;
            }
        }
        any = __any_sync(FULL, any != 0);
        if (lane == 0) s_live[kb] = any ? 1 : 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int n = 0;
        for (int kb = 0; kb < nkb; ++kb)
            if (s_live[kb]) kb_list[(long long)tp * nkb + n++] = kb;
        kb_count[tp] = n;
    }
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" int sffn_tile_scan_counts(const int32_t* tile_counts, int64_t ntiles, int32_t* prefix,
                                     int32_t* offset_dev, int32_t* vals_offset_dev, uint32_t* status_dev,
                                     void* stream) {
    if (ntiles <= 0 || !tile_counts || !prefix || !offset_dev || !vals_offset_dev || !status_dev)
        return SFFN_ERR_ARG;
    if (offset_dev == vals_offset_dev) return SFFN_ERR_ARG;
    if (int rc = bind_device_of(tile_counts)) return rc;
    tile_scan_kernel<<<1, SCAN_NT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        tile_counts, ntiles, prefix, offset_dev, vals_offset_dev, status_dev);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_tile_gather_slots(const void* slots, int tile_elems, const int32_t* prefix,
                                      const int32_t* vals_offset_dev, int64_t ntiles, void* vals,
                                      int64_t vals_capacity, int dtype, uint32_t* status_dev, void* stream) {
    if (dtype != SFFN_BF16 && dtype != SFFN_F16) return SFFN_ERR_DTYPE;
    if (ntiles <= 0 || tile_elems <= 0 || !slots || !prefix || !vals_offset_dev || !vals || !status_dev)
        return SFFN_ERR_ARG;
    if (int rc = bind_device_of(vals)) return rc;
    slot_gather_kernel<<<(unsigned)ntiles, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(slots), tile_elems, prefix, vals_offset_dev, static_cast<uint16_t*>(vals),
        vals_capacity, status_dev);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_live_kblocks(const uint8_t* bitmask, int64_t M, int64_t N, int32_t* kb_list,
                                 int32_t* kb_count, void* stream) {
    if (M <= 0 || N <= 0 || !bitmask || !kb_list || !kb_count) return SFFN_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(bitmask) & 7u) return SFFN_ERR_ALIGN;
    const long long gm = (M + 127) / 128, gp = (M + 255) / 256, gn_f = (N + 127) / 128, nkb = (N + 63) / 64;
    if (nkb > 12288) return SFFN_ERR_UNSUPPORTED;  // shared-memory flag array
    if (int rc = bind_device_of(bitmask)) return rc;
    live_kblocks_kernel<<<(unsigned)gp, 256, (size_t)nkb * sizeof(int), reinterpret_cast<cudaStream_t>(stream)>>>(
        bitmask, (int)gm, (int)gn_f, (int)nkb, kb_list, kb_count);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}
