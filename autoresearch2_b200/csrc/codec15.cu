// 15-bit sign-strip codec (bitshifting/code.py) for sm_100a.
//
// Format: n 16-bit words (bf16 / fp16 bit patterns, non-negative by intent)
// become a byte stream of ceil(15 n / 8) bytes with value i at stream bits
// [15 i, 15 i + 15), little-endian.  The reference builds each output byte b
// as ((v[i] >> o) | (v[i+1] << (15 - o))) & 0xFF, i = 8b / 15, o = 8b % 15
// (code.py:39-69), from the full 16-bit words; a set sign bit of v[i] thus
// lands on stream bit 15 (i + 1) unless that bit starts a byte, i.e. unless
// i % 8 == 7.  Here: stream = OR over i of (t_i << 15 i), t_i = v[i] with its
// sign bit cleared where i % 8 == 7 -- the same bytes for every input.
// Decoding (code.py:98-122) takes field i and clears nothing else.
//
// Work unit: a group of 16 values = 240 bits = 30 bytes, self-contained
// (15 * 16 % 8 == 0, and value 16g + 15 has i % 8 == 7).  One thread per
// group, 256 groups (4096 values, 7680 bytes) per tile; the 30-byte records
// are staged in shared memory so that global reads and writes of the packed
// side are 16-byte vectors at 16-byte aligned offsets (7680 = 480 * 16).
// Compress: one tile per CTA, values loaded straight into registers.
// Uncompress: persistent CTAs, the next tile's stream bytes copied into a
// second shared buffer (cp.async) while the current tile is decoded.
// Both kernels are HBM-bound: 2 n + ceil(15 n / 8) bytes per call.
#include "common.cuh"

namespace sffn {
namespace {

constexpr int C15_T = 256;
constexpr int C15_GROUP_BYTES = 30;
constexpr int C15_BLOCK_BYTES = C15_T * C15_GROUP_BYTES;  // 7680
constexpr long long C15_BLOCK_VALS = C15_T * 16;          // 4096
static_assert(C15_BLOCK_BYTES % 16 == 0, "packed block must be whole 16-byte vectors");

__device__ __forceinline__ void c15_split(const uint4 q, uint32_t* v) {
    v[0] = q.x & 0xFFFFu; v[1] = q.x >> 16;
    v[2] = q.y & 0xFFFFu; v[3] = q.y >> 16;
    v[4] = q.z & 0xFFFFu; v[5] = q.z >> 16;
    v[6] = q.w & 0xFFFFu; v[7] = q.w >> 16;
}

__device__ __forceinline__ uint32_t c15_join(uint32_t lo, uint32_t hi) { return (lo & 0xFFFFu) | (hi << 16); }

// 16 words of group starting at value v0 (zeros past n).
__device__ __forceinline__ void c15_load(const uint16_t* __restrict__ src, long long n, long long v0, bool vec,
                                         uint32_t (&v)[16]) {
    if (vec && v0 + 16 <= n) {
        const uint4* p = reinterpret_cast<const uint4*>(src + v0);
        c15_split(__ldg(p), v);
        c15_split(__ldg(p + 1), v + 8);
        return;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = v0 + i < n ? (uint32_t)__ldg(src + v0 + i) : 0u;
}

// The group's 240-bit stream in 8 words (w[7] uses its low 16 bits).
__device__ __forceinline__ void c15_pack(const uint32_t (&v)[16], uint32_t (&w)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const uint32_t t = (i % 8 == 7) ? (v[i] & 0x7FFFu) : v[i];
        const int p = 15 * i;
        w[p >> 5] |= t << (p & 31);
        if ((p & 31) > 16) w[(p >> 5) + 1] |= t >> (32 - (p & 31));
    }
}

__global__ void __launch_bounds__(C15_T) codec15_compress_kernel(const uint16_t* __restrict__ src, long long n,
                                                                 uint8_t* __restrict__ dst, long long nbytes,
                                                                 bool vec_in, bool vec_out) {
    __shared__ __align__(16) uint8_t sbuf[C15_BLOCK_BYTES];
    const long long blk_b = (long long)blockIdx.x * C15_BLOCK_BYTES;
    uint32_t v[16], w[8];
    c15_load(src, n, (long long)blockIdx.x * C15_BLOCK_VALS + 16 * threadIdx.x, vec_in, v);
    c15_pack(v, w);
    // 30 bytes at 30 * tid: 2-byte aligned, 15 halfword stores
    uint16_t* s16 = reinterpret_cast<uint16_t*>(sbuf + C15_GROUP_BYTES * threadIdx.x);
#pragma unroll
    for (int j = 0; j < 15; ++j) s16[j] = (uint16_t)((j & 1) ? (w[j >> 1] >> 16) : w[j >> 1]);
    __syncthreads();
    const long long left = nbytes - blk_b;
    const int bytes = left < C15_BLOCK_BYTES ? (int)left : C15_BLOCK_BYTES;
    if (vec_out && bytes == C15_BLOCK_BYTES) {
        uint4* d = reinterpret_cast<uint4*>(dst + blk_b);
        const uint4* s = reinterpret_cast<const uint4*>(sbuf);
        for (int q = threadIdx.x; q < C15_BLOCK_BYTES / 16; q += C15_T) d[q] = s[q];
    } else {
        for (int q = threadIdx.x; q < bytes; q += C15_T) dst[blk_b + q] = sbuf[q];
    }
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Stream bytes of tile t into a shared buffer: whole 16-byte-aligned tiles by
// asynchronous 16-byte copies, the last (partial) tile or an unaligned
// stream by plain byte loads with zero fill.  Always closes one copy group.
__device__ __forceinline__ void c15_fetch(const uint8_t* __restrict__ src, long long nbytes, long long t,
                                          long long tiles, bool vec_in, uint8_t* buf) {
    if (t < tiles) {
        const long long b0 = t * C15_BLOCK_BYTES;
        const long long left = nbytes - b0;
        if (vec_in && left >= C15_BLOCK_BYTES) {
            for (int q = threadIdx.x; q < C15_BLOCK_BYTES / 16; q += C15_T) cp_async16(buf + 16 * q, src + b0 + 16 * q);
        } else {
            for (int q = threadIdx.x; q < C15_BLOCK_BYTES; q += C15_T) buf[q] = q < left ? __ldg(src + b0 + q) : 0;
        }
    }
    cp_async_commit();
}

// Persistent over tiles (stride gridDim.x), two shared buffers: the next
// tile's bytes are in flight while the current one is decoded and stored.
__global__ void __launch_bounds__(C15_T) codec15_uncompress_kernel(const uint8_t* __restrict__ src,
                                                                   long long nbytes, long long n,
                                                                   uint16_t* __restrict__ dst, bool vec_in,
                                                                   bool vec_out) {
    __shared__ __align__(16) uint8_t sbuf[2][C15_BLOCK_BYTES];
    const long long tiles = (n + C15_BLOCK_VALS - 1) / C15_BLOCK_VALS;
    int stage = 0;
    c15_fetch(src, nbytes, blockIdx.x, tiles, vec_in, sbuf[0]);
    for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
        c15_fetch(src, nbytes, t + gridDim.x, tiles, vec_in, sbuf[stage ^ 1]);
        cp_async_wait_one();  // this thread's copies of tile t have landed
        __syncthreads();      // ... and every thread's
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(sbuf[stage] + C15_GROUP_BYTES * threadIdx.x);
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 7; ++j) w[j] = c15_join(s16[2 * j], s16[2 * j + 1]);
        w[7] = s16[14];
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int p = 15 * i;
            uint32_t x = w[p >> 5] >> (p & 31);
            if ((p & 31) > 17) x |= w[(p >> 5) + 1] << (32 - (p & 31));
            v[i] = x & 0x7FFFu;
        }
        const long long v0 = t * C15_BLOCK_VALS + 16 * threadIdx.x;
        if (vec_out && v0 + 16 <= n) {
            uint4* d = reinterpret_cast<uint4*>(dst + v0);
            d[0] = make_uint4(c15_join(v[0], v[1]), c15_join(v[2], v[3]), c15_join(v[4], v[5]),
                              c15_join(v[6], v[7]));
            d[1] = make_uint4(c15_join(v[8], v[9]), c15_join(v[10], v[11]), c15_join(v[12], v[13]),
                              c15_join(v[14], v[15]));
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (v0 + i < n) dst[v0 + i] = (uint16_t)v[i];
        }
        __syncthreads();  // sbuf[stage] is refilled two tiles from now
        stage ^= 1;
    }
}

// Host checks shared by both directions: sizes, pointers, overlap, grid.
int c15_check(const void* words, int64_t n, const void* bytes, int64_t bytes_len, unsigned& blocks) {
    if (n < 0 || n > (int64_t(1) << 40) || bytes_len < 0) return SFFN_ERR_ARG;
    const int64_t nb = sffn_codec15_bytes(n);
    if (n == 0) return SFFN_OK;
    if (!words || !bytes || bytes_len < nb) return SFFN_ERR_ARG;
    const uintptr_t w0 = reinterpret_cast<uintptr_t>(words), b0 = reinterpret_cast<uintptr_t>(bytes);
    if (w0 % 2) return SFFN_ERR_ALIGN;
    if (w0 < b0 + (uintptr_t)nb && b0 < w0 + 2 * (uintptr_t)n) return SFFN_ERR_ARG;  // overlap
    blocks = (unsigned)((n + C15_BLOCK_VALS - 1) / C15_BLOCK_VALS);
    return SFFN_OK;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" int64_t sffn_codec15_bytes(int64_t n) { return n < 0 ? -1 : (15 * n + 7) / 8; }

extern "C" int sffn_codec15_compress(const void* src, int64_t n, uint8_t* dst, int64_t dst_bytes, void* stream) {
    unsigned blocks = 0;
    if (int rc = c15_check(src, n, dst, dst_bytes, blocks)) return rc;
    if (n == 0) return SFFN_OK;
    SFFN_BIND(dev_scope, src);
    const bool vec_in = reinterpret_cast<uintptr_t>(src) % 16 == 0;
    const bool vec_out = reinterpret_cast<uintptr_t>(dst) % 16 == 0;
    codec15_compress_kernel<<<blocks, C15_T, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(src), n, dst, sffn_codec15_bytes(n), vec_in, vec_out);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_codec15_uncompress(const uint8_t* src, int64_t src_bytes, int64_t n, void* dst,
                                       void* stream) {
    unsigned blocks = 0;
    if (int rc = c15_check(dst, n, src, src_bytes, blocks)) return rc;
    if (n == 0) return SFFN_OK;
    SFFN_BIND(dev_scope, src);
    const bool vec_in = reinterpret_cast<uintptr_t>(src) % 16 == 0;
    const bool vec_out = reinterpret_cast<uintptr_t>(dst) % 16 == 0;
    // persistent: 8 CTAs (2048 threads) per SM at most
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned cap = 8u * (unsigned)(sms > 0 ? sms : 148);
    codec15_uncompress_kernel<<<blocks < cap ? blocks : cap, C15_T, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        src, sffn_codec15_bytes(n), n, static_cast<uint16_t*>(dst), vec_in, vec_out);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}
