// Flat bitmask format: single-pass pack and unpack (sm_100a).
//
// Reference: old/sparse_pack.py:6-106 (count/pack, serial prefix, vals --
// three kernels, two reads of the dense tensor) and old/sparse_unpack.py:6-97
// (popcount, serial prefix, reconstruct).  Here each direction is ONE kernel:
// a CTA takes the next 8192-element chunk by ticket, builds its mask bytes /
// ranks in registers, resolves its global offset by decoupled look-back over
// the preceding chunks and writes its values through shared memory, so the
// dense tensor is read (pack) or written (unpack) exactly once.
//
// Thread layout: 256 threads x 4 iterations x 8 elements.  A thread's 8
// consecutive elements form one mask byte; lanes 4k..4k+3 form one
// little-endian uint32 mask word (bit f%32 of word f/32 == bit f%8 of byte f/8).
#include "common.cuh"

namespace sffn {
namespace {

constexpr int FL_NT = 256;
constexpr int FL_U = 4;
constexpr int FL_CHUNK = FL_NT * 8 * FL_U;  // 8192 elements
static_assert(FL_U * (FL_NT / 32) == 32, "one warp scans the (iteration, warp) totals");

template <typename B>
__device__ __forceinline__ void load8(const B* __restrict__ p, B (&v)[8]) {
    if constexpr (sizeof(B) == 2) {
        uint4 q = __ldcs(reinterpret_cast<const uint4*>(p));
        const B* s = reinterpret_cast<const B*>(&q);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = s[j];
    } else {
        uint4 q0 = __ldcs(reinterpret_cast<const uint4*>(p));
        uint4 q1 = __ldcs(reinterpret_cast<const uint4*>(p) + 1);
        v[0] = q0.x; v[1] = q0.y; v[2] = q0.z; v[3] = q0.w;
        v[4] = q1.x; v[5] = q1.y; v[6] = q1.z; v[7] = q1.w;
    }
}

template <typename B>
__device__ __forceinline__ void store8(B* __restrict__ p, const B (&v)[8]) {
    if constexpr (sizeof(B) == 2) {
        uint4 q;
        B* d = reinterpret_cast<B*>(&q);
#pragma unroll
        for (int j = 0; j < 8; ++j) d[j] = v[j];
        __stcs(reinterpret_cast<uint4*>(p), q);
    } else {
        __stcs(reinterpret_cast<uint4*>(p), make_uint4(v[0], v[1], v[2], v[3]));
        __stcs(reinterpret_cast<uint4*>(p) + 1, make_uint4(v[4], v[5], v[6], v[7]));
    }
}

// Scan the 32 (iteration, warp) totals held in s_wx (in place -> exclusive);
// returns nothing, writes the chunk aggregate to *s_agg.
__device__ __forceinline__ void scan32(int* s_wx, int* s_agg, int lane) {
    int t = s_wx[lane];
    int inc = warp_incl_scan(t, lane);
    s_wx[lane] = inc - t;
    if (lane == 31) *s_agg = inc;
}

template <typename B>
__global__ void __launch_bounds__(FL_NT) flat_pack_kernel(
    const B* __restrict__ dense, long long n, uint8_t* __restrict__ mask, B* __restrict__ vals,
    long long cap, long long* __restrict__ nnz_out, unsigned long long* __restrict__ states,
    unsigned* __restrict__ ticket, uint32_t* __restrict__ status, long long nchunks) {
    __shared__ __align__(16) B s_vals[FL_CHUNK];
    __shared__ int s_wx[32];
    __shared__ int s_agg;
    __shared__ long long s_chunk;
    __shared__ unsigned long long s_excl;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_chunk = atomicAdd(ticket, 1u);
    __syncthreads();
    const long long chunk = s_chunk;
    const long long base = chunk * FL_CHUNK;
    const long long nbytes = (n + 7) >> 3;

    B v[FL_U][8];
    uint32_t bits[FL_U];
    int lex[FL_U];
#pragma unroll
    for (int it = 0; it < FL_U; ++it) {
        const long long f0 = base + (long long)(it * FL_NT + tid) * 8;
        if (f0 + 8 <= n) {
            load8(dense + f0, v[it]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[it][j] = (f0 + j < n) ? dense[f0 + j] : B(0);
        }
        uint32_t b = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) b |= (uint32_t)nonzero_bits(v[it][j]) << j;
        bits[it] = b;
        const uint32_t w = bytes_to_word(b, lane);
        if ((lane & 3) == 0 && f0 < n) {
            const long long byte = f0 >> 3;
            if (byte + 4 <= nbytes) {
                *reinterpret_cast<uint32_t*>(mask + byte) = w;
            } else {
                for (int k = 0; k < 4; ++k)
                    if (byte + k < nbytes) mask[byte + k] = (uint8_t)(w >> (8 * k));
            }
        }
        const int c = __popc(b);
        const int inc = warp_incl_scan(c, lane);
        lex[it] = inc - c;
        if (lane == 31) s_wx[it * (FL_NT / 32) + warp] = inc;
    }
    __syncthreads();
    if (warp == 0) scan32(s_wx, &s_agg, lane);
    __syncthreads();
#pragma unroll
    for (int it = 0; it < FL_U; ++it) {
        int r = s_wx[it * (FL_NT / 32) + warp] + lex[it];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if ((bits[it] >> j) & 1u) s_vals[r++] = v[it][j];
    }
    const int agg = s_agg;
    if (warp == 0) {
        unsigned long long ex = lookback(states, chunk, (unsigned long long)agg, status, lane);
        if (lane == 0) s_excl = ex;
    }
    __syncthreads();
    const long long ex = (long long)s_excl;
    for (int i = tid; i < agg; i += FL_NT) {
        const long long p = ex + i;
        if (p < cap) vals[p] = s_vals[i];
    }
    if (tid == 0) {
        if (ex + agg > cap) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
        if (chunk == nchunks - 1) *nnz_out = ex + agg;
    }
}

template <typename B>
__global__ void __launch_bounds__(FL_NT) flat_unpack_kernel(
    const B* __restrict__ vals, long long vals_len, const uint8_t* __restrict__ mask, long long n,
    B* __restrict__ out, unsigned long long* __restrict__ states, unsigned* __restrict__ ticket,
    uint32_t* __restrict__ status) {
    __shared__ __align__(16) B s_vals[FL_CHUNK];
    __shared__ int s_wx[32];
    __shared__ int s_agg;
    __shared__ long long s_chunk;
    __shared__ unsigned long long s_excl;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_chunk = atomicAdd(ticket, 1u);
    __syncthreads();
    const long long chunk = s_chunk;
    const long long base = chunk * FL_CHUNK;
    const long long nbytes = (n + 7) >> 3;

    uint32_t bits[FL_U];
    int lex[FL_U];
#pragma unroll
    for (int it = 0; it < FL_U; ++it) {
        const long long f0 = base + (long long)(it * FL_NT + tid) * 8;
        const long long byte = f0 >> 3;
        uint32_t w = 0;
        if ((lane & 3) == 0 && byte < nbytes) {
            if (byte + 4 <= nbytes) {
                w = __ldcs(reinterpret_cast<const unsigned int*>(mask + byte));
            } else {
                for (int k = 0; k < 4; ++k)
                    if (byte + k < nbytes) w |= (uint32_t)mask[byte + k] << (8 * k);
            }
        }
        w = __shfl_sync(FULL, w, lane & ~3);
        uint32_t b = (w >> (8 * (lane & 3))) & 0xFFu;
        if (f0 >= n) b = 0;
        else if (f0 + 8 > n) b &= (1u << (n - f0)) - 1u;
        bits[it] = b;
        const int c = __popc(b);
        const int inc = warp_incl_scan(c, lane);
        lex[it] = inc - c;
        if (lane == 31) s_wx[it * (FL_NT / 32) + warp] = inc;
    }
    __syncthreads();
    if (warp == 0) scan32(s_wx, &s_agg, lane);
    __syncthreads();
    const int agg = s_agg;
    if (warp == 0) {
        unsigned long long ex = lookback(states, chunk, (unsigned long long)agg, status, lane);
        if (lane == 0) s_excl = ex;
    }
    __syncthreads();
    const long long ex = (long long)s_excl;
    for (int i = tid; i < agg; i += FL_NT) {
        const long long p = ex + i;
        s_vals[i] = p < vals_len ? vals[p] : B(0);
    }
    if (tid == 0 && ex + agg > vals_len) atomicOr(status, SFFN_STATUS_VALS_SHORT);
    __syncthreads();
#pragma unroll
    for (int it = 0; it < FL_U; ++it) {
        const long long f0 = base + (long long)(it * FL_NT + tid) * 8;
        if (f0 >= n) continue;
        int r = s_wx[it * (FL_NT / 32) + warp] + lex[it];
        B o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = ((bits[it] >> j) & 1u) ? s_vals[r++] : B(0);
        if (f0 + 8 <= n) {
            store8(out + f0, o);
        } else {
            for (int j = 0; j < 8; ++j)
                if (f0 + j < n) out[f0 + j] = o[j];
        }
    }
}

struct FlatWs {
    unsigned* ticket;
    unsigned long long* states;
    size_t used;
};

inline long long flat_chunks(long long n) { return (n + FL_CHUNK - 1) / FL_CHUNK; }

inline FlatWs flat_ws(void* ws, long long n) {
    FlatWs w;
    w.ticket = reinterpret_cast<unsigned*>(ws);
    w.states = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(ws) + 16);
    w.used = 16 + (size_t)flat_chunks(n) * 8;
    return w;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" size_t sffn_flat_workspace_bytes(int64_t n) {
    if (n < 0) return 0;
    return 16 + (size_t)flat_chunks(n) * 8;
}

extern "C" int sffn_flat_pack(const void* dense, int dtype, int64_t n, uint8_t* packed_mask,
                              void* vals, int64_t vals_capacity, int64_t* nnz_dev, void* workspace,
                              size_t workspace_bytes, uint32_t* status_dev, void* stream) {
    if (!dtype_ok(dtype)) return SFFN_ERR_DTYPE;
    if (n < 0 || vals_capacity < 0 || !nnz_dev || !status_dev) return SFFN_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n == 0) {
        SFFN_CUDA_TRY(cudaMemsetAsync(nnz_dev, 0, sizeof(int64_t), st));
        return SFFN_OK;
    }
    if (!dense || !packed_mask || (!vals && vals_capacity > 0) || !workspace) return SFFN_ERR_ARG;
    if (!aligned16(dense) || (reinterpret_cast<uintptr_t>(packed_mask) & 3u)) return SFFN_ERR_ALIGN;
    if (workspace_bytes < sffn_flat_workspace_bytes(n)) return SFFN_ERR_WORKSPACE;
    FlatWs w = flat_ws(workspace, n);
    SFFN_CUDA_TRY(cudaMemsetAsync(workspace, 0, w.used, st));
    const long long nch = flat_chunks(n);
    if (dtype == SFFN_F32) {
        flat_pack_kernel<uint32_t><<<(unsigned)nch, FL_NT, 0, st>>>(
            (const uint32_t*)dense, n, packed_mask, (uint32_t*)vals, vals_capacity,
            (long long*)nnz_dev, w.states, w.ticket, status_dev, nch);
    } else {
        flat_pack_kernel<uint16_t><<<(unsigned)nch, FL_NT, 0, st>>>(
            (const uint16_t*)dense, n, packed_mask, (uint16_t*)vals, vals_capacity,
            (long long*)nnz_dev, w.states, w.ticket, status_dev, nch);
    }
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
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
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    FlatWs w = flat_ws(workspace, n);
    SFFN_CUDA_TRY(cudaMemsetAsync(workspace, 0, w.used, st));
    const long long nch = flat_chunks(n);
    if (dtype == SFFN_F32) {
        flat_unpack_kernel<uint32_t><<<(unsigned)nch, FL_NT, 0, st>>>(
            (const uint32_t*)vals, vals_len, packed_mask, n, (uint32_t*)out, w.states, w.ticket,
            status_dev);
    } else {
        flat_unpack_kernel<uint16_t><<<(unsigned)nch, FL_NT, 0, st>>>(
            (const uint16_t*)vals, vals_len, packed_mask, n, (uint16_t*)out, w.states, w.ticket,
            status_dev);
    }
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}
