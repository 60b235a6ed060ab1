// Shared device helpers for the sparse-FFN kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <initializer_list>
#include <type_traits>

#include "../../include/sparseffn.h"

namespace sffn {

constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------------------
// Host-side error plumbing
// ---------------------------------------------------------------------------
void set_cuda_error(cudaError_t e);
void set_error_text(const char* msg);

#define SFFN_CHECK_LAUNCH()                                  \
    do {                                                     \
        cudaError_t _e = cudaGetLastError();                 \
        if (_e != cudaSuccess) {                             \
            ::sffn::set_cuda_error(_e);                      \
            return SFFN_ERR_CUDA;                            \
        }                                                    \
    } while (0)

#define SFFN_CUDA_TRY(call)                                  \
    do {                                                     \
        cudaError_t _e = (call);                             \
        if (_e != cudaSuccess) {                             \
            ::sffn::set_cuda_error(_e);                      \
            return SFFN_ERR_CUDA;                            \
        }                                                    \
    } while (0)

// Device of a device (or managed) pointer, or -1 (the failed query cleared).
int device_of(const void* p);
// Unique id of the thread's current CUDA context (ids are never reused, also
// not after a device reset creates a new primary context), or 0 if unknown.
unsigned long long current_context_id();

// For the length of one entry-point call: makes the device that owns a
// pointer current on the calling thread, with its primary context bound
// (driver calls such as cuTensorMapEncodeTiled need one), and on every return
// path puts back the context that was current when the call began -- which
// may be another device's, or none.  Callers arrive on any host thread (an
// autograd worker, a plug-in host's thread) and keep their own device.
class DeviceScope {
  public:
    DeviceScope() = default;
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;
    ~DeviceScope();
    // SFFN_OK, SFFN_ERR_ARG (not device memory) or SFFN_ERR_CUDA.
    int bind(const void* p);
    // Also SFFN_ERR_ARG unless every non-null pointer of `others` lives on the bound device.
    int bind_same(const void* p, std::initializer_list<const void*> others);
    int device() const { return dev_; }

  private:
    void* saved_ = nullptr;  // CUcontext current at bind()
    bool restore_ = false;
    int dev_ = -1;
};

// One-line form for the entry points: `SFFN_BIND(scope, ptr)` declares a
// DeviceScope named `scope` bound to ptr's device, returning on failure.
#define SFFN_BIND(scope, p)                              \
    ::sffn::DeviceScope scope;                           \
    if (int _rc = scope.bind(p)) return _rc

inline int esize_of(int dtype) { return dtype == SFFN_F32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == SFFN_F32 || dtype == SFFN_BF16 || dtype == SFFN_F16; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Element predicates on raw bit patterns (exactly IEEE compares)
// ---------------------------------------------------------------------------
// x != 0: magnitude bits non-zero (-0.0 -> false, NaN -> true).
__device__ __forceinline__ bool nonzero_bits(uint16_t b) { return (b & 0x7FFFu) != 0; }
// The float32 bit pattern `u` rounded to the nearest TF32 value (10 explicit
// mantissa bits), ties away from zero: half of the 13 dropped bits' weight
// added to the magnitude, then those bits cleared (a carry moves into the
// exponent, up to infinity); infinities and NaNs unchanged.
__device__ __forceinline__ uint32_t tf32_round_bits(uint32_t u) {
    return (u & 0x7F800000u) == 0x7F800000u ? u : (u + 0x1000u) & 0xFFFFE000u;
}
__device__ __forceinline__ bool nonzero_bits(uint32_t b) { return (b & 0x7FFFFFFFu) != 0; }

// x > 0: sign clear, non-zero, not NaN.  INF16 is the +inf pattern of the
// 16-bit type (0x7F80 bf16, 0x7C00 fp16).
__device__ __forceinline__ bool positive_bits(uint16_t b, uint16_t inf16) {
    return (int16_t)b > 0 && b <= inf16;
}
__device__ __forceinline__ bool positive_bits(uint32_t b, uint16_t) {
    return (int32_t)b > 0 && b <= 0x7F800000u;
}

inline uint16_t inf16_of(int dtype) { return dtype == SFFN_F16 ? 0x7C00 : 0x7F80; }

// Storage-dtype arithmetic (products of two 16-bit floats are exact in fp32,
// so computing in fp32 and rounding once equals the 16-bit operation).
template <int DT> struct Elt;
template <> struct Elt<SFFN_F32> {
    using bits = uint32_t;
    __device__ static float to_f(bits b) { return __uint_as_float(b); }
    __device__ static bits from_f(float f) { return __float_as_uint(f); }
};
template <> struct Elt<SFFN_BF16> {
    using bits = uint16_t;
    __device__ static float to_f(bits b) { return __uint_as_float(((uint32_t)b) << 16); }
    __device__ static bits from_f(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
};
template <> struct Elt<SFFN_F16> {
    using bits = uint16_t;
    __device__ static float to_f(bits b) { return __half2float(__ushort_as_half(b)); }
    __device__ static bits from_f(float f) { return __half_as_ushort(__float2half_rn(f)); }
};

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(FULL, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

// Combine one mask byte per lane into little-endian 32-bit words: lanes
// 4k..4k+3 hold consecutive bytes; every lane gets its group's word.
__device__ __forceinline__ uint32_t bytes_to_word(uint32_t byte, int lane) {
    uint32_t w = byte << (8 * (lane & 3));
    w |= __shfl_xor_sync(FULL, w, 1);
    w |= __shfl_xor_sync(FULL, w, 2);
    return w;
}

// ---------------------------------------------------------------------------
// Decoupled look-back over a sequence of partitions (single-pass scan).
// State word per partition: bits 63:62 = flag (0 none, 1 aggregate, 2 inclusive),
// bits 61:0 = value.  Partitions are processed in an order in which every
// predecessor of a running partition has started, so the wait ends; it is
// still bounded: after kLookbackLimitNs of wall time the partition records
// SFFN_STATUS_WAIT_TIMEOUT, publishes what it has and returns.
// ---------------------------------------------------------------------------
constexpr unsigned long long LB_AGG = 1ull << 62;
constexpr unsigned long long LB_INCL = 2ull << 62;
constexpr unsigned long long LB_VAL = (1ull << 62) - 1;
constexpr unsigned long long kLookbackLimitNs = 500ull * 1000 * 1000;  // wall-time bound

__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Publish this partition's aggregate (or, for partition 0, its inclusive
// prefix).  Called by one thread, before lookback().  The release orders
// every earlier memory access of that thread before the publication.
__device__ __forceinline__ void lookback_publish(unsigned long long* states, long long part,
                                                 unsigned long long agg) {
    st_release_u64(&states[part], (part == 0 ? LB_INCL : LB_AGG) | (agg & LB_VAL));
}

// Called by one full warp after lookback_publish().  Returns the exclusive
// prefix of partition `part` and publishes its inclusive prefix.  Each lane
// inspects W consecutive predecessors per round, so one round covers 32*W
// partitions: the resolved frontier advances 32*W partitions per L2 round
// trip, which bounds the scan's throughput.
template <int W>
__device__ __forceinline__ unsigned long long lookback(unsigned long long* states, long long part,
                                                      unsigned long long agg, uint32_t* status,
                                                      int lane,
                                                      unsigned long long limit_ns = kLookbackLimitNs) {
    if (part == 0) return 0;
    unsigned long long excl = 0;
    long long pred = part - 1;
    unsigned long long t0 = 0;
    while (true) {
        unsigned long long s[W];
#pragma unroll
        for (int k = 0; k < W; ++k) {
            const long long idx = pred - (long long)lane * W - k;
            s[k] = idx >= 0 ? ld_relaxed_u64(&states[idx]) : LB_INCL;
        }
        // nearest inclusive entry of this lane, and whether an empty entry precedes it
        int kin = W;
#pragma unroll
        for (int k = W - 1; k >= 0; --k)
            if ((s[k] >> 62) == 2) kin = k;
        bool empty_before = false;
#pragma unroll
        for (int k = 0; k < W; ++k)
            if (k <= kin && k < W && (s[k] >> 62) == 0) empty_before = true;
        const unsigned incl = __ballot_sync(FULL, kin < W);
        const int first = incl ? __ffs(incl) - 1 : 32;  // nearest lane holding an inclusive entry
        const bool need_lane = lane <= first;
        const unsigned waiting = __ballot_sync(FULL, need_lane && empty_before);
        if (waiting) {
            unsigned long long now;
            asm volatile("mov.u64 %0, %globaltimer;" : "=l"(now));
            if (t0 == 0) t0 = now;
            // lane 0's clock decides for the whole warp
            if (__shfl_sync(FULL, now - t0 > limit_ns ? 1 : 0, 0)) {
                if (lane == 0) atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                break;
            }
            __nanosleep(32);
            continue;
        }
        unsigned long long v = 0;
        if (need_lane) {
            const int upto = lane == first ? kin : W - 1;
#pragma unroll
            for (int k = 0; k < W; ++k)
                if (k <= upto) v += s[k] & LB_VAL;
        }
        excl += warp_sum_u64(v);
        if (incl) break;
        pred -= 32LL * W;
    }
    if (lane == 0) st_release_u64(&states[part], LB_INCL | ((excl + agg) & LB_VAL));
    return excl;
}

// Publication for lookback_rows(): a relaxed store.  A state word carries
// its flag and count together in one aligned 64-bit store, and no reader pairs
// it with other data written by the publishing partition, so it needs no
// release -- a release would stall until all of the thread's earlier stores
// are acknowledged, which under full memory load takes microseconds.
__device__ __forceinline__ void lookback_publish_relaxed(unsigned long long* states, long long part,
                                                         unsigned long long agg) {
    st_relaxed_u64(&states[part], (part == 0 ? LB_INCL : LB_AGG) | (agg & LB_VAL));
}

// Warp-collective look-back like lookback(), reading W*32 predecessors per
// round in coalesced rows: in row k lane l reads partition pred - 32*k - l,
// so each load instruction fetches 32 consecutive states (256 bytes).  The
// nearest inclusive entry is the first (row, lane) in that order that holds
// one; every entry before it must be at least an aggregate.  A wide window
// lets the resolved frontier advance 32*W partitions per L2 round trip.
template <int W>
__device__ __forceinline__ unsigned long long lookback_rows(unsigned long long* states, long long part,
                                                           unsigned long long agg, uint32_t* status,
                                                           int lane,
                                                           unsigned long long limit_ns = kLookbackLimitNs) {
    if (part == 0) return 0;
    unsigned long long excl = 0;
    long long pred = part - 1;
    unsigned long long t0 = 0;
    while (true) {
        unsigned long long s[W];
#pragma unroll
        for (int k = 0; k < W; ++k) {
            const long long idx = pred - 32LL * k - lane;
            s[k] = idx >= 0 ? ld_relaxed_u64(&states[idx]) : LB_INCL;
        }
        int krow = W;  // first row holding an inclusive entry (warp-uniform)
        unsigned lanes = 0;
#pragma unroll
        for (int k = 0; k < W; ++k) {
            const unsigned b = __ballot_sync(FULL, (s[k] >> 62) == 2);
            if (krow == W && b) {
                krow = k;
                lanes = b;
            }
        }
        const int cut = krow < W ? 32 * krow + (__ffs(lanes) - 1) : 32 * W;  // position of that entry
        bool empty = false;
        unsigned long long v = 0;
#pragma unroll
        for (int k = 0; k < W; ++k) {
            if (32 * k + lane <= cut) {
                if ((s[k] >> 62) == 0) empty = true;
                v += s[k] & LB_VAL;
            }
        }
        if (__any_sync(FULL, empty)) {
            unsigned long long now;
            asm volatile("mov.u64 %0, %globaltimer;" : "=l"(now));
            if (t0 == 0) t0 = now;
            // lane 0's clock decides for the whole warp
            if (__shfl_sync(FULL, now - t0 > limit_ns ? 1 : 0, 0)) {
                if (lane == 0) atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                break;
            }
            __nanosleep(32);
            continue;
        }
        excl += warp_sum_u64(v);
        if (krow < W) break;
        pred -= 32LL * W;
    }
    if (lane == 0) st_relaxed_u64(&states[part], LB_INCL | ((excl + agg) & LB_VAL));
    return excl;
}

// Copy of n 16-bit values from src (16-byte aligned) to dst by the NT threads
// r = 0 .. NT-1, where dst + H is 16-byte aligned (H = 0..7): H head values one
// by one, then 16-byte stores whose eight values straddle two aligned source
// vectors (shifted by H values), then the tail.  Source reads stay below the
// aligned end of src[0 .. n+7).
template <int H, int NT>
__device__ __forceinline__ void copy_run(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int n,
                                         int r) {
    const int body = n > H ? (n - H) >> 3 : 0;
    const int tail0 = n > H ? H + body * 8 : n;
    if (r < H && r < n) dst[r] = src[r];
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst + H);
#pragma unroll 4
    for (int k = r; k < body; k += NT) {
        if constexpr (H == 0) {
            d4[k] = __ldcs(s4 + k);
        } else {
            const uint4 a = __ldg(s4 + k), b = __ldg(s4 + k + 1);
            const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if constexpr (H % 2 == 0) o[j] = w[j + H / 2];
                else o[j] = __funnelshift_r(w[j + H / 2], w[j + H / 2 + 1], 16);
            }
            d4[k] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
    for (int i = tail0 + r; i < n; i += NT) dst[i] = src[i];
}

// copy_run with H taken from dst's alignment (dst at least 2-byte aligned).
template <int NT>
__device__ __forceinline__ void copy_run16(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int n,
                                           int r) {
    switch ((int)((16u - (uint32_t)(reinterpret_cast<uintptr_t>(dst) & 15u)) & 15u) >> 1) {
        case 0: copy_run<0, NT>(src, dst, n, r); break;
        case 1: copy_run<1, NT>(src, dst, n, r); break;
        case 2: copy_run<2, NT>(src, dst, n, r); break;
        case 3: copy_run<3, NT>(src, dst, n, r); break;
        case 4: copy_run<4, NT>(src, dst, n, r); break;
        case 5: copy_run<5, NT>(src, dst, n, r); break;
        case 6: copy_run<6, NT>(src, dst, n, r); break;
        default: copy_run<7, NT>(src, dst, n, r); break;
    }
}

}  // namespace sffn
