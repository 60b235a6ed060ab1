// Flat bitmask format: pack and unpack (sm_100a).
//
// Reference: old/sparse_pack.py:6-106 (count/pack kernel, one-program serial
// prefix, vals kernel -- the dense tensor is read twice) and
// old/sparse_unpack.py:6-97 (popcount, one-program serial prefix, rebuild).
//
// Pack is ONE persistent kernel, launched cooperatively so that all its CTAs
// are resident.  CTA c owns chunks c, c+G, c+2G, ... (G = grid size) of 32 KB
// and streams them through a 3-stage ring of shared memory filled by 1-D TMA
// bulk copies, so the copies of its next two chunks are in flight while it
// works on one.  Per chunk: mask bytes and counts in registers, a block scan,
// the compacted values written back into the stage buffer, a decoupled
// look-back (256 predecessors per round) for the chunk's global offset, then a
// coalesced copy of the values to `vals`.  Because every chunk of round k is
// being worked on at the same time and round k-1 is resolved, a look-back
// needs at most two rounds of loads.  The dense tensor is read exactly once.
//
// Unpack needs no look-back: a small kernel popcounts the mask per 16K-element
// chunk and the last CTA to finish scans the counts; the expand kernel then
// streams every chunk independently (mask + its contiguous vals -> dense).
//
// Thread layout: 256 threads; in sub-step `sub` thread `tid` owns the 8
// consecutive elements f = 8*(sub*256 + tid) .. +7 of its chunk, i.e. one mask
// byte; lanes 4k..4k+3 form one little-endian uint32 mask word
// (bit f%32 of word f/32 == bit f%8 of byte f/8).
#include <stdio.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace sffn {
namespace {

constexpr int FL_NT = 256;
constexpr int FL_NW = FL_NT / 32;
constexpr int PACK_CHUNK_BYTES = 32768;
constexpr int PACK_STAGES = 3;
constexpr int LB_W = 8;  // look-back: 8 states per lane, 256 per round

template <typename B>
struct PackCfg {
    static constexpr int CE = PACK_CHUNK_BYTES / (int)sizeof(B);  // elements per chunk
    static constexpr int SUBS = CE / (FL_NT * 8);
    static constexpr int NE = SUBS * FL_NW;  // (sub-step, warp) partial counts
    static_assert(NE == 32 || NE == 64, "scan_pairs handles 32 or 64 entries");
};

// Exclusive scan, by one warp, of NE (32 or 64) ints in shared memory.
template <int NE>
__device__ __forceinline__ void scan_pairs(int* s, int* s_total, int lane) {
    if constexpr (NE == 32) {
        int t = s[lane];
        int inc = warp_incl_scan(t, lane);
        s[lane] = inc - t;
        if (lane == 31) *s_total = inc;
    } else {
        int a = s[2 * lane], b = s[2 * lane + 1];
        int inc = warp_incl_scan(a + b, lane);
        s[2 * lane] = inc - a - b;
        s[2 * lane + 1] = inc - b;
        if (lane == 31) *s_total = inc;
    }
}

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
template <typename B>
__global__ void __launch_bounds__(FL_NT, 2) flat_pack_kernel(
    const B* __restrict__ dense, long long n, uint8_t* __restrict__ mask, B* __restrict__ vals,
    long long cap, long long* __restrict__ nnz_out, unsigned long long* __restrict__ states,
    uint32_t* __restrict__ status, long long nchunks) {
    using C = PackCfg<B>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    B* stage = reinterpret_cast<B*>(smem_raw);  // [PACK_STAGES][CE]
    __shared__ __align__(8) uint64_t bars[PACK_STAGES];
    __shared__ long long s_tick[PACK_STAGES];
    __shared__ int s_wx[C::NE];
    __shared__ int s_agg;
    __shared__ unsigned long long s_excl;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long nbytes = (n + 7) >> 3;

    // Producer (thread 0): start the bulk copy of this CTA's k-th chunk into stage s.
    auto issue = [&](int s, long long k) {
        const long long t = (long long)blockIdx.x + k * gridDim.x;
        s_tick[s] = t;
        if (t < nchunks) {
            const long long nvalid = min((long long)C::CE, n - t * C::CE);
            const uint32_t bytes = (uint32_t)(nvalid * sizeof(B)) & ~15u;
            mbar_arrive_expect_tx(&bars[s], bytes);
            if (bytes) bulk_g2s(stage + (size_t)s * C::CE, dense + t * C::CE, bytes, &bars[s]);
        }
    };

    if (tid == 0) {
        for (int s = 0; s < PACK_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < PACK_STAGES; ++s) issue(s, s);
    __syncthreads();

    for (int it = 0;; ++it) {
        const int s = it % PACK_STAGES;
        const uint32_t parity = (uint32_t)(it / PACK_STAGES) & 1u;
        const long long t = s_tick[s];
        if (t >= nchunks) break;
        const bool ok = mbar_wait_bounded(&bars[s], parity);
        if (__syncthreads_or(!ok)) {
            // Give up: wait (bounded) for this CTA's copies still in flight --
            // stages of iterations it .. it+STAGES-1 -- before exiting.
            if (tid == 0) {
                atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                for (int j = 0; j < PACK_STAGES; ++j) {
                    const int sj = (it + j) % PACK_STAGES;
                    if (s_tick[sj] < nchunks)
                        (void)mbar_wait_bounded(&bars[sj], (uint32_t)((it + j) / PACK_STAGES) & 1u);
                }
            }
            break;
        }
        B* buf = stage + (size_t)s * C::CE;
        const long long base = t * C::CE;
        const int nvalid = (int)min((long long)C::CE, n - base);
        const int tma_elems = (int)(((long long)nvalid * sizeof(B)) & ~15ll) / (int)sizeof(B);

        Vec8<B> v[C::SUBS];
        uint32_t bits[C::SUBS];
        int lex[C::SUBS];
#pragma unroll
        for (int sub = 0; sub < C::SUBS; ++sub) {
            const int f = 8 * (sub * FL_NT + tid);
            if (f + 8 <= tma_elems) {
                v[sub].load_smem(buf + f);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int fe = f + j;
                    B e = B(0);
                    if (fe < tma_elems) e = buf[fe];
                    else if (fe < nvalid) e = dense[base + fe];
                    v[sub].set(j, e);
                }
            }
            uint32_t b = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) b |= (uint32_t)nonzero_bits(v[sub].get(j)) << j;
            bits[sub] = b;
            const uint32_t w = bytes_to_word(b, lane);
            const long long byte = (base + f) >> 3;
            if ((lane & 3) == 0 && f < nvalid) {
                if (byte + 4 <= nbytes) {
                    *reinterpret_cast<uint32_t*>(mask + byte) = w;
                } else {
                    for (int k = 0; k < 4; ++k)
                        if (byte + k < nbytes) mask[byte + k] = (uint8_t)(w >> (8 * k));
                }
            }
            const int c = __popc(b);
            const int inc = warp_incl_scan(c, lane);
            lex[sub] = inc - c;
            if (lane == 31) s_wx[sub * FL_NW + warp] = inc;
        }
        __syncthreads();  // all reads of the stage are in registers; s_wx complete
        if (warp == 0) {
            scan_pairs<C::NE>(s_wx, &s_agg, lane);
            __syncwarp();
            if (lane == 0) lookback_publish(states, t, (unsigned long long)s_agg);
        }
        __syncthreads();
        // compact into the (now free) stage buffer
#pragma unroll
        for (int sub = 0; sub < C::SUBS; ++sub) {
            int r = s_wx[sub * FL_NW + warp] + lex[sub];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if ((bits[sub] >> j) & 1u) buf[r++] = v[sub].get(j);
        }
        const int agg = s_agg;
        if (warp == 0) {
            const unsigned long long ex = lookback<LB_W>(states, t, (unsigned long long)agg, status, lane);
            if (lane == 0) s_excl = ex;
        }
        __syncthreads();
        const long long ex = (long long)s_excl;
        for (int i = tid; i < agg; i += FL_NT) {
            const long long p = ex + i;
            if (p < cap) vals[p] = buf[i];
        }
        if (tid == 0) {
            if (ex + agg > cap) atomicOr(status, SFFN_STATUS_VALS_OVERFLOW);
            if (t == nchunks - 1) *nnz_out = ex + agg;
        }
        // The stage was written through the generic proxy; order that before
        // the next bulk copy (async proxy) into it.
        fence_proxy_async_smem();
        __syncthreads();  // stage s fully consumed
        if (tid == 0) issue(s, it + PACK_STAGES);
        __syncthreads();
    }
}

// ---------------------------------------------------------------- unpack ----
constexpr int UNP_CE = 16384;               // elements per unpack chunk
constexpr int UNP_SUBS = UNP_CE / (FL_NT * 8);  // 8
constexpr int UNP_NE = UNP_SUBS * FL_NW;        // 64
constexpr int CNT_CHUNKS_PER_CTA = 16;

// Popcount of each chunk's mask; the last CTA to finish scans all counts into
// cprefix[0..nchunks] (exclusive prefix, cprefix[nchunks] = total).
__global__ void __launch_bounds__(FL_NT) flat_count_kernel(
    const uint8_t* __restrict__ mask, long long n, long long nchunks, int* __restrict__ counts,
    long long* __restrict__ cprefix, unsigned* __restrict__ done) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long nbytes = (n + 7) >> 3;
    const long long c0 = (long long)blockIdx.x * CNT_CHUNKS_PER_CTA;
    for (int k = warp; k < CNT_CHUNKS_PER_CTA; k += FL_NW) {
        const long long c = c0 + k;
        if (c >= nchunks) break;
        const long long b0 = c * (UNP_CE / 8), b1 = min(b0 + UNP_CE / 8, nbytes);
        int cnt = 0;
        // 2 KB per chunk: 32 lanes x 16 words, coalesced 128 B per warp load;
        // all 16 loads are issued before any is used.
        if (b0 + UNP_CE / 8 <= nbytes) {
            unsigned int w[16];
#pragma unroll
            for (int k = 0; k < 16; ++k)
                w[k] = __ldcs(reinterpret_cast<const unsigned int*>(mask + b0 + 4 * (lane + 32 * k)));
#pragma unroll
            for (int k = 0; k < 16; ++k) cnt += __popc(w[k]);
        } else {
            for (long long b = b0 + lane * 4; b < b1; b += 32 * 4) {
                if (b + 4 <= b1) {
                    cnt += __popc(__ldcs(reinterpret_cast<const unsigned int*>(mask + b)));
                } else {
                    for (long long e = b; e < b1; ++e) cnt += __popc((uint32_t)mask[e]);
                }
            }
        }
        // bits of the last byte past n are ignored
        if (c == nchunks - 1 && (n & 7) && lane == 0)
            cnt -= __popc((uint32_t)mask[nbytes - 1] & ~((1u << (n & 7)) - 1u));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(FULL, cnt, o);
        if (lane == 0) counts[c] = cnt;
    }
    __threadfence();
    __syncthreads();
    __shared__ unsigned s_last;
    if (tid == 0) s_last = (atomicAdd(done, 1u) == gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // last CTA: exclusive scan of counts[0..nchunks)
    __shared__ long long s_part[FL_NT];
    const long long per = (nchunks + FL_NT - 1) / FL_NT;
    const long long lo = tid * per, hi = min(lo + per, nchunks);
    long long sum = 0;
    for (long long c = lo; c < hi; ++c) sum += __ldcg(counts + c);
    s_part[tid] = sum;
    __syncthreads();
    if (tid == 0) {
        long long run = 0;
        for (int i = 0; i < FL_NT; ++i) {
            const long long x = s_part[i];
            s_part[i] = run;
            run += x;
        }
        cprefix[nchunks] = run;
    }
    __syncthreads();
    long long run = s_part[tid];
    for (long long c = lo; c < hi; ++c) {
        cprefix[c] = run;
        run += __ldcg(counts + c);
    }
}

template <typename B>
__global__ void __launch_bounds__(FL_NT) flat_expand_kernel(
    const B* __restrict__ vals, long long vals_len, const uint8_t* __restrict__ mask, long long n,
    const long long* __restrict__ cprefix, B* __restrict__ out, uint32_t* __restrict__ status) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    B* s_vals = reinterpret_cast<B*>(smem_raw);  // [UNP_CE]
    __shared__ int s_wx[UNP_NE];
    __shared__ int s_agg;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long c = blockIdx.x;
    const long long base = c * UNP_CE;
    const long long nbytes = (n + 7) >> 3;
    const long long start = cprefix[c];
    const int cnt = (int)min((long long)UNP_CE, cprefix[c + 1] - start);
    for (int i = tid; i < cnt; i += FL_NT) {
        const long long p = start + i;
        s_vals[i] = (p >= 0 && p < vals_len) ? vals[p] : B(0);
    }
    if (tid == 0 && start + cnt > vals_len) atomicOr(status, SFFN_STATUS_VALS_SHORT);

    uint32_t bits[UNP_SUBS];
    int lex[UNP_SUBS];
#pragma unroll
    for (int sub = 0; sub < UNP_SUBS; ++sub) {
        const long long f0 = base + 8LL * (sub * FL_NT + tid);
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
        bits[sub] = b;
        const int cc = __popc(b);
        const int inc = warp_incl_scan(cc, lane);
        lex[sub] = inc - cc;
        if (lane == 31) s_wx[sub * FL_NW + warp] = inc;
    }
    __syncthreads();
    if (warp == 0) scan_pairs<UNP_NE>(s_wx, &s_agg, lane);
    __syncthreads();
#pragma unroll
    for (int sub = 0; sub < UNP_SUBS; ++sub) {
        const long long f0 = base + 8LL * (sub * FL_NT + tid);
        if (f0 >= n) continue;
        int r = s_wx[sub * FL_NW + warp] + lex[sub];
        Vec8<B> o;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            B e = B(0);
            if ((bits[sub] >> j) & 1u) {
                e = r < UNP_CE ? s_vals[r] : B(0);
                ++r;
            }
            o.set(j, e);
        }
        if (f0 + 8 <= n) {
            o.store_global_cs(out + f0);
        } else {
            for (int j = 0; j < 8; ++j)
                if (f0 + j < n) out[f0 + j] = o.get(j);
        }
    }
}

inline long long pack_chunks(long long n, int esz) {
    const long long ce = PACK_CHUNK_BYTES / esz;
    return (n + ce - 1) / ce;
}
inline long long unpack_chunks(long long n) { return (n + UNP_CE - 1) / UNP_CE; }

int num_sms() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

template <typename K>
cudaError_t allow_smem(K kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Cooperative launch: every CTA is resident, which the look-back's waits on
// the other CTAs of the same round rely on.
template <typename B>
int launch_pack(const void* dense, long long n, uint8_t* mask, void* vals, long long cap,
                int64_t* nnz_dev, unsigned long long* states, uint32_t* status, long long nch,
                cudaStream_t st) {
    const int smem = PACK_STAGES * PACK_CHUNK_BYTES;
    auto k = flat_pack_kernel<B>;
    SFFN_CUDA_TRY(allow_smem(k, smem));
    int per_sm = 0;
    SFFN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, FL_NT, smem));
    if (per_sm < 1) return SFFN_ERR_CUDA;
    const long long grid = std::min<long long>(nch, (long long)per_sm * num_sms());
    const B* d = static_cast<const B*>(dense);
    B* v = static_cast<B*>(vals);
    long long* nz = reinterpret_cast<long long*>(nnz_dev);
    void* args[] = {(void*)&d, (void*)&n, (void*)&mask, (void*)&v, (void*)&cap, (void*)&nz,
                    (void*)&states, (void*)&status, (void*)&nch};
    SFFN_CUDA_TRY(cudaLaunchCooperativeKernel((const void*)k, dim3((unsigned)grid), dim3(FL_NT), args,
                                              (size_t)smem, st));
    return SFFN_OK;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

// Workspace: [0,16) ticket / done counter, then per-chunk state.
//   pack:   8 bytes per 32 KB chunk (look-back states)
//   unpack: 12 bytes per 16K-element chunk (counts + int64 prefix) + 8
extern "C" size_t sffn_flat_workspace_bytes(int64_t n) {
    if (n < 0) return 0;
    const size_t a = 16 + (size_t)pack_chunks(n, 2) * 8;
    const size_t b = 16 + (size_t)unpack_chunks(n) * 12 + 16;
    return a > b ? a : b;
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
    if (int rc = bind_device_of(dense)) return rc;
    const int esz = esize_of(dtype);
    const long long nch = pack_chunks(n, esz);
    auto* states = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(workspace) + 16);
    SFFN_CUDA_TRY(cudaMemsetAsync(workspace, 0, 16 + (size_t)nch * 8, st));
    if (esz == 4)
        return launch_pack<uint32_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, states,
                                     status_dev, nch, st);
    return launch_pack<uint16_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, states,
                                 status_dev, nch, st);
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
    if (int rc = bind_device_of(out)) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const long long nch = unpack_chunks(n);
    unsigned* done = reinterpret_cast<unsigned*>(workspace);
    auto* cprefix = reinterpret_cast<long long*>(reinterpret_cast<char*>(workspace) + 16);
    int* counts = reinterpret_cast<int*>(cprefix + nch + 1);
    SFFN_CUDA_TRY(cudaMemsetAsync(workspace, 0, 16, st));
    const long long g1 = (nch + CNT_CHUNKS_PER_CTA - 1) / CNT_CHUNKS_PER_CTA;
    flat_count_kernel<<<(unsigned)g1, FL_NT, 0, st>>>(packed_mask, n, nch, counts, cprefix, done);
    SFFN_CHECK_LAUNCH();
    const int esz = esize_of(dtype);
    const int smem = UNP_CE * esz;
    if (esz == 4) {
        auto k = flat_expand_kernel<uint32_t>;
        SFFN_CUDA_TRY(allow_smem(k, smem));
        k<<<(unsigned)nch, FL_NT, smem, st>>>((const uint32_t*)vals, vals_len, packed_mask, n, cprefix,
                                             (uint32_t*)out, status_dev);
    } else {
        auto k = flat_expand_kernel<uint16_t>;
        SFFN_CUDA_TRY(allow_smem(k, smem));
        k<<<(unsigned)nch, FL_NT, smem, st>>>((const uint16_t*)vals, vals_len, packed_mask, n, cprefix,
                                             (uint16_t*)out, status_dev);
    }
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
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

constexpr long long kNoAllocMaxChunks = 4096;  // 4096 chunks of 32 KB of input
static __device__ __align__(256) unsigned char g_noalloc_scratch[16 + kNoAllocMaxChunks * 8];

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
    return kNoAllocMaxChunks * (PACK_CHUNK_BYTES / esize_of(dtype));
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
    const int esz = esize_of(dtype);
    const long long nch = pack_chunks(n, esz);
    auto* states = reinterpret_cast<unsigned long long*>(static_cast<char*>(scratch) + 16);
    // clear what the look-back needs at zero (the previous call left its states)
    SFFN_CUDA_TRY(cudaMemsetAsync(scratch, 0, 16 + (size_t)nch * 8, st));
    if (esz == 4)
        return launch_pack<uint32_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, states,
                                     status_dev, nch, st);
    return launch_pack<uint16_t>(dense, n, packed_mask, vals, vals_capacity, nnz_dev, states,
                                 status_dev, nch, st);
}
