// 2:4 structured form for the sparse tensor-core GEMMs (sm_100a): compression
// and the overflow correction.
//
// The FFN activations (and their gradients) are ~90% zeros in no fixed
// pattern.  tcgen05.mma.sp multiplies a 2:4 structured A (at most two
// non-zeros in every group of four consecutive K elements) at twice the dense
// rate.  A sparse matrix is split into
//   * its 2:4 part: per group, the first two non-zeros (by position) --
//     compressed values [M, K/2] plus 4-bit index pairs ("metadata"), laid out
//     per 128-row tile and 128-wide K block exactly as one tcgen05.st of 128
//     lanes x 4 columns puts them into tensor memory: word j of lane
//     dp = m0 + 8*k1 + 16*m2 holds the index nibbles of K-half k1 of the j-th
//     32-wide K step, for row 16*m2 + m0 in bits 0-15 and row 16*m2 + m0 + 8
//     in bits 16-31 (group g of the half at bits 4g; idx0 in bits 0-1, idx1 in
//     bits 2-3, idx0 < idx1; a group with fewer non-zeros keeps zero slots);
//   * its overflow: the 3rd and 4th non-zero of a group (0.4% of the groups
//     at 90% zeros), kept per row as (column, value) and added afterwards by
//     sffn_sp24_overflow_add on the CUDA cores.
// The reference has no counterpart: its products are dense cuBLAS matmuls
// (old/lib_sparse/sparse.py:75,95-100,118,136-139); the path is checked end to
// end against dense products.
#include "common.cuh"
#include "sp24.cuh"

namespace sffn {
namespace {

constexpr int SP_TILE = 128;  // rows per tile, K per block

// One CTA per (128-row tile, 128-wide K block); thread = row of the tile.
// TRANS: the logical A is X^T for X = src [K, M] (row stride ld), i.e. the
// compression runs along X's rows (the token dimension of an activation).
template <bool TRANS>
__global__ void __launch_bounds__(SP_TILE) sp24_compress_kernel(
    const uint16_t* __restrict__ src, long long ld, int M, int K, uint16_t* __restrict__ vals,
    uint32_t* __restrict__ meta, uint16_t* __restrict__ ovf_cols, uint16_t* __restrict__ ovf_vals,
    int* __restrict__ ovf_count) {
    __shared__ __align__(16) uint16_t s_tile[SP_TILE * SP_TILE];  // 32 KB
    __shared__ uint32_t s_rowmeta[SP_TILE][4];
    const int tm = blockIdx.x, kb = blockIdx.y, t = threadIdx.x;
    // Coalesced 16-byte loads of the 128 x 128 tile.  Untransposed tiles are
    // read back one row per thread, so their 16-byte chunks are swizzled by
    // row; transposed tiles are read one column per thread (conflict-free).
    for (int i = t; i < SP_TILE * 16; i += SP_TILE) {
        const int r = i >> 4, c = i & 15;
        const long long grow = TRANS ? (long long)kb * SP_TILE + r : (long long)tm * SP_TILE + r;
        const long long gcol = TRANS ? (long long)tm * SP_TILE + c * 8 : (long long)kb * SP_TILE + c * 8;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + grow * ld + gcol));
        const int pc = TRANS ? c : (c ^ (r & 15));
        *reinterpret_cast<uint4*>(&s_tile[r * SP_TILE + pc * 8]) = v;
    }
    __syncthreads();
    const int m = t;
    const long long row = (long long)tm * SP_TILE + m;
    uint32_t rowmeta[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // 32-wide K steps of the block
        uint32_t w[16];
        if (TRANS) {
#pragma unroll
            for (int q = 0; q < 16; ++q)
                w[q] = (uint32_t)s_tile[(32 * j + 2 * q) * SP_TILE + m] |
                       ((uint32_t)s_tile[(32 * j + 2 * q + 1) * SP_TILE + m] << 16);
        } else {
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const int c = 4 * j + h;  // 16-byte chunk of the row
                const uint4 v = *reinterpret_cast<const uint4*>(&s_tile[m * SP_TILE + ((c ^ (m & 15)) << 3)]);
                w[4 * h] = v.x;
                w[4 * h + 1] = v.y;
                w[4 * h + 2] = v.z;
                w[4 * h + 3] = v.w;
            }
        }
        uint32_t cw[8], nib, ov;
        sp24_chunk(w, cw, nib, ov);
        rowmeta[j] = nib;
        uint4* vdst = reinterpret_cast<uint4*>(vals + row * (K / 2) + (long long)kb * 64 + 16 * j);
        vdst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
        vdst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
        if (ov) {
            int pos = atomicAdd(&ovf_count[row], __popc(ov));
            const long long base = row * (long long)(K / 2);
            sp24_for_overflow(w, ov, [&](int e, uint32_t v) {
                ovf_cols[base + pos] = (uint16_t)(kb * SP_TILE + 32 * j + e);
                ovf_vals[base + pos] = (uint16_t)v;
                ++pos;
            });
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) s_rowmeta[m][j] = rowmeta[j];
    __syncthreads();
    // tensor-memory lane order: lane dp = m0 + 8*k1 + 16*m2
    {
        const int dp = t, m0 = dp & 7, k1 = (dp >> 3) & 1, m2 = dp >> 4;
        const int ra = 16 * m2 + m0, rb = ra + 8;
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = ((s_rowmeta[ra][j] >> (16 * k1)) & 0xFFFFu) | (((s_rowmeta[rb][j] >> (16 * k1)) & 0xFFFFu) << 16);
        reinterpret_cast<uint4*>(meta)[((long long)tm * (K / SP_TILE) + kb) * SP_TILE + dp] =
            make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// C[r, :] += sum over the overflow entries (k, v) of row r of v * Bt[k, :],
// in fp32, then rounded once more to bf16.  One CTA of 256 threads per row;
// thread t owns the 16 columns 16t .. 16t+15 of each 4096-column block, and
// four entries' loads are in flight at a time.
constexpr int OV_NT = 256;
constexpr int OV_COLS = OV_NT * 16;  // columns per block
__global__ void __launch_bounds__(OV_NT) sp24_overflow_kernel(
    const uint16_t* __restrict__ ovf_cols, const uint16_t* __restrict__ ovf_vals,
    const int* __restrict__ ovf_count, long long ovf_ld, const uint16_t* __restrict__ bt, long long ldb,
    uint16_t* __restrict__ C, long long ldc, int N) {
    const long long r = blockIdx.x;
    const int n = ovf_count[r];
    if (n == 0) return;
    const int t = threadIdx.x;
    const uint16_t* oc = ovf_cols + r * ovf_ld;
    const uint16_t* ov = ovf_vals + r * ovf_ld;
    uint16_t* crow = C + r * ldc;
    for (int c0 = 0; c0 < N; c0 += OV_COLS) {
        const int col = c0 + 16 * t;
        if (col >= N) break;  // N % 16 == 0: whole 16-column groups
        float acc[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[e] = 0.f;
        for (int e0 = 0; e0 < n; e0 += 4) {
            uint4 q[4][2];
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = min(e0 + u, n - 1);
                v[u] = e0 + u < n ? __uint_as_float((uint32_t)__ldg(ov + e) << 16) : 0.f;
                const uint4* brow = reinterpret_cast<const uint4*>(bt + (long long)__ldg(oc + e) * ldb + col);
                q[u][0] = __ldg(brow);
                q[u][1] = __ldg(brow + 1);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t w[8] = {q[u][0].x, q[u][0].y, q[u][0].z, q[u][0].w,
                                       q[u][1].x, q[u][1].y, q[u][1].z, q[u][1].w};
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    acc[2 * h] += v[u] * __uint_as_float(w[h] << 16);
                    acc[2 * h + 1] += v[u] * __uint_as_float(w[h] & 0xFFFF0000u);
                }
            }
        }
        uint4* p = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
        for (int hv = 0; hv < 2; ++hv) {
            const uint4 qc = p[hv];
            const uint32_t w[4] = {qc.x, qc.y, qc.z, qc.w};
            uint32_t o[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float lo = __uint_as_float(w[h] << 16) + acc[8 * hv + 2 * h];
                const float hi = __uint_as_float(w[h] & 0xFFFF0000u) + acc[8 * hv + 2 * h + 1];
                o[h] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
                       ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
            }
            p[hv] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" int sffn_sp24_compress(const void* src, int64_t ld, int trans, int64_t M, int64_t K, void* vals,
                                  uint32_t* meta, void* ovf_cols, void* ovf_vals, int32_t* ovf_count,
                                  void* stream) {
    if (M <= 0 || K <= 0 || M % SP_TILE || K % SP_TILE || K > 65536 || M > 0x7FFFFFFF) return SFFN_ERR_UNSUPPORTED;
    if (!src || !vals || !meta || !ovf_cols || !ovf_vals || !ovf_count) return SFFN_ERR_ARG;
    if (ld < (trans ? M : K) || (ld * 2) % 16 || !aligned16(src) || !aligned16(vals) || !aligned16(meta))
        return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, src);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    SFFN_CUDA_TRY(cudaMemsetAsync(ovf_count, 0, (size_t)M * sizeof(int32_t), st));
    const dim3 grid((unsigned)(M / SP_TILE), (unsigned)(K / SP_TILE));
    const uint16_t* s = static_cast<const uint16_t*>(src);
    uint16_t* v = static_cast<uint16_t*>(vals);
    uint16_t* oc = static_cast<uint16_t*>(ovf_cols);
    uint16_t* ov = static_cast<uint16_t*>(ovf_vals);
    if (trans)
        sp24_compress_kernel<true><<<grid, SP_TILE, 0, st>>>(s, ld, (int)M, (int)K, v, meta, oc, ov, ovf_count);
    else
        sp24_compress_kernel<false><<<grid, SP_TILE, 0, st>>>(s, ld, (int)M, (int)K, v, meta, oc, ov, ovf_count);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

extern "C" int sffn_sp24_overflow_add(const void* ovf_cols, const void* ovf_vals, const int32_t* ovf_count,
                                      int64_t M, int64_t K, const void* bt, int64_t ldb, int64_t N, void* C,
                                      int64_t ldc, void* stream) {
    if (M <= 0 || N <= 0 || K <= 0 || N % 16) return SFFN_ERR_UNSUPPORTED;
    if (!ovf_cols || !ovf_vals || !ovf_count || !bt || !C) return SFFN_ERR_ARG;
    if (!aligned16(bt) || !aligned16(C) || (ldb * 2) % 16 || (ldc * 2) % 16 || ldb < N || ldc < N)
        return SFFN_ERR_ALIGN;
    SFFN_BIND(dev_scope, C);
    sp24_overflow_kernel<<<(unsigned)M, OV_NT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(ovf_cols), static_cast<const uint16_t*>(ovf_vals), ovf_count, K / 2,
        static_cast<const uint16_t*>(bt), ldb, static_cast<uint16_t*>(C), ldc, (int)N);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}
