// tcgen05 (5th-generation tensor core) bf16 GEMM for sm_100a with fused
// sparse-FFN epilogues.
//
//   C[M, N] = A[M, K] * B[N, K]^T, fp32 accumulation in tensor memory.
//   A is K-major ([M][lda], K contiguous) or MN-major ([K][lda], M contiguous);
//   B likewise with N.  This covers all six FFN GEMMs without transposes.
//
// Design (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0       TMA producer: 2-D tiled bulk-tensor loads (128-byte swizzle)
//                of A and B k-blocks (64 wide) into a 4-stage shared-memory ring.
//   warp 1       MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16)
//                into one of two TMEM accumulators, commits stage releases and
//                accumulator-ready signals through mbarriers.
//   warp 2       allocates / frees the 2*BN TMEM columns.
//   warps 4..7   epilogue: each thread owns one accumulator row (TMEM lane),
//                reads 32 columns per tcgen05.ld, applies the epilogue and
//                stores with 16-byte vector stores; the second accumulator
//                lets the next tile's MMAs run meanwhile.
// Tiles are visited in groups of 16 row-tiles so that a wave of CTAs shares
// A and B tiles in L2.  An optional per-row-tile list of live k-blocks lets
// the down-projection skip 64-wide K blocks whose activations are all zero.
//
// Epilogues:
//   STORE  bf16 C.
//   UP     (x @ W1^T + b1): pre = bf16(acc [+ b1]); z = relu(pre); writes
//          act = z^2 (ReLU^2) or z (ReLU) densely for the down-projection, the
//          tiled 128x128 bitmask of z > 0 (one 16-byte store of four uint32
//          words per tile row), per-tile counts and z compacted, row-major in
//          the tile, into a per-tile slot -- the arena offset is applied by
//          sffn_tile_gather_slots once all counts are scanned.
//   DGRAD  (dout @ W2): g = bf16(acc); with z gathered from the packed vals,
//          ReLU^2: dpre = bf16((g*2) * z) and act2 = bf16(z*z) (for dW2);
//          ReLU:   dpre = bit ? g : 0 and act2 = z.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <stdio.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace sffn {
namespace {

constexpr int G_BM = 128;
constexpr int G_BK = 64;
constexpr int G_THREADS = 256;
constexpr int G_STAGES = 4;
constexpr int G_GROUP_M = 16;
constexpr int FT = 128;            // format tile (BLOCK_M = BLOCK_N = 128)
constexpr int FT_BYTES = FT * FT / 8;
constexpr int FT_ELEMS = FT * FT;

enum { EPI_STORE = 0, EPI_UP = 1, EPI_DGRAD = 2 };
enum { ACT_RELU = 0, ACT_RELU2 = 1 };

struct GemmArgs {
    int M, N, K;
    int tiles_m, tiles_n;
    uint16_t* out;  // STORE: C; UP: act (z^2 or z); DGRAD: dpre
    long long ldc;
    int vec_out;  // out (and out2) 16-byte aligned with ldc*2 % 16 == 0
    const int* kb_list;  // optional live k-blocks per row tile
    const int* kb_count;
    int kb_stride;
    int act;
    const uint16_t* bias;  // UP: optional [N]
    uint8_t* mask;         // UP: written; DGRAD: read (tiled 128x128, grid_n = ceil(N/128))
    int* tile_counts;      // UP
    uint16_t* slots;       // UP: [num_tiles][128*128]
    uint16_t* out2;        // DGRAD: act2
    const uint16_t* vals;  // DGRAD
    long long vals_len;
    const int* prefix;
    const int* vals_offset;
    uint32_t* status;
};

__device__ __forceinline__ void raster(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
    const int per_group = G_GROUP_M * tiles_n;
    const int group = tile / per_group;
    const int first_m = group * G_GROUP_M;
    const int gsize = min(tiles_m - first_m, G_GROUP_M);
    const int r = tile - group * per_group;
    tm = first_m + r % gsize;
    tn = r / gsize;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
    const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
    return l | (h << 16);
}
__device__ __forceinline__ float bf16_to_f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ uint16_t f_to_bf16(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Store 32 bf16 values (16 packed words) to row[gcol .. gcol+32), bounds-checked.
__device__ __forceinline__ void store_row32(uint16_t* row, int gcol, int N, bool vec, const uint32_t (&w)[16]) {
    if (vec && gcol + 32 <= N) {
        uint4* p = reinterpret_cast<uint4*>(row + gcol);
#pragma unroll
        for (int q = 0; q < 4; ++q) p[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (gcol + j < N) row[gcol + j] = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
    }
}

// 128-thread exclusive scan of one count per epilogue thread (ew = warp 0..3).
__device__ __forceinline__ int epi_scan128(int cnt, int ew, int lane, int* s_part, int* total) {
    const int inc = warp_incl_scan(cnt, lane);
    if (lane == 31) s_part[ew] = inc;
    named_bar_sync(1, 128);
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const int v = s_part[w];
        if (w < ew) before += v;
        all += v;
    }
    *total = all;
    return before + inc - cnt;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(G_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const GemmArgs args) {
    constexpr int A_BYTES = G_BM * G_BK * 2;
    constexpr int B_BYTES = BN * G_BK * 2;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr uint32_t IDESC = idesc_bf16_f32(G_BM, BN, A_MN, B_MN);
    constexpr int TMEM_COLS = 2 * BN;
    constexpr uint32_t MN_LBO = G_BK * 128;  // MN-major: 64-element blocks are K rows x 128 B apart

    extern __shared__ __align__(1024) unsigned char g_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(g_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t full_bar[G_STAGES];
    __shared__ __align__(8) uint64_t empty_bar[G_STAGES];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ int s_scan[2][4];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = args.tiles_m * args.tiles_n;
    const int nkb_full = (args.K + G_BK - 1) / G_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 4);
        }
        s_abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 2) {
        tmem_alloc(&s_tmem, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem;

    if (warp == 0) {
        // ------------------------------------------------------ producer --
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int armed[G_STAGES] = {0};
            for (int tile = blockIdx.x; tile < ntiles && !s_abort; tile += gridDim.x) {
                int tm, tn;
                raster(tile, args.tiles_m, args.tiles_n, tm, tn);
                const int nkb = args.kb_count ? args.kb_count[tm] : nkb_full;
                for (int i = 0; i < nkb; ++i) {
                    const int kb = args.kb_list ? args.kb_list[(size_t)tm * args.kb_stride + i] : i;
                    if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u)) {
                        atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES);
                    ++armed[stage];
                    unsigned char* sa = smem + (size_t)stage * STAGE_BYTES;
                    unsigned char* sb = sa + A_BYTES;
                    if constexpr (!A_MN) {
                        tma_load_2d(sa, &tmA, kb * G_BK, tm * G_BM, &full_bar[stage]);
                    } else {
#pragma unroll
                        for (int j = 0; j < G_BM / 64; ++j)
                            tma_load_2d(sa + j * MN_LBO, &tmA, tm * G_BM + j * 64, kb * G_BK, &full_bar[stage]);
                    }
                    if constexpr (!B_MN) {
                        tma_load_2d(sb, &tmB, kb * G_BK, tn * BN, &full_bar[stage]);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d(sb + j * MN_LBO, &tmB, tn * BN + j * 64, kb * G_BK, &full_bar[stage]);
                    }
                    if (++stage == G_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // No copy may still be landing in shared memory when the CTA exits.
            for (int s = 0; s < G_STAGES; ++s)
                if (armed[s]) (void)mbar_wait_bounded(&full_bar[s], (uint32_t)(armed[s] - 1) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA --
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int tile = blockIdx.x; tile < ntiles && !s_abort; tile += gridDim.x) {
                int tm, tn;
                raster(tile, args.tiles_m, args.tiles_n, tm, tn);
                const int nkb = args.kb_count ? args.kb_count[tm] : nkb_full;
                if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1u)) {
                    atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int i = 0; i < nkb; ++i) {
                    if (!mbar_wait_bounded(&full_bar[stage], phase)) {
                        atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + (size_t)stage * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int k = 0; k < G_BK / 16; ++k) {
                        const uint64_t ad = A_MN ? umma_desc_sw128(sa + k * 2048, MN_LBO, 1024)
                                                 : umma_desc_sw128(sa + k * 32, 16, 1024);
                        const uint64_t bd = B_MN ? umma_desc_sw128(sb + k * 2048, MN_LBO, 1024)
                                                 : umma_desc_sw128(sb + k * 32, 16, 1024);
                        tc_mma_f16(d, ad, bd, IDESC, (i | k) != 0 ? 1u : 0u);
                    }
                    tc_commit(&empty_bar[stage]);
                    if (++stage == G_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                tc_commit(&tfull_bar[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ------------------------------------------------------ epilogue --
        const int ew = warp - 4;
        const int row = ew * 32 + lane;
        const int gn_f = (args.N + FT - 1) / FT;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            int tm, tn;
            raster(tile, args.tiles_m, args.tiles_n, tm, tn);
            const int nkb = args.kb_count ? args.kb_count[tm] : nkb_full;
            // every lane must take the same branch before the warp-collective tcgen05.ld
            const bool ok = __all_sync(FULL, mbar_wait_bounded(&tfull_bar[acc], acc_phase));
            if (!ok || __any_sync(FULL, s_abort != 0)) {
                if (lane == 0) atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
            const int grow = tm * G_BM + row;
            const bool row_ok = grow < args.M;
            uint16_t* orow = args.out + (size_t)grow * args.ldc;
            const bool vec = args.vec_out != 0;

            if constexpr (EPI == EPI_STORE) {
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_wait_ld();
                    uint32_t w[16];
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        w[q] = nkb ? pack_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1])) : 0u;
                    if (row_ok) store_row32(orow, tn * BN + c * 32, args.N, vec, w);
                }
            } else if constexpr (EPI == EPI_UP) {
#pragma unroll 1
                for (int h = 0; h < BN / FT; ++h) {
                    const int tnf = tn * (BN / FT) + h;
                    const int gcol0 = tnf * FT;
                    if (gcol0 >= args.N) break;  // uniform over the 128 epilogue threads
                    const long long tf = (long long)tm * gn_f + tnf;
                    uint32_t words[4];
                    int cnt = 0;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t r[32];
                        tmem_ld32(tbase + h * FT + c * 32, r);
                        tmem_wait_ld();
                        const int gcol = gcol0 + c * 32;
                        uint32_t bits = 0, w[16];
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            float v0 = nkb ? __uint_as_float(r[j]) : 0.f;
                            float v1 = nkb ? __uint_as_float(r[j + 1]) : 0.f;
                            if (args.bias) {
                                if (gcol + j < args.N) v0 += bf16_to_f(args.bias[gcol + j]);
                                if (gcol + j + 1 < args.N) v1 += bf16_to_f(args.bias[gcol + j + 1]);
                            }
                            // pre rounded to bf16, z = relu(pre) (NaN stays NaN, as in torch)
                            const uint16_t p0 = f_to_bf16(v0), p1 = f_to_bf16(v1);
                            const uint16_t z0 = ((int16_t)p0 < 0 && (p0 & 0x7FFF) <= 0x7F80) ? 0 : p0;
                            const uint16_t z1 = ((int16_t)p1 < 0 && (p1 & 0x7FFF) <= 0x7F80) ? 0 : p1;
                            const bool in0 = row_ok && gcol + j < args.N, in1 = row_ok && gcol + j + 1 < args.N;
                            bits |= (uint32_t)(in0 && positive_bits(z0, 0x7F80)) << j;
                            bits |= (uint32_t)(in1 && positive_bits(z1, 0x7F80)) << (j + 1);
                            float a0 = bf16_to_f(z0), a1 = bf16_to_f(z1);
                            if (args.act == ACT_RELU2) {
                                a0 *= a0;
                                a1 *= a1;
                            }
                            w[j >> 1] = pack_bf16x2(a0, a1);
                        }
                        if (row_ok) store_row32(orow, gcol, args.N, vec, w);
                        words[c] = bits;
                        cnt += __popc(bits);
                    }
                    *reinterpret_cast<uint4*>(args.mask + tf * FT_BYTES + row * 16) =
                        make_uint4(words[0], words[1], words[2], words[3]);
                    int total;
                    const int rex = epi_scan128(cnt, ew, lane, s_scan[h], &total);
                    if (row == FT - 1) args.tile_counts[tf] = total;
                    // second pass: z values of this row, compacted into the tile's slot
                    uint16_t* slot = args.slots + tf * FT_ELEMS + rex;
                    int k = 0;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        // tcgen05.ld is warp-collective: skip only if no lane needs it
                        if (!__any_sync(FULL, words[c] != 0)) continue;
                        uint32_t r[32];
                        tmem_ld32(tbase + h * FT + c * 32, r);
                        tmem_wait_ld();
                        const int gcol = gcol0 + c * 32;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if ((words[c] >> j) & 1u) {
                                float v = __uint_as_float(r[j]);
                                if (args.bias) v += bf16_to_f(args.bias[gcol + j]);
                                slot[k++] = f_to_bf16(v);
                            }
                        }
                    }
                }
            } else {  // EPI_DGRAD
                uint16_t* orow2 = args.out2 + (size_t)grow * args.ldc;
                const long long voff = (long long)*args.vals_offset;
#pragma unroll 1
                for (int h = 0; h < BN / FT; ++h) {
                    const int tnf = tn * (BN / FT) + h;
                    const int gcol0 = tnf * FT;
                    if (gcol0 >= args.N) break;  // uniform over the 128 epilogue threads
                    const long long tf = (long long)tm * gn_f + tnf;
                    uint4 mw = make_uint4(0, 0, 0, 0);
                    if (row_ok) mw = *reinterpret_cast<const uint4*>(args.mask + tf * FT_BYTES + row * 16);
                    const uint32_t words[4] = {mw.x, mw.y, mw.z, mw.w};
                    const int cnt = __popc(mw.x) + __popc(mw.y) + __popc(mw.z) + __popc(mw.w);
                    int total;
                    const int rex = epi_scan128(cnt, ew, lane, s_scan[h], &total);
                    long long vbase = voff + args.prefix[tf] + rex;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t r[32];
                        tmem_ld32(tbase + h * FT + c * 32, r);
                        tmem_wait_ld();
                        const uint32_t bits = words[c];
                        uint32_t wd[16], wa[16];
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            float out_v[2], act_v[2];
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int jj = j + e;
                                const float g = bf16_to_f(f_to_bf16(nkb ? __uint_as_float(r[jj]) : 0.f));
                                float z = 0.f;
                                if ((bits >> jj) & 1u) {
                                    const long long p = vbase + __popc(bits & ((1u << jj) - 1u));
                                    z = (p >= 0 && p < args.vals_len) ? bf16_to_f(args.vals[p]) : 0.f;
                                }
                                if (args.act == ACT_RELU2) {
                                    out_v[e] = (g * 2.0f) * z;
                                    act_v[e] = z * z;
                                } else {
                                    out_v[e] = ((bits >> jj) & 1u) ? g : 0.f;
                                    act_v[e] = z;
                                }
                            }
                            wd[j >> 1] = pack_bf16x2(out_v[0], out_v[1]);
                            wa[j >> 1] = pack_bf16x2(act_v[0], act_v[1]);
                        }
                        vbase += __popc(bits);
                        if (row_ok) {
                            store_row32(orow, gcol0 + c * 32, args.N, vec, wd);
                            store_row32(orow2, gcol0 + c * 32, args.N, vec, wa);
                        }
                    }
                }
            }
            // release this accumulator to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host ----
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e == cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            set_error_text("cuTensorMapEncodeTiled entry point not found");
    }
    return fn;
}

// 2-D bf16 tensor map: `inner` contiguous elements per row, `outer` rows,
// row stride `ld` elements, box = box_inner x box_outer, 128-byte swizzle.
bool make_tmap(CUtensorMap* m, const void* base, long long inner, long long outer, long long ld,
               int box_inner, int box_outer) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                          box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char msg[200];
        snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled -> %d (base %p dims %lld x %lld ld %lld box %d x %d)",
                 (int)r, base, inner, outer, ld, box_inner, box_outer);
        set_error_text(msg);
        return false;
    }
    return true;
}

int g_num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

bool device_is_sm100() {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
    return major == 10;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
int launch_gemm(const void* A, long long lda, const void* B, long long ldb, GemmArgs args,
                cudaStream_t st) {
    CUtensorMap ta, tb;
    // K-major operand [rows][K]: inner = K; MN-major operand [K][rows]: inner = rows.
    const bool okA = A_MN ? make_tmap(&ta, A, args.M, args.K, lda, 64, G_BK)
                          : make_tmap(&ta, A, args.K, args.M, lda, G_BK, G_BM);
    const bool okB = B_MN ? make_tmap(&tb, B, args.N, args.K, ldb, 64, G_BK)
                          : make_tmap(&tb, B, args.K, args.N, ldb, G_BK, BN);
    if (!okA || !okB) return SFFN_ERR_CUDA;
    constexpr int smem = G_STAGES * (G_BM * G_BK * 2 + BN * G_BK * 2) + 1024;
    auto k = gemm_kernel<BN, A_MN, B_MN, EPI>;
    SFFN_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int ntiles = args.tiles_m * args.tiles_n;
    const int grid = std::min(ntiles, g_num_sms());
    if (grid <= 0) return SFFN_OK;
    k<<<grid, G_THREADS, smem, st>>>(ta, tb, args);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <int EPI>
int dispatch(bool a_mn, bool b_mn, const void* A, long long lda, const void* B, long long ldb,
             GemmArgs args, cudaStream_t st) {
    constexpr int BN = 256;
    if (!a_mn && !b_mn) return launch_gemm<BN, false, false, EPI>(A, lda, B, ldb, args, st);
    if (!a_mn && b_mn) return launch_gemm<BN, false, true, EPI>(A, lda, B, ldb, args, st);
    if (a_mn && b_mn) return launch_gemm<BN, true, true, EPI>(A, lda, B, ldb, args, st);
    return launch_gemm<BN, true, false, EPI>(A, lda, B, ldb, args, st);
}

// Common argument checks.  TMA needs 16-byte aligned bases and row strides,
// and every inner coordinate we issue is a multiple of 64 elements.
int check_operands(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn,
                   long long M, long long N, long long K) {
    if (M <= 0 || N <= 0 || K <= 0) return SFFN_ERR_ARG;
    if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return SFFN_ERR_ARG;
    if (!A || !B) return SFFN_ERR_ARG;
    if (!aligned16(A) || !aligned16(B) || (lda * 2) % 16 || (ldb * 2) % 16) return SFFN_ERR_ALIGN;
    if (lda < (a_mn ? M : K) || ldb < (b_mn ? N : K)) return SFFN_ERR_ARG;
    if (int rc = bind_device_of(A)) return rc;
    if (!device_is_sm100()) return SFFN_ERR_DEVICE;
    return SFFN_OK;
}

GemmArgs base_args(long long M, long long N, long long K, void* out, long long ldc) {
    GemmArgs a{};
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.tiles_m = (int)((M + G_BM - 1) / G_BM);
    a.tiles_n = (int)((N + 255) / 256);
    a.out = static_cast<uint16_t*>(out);
    a.ldc = ldc;
    a.vec_out = aligned16(out) && (ldc * 2) % 16 == 0;
    return a;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" int sffn_gemm_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                              void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                              const int32_t* kb_list, const int32_t* kb_count, int kb_stride,
                              uint32_t* status_dev, void* stream) {
    int rc = check_operands(A, lda, a_mn, B, ldb, b_mn, M, N, K);
    if (rc) return rc;
    if (!C || ldc < N || !status_dev) return SFFN_ERR_ARG;
    if ((kb_list == nullptr) != (kb_count == nullptr)) return SFFN_ERR_ARG;
    GemmArgs a = base_args(M, N, K, C, ldc);
    a.kb_list = kb_list;
    a.kb_count = kb_count;
    a.kb_stride = kb_stride;
    a.status = status_dev;
    return dispatch<EPI_STORE>(a_mn != 0, b_mn != 0, A, lda, B, ldb, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sffn_ffn_up(const void* x, int64_t ldx, const void* w1, int64_t ldw1, const void* b1,
                           int64_t T, int64_t D, int64_t F, int act, void* act_out, int64_t ld_act,
                           uint8_t* bitmask, int32_t* tile_counts, void* slots, uint32_t* status_dev,
                           void* stream) {
    int rc = check_operands(x, ldx, false, w1, ldw1, false, T, F, D);
    if (rc) return rc;
    if (act != ACT_RELU && act != ACT_RELU2) return SFFN_ERR_ARG;
    if (!act_out || ld_act < F || !bitmask || !tile_counts || !slots || !status_dev) return SFFN_ERR_ARG;
    if (!aligned16(bitmask)) return SFFN_ERR_ALIGN;
    if (T * F > 0x7FFFFFFFll) return SFFN_ERR_ARG;
    GemmArgs a = base_args(T, F, D, act_out, ld_act);
    a.act = act;
    a.bias = static_cast<const uint16_t*>(b1);
    a.mask = bitmask;
    a.tile_counts = tile_counts;
    a.slots = static_cast<uint16_t*>(slots);
    a.status = status_dev;
    return dispatch<EPI_UP>(false, false, x, ldx, w1, ldw1, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sffn_ffn_dgrad(const void* dout, int64_t ld_dout, const void* w2, int64_t ldw2,
                              int64_t T, int64_t D, int64_t F, int act, const void* vals,
                              int64_t vals_len, const uint8_t* bitmask, const int32_t* prefix,
                              const int32_t* vals_offset_dev, void* dpre_out, void* act_out,
                              int64_t ld_out, uint32_t* status_dev, void* stream) {
    // dA[T, F] = dout[T, D] @ W2[D, F]: B = W2 is [K=D][N=F], N contiguous (MN-major).
    int rc = check_operands(dout, ld_dout, false, w2, ldw2, true, T, F, D);
    if (rc) return rc;
    if (act != ACT_RELU && act != ACT_RELU2) return SFFN_ERR_ARG;
    if (!vals || !bitmask || !prefix || !vals_offset_dev || !dpre_out || !act_out || ld_out < F ||
        !status_dev)
        return SFFN_ERR_ARG;
    if (!aligned16(bitmask)) return SFFN_ERR_ALIGN;
    if (!aligned16(dpre_out) != !aligned16(act_out)) return SFFN_ERR_ALIGN;
    GemmArgs a = base_args(T, F, D, dpre_out, ld_out);
    a.act = act;
    a.out2 = static_cast<uint16_t*>(act_out);
    a.mask = const_cast<uint8_t*>(bitmask);
    a.vals = static_cast<const uint16_t*>(vals);
    a.vals_len = vals_len;
    a.prefix = prefix;
    a.vals_offset = vals_offset_dev;
    a.status = status_dev;
    return dispatch<EPI_DGRAD>(false, true, dout, ld_dout, w2, ldw2, a, reinterpret_cast<cudaStream_t>(stream));
}
