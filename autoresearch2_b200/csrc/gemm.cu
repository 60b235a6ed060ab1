// tcgen05 (5th-generation tensor core) bf16 GEMM for sm_100a with fused
// sparse-FFN epilogues.
//
//   C[M, N] = A[M, K] * B[N, K]^T, fp32 accumulation in tensor memory.
//   A is K-major ([M][lda], K contiguous) or MN-major ([K][lda], M contiguous);
//   B likewise with N.  This covers all six FFN GEMMs without transposes.
//
// Design (one CTA per SM, CTA pairs (clusters of 2) persistent over output
// tiles of 256 x BN; each CTA of the pair owns 128 rows):
//   warps 0,2,3,12  TMA producers (both CTAs): 2-D tiled bulk-tensor loads
//                (128-byte swizzle) of this CTA's half of the A (warps 0, 2)
//                and B (warps 3, 12) k-blocks (64 wide; even / odd k-blocks)
//                into a 6-stage shared-memory ring; the bytes complete on the
//                leader CTA's barrier.
//   warp 1       MMA issuer (leader CTA only): one thread issues
//                tcgen05.mma.cta_group::2 (M=256, N=BN, K=16), which reads the A
//                and B halves from both CTAs' shared memory and accumulates rows
//                0-127 in the leader's TMEM and 128-255 in the peer's, into one
//                of two accumulators; commits are multicast to both CTAs.
//   warp 2       also allocates / frees the 2*BN TMEM columns (pair allocation).
//   warps 4..11  epilogue, two warpgroups each owning half of the tile's
//                columns: each thread owns one accumulator row (TMEM lane),
//                reads 32 columns per tcgen05.ld, applies the epilogue and
//                stages the warp's 32 x 32 block in a 2 KB swizzled shared
//                buffer that one bulk-tensor store writes out (whole 64-byte
//                row segments instead of 32 scattered rows per instruction);
//                the second accumulator lets the next tile's MMAs run meanwhile.
// Splitting B between the two CTAs halves the shared-memory bytes each SM
// needs per k-block (32 KB instead of 48 KB), which buys a 6-stage ring.
// Tiles are visited in groups of 16 row-tiles so that a wave of CTAs shares
// A and B tiles in L2.  An optional per-256-row-tile list of live k-blocks
// lets the down-projection skip 64-wide K blocks whose activations are all zero.
//
// Epilogues:
//   STORE  bf16 C.
//   UP     (x @ W1^T + b1): pre = bf16(acc [+ b1]); z = relu(pre); writes
//          act = z^2 (ReLU^2) or z (ReLU) densely for the down-projection, the
//          tiled 128x128 bitmask of z > 0 (one 16-byte store of four uint32
//          words per tile row), per-warp partial tile counts, and each row's
//          z values compacted into that row's own 128-element segment of the
//          tile's slot -- no cross-thread scan in the epilogue; the tile scan
//          and the in-tile row scan happen in sffn_tile_scan_counts /
//          sffn_tile_gather_slots.
//   DGRAD  (dout @ W2): g = bf16(acc); z gathered from the packed vals at
//          the row's precomputed offset (sffn_tile_row_offsets);
//          ReLU^2: dpre = bf16((g*2) * z) and act2 = bf16(z*z) (for dW2);
//          ReLU:   dpre = bit ? g : 0 and act2 = z.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <stdio.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "sp24.cuh"

namespace sffn {
namespace {

constexpr int G_BM = 128;
constexpr int G_BK = 64;
constexpr int G_THREADS = 416;  // 4 control warps, 2 epilogue warpgroups (warps 4-11), 1 more producer
constexpr int G_STAGES = 6;  // even: two issuers per operand take alternate k-blocks
constexpr int G_GROUP_M = 8;  // pair-tile rows per raster group (16 row tiles of 128)
constexpr int G_CTAS = 2;     // CTA pairs (cta_group::2)
constexpr int FT = 128;            // format tile (BLOCK_M = BLOCK_N = 128)
constexpr int FT_BYTES = FT * FT / 8;
constexpr int FT_ELEMS = FT * FT;
enum { EPI_STORE = 0, EPI_UP = 1, EPI_DGRAD = 2 };
// The fused epilogues keep more in shared memory: the activation gradient
// prefetches each tile's packed z values (one buffer per warpgroup: a whole
// 128x128 format tile's values plus 16-byte alignment slack), the
// up-projection gathers each row's z values (256 bytes per row, 8 KB per
// warp).  Their rings have four stages to make room (the main loop runs as
// fast with four as with six).
constexpr int G_ZBUF = FT_ELEMS * 2 + 64;
template <int EPI>
constexpr int gemm_stages() { return EPI == EPI_STORE ? G_STAGES : 4; }
template <int EPI>
constexpr int gemm_smem_bytes(int BN) {
    return gemm_stages<EPI>() * (G_BM * G_BK * 2 + (BN / G_CTAS) * G_BK * 2) + 8 * 2048 +
           (EPI == EPI_DGRAD ? 2 * G_ZBUF : EPI == EPI_UP ? 8 * 32 * 256 : 0) + 1024;
}

enum { ACT_RELU = 0, ACT_RELU2 = 1 };

// One matrix written in the 2:4 form of sp24.cu by a fused epilogue.
struct Sp24Out {
    uint16_t* vals;   // [rows][vals_ld] kept values
    uint32_t* meta;   // [rows/128][nkb][128 lanes][4]
    uint16_t* ocols;  // [rows][vals_ld] overflow columns
    uint16_t* ovals;  //                 and values
    int* ocount;      // [rows]
    long long vals_ld;  // K/2 of the matrix
    int nkb;            // K/128
};

struct GemmArgs {
    int M, N, K;
    int tiles_m, tiles_n;
    uint16_t* out;  // STORE: C; UP: act (z^2 or z); DGRAD: dpre
    long long ldc;
    int vec_out;  // out (and out2) 16-byte aligned with ldc*2 % 16 == 0: bulk-tensor stores
    const int* kb_list;  // optional live k-blocks per row tile
    const int* kb_count;
    int kb_stride;
    int act;
    const uint16_t* bias;  // UP: optional [N]
    uint8_t* mask;         // UP: written; DGRAD: read (tiled 128x128, grid_n = ceil(N/128))
    int* tile_counts;      // UP: [num_tiles][4] per-warp partial counts
    uint16_t* slots;       // UP: [num_tiles][16384]: z values per row at r*128, or tile-packed
    int* slot_rows;        // UP: tile-packed slots; [num_tiles][128] row offsets in the tile
    uint16_t* out2;        // DGRAD: act2
    const uint16_t* vals;  // DGRAD
    long long vals_len;
    const int* row_offsets;  // DGRAD: [num_tiles][128] prefix[t] + in-tile row prefix
    const int* vals_offset;
    float* colsum;  // DGRAD: optional fp32 [N] += column sums of dpre
    int c_trans;    // STORE: write C^T ([N][ldc]) instead of C
    float* out_f32; // STORE: C in float32 ([M][ldc]) instead of bf16
    int acc_f32;    // with out_f32: C += the product (round to nearest, on the CUDA cores)
    int relu_out;   // STORE: C = max(C, 0) as stored (bf16 or float32)
    int kb0;        // first K block of the product (K blocks kb0 .. kb0 + ceil(K/64) - 1)
    int sp_on;      // UP: a, DGRAD: dpre, dpre^T and a^T in 2:4 form instead of dense
    Sp24Out sp[3];  // UP: [0] a; DGRAD: [0] dpre, [1] dpre^T, [2] a^T
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
__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

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

// Epilogue output through shared memory: the warp's 32 rows x 32 columns (lane
// = row, 16 packed words) go to its 2 KB staging buffer in the layout of a
// tensor map with 64-byte swizzle (16-byte chunk ch of row r at
// r*64 + 16*(ch ^ ((r >> 1) & 3)), conflict-free for a quarter warp), then
// one bulk-tensor store writes whole 64-byte row segments at (col, row0);
// rows and columns past the tensor's extent are clipped by the store.
__device__ __forceinline__ void stage_store32(const CUtensorMap* tmap, unsigned char* sbuf, int lane,
                                              const uint32_t (&w)[16], int col, int row0) {
    if (lane == 0) bulk_wait_group_read0();  // the previous store has read the buffer
    __syncwarp();
    const uint32_t rb = smem_u32(sbuf) + (uint32_t)lane * 64u;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rb + 16u * (uint32_t)(ch ^ sw)),
                     "r"(w[4 * ch]), "r"(w[4 * ch + 1]), "r"(w[4 * ch + 2]), "r"(w[4 * ch + 3])
                     : "memory");
    fence_proxy_async_smem();  // these generic-proxy writes, before the async-proxy read
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(tmap, sbuf, col, row0);
        bulk_commit_group();
    }
}

// The warp's 32 x 32 block (lane = row) into its staging buffer, same layout
// as stage_store32, without a store to global memory.
__device__ __forceinline__ void stage_words(unsigned char* sbuf, int lane, const uint32_t (&w)[16]) {
    const uint32_t rb = smem_u32(sbuf) + (uint32_t)lane * 64u;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rb + 16u * (uint32_t)(ch ^ sw)),
                     "r"(w[4 * ch]), "r"(w[4 * ch + 1]), "r"(w[4 * ch + 2]), "r"(w[4 * ch + 3])
                     : "memory");
}
// Column `lane` of the staged block (rows 0..31, two per word) and its sum.
__device__ __forceinline__ void staged_column(const unsigned char* sbuf, int lane, uint32_t (&wt)[16], float& sum) {
    const uint32_t sb0 = smem_u32(sbuf);
    const int ch = lane >> 3, sub = (lane & 7) * 2;
    sum = 0.f;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        uint16_t h0, h1;
        const int r0 = 2 * q, r1 = 2 * q + 1;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h0) : "r"(sb0 + (uint32_t)(r0 * 64 + 16 * (ch ^ ((r0 >> 1) & 3)) + sub)));
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h1) : "r"(sb0 + (uint32_t)(r1 * 64 + 16 * (ch ^ ((r1 >> 1) & 3)) + sub)));
        wt[q] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        sum += bf16_to_f(h0) + bf16_to_f(h1);
    }
}
// Element e of row r of a block staged by stage_words.
__device__ __forceinline__ uint32_t staged_elem(const unsigned char* sbuf, int r, int e) {
    uint16_t h;
    asm volatile("ld.shared.u16 %0, [%1];"
                 : "=h"(h)
                 : "r"(smem_u32(sbuf) + (uint32_t)(r * 64 + 16 * ((e >> 3) ^ ((r >> 1) & 3)) + 2 * (e & 7))));
    return h;
}
// 2:4 form of row `row` (elements k0 .. k0+31 in w) of a matrix: kept values
// and overflow to global memory; returns the tensor-memory-order metadata
// word of this lane (warp-collective: every lane calls it).  The overflow
// values, rare, are read back by val(e) from the staged block rather than
// from w, which a rolled loop could only index through local memory.
template <typename ValFn>
__device__ __forceinline__ uint32_t sp24_emit(const Sp24Out& o, const uint32_t (&w)[16], long long row, int k0,
                                              int lane, ValFn&& val) {
    uint32_t cw[8], nib, ov;
    sp24_chunk(w, cw, nib, ov);
    uint4* dst = reinterpret_cast<uint4*>(o.vals + row * o.vals_ld + k0 / 2);
    dst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
    dst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
    if (ov) {
        int pos = atomicAdd(o.ocount + row, __popc(ov));
        const long long base = row * o.vals_ld;
#pragma unroll 1
        while (ov) {
            const int e = __ffs(ov) - 1;
            ov &= ov - 1u;
            o.ocols[base + pos] = (uint16_t)(k0 + e);
            o.ovals[base + pos] = (uint16_t)val(e);
            ++pos;
        }
    }
    return sp24_lane_word(nib, lane);
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool TF32 = false>
__global__ void __cluster_dims__(G_CTAS, 1, 1) __launch_bounds__(G_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
                const GemmArgs args) {
    constexpr int BN_CTA = BN / G_CTAS;  // B rows (N) loaded by each CTA
    constexpr int A_BYTES = G_BM * G_BK * 2;
    constexpr int B_BYTES = BN_CTA * G_BK * 2;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // TF32: float32 operands, the same 128-byte k-block rows holding 32 K
    // elements instead of 64 (K-major operands, plain or float32 C only)
    constexpr uint32_t IDESC = TF32 ? idesc_tf32_f32(G_BM * G_CTAS, BN, A_MN, B_MN)
                                    : idesc_bf16_f32(G_BM * G_CTAS, BN, A_MN, B_MN);
    constexpr int KB_ELEMS = TF32 ? G_BK / 2 : G_BK;  // K elements per k-block
    static_assert(!TF32 || (!A_MN && !B_MN && EPI == EPI_STORE), "tf32: K-major operands, plain epilogue");
    constexpr int TMEM_COLS = 2 * BN;
    constexpr uint32_t MN_LBO = G_BK * 128;  // MN-major: 64-element blocks are K rows x 128 B apart
    static_assert(BN_CTA % 64 == 0, "each CTA loads whole 64-row B blocks");
    // the even / odd k-block issuers each own every other use of a stage only
    // if the stage count is even (their final drain counts their own phases)
    constexpr int NST = gemm_stages<EPI>();
    static_assert(NST % 2 == 0, "an even number of stages");

    extern __shared__ __align__(1024) unsigned char g_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(g_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t full_bar[NST];
    __shared__ __align__(8) uint64_t empty_bar[NST];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ float s_bias[2][2][FT];  // [warpgroup][tile parity][column]
    __shared__ __align__(8) uint64_t z_bar[2];  // DGRAD: the z buffer of each warpgroup has landed
    __shared__ long long s_zb0[2];              // DGRAD: arena index of the buffer's first value, or -1

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Pair tiles: 256 rows (two 128-row tiles, one per CTA) x BN columns.
    const int tiles_mp = (args.tiles_m + 1) / 2;
    const int ntiles = tiles_mp * args.tiles_n;
    const int nkb_full = (args.K + KB_ELEMS - 1) / KB_ELEMS;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int first_tile = (int)cluster_id_x();
    const int tile_stride = (int)cluster_count_x();

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full_bar[s], 1);   // leader: its own arrive.expect_tx for both CTAs' bytes
            mbar_init(&empty_bar[s], 1);  // one multicast commit per use
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 8 * G_CTAS);  // every epilogue warp of both CTAs
            mbar_init(&z_bar[a], 1);
        }
        s_abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 2) {
        tmem_alloc_pair(&s_tmem, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    // barriers and TMEM of both CTAs are set up before any cross-CTA traffic
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem;

    if (warp == 0 || warp == 2 || warp == 3 || warp == 12) {
        // ----------------------------------------------------- producers --
        // Four issuing threads, one per (operand, k-block parity): warps 0 / 2
        // load A of the even / odd k-blocks and arm those stages (both
        // operands' bytes of both CTAs, on the leader's barrier), warps 3 / 12
        // load B of the even / odd k-blocks.  One thread's bulk-tensor copies
        // complete one after another (about one per L2 round trip), so the
        // four issuers keep four copies in flight per SM.  (B's bytes may land
        // before the arming; the barrier's transaction count may go negative
        // meanwhile, and the phase cannot complete before the arrival.)
        const bool loads_a = warp == 0 || warp == 2;
        const int par = (warp == 0 || warp == 3) ? 0 : 1;
        if (lane == 0) {
            int armed[NST] = {0};
            long long kc = 0;  // k-blocks of this CTA so far (all tiles)
            for (int tile = first_tile; tile < ntiles && !s_abort; tile += tile_stride) {
                int pm, tn;
                raster(tile, tiles_mp, args.tiles_n, pm, tn);
                const int nkb = args.kb_count ? args.kb_count[pm] : nkb_full;
                const int arow = pm * G_BM * G_CTAS + (int)rank * G_BM;   // this CTA's A rows
                const int brow = tn * BN + (int)rank * BN_CTA;            // this CTA's B rows (N)
                bool stop = false;
                for (int i = 0; i < nkb; ++i, ++kc) {
                    if ((int)(kc & 1) != par) continue;
                    const int stage = (int)(kc % NST);
                    const uint32_t phase = (uint32_t)((kc / NST) & 1);
                    // a full list (every block live) is not read: no dependent load per k-block
                    const int kb = args.kb_list && nkb != nkb_full ? args.kb_list[(size_t)pm * args.kb_stride + i]
                                                                   : args.kb0 + i;
                    // the stage is free once the leader's MMAs reading it are done
                    if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u)) {
                        atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        stop = true;
                        break;
                    }
                    unsigned char* sa = smem + (size_t)stage * STAGE_BYTES;
                    unsigned char* sb = sa + A_BYTES;
                    if (loads_a) {
                        if (leader) {
                            mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES * G_CTAS);
                            ++armed[stage];
                        }
                        if constexpr (!A_MN) {
                            tma_load_2d_pair(sa, &tmA, kb * KB_ELEMS, arow, &full_bar[stage]);
                        } else {
#pragma unroll
                            for (int j = 0; j < G_BM / 64; ++j)
                                tma_load_2d_pair(sa + j * MN_LBO, &tmA, arow + j * 64, kb * G_BK, &full_bar[stage]);
                        }
                    } else {
                        if constexpr (!B_MN) {
                            tma_load_2d_pair(sb, &tmB, kb * KB_ELEMS, brow, &full_bar[stage]);
                        } else {
#pragma unroll
                            for (int j = 0; j < BN_CTA / 64; ++j)
                                tma_load_2d_pair(sb + j * MN_LBO, &tmB, brow + j * 64, kb * G_BK, &full_bar[stage]);
                        }
                    }
                }
                if (stop) break;
            }
            // The leader's full barriers count both CTAs' bytes of both
            // operands: once the last phases armed by this thread complete, no
            // copy of those stages is still landing in either CTA.
            if (leader && loads_a)
                for (int s = 0; s < NST; ++s)
                    if (armed[s]) (void)mbar_wait_bounded(&full_bar[s], (uint32_t)(armed[s] - 1) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA --
        if (lane == 0 && leader) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int tile = first_tile; tile < ntiles && !s_abort; tile += tile_stride) {
                int pm, tn;
                raster(tile, tiles_mp, args.tiles_n, pm, tn);
                const int nkb = args.kb_count ? args.kb_count[pm] : nkb_full;
                if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1u)) {
                    atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                // The operands reach shared memory by TMA and are read by the MMAs
                // through the async proxy, ordered by the full barrier alone: no
                // tcgen05 fence per k-block.  The next k-block's barrier is
                // tested while the current MMAs run, so its latency is hidden.
                bool ready = nkb > 0 && mbar_try_wait(&full_bar[stage], phase);
                for (int i = 0; i < nkb; ++i) {
                    if (!ready && !mbar_wait_bounded(&full_bar[stage], phase)) {
                        atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        break;
                    }
                    const uint32_t sa = smem_u32(smem + (size_t)stage * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int k = 0; k < G_BK / 16; ++k) {
                        const uint64_t ad = A_MN ? umma_desc_sw128(sa + k * 2048, MN_LBO, 1024)
                                                 : umma_desc_sw128(sa + k * 32, 16, 1024);
                        const uint64_t bd = B_MN ? umma_desc_sw128(sb + k * 2048, MN_LBO, 1024)
                                                 : umma_desc_sw128(sb + k * 32, 16, 1024);
                        if constexpr (TF32)
                            tc_mma_tf32_pair(d, ad, bd, IDESC, (i | k) != 0 ? 1u : 0u);
                        else
                            tc_mma_f16_pair(d, ad, bd, IDESC, (i | k) != 0 ? 1u : 0u);
                    }
                    tc_commit_pair_multicast(&empty_bar[stage], 0x3);
                    if (++stage == NST) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    ready = i + 1 < nkb && mbar_try_wait(&full_bar[stage], phase);
                }
                tc_commit_pair_multicast(&tfull_bar[acc], 0x3);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------ epilogue --
        // Two warpgroups: warps 4-7 own accumulator columns [0, BN/2), warps
        // 8-11 own [BN/2, BN).  Warp w reads TMEM lanes 32*(w%4) .. +31 (the
        // lane quarter tcgen05.ld gives it), so thread = accumulator row.
        constexpr int HALF = BN / 2;
        static_assert(EPI == EPI_STORE || HALF == FT, "fused epilogues map one warpgroup to one format tile");
        const int wg = (warp - 4) >> 2;
        const int ew = warp & 3;
        const int row = ew * 32 + lane;
        const int gn_f = (args.N + FT - 1) / FT;
        const int bar_id = 1 + wg;
        const uint16_t* __restrict__ vals = args.vals;
        const uint16_t* __restrict__ bias = args.bias;
        const uint32_t tempty_leader[2] = {leader_smem_addr(&tempty_bar[0]), leader_smem_addr(&tempty_bar[1])};
        int acc = 0;
        uint32_t acc_phase = 0;
        int it = 0;
        uint32_t z_phase = 0;
        for (int tile = first_tile; tile < ntiles; tile += tile_stride, ++it) {
            int pm, tn;
            raster(tile, tiles_mp, args.tiles_n, pm, tn);
            const int tm = pm * G_CTAS + (int)rank;  // this CTA's 128-row tile
            const bool tile_ok = tm < args.tiles_m;   // false for the empty half of an odd last pair
            const int nkb = args.kb_count ? args.kb_count[pm] : nkb_full;
            // DGRAD: the format tile's packed z values are one contiguous run of
            // the arena; one bulk copy brings it (16-byte aligned superset) into
            // this warpgroup's buffer while the tile's MMAs still run.  A run
            // whose aligned superset would leave the arena is read from global
            // memory instead (zb0 = -1).
            long long zb0 = -1;
            if constexpr (EPI == EPI_DGRAD) {
                if (tile_ok && tn * BN + wg * HALF < args.N) {  // uniform over the warpgroup
                    named_bar_sync(bar_id, 128);  // the previous tile's reads of the buffer are done
                    if (ew == 0 && lane == 0) {
                        long long b0 = -1;
                        const long long tfz = (long long)tm * gn_f + (tn * BN + wg * HALF) / FT;
                        const uint4 m127 = __ldg(reinterpret_cast<const uint4*>(args.mask + tfz * FT_BYTES + 127 * 16));
                        const long long base = (long long)*args.vals_offset;
                        const long long start = base + __ldg(args.row_offsets + tfz * FT);
                        const long long end = base + __ldg(args.row_offsets + tfz * FT + 127) + __popc(m127.x) +
                                              __popc(m127.y) + __popc(m127.z) + __popc(m127.w);
                        if (start >= 0 && end > start && end <= args.vals_len && end - start <= FT_ELEMS) {
                            const uintptr_t vp = reinterpret_cast<uintptr_t>(args.vals);
                            const uintptr_t lo = (vp + 2 * (uintptr_t)start) & ~(uintptr_t)15;
                            const uintptr_t hi = (vp + 2 * (uintptr_t)end + 15) & ~(uintptr_t)15;
                            if (lo >= vp && hi <= vp + 2 * (uintptr_t)args.vals_len) {
                                b0 = (long long)((lo - vp) >> 1);
                                unsigned char* zbuf = smem + (size_t)NST * STAGE_BYTES + 8 * 2048 + (size_t)wg * G_ZBUF;
                                mbar_arrive_expect_tx(&z_bar[wg], (uint32_t)(hi - lo));
                                bulk_g2s(zbuf, reinterpret_cast<const void*>(lo), (uint32_t)(hi - lo), &z_bar[wg]);
                            }
                        }
                        s_zb0[wg] = b0;
                    }
                    named_bar_sync(bar_id, 128);
                    zb0 = s_zb0[wg];
                    if (zb0 >= 0) {
                        if (!__all_sync(FULL, mbar_wait_bounded(&z_bar[wg], z_phase))) {
                            if (lane == 0) atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                            break;
                        }
                        z_phase ^= 1u;
                    }
                }
            }
            // every lane must take the same branch before the warp-collective tcgen05.ld
            const bool ok = __all_sync(FULL, mbar_wait_bounded(&tfull_bar[acc], acc_phase));
            if (!ok || __any_sync(FULL, s_abort != 0)) {
                if (lane == 0) atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN + wg * HALF);
            const int grow = tm * G_BM + row;
            const bool row_ok = grow < args.M;
            const int gcol0 = tn * BN + wg * HALF;  // first column of this warpgroup
            uint16_t* orow = args.out + (size_t)grow * args.ldc;
            const bool vec = args.vec_out != 0;
            const int par = it & 1;
            const int row0 = tm * G_BM + ew * 32;  // first row of this warp
            unsigned char* sbuf = smem + (size_t)NST * STAGE_BYTES + (size_t)(warp - 4) * 2048;

            if constexpr (EPI == EPI_STORE) {
#pragma unroll 1
                for (int c = 0; c < HALF / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_wait_ld();
                    if (args.out_f32) {
                        // float32 C: each lane stores its row's 32 values (128 contiguous bytes)
                        const int gcol = gcol0 + c * 32;
                        if (row_ok && gcol < args.N) {
                            float* frow = args.out_f32 + (size_t)grow * args.ldc + gcol;
                            if (vec && gcol + 32 <= args.N) {
#pragma unroll
                                for (int q = 0; q < 8; ++q) {
                                    float4 v = nkb ? make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                                 __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]))
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                                    if (args.acc_f32) {
                                        const float4 o = reinterpret_cast<const float4*>(frow)[q];
                                        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
                                    }
                                    if (args.relu_out)
                                        v = make_float4(fmaxf(v.x, 0.f), fmaxf(v.y, 0.f), fmaxf(v.z, 0.f),
                                                        fmaxf(v.w, 0.f));
                                    reinterpret_cast<float4*>(frow)[q] = v;
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < 32; ++j) {
                                    if (gcol + j < args.N) {
                                        const float v = nkb ? __uint_as_float(r[j]) : 0.f;
                                        const float o = args.acc_f32 ? frow[j] + v : v;
                                        frow[j] = args.relu_out ? fmaxf(o, 0.f) : o;
                                    }
                                }
                            }
                        }
                        continue;
                    }
                    uint32_t w[16];
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        w[q] = nkb ? pack_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1])) : 0u;
                    if (args.relu_out) {
                        // max(x, 0) on the packed halves: a set sign bit (negative or -0) gives +0
#pragma unroll
                        for (int q = 0; q < 16; ++q)
                            w[q] &= ((w[q] & 0x8000u) ? 0u : 0xFFFFu) | ((w[q] & 0x80000000u) ? 0u : 0xFFFF0000u);
                    }
                    if (args.c_trans) {
                        // the 32 x 32 block transposed through the staging buffer:
                        // lane takes column `lane`, row gcol0 + 32c + lane of C^T
                        if (tile_ok) {
                            if (lane == 0) bulk_wait_group_read0();
                            __syncwarp();
                            stage_words(sbuf, lane, w);
                            __syncwarp();
                            uint32_t wt[16];
                            float unused;
                            staged_column(sbuf, lane, wt, unused);
                            stage_store32(&tmC, sbuf, lane, wt, row0, gcol0 + c * 32);
                        }
                    } else if (vec) {
                        if (tile_ok) stage_store32(&tmC, sbuf, lane, w, gcol0 + c * 32, row0);
                    } else if (row_ok) {
                        store_row32(orow, gcol0 + c * 32, args.N, false, w);
                    }
                }
            } else if constexpr (EPI == EPI_UP) {
                if (gcol0 < args.N && tile_ok) {  // uniform over the warpgroup
                    const long long tf = (long long)tm * gn_f + gcol0 / FT;
                    float* sb = s_bias[wg][par];
                    if (bias) {
                        sb[row] = gcol0 + row < args.N ? bf16_to_f(bias[gcol0 + row]) : 0.f;
                        named_bar_sync(bar_id, 128);
                    }
                    // Chunk c of this row from the accumulator: z (packed bf16
                    // pairs), the activation words and the mask bits of z > 0.
                    auto zchunk = [&](int c, uint32_t (&zw)[16], uint32_t (&w)[16]) -> uint32_t {
                        uint32_t r[32];
                        tmem_ld32(tbase + c * 32, r);
                        tmem_wait_ld();
                        const int gcol = gcol0 + c * 32;
                        // columns past N (and rows past M) carry no bits
                        const int ncol = row_ok ? min(32, args.N - gcol) : 0;
                        const uint32_t colmask = ncol >= 32 ? 0xFFFFFFFFu : ((1u << max(ncol, 0)) - 1u);
                        uint32_t bits = 0;
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            float v0 = nkb ? __uint_as_float(r[2 * q]) : 0.f;
                            float v1 = nkb ? __uint_as_float(r[2 * q + 1]) : 0.f;
                            if (bias) {
                                v0 += sb[c * 32 + 2 * q];
                                v1 += sb[c * 32 + 2 * q + 1];
                            }
                            // pre = bf16(v); z = relu(pre) on the packed pair (NaN stays NaN,
                            // as in torch); the bf16 product z*z is exact before its one
                            // rounding, so __hmul2 gives bf16(z^2) exactly
                            const __nv_bfloat162 pre = __floats2bfloat162_rn(v0, v1);
                            const __nv_bfloat162 zb = __hmax2_nan(pre, __float2bfloat162_rn(0.f));
                            const uint32_t z = bf162_bits(zb);
                            // z > 0: magnitude non-zero and not NaN (+inf counts)
                            const uint32_t mag = z & 0x7FFF7FFFu;
                            const uint32_t pos = __vcmpgtu2(mag, 0u) & __vcmpleu2(mag, 0x7F807F80u) &
                                                 ~(((z >> 15) & 0x00010001u) * 0xFFFFu);
                            bits |= ((pos & 1u) | ((pos >> 15) & 2u)) << (2 * q);
                            zw[q] = z;
                            w[q] = args.act == ACT_RELU2 ? bf162_bits(__hmul2(zb, zb)) : z;
                        }
                        return bits & colmask;
                    };
                    uint32_t words[4];
                    int cnt = 0;
                    if (args.slot_rows) {
                        // Warp-packed slots: the warp's 32 rows' values in arena order
                        // from slots[tf * 16384 + ew * 4096].  In one pass over the
                        // accumulator each lane appends its row's values to the row's
                        // 256-byte area in shared memory (rotated by 2 * lane values
                        // so that lanes writing the same position hit different
                        // banks); a warp scan of the row counts gives each row's
                        // offset in the warp's run, and each row then leaves as one
                        // coalesced run (lane = value).
                        const uint32_t zrows = smem_u32(smem + (size_t)NST * STAGE_BYTES + 8 * 2048 +
                                                        (size_t)(warp - 4) * (32 * 256));
                        const uint32_t ra = zrows + (uint32_t)lane * 256u;
                        uint32_t mw[4] = {0, 0, 0, 0};  // 2:4 metadata words (sp_on)
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const int gcol = gcol0 + c * 32;
                            uint32_t zw[16], w[16];
                            const uint32_t bits = zchunk(c, zw, w);
                            if (args.sp_on) {
                                stage_words(sbuf, lane, w);  // own row: read back by this lane only
                                mw[c] = sp24_emit(args.sp[0], w, grow, gcol, lane,
                                                  [&](int e) { return staged_elem(sbuf, lane, e); });
                            } else if (args.out) {
                                if (vec) stage_store32(&tmC, sbuf, lane, w, gcol, row0);
                                else if (row_ok) store_row32(orow, gcol, args.N, false, w);
                            }
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                if ((bits >> (2 * q)) & 1u) {
                                    asm volatile("st.shared.u16 [%0], %1;" ::"r"(ra + 2u * (uint32_t)((cnt + 2 * lane) & 127)),
                                                 "h"((uint16_t)zw[q]) : "memory");
                                    ++cnt;
                                }
                                if ((bits >> (2 * q + 1)) & 1u) {
                                    asm volatile("st.shared.u16 [%0], %1;" ::"r"(ra + 2u * (uint32_t)((cnt + 2 * lane) & 127)),
                                                 "h"((uint16_t)(zw[q] >> 16)) : "memory");
                                    ++cnt;
                                }
                            }
                            words[c] = bits;
                        }
                        const int incl = warp_incl_scan(cnt, lane);
                        args.slot_rows[tf * FT + row] = incl - cnt;  // offset in the warp's run
                        uint16_t* wslot = args.slots + tf * FT_ELEMS + ew * (FT_ELEMS / 4);
                        __syncwarp();
#pragma unroll 1
                        for (int i = 0; i < 32; ++i) {
                            const int ci = __shfl_sync(FULL, cnt, i);
                            const int ri = __shfl_sync(FULL, incl, i) - ci;
                            for (int j = lane; j < ci; j += 32) {
                                uint16_t v;
                                asm volatile("ld.shared.u16 %0, [%1];"
                                             : "=h"(v)
                                             : "r"(zrows + (uint32_t)i * 256u + 2u * (uint32_t)((j + 2 * i) & 127)));
                                wslot[ri + j] = v;
                            }
                        }
                        __syncwarp();  // the row areas are read before the next tile writes them
                        if (args.sp_on)  // the 128 columns are one K block of the 2:4 form
                            reinterpret_cast<uint4*>(args.sp[0].meta)[((long long)tm * args.sp[0].nkb + gcol0 / 128) * 128 +
                                                                      ew * 32 + lane] = make_uint4(mw[0], mw[1], mw[2], mw[3]);
                    } else {
                        // Per-row slots: row r's values at slots[tf * 16384 + r * 128].
                        uint16_t* slot_row = args.slots + tf * FT_ELEMS + row * FT;
                        uint32_t mw[4] = {0, 0, 0, 0};  // 2:4 metadata words (sp_on)
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const int gcol = gcol0 + c * 32;
                            uint32_t zw[16], w[16];
                            const uint32_t bits = zchunk(c, zw, w);
                            if (args.sp_on) {
                                stage_words(sbuf, lane, w);  // own row: read back by this lane only
                                mw[c] = sp24_emit(args.sp[0], w, grow, gcol, lane,
                                                  [&](int e) { return staged_elem(sbuf, lane, e); });
                            } else if (args.out) {  // no dense activation when the caller passed none
                                if (vec) stage_store32(&tmC, sbuf, lane, w, gcol, row0);
                                else if (row_ok) store_row32(orow, gcol, args.N, false, w);
                            }
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                const uint32_t b2 = (bits >> (2 * q)) & 3u;
                                if (b2) {
                                    if (b2 & 1u) slot_row[cnt++] = (uint16_t)zw[q];
                                    if (b2 & 2u) slot_row[cnt++] = (uint16_t)(zw[q] >> 16);
                                }
                            }
                            words[c] = bits;
                        }
                        if (args.sp_on)  // the 128 columns are one K block of the 2:4 form
                            reinterpret_cast<uint4*>(args.sp[0].meta)[((long long)tm * args.sp[0].nkb + gcol0 / 128) * 128 +
                                                                      ew * 32 + lane] = make_uint4(mw[0], mw[1], mw[2], mw[3]);
                    }
                    *reinterpret_cast<uint4*>(args.mask + tf * FT_BYTES + row * 16) =
                        make_uint4(words[0], words[1], words[2], words[3]);
                    // per-warp partial count of the tile (summed by the scan kernel)
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(FULL, cnt, o);
                    if (lane == 0) args.tile_counts[tf * 4 + ew] = cnt;
                }
            } else {  // EPI_DGRAD
                const uint32_t zsm = smem_u32(smem + (size_t)NST * STAGE_BYTES + 8 * 2048 + (size_t)wg * G_ZBUF);
                if (gcol0 < args.N && tile_ok) {  // uniform over the warpgroup
                    uint16_t* orow2 = args.out2 + (size_t)grow * args.ldc;
                    const long long tf = (long long)tm * gn_f + gcol0 / FT;
                    uint4 mw = make_uint4(0, 0, 0, 0);
                    long long vbase = 0;
                    if (row_ok) {
                        mw = __ldg(reinterpret_cast<const uint4*>(args.mask + tf * FT_BYTES + row * 16));
                        vbase = (long long)*args.vals_offset + __ldg(args.row_offsets + tf * FT + row);
                    }
                    // chunk c (columns gcol0 + 32c ..): dpre and the activation, from
                    // the accumulator and z gathered from the packed values
                    auto chunk = [&](int c, uint32_t bits, uint32_t (&wd)[16], uint32_t (&wa)[16]) {
                        // gather this chunk's z first (from the tile's buffer, or
                        // global memory): read-only loads, free to run ahead
                        // (one branch per chunk, so each path's loads issue together)
                        uint32_t zb[16];
                        if (zb0 >= 0) {
                            const long long k0 = vbase - zb0;  // this row's first value in the buffer
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                uint16_t lo = 0, hi = 0;
                                const long long k1 = k0 + __popc(bits & ((1u << (2 * q)) - 1u));
                                const long long k2 = k0 + __popc(bits & ((2u << (2 * q)) - 1u));
                                if (((bits >> (2 * q)) & 1u) && k1 >= 0 && k1 < G_ZBUF / 2)
                                    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(lo) : "r"(zsm + 2u * (uint32_t)k1));
                                if (((bits >> (2 * q + 1)) & 1u) && k2 >= 0 && k2 < G_ZBUF / 2)
                                    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(hi) : "r"(zsm + 2u * (uint32_t)k2));
                                zb[q] = (uint32_t)lo | ((uint32_t)hi << 16);
                            }
                        } else {
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                uint32_t lo = 0, hi = 0;
                                if ((bits >> (2 * q)) & 1u) {
                                    const long long p = vbase + __popc(bits & ((1u << (2 * q)) - 1u));
                                    if (p < args.vals_len) lo = __ldg(vals + p);
                                }
                                if ((bits >> (2 * q + 1)) & 1u) {
                                    const long long p = vbase + __popc(bits & ((2u << (2 * q)) - 1u));
                                    if (p < args.vals_len) hi = __ldg(vals + p);
                                }
                                zb[q] = lo | (hi << 16);
                            }
                        }
                        vbase += __popc(bits);
                        uint32_t r[32];
                        tmem_ld32(tbase + c * 32, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            // g = bf16(acc); z from the packed values (0 off the mask)
                            const uint32_t gw = nkb ? pack_bf16x2(__uint_as_float(r[2 * q]),
                                                                  __uint_as_float(r[2 * q + 1]))
                                                    : 0u;
                            const float g0 = __uint_as_float(gw << 16), g1 = __uint_as_float(gw & 0xFFFF0000u);
                            const float z0 = __uint_as_float(zb[q] << 16), z1 = __uint_as_float(zb[q] & 0xFFFF0000u);
                            if (args.act == ACT_RELU2) {
                                wd[q] = pack_bf16x2((g0 * 2.0f) * z0, (g1 * 2.0f) * z1);
                                wa[q] = pack_bf16x2(z0 * z0, z1 * z1);
                            } else {
                                const uint32_t keep = (((bits >> (2 * q)) & 1u) ? 0x0000FFFFu : 0u) |
                                                      (((bits >> (2 * q + 1)) & 1u) ? 0xFFFF0000u : 0u);
                                wd[q] = gw & keep;
                                wa[q] = zb[q];
                            }
                        }
                    };
                    if (args.sp_on) {
                        // dpre by rows (for dX), dpre^T and a^T by columns (for dW1,
                        // dW2): the block's column `lane` is row f = gcol0 + 32c + lane
                        // of the transposed matrices, 32 consecutive tokens of its K.
                        // A rolled loop: the three compressions per chunk would not
                        // fit the instruction cache four times over.
                        uint32_t spw0 = 0, spw1 = 0, spw2 = 0, spw3 = 0;
#pragma unroll 1
                        for (int c = 0; c < 4; ++c) {
                            const uint32_t bits = c == 0 ? mw.x : c == 1 ? mw.y : c == 2 ? mw.z : mw.w;
                            uint32_t wd[16], wa[16];
                            chunk(c, bits, wd, wa);
                            auto own = [&](int e) { return staged_elem(sbuf, lane, e); };
                            auto col = [&](int e) { return staged_elem(sbuf, e, lane); };
                            stage_words(sbuf, lane, wd);
                            const uint32_t lw = sp24_emit(args.sp[0], wd, grow, gcol0 + c * 32, lane, own);
                            spw0 = c == 0 ? lw : spw0;
                            spw1 = c == 1 ? lw : spw1;
                            spw2 = c == 2 ? lw : spw2;
                            spw3 = c == 3 ? lw : spw3;
                            const long long f = gcol0 + c * 32 + lane;
                            const long long tmeta =
                                ((long long)(gcol0 / 128) * args.sp[1].nkb + tm) * 128 + c * 32 + lane;
                            const int tk0 = tm * G_BM + ew * 32;
                            uint32_t wt[16];
                            float csum;
                            __syncwarp();
                            staged_column(sbuf, lane, wt, csum);
                            if (args.colsum) atomicAdd(args.colsum + f, csum);
                            args.sp[1].meta[tmeta * 4 + ew] = sp24_emit(args.sp[1], wt, f, tk0, lane, col);
                            __syncwarp();
                            stage_words(sbuf, lane, wa);
                            __syncwarp();
                            staged_column(sbuf, lane, wt, csum);
                            args.sp[2].meta[tmeta * 4 + ew] = sp24_emit(args.sp[2], wt, f, tk0, lane, col);
                            __syncwarp();
                        }
                        reinterpret_cast<uint4*>(args.sp[0].meta)[((long long)tm * args.sp[0].nkb + gcol0 / 128) * 128 +
                                                                  ew * 32 + lane] = make_uint4(spw0, spw1, spw2, spw3);
                    } else {
                        const uint32_t words[4] = {mw.x, mw.y, mw.z, mw.w};
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            uint32_t wd[16], wa[16];
                            chunk(c, words[c], wd, wa);
                            if (vec) {
                                stage_store32(&tmC, sbuf, lane, wd, gcol0 + c * 32, row0);
                                if (args.colsum) {
                                    // lane = column: sum the staged dpre block over its rows
                                    // (rows past M hold zeros); conflict-free swizzled reads
                                    const uint32_t sb0 = smem_u32(sbuf);
                                    const int ch = lane >> 3, sub = (lane & 7) * 2;
                                    float acc = 0.f;
#pragma unroll 8
                                    for (int rr = 0; rr < 32; ++rr) {
                                        uint16_t h;
                                        asm volatile("ld.shared.u16 %0, [%1];"
                                                     : "=h"(h)
                                                     : "r"(sb0 + (uint32_t)(rr * 64 + 16 * (ch ^ ((rr >> 1) & 3)) + sub)));
                                        acc += bf16_to_f(h);
                                    }
                                    const int col = gcol0 + c * 32 + lane;
                                    if (col < args.N) atomicAdd(args.colsum + col, acc);
                                }
                                if (args.out2) stage_store32(&tmC2, sbuf, lane, wa, gcol0 + c * 32, row0);
                            } else {
                                if (row_ok) {
                                    store_row32(orow, gcol0 + c * 32, args.N, false, wd);
                                    if (args.out2) store_row32(orow2, gcol0 + c * 32, args.N, false, wa);
                                }
                                if (args.colsum) {
                                    // column sums by shuffles (rows past M contribute zeros)
#pragma unroll
                                    for (int j = 0; j < 32; ++j) {
                                        float v = row_ok ? bf16_to_f((uint16_t)(wd[j >> 1] >> (16 * (j & 1)))) : 0.f;
#pragma unroll
                                        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
                                        const int col = gcol0 + c * 32 + j;
                                        if (lane == 0 && col < args.N) atomicAdd(args.colsum + col, v);
                                    }
                                }
                            }
                        }
                    }
                }
            }
            // release this accumulator to the leader's MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_group0();  // this warp's stores are complete
        __syncwarp();
    }
    // No CTA may leave while its peer can still touch its shared memory,
    // barriers or TMEM.
    tc_fence_before();
    cluster_sync();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------------- 2:4 GEMM ----
// C[M, N] = A24[M, K] * B[N, K]^T with A in the 2:4 form of sp24.cu
// (compressed values [M, K/2] + tensor-memory-ordered metadata); B K-major
// ([N][ldb]) or MN-major ([K][ldb]).  Pair tiles of 256 x 256 as in
// gemm_kernel; a stage is 128 logical K (four tcgen05.mma.sp of K = 32):
// 16 KB of compressed A + 32 KB of B + 2 KB of metadata per CTA, 4 stages.
//   warps 0-7   TMA issuers, one per (copy A / B0 / B1 / metadata, even / odd
//               stage), since one thread's copies complete one after another;
//               the A issuers of the leader arm the stage barrier
//   warp 8      MMA issuer (leader): per stage one tcgen05.cp moves the
//               stage's metadata (128 lanes x 16 bytes, in each CTA) from
//               shared into 4 tensor-memory columns, then four tcgen05.mma.sp
//   warps 9-16  epilogue: two warpgroups of 128 accumulator columns.  There is
//               one accumulator (256 columns) because the metadata ring needs
//               tensor memory too; the epilogue frees it fast by converting
//               each 32-column chunk to bf16 into spare tensor-memory columns,
//               then stores from there while the next tile accumulates.
constexpr int S_BK = 128;
constexpr int S_STAGES = 4;
constexpr int S_THREADS = 17 * 32;
constexpr int S_EPI0 = 9;  // first epilogue warp
constexpr int S_META_COL = 256;  // metadata ring: 4 columns per stage
constexpr int S_PACK_COL = 272;  // bf16 staging: 64 columns per warpgroup

// The 2:4 GEMM's store phase: the overflow of A added in fp32 (rows of B
// read from bt, B as row-major [K][ldbt]) and C stored as is or transposed.
struct Sp24Epi {
    const uint16_t* ocols;  // NULL: no overflow to add
    const uint16_t* ovals;
    const int* ocount;
    long long ovf_ld;  // K/2
    const uint16_t* bt;
    long long ldbt;
    int c_trans;  // store C^T ([N][ldc]) instead of C
};

template <bool B_MN>
__global__ void __cluster_dims__(G_CTAS, 1, 1) __launch_bounds__(S_THREADS, 1)
    gemm_sp24_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmE, int M, int N,
                     int K, const Sp24Epi epi, uint32_t* __restrict__ status) {
    constexpr int A_BYTES = G_BM * (S_BK / 2) * 2;  // 16 KB
    constexpr int B_HALF = 128 * 64 * 2;             // one 16 KB box
    constexpr int META_BYTES = 128 * 16;  // 2 KB
    constexpr int TMA_BYTES = A_BYTES + 2 * B_HALF;
    constexpr int STAGE_BYTES = TMA_BYTES + META_BYTES;  // all of it completes on the leader's full barrier
    constexpr uint32_t IDESC = idesc_bf16_f32(G_BM * G_CTAS, 256, false, B_MN) | (1u << 2);
    extern __shared__ __align__(1024) unsigned char g_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(g_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t full_bar[S_STAGES], empty_bar[S_STAGES];
    __shared__ __align__(8) uint64_t tfull_bar, tempty_bar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = M / G_BM, tiles_n = (N + 255) / 256;
    const int tiles_mp = (tiles_m + 1) / 2;
    const int ntiles = tiles_mp * tiles_n;
    const int nkb = K / S_BK;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int first_tile = (int)cluster_id_x();
    const int tile_stride = (int)cluster_count_x();

    if (threadIdx.x == 0) {
        for (int s = 0; s < S_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&tfull_bar, 1);
        mbar_init(&tempty_bar, 8 * G_CTAS);  // the 8 epilogue warps of both CTAs
        s_abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        prefetch_tmap(&tmE);
    }
    if (warp == 0) {
        tmem_alloc_pair(&s_tmem, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem;

    if (warp < 8) {
        // ------------------------------------------------------ producers --
        const int op = warp & 3;   // 0: A, 1: B (first half), 2: B (second half), 3: metadata
        const int par = warp >> 2;  // even / odd stages
        if (lane == 0) {
            int armed[S_STAGES] = {0};
            long long kc = 0;
            bool stop = false;
            for (int tile = first_tile; tile < ntiles && !stop && !s_abort; tile += tile_stride) {
                int pm, tn;
                raster(tile, tiles_mp, tiles_n, pm, tn);
                const int arow = (pm * G_CTAS + (int)rank) * G_BM;
                const int brow = tn * 256 + (int)rank * 128;
                for (int kb = 0; kb < nkb; ++kb, ++kc) {
                    if ((int)(kc & 1) != par) continue;
                    const int stage = (int)(kc % S_STAGES);
                    const uint32_t phase = (uint32_t)((kc / S_STAGES) & 1);
                    if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u)) {
                        atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        stop = true;
                        break;
                    }
                    unsigned char* sa = smem + (size_t)stage * STAGE_BYTES;
                    unsigned char* sb = sa + A_BYTES;
                    if (op == 0) {
                        if (leader) {
                            mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES * G_CTAS);
                            ++armed[stage];
                        }
                        tma_load_2d_pair(sa, &tmA, kb * (S_BK / 2), arow, &full_bar[stage]);
                    } else if (op == 3) {
                        // this CTA's 128-row tile; the empty half of an odd last pair
                        // copies the previous tile's metadata (its A rows are zero)
                        const int tm = min(pm * G_CTAS + (int)rank, tiles_m - 1);
                        tma_load_2d_pair(sa + TMA_BYTES, &tmE, 0, ((tm * nkb) + kb) * 128, &full_bar[stage]);
                    } else {
                        const int h = op - 1;
                        if constexpr (!B_MN)  // [N][K]: K offsets 0 / 64 of the stage
                            tma_load_2d_pair(sb + h * B_HALF, &tmB, kb * S_BK + h * 64, brow, &full_bar[stage]);
                        else  // [K][N]: N blocks 0 / 64, 128 K rows each
                            tma_load_2d_pair(sb + h * B_HALF, &tmB, brow + h * 64, kb * S_BK, &full_bar[stage]);
                    }
                }
            }
            if (leader && op == 0)
                for (int s = 0; s < S_STAGES; ++s)
                    if (armed[s]) (void)mbar_wait_bounded(&full_bar[s], (uint32_t)(armed[s] - 1) & 1u);
        }
        __syncwarp();
    } else if (warp == 8) {
        // ----------------------------------------------------------- MMA --
        if (lane == 0 && leader) {
            long long kc = 0;
            int it = 0;
            for (int tile = first_tile; tile < ntiles && !s_abort; tile += tile_stride, ++it) {
                if (!mbar_wait_bounded(&tempty_bar, ((uint32_t)it & 1u) ^ 1u)) {
                    atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                bool fail = false;
                for (int kb = 0; kb < nkb; ++kb, ++kc) {
                    const int stage = (int)(kc % S_STAGES);
                    const uint32_t phase = (uint32_t)((kc / S_STAGES) & 1);
                    if (!mbar_wait_bounded(&full_bar[stage], phase)) {
                        atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        fail = true;
                        break;
                    }
                    const uint32_t sa = smem_u32(smem + (size_t)stage * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
                    const uint32_t e0 = tmem_base + S_META_COL + 4 * stage;
                    tc_cp_pair_128x128b(e0, smem_desc_rows16(sa + TMA_BYTES));
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t ad = umma_desc_sw128(sa + 32 * j, 16, 1024);
                        const uint64_t bd = B_MN ? umma_desc_sw128(sb + 4096 * j, B_HALF, 1024)
                                                 : umma_desc_sw128(sb + (j >> 1) * B_HALF + 64 * (j & 1), 16, 1024);
                        tc_mma_sp_pair(tmem_base, ad, bd, e0 + (uint32_t)(j & ~1), IDESC | (uint32_t)(j & 1),
                                       (kb | j) != 0 ? 1u : 0u);
                    }
                    tc_commit_pair_multicast(&empty_bar[stage], 0x3);
                }
                if (fail) break;
                tc_commit_pair_multicast(&tfull_bar, 0x3);
            }
        }
        __syncwarp();
    } else if (warp < S_EPI0) {
    } else {
        // ------------------------------------------------------ epilogue --
        const int ew = warp & 3;          // lane quarter: accumulator rows 32*ew ..
        const int wg = (warp - S_EPI0) >> 2;  // columns 128*wg ..
        unsigned char* sbuf = smem + (size_t)S_STAGES * STAGE_BYTES + (size_t)(warp - S_EPI0) * 2048;
        const uint32_t tempty_leader = leader_smem_addr(&tempty_bar);
        const uint32_t lane_base = tmem_base + ((uint32_t)(ew * 32) << 16);
        int it = 0;
        for (int tile = first_tile; tile < ntiles; tile += tile_stride, ++it) {
            int pm, tn;
            raster(tile, tiles_mp, tiles_n, pm, tn);
            const int tm = pm * G_CTAS + (int)rank;
            const bool ok = __all_sync(FULL, mbar_wait_bounded(&tfull_bar, (uint32_t)it & 1u));
            if (!ok || __any_sync(FULL, s_abort != 0)) {
                if (lane == 0 && !ok) atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
                break;
            }
            tc_fence_after();
            // accumulator -> bf16 in the spare columns, then free the accumulator
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t r[32], w[16];
                tmem_ld32(lane_base + (uint32_t)(wg * 128 + c * 32), r);
                tmem_wait_ld();
#pragma unroll
                for (int q2 = 0; q2 < 16; ++q2)
                    w[q2] = pack_bf16x2(__uint_as_float(r[2 * q2]), __uint_as_float(r[2 * q2 + 1]));
                tmem_st16(lane_base + (uint32_t)(S_PACK_COL + wg * 64 + c * 16), w);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader);
            if (tm < tiles_m && tn * 256 + wg * 128 < N) {
                const long long grow = (long long)tm * G_BM + ew * 32 + lane;
                const int novf = epi.ocols ? min(max(__ldg(epi.ocount + grow), 0), (int)epi.ovf_ld) : 0;
                const bool any_ovf = __any_sync(FULL, novf > 0);  // warp-uniform
                const uint16_t* ocol = epi.ocols + grow * epi.ovf_ld;
                const uint16_t* oval = epi.ovals + grow * epi.ovf_ld;
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    const int col0 = tn * 256 + wg * 128 + c * 32;
                    if (col0 >= N) break;  // uniform; N is a multiple of 32 with overflow
                    uint32_t w[16];
                    if (any_ovf) {
                        // this row's overflow entries (k, v): C[row, col0 ..] += v * B[k, col0 ..],
                        // summed from zero in entry order, then added to the bf16 C (as
                        // sffn_sp24_overflow_add does).  Two entries' rows of B in flight,
                        // the next pair's (k, v) fetched alongside them.
                        // (per-lane loop: no warp-collective instruction inside)
                        float acc[32];
#pragma unroll
                        for (int q = 0; q < 32; ++q) acc[q] = 0.f;
                        int k0 = novf > 0 ? __ldg(ocol) : 0, k1 = novf > 1 ? __ldg(ocol + 1) : k0;
                        float v0 = novf > 0 ? bf16_to_f(__ldg(oval)) : 0.f;
                        float v1 = novf > 1 ? bf16_to_f(__ldg(oval + 1)) : 0.f;
#pragma unroll 1
                        for (int i = 0; i < novf; i += 2) {
                            const uint4* r0 = reinterpret_cast<const uint4*>(epi.bt + (long long)k0 * epi.ldbt + col0);
                            const uint4* r1 = reinterpret_cast<const uint4*>(epi.bt + (long long)k1 * epi.ldbt + col0);
                            uint4 b0[4], b1[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                b0[u] = __ldg(r0 + u);
                                b1[u] = __ldg(r1 + u);
                            }
                            const float cv0 = v0, cv1 = v1;
                            if (i + 2 < novf) {
                                k0 = __ldg(ocol + i + 2);
                                v0 = bf16_to_f(__ldg(oval + i + 2));
                                k1 = i + 3 < novf ? __ldg(ocol + i + 3) : k0;
                                v1 = i + 3 < novf ? bf16_to_f(__ldg(oval + i + 3)) : 0.f;
                            }
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const uint32_t bw0[4] = {b0[u].x, b0[u].y, b0[u].z, b0[u].w};
                                const uint32_t bw1[4] = {b1[u].x, b1[u].y, b1[u].z, b1[u].w};
#pragma unroll
                                for (int h = 0; h < 4; ++h) {
                                    float& lo = acc[8 * u + 2 * h];
                                    float& hi = acc[8 * u + 2 * h + 1];
                                    lo = fmaf(cv0, __uint_as_float(bw0[h] << 16), lo);
                                    hi = fmaf(cv0, __uint_as_float(bw0[h] & 0xFFFF0000u), hi);
                                    lo = fmaf(cv1, __uint_as_float(bw1[h] << 16), lo);
                                    hi = fmaf(cv1, __uint_as_float(bw1[h] & 0xFFFF0000u), hi);
                                }
                            }
                        }
                        // the bf16 C chunk only now, to keep the loop's registers free
                        // (tcgen05.ld is warp-collective: every lane gets here)
                        __syncwarp();
                        tmem_ld16(lane_base + (uint32_t)(S_PACK_COL + wg * 64 + c * 16), w);
                        tmem_wait_ld();
                        if (novf > 0)  // rows without overflow stay as they are (signed zeros too)
#pragma unroll
                            for (int q = 0; q < 16; ++q)
                                w[q] = pack_bf16x2(__uint_as_float(w[q] << 16) + acc[2 * q],
                                                   __uint_as_float(w[q] & 0xFFFF0000u) + acc[2 * q + 1]);
                    } else {
                        tmem_ld16(lane_base + (uint32_t)(S_PACK_COL + wg * 64 + c * 16), w);
                        tmem_wait_ld();
                    }
                    if (!epi.c_trans) {
                        stage_store32(&tmC, sbuf, lane, w, col0, tm * G_BM + ew * 32);
                    } else {
                        // transpose through the staging buffer: lane takes column `lane`
                        // of the block, row col0 + lane of C^T
                        if (lane == 0) bulk_wait_group_read0();
                        __syncwarp();
                        stage_words(sbuf, lane, w);
                        __syncwarp();
                        uint32_t wt[16];
                        float unused;
                        staged_column(sbuf, lane, wt, unused);
                        stage_store32(&tmC, sbuf, lane, wt, tm * G_BM + ew * 32, col0);
                    }
                }
            }
        }
        if (lane == 0) bulk_wait_group0();
        __syncwarp();
    }
    tc_fence_before();
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

// ------------------------------------------------------- compacted-K GEMM ----
// C[M, N] = sum over j < K(tm) of Ac[row, j] * B[idx[tm][j], :] for the rows
// of each 128-row tile tm: the contraction of the bitmask-sparse
// down-projection (and of dX) over the tile's live columns only.  Ac is the
// activation with those columns compacted (K-major, [M][lda]); B is the other
// operand with rows = the contraction index ([K rows][ldb], N contiguous), of
// which each stage gathers the 64 rows the list names by TMA tile::gather4 (a
// one-row box, four rows per copy, this GPU's memory only).  The list of tile
// tm is padded to a multiple of 64 with a column that is zero in every row of
// the tile, so the padding adds nothing.
//
// One CTA per SM, single-CTA (cta_group::1) tcgen05.mma of M = 128, N = 256,
// K = 16 (a pair of SMs would need one list for 256 rows, whose union of live
// columns is larger).  Tiles of 128 x 256 are visited in groups of
// CK_GROUP_M row tiles, row tile fastest, so that the CTAs in flight share
// Ac tiles and the gathered rows of B (which together exceed L2) across a
// group.
//   warp 0       A producer: arms the stage (A and B bytes) and loads the
//                128 x 64 Ac block (128-byte swizzle).
//   warp 3       B producer: lane l holds four list entries (K rows 4(l%16)
//                .., loaded a stage ahead).  When the stage's 64 rows are
//                consecutive (whole live column runs, as clustered sparsity
//                gives) lane 0 loads them as four tiled 64 x 64 boxes;
//                otherwise each lane gathers its four rows for two of the
//                four 64-column N blocks.
//   warp 1       MMA issuer (one thread), two accumulators of 256 columns.
//   warp 2       allocates / frees the 512 tensor-memory columns.
//   warps 4..11  epilogue, two warpgroups of 128 columns (thread = row).
constexpr int CK_STAGES = 4;
constexpr int CK_BN = 256;
constexpr int CK_THREADS = 12 * 32;
constexpr int CK_A_BYTES = G_BM * G_BK * 2;      // 16 KB
constexpr int CK_B_BYTES = CK_BN * G_BK * 2;     // 32 KB: four MN blocks of 64 K rows x 128 B
constexpr int CK_STAGE_BYTES = CK_A_BYTES + CK_B_BYTES;
constexpr int CK_SMEM = CK_STAGES * CK_STAGE_BYTES + 8 * 2048 + 1024;
constexpr int CK_GROUP_M = 16;

__device__ __forceinline__ void ck_raster(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
    const int per_group = CK_GROUP_M * tiles_n;
    const int group = tile / per_group;
    const int first_m = group * CK_GROUP_M;
    const int gsize = min(tiles_m - first_m, CK_GROUP_M);
    const int r = tile - group * per_group;
    tm = first_m + r % gsize;
    tn = r / gsize;
}

struct CkArgs {
    int M, N;
    int tiles_m, tiles_n;
    const int* idx;     // [tiles_m][ld_idx] row of B for each compacted column
    long long ld_idx;
    const int* kcount;  // [tiles_m] live columns of the tile (its list is padded to 64)
    int vec_out;
    uint16_t* out;
    long long ldc;
    uint32_t* status;
};

__global__ void __launch_bounds__(CK_THREADS, 1)
    gemm_ck_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmBt, const __grid_constant__ CUtensorMap tmC,
                   const CkArgs args) {
    constexpr uint32_t IDESC = idesc_bf16_f32(G_BM, CK_BN, false, true);
    constexpr uint32_t MN_LBO = G_BK * 128;
    extern __shared__ __align__(1024) unsigned char g_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(g_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t full_bar[CK_STAGES];
    __shared__ __align__(8) uint64_t empty_bar[CK_STAGES];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = args.tiles_m * args.tiles_n;
    if (threadIdx.x == 0) {
        for (int s = 0; s < CK_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);   // the A producer's arrive.expect_tx
            mbar_init(&empty_bar[s], 1);  // one commit per use
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 8);  // every epilogue warp
        }
        s_abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        prefetch_tmap(&tmBt);
    }
    if (warp == 2) {
        tmem_alloc(&s_tmem, 2 * CK_BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem;

    auto nkb_of = [&](int tm) { return (__ldg(args.kcount + tm) + G_BK - 1) / G_BK; };

    if (warp == 0 || warp == 3) {
        // ----------------------------------------------------- producers --
        const bool loads_a = warp == 0;
        if (loads_a ? lane == 0 : true) {
            int armed[CK_STAGES] = {0};
            long long kc = 0;
            bool stop = false;
            const int g = lane & 15, h = lane >> 4;  // B: K rows 4g .. 4g+3, N blocks 2h, 2h+1
            for (int tile = blockIdx.x; tile < ntiles && !stop; tile += gridDim.x) {
                bool ab = s_abort != 0;
                if (!loads_a) ab = __any_sync(FULL, ab);  // the B warp's lanes stay converged
                if (ab) break;
                int tm, tn;
                ck_raster(tile, args.tiles_m, args.tiles_n, tm, tn);
                const int nkb = nkb_of(tm);
                const int* list = args.idx + (long long)tm * args.ld_idx;
                int4 r4 = make_int4(0, 0, 0, 0);
                if (!loads_a && nkb > 0) r4 = __ldg(reinterpret_cast<const int4*>(list + 4 * g));
                for (int i = 0; i < nkb; ++i, ++kc) {
                    const int stage = (int)(kc % CK_STAGES);
                    const uint32_t phase = (uint32_t)((kc / CK_STAGES) & 1);
                    // the B warp decides together: its lanes shuffle and vote below
                    const bool freed = loads_a ? mbar_wait_bounded(&empty_bar[stage], phase ^ 1u)
                                               : __all_sync(FULL, mbar_wait_bounded(&empty_bar[stage], phase ^ 1u));
                    if (!freed) {
                        atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        stop = true;
                        break;
                    }
                    unsigned char* sa = smem + (size_t)stage * CK_STAGE_BYTES;
                    unsigned char* sb = sa + CK_A_BYTES;
                    ++armed[stage];
                    if (loads_a) {
                        mbar_arrive_expect_tx(&full_bar[stage], CK_STAGE_BYTES);
                        tma_load_2d(sa, &tmA, i * G_BK, tm * G_BM, &full_bar[stage]);
                    } else {
                        const int4 cur = r4;
                        if (i + 1 < nkb)  // the next stage's entries, in flight while this one is issued
                            r4 = __ldg(reinterpret_cast<const int4*>(list + (i + 1) * G_BK + 4 * g));
                        const int base = __shfl_sync(FULL, cur.x, 0);
                        const bool run = cur.x == base + 4 * g && cur.y == base + 4 * g + 1 &&
                                         cur.z == base + 4 * g + 2 && cur.w == base + 4 * g + 3;
                        if (__all_sync(FULL, run)) {
                            // 64 consecutive rows of B: four tiled 64 x 64 boxes
                            if (lane == 0)
#pragma unroll
                                for (int blk = 0; blk < 4; ++blk)
                                    tma_load_2d(sb + blk * MN_LBO, &tmBt, tn * CK_BN + blk * 64, base, &full_bar[stage]);
                        } else {
#pragma unroll
                            for (int b = 0; b < 2; ++b) {
                                const int blk = 2 * h + b;
                                tma_gather4(sb + blk * MN_LBO + g * 512, &tmB, tn * CK_BN + blk * 64, cur.x, cur.y,
                                            cur.z, cur.w, &full_bar[stage]);
                            }
                        }
                    }
                }
            }
            // the full barriers count both operands' bytes: once the last phase
            // this thread loaded into completes, none of its copies is landing
            for (int s = 0; s < CK_STAGES; ++s)
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
                ck_raster(tile, args.tiles_m, args.tiles_n, tm, tn);
                const int nkb = nkb_of(tm);
                if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1u)) {
                    atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * CK_BN);
                bool ready = nkb > 0 && mbar_try_wait(&full_bar[stage], phase);
                bool fail = false;
                for (int i = 0; i < nkb; ++i) {
                    if (!ready && !mbar_wait_bounded(&full_bar[stage], phase)) {
                        atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                        s_abort = 1;
                        fail = true;
                        break;
                    }
                    const uint32_t sa = smem_u32(smem + (size_t)stage * CK_STAGE_BYTES);
                    const uint32_t sb = sa + CK_A_BYTES;
#pragma unroll
                    for (int k = 0; k < G_BK / 16; ++k)
                        tc_mma_f16(d, umma_desc_sw128(sa + k * 32, 16, 1024), umma_desc_sw128(sb + k * 2048, MN_LBO, 1024),
                                   IDESC, (i | k) != 0 ? 1u : 0u);
                    tc_commit(&empty_bar[stage]);
                    if (++stage == CK_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    ready = i + 1 < nkb && mbar_try_wait(&full_bar[stage], phase);
                }
                if (fail) break;
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
        const int wg = (warp - 4) >> 2;
        const int ew = warp & 3;
        unsigned char* sbuf = smem + (size_t)CK_STAGES * CK_STAGE_BYTES + (size_t)(warp - 4) * 2048;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            int tm, tn;
            ck_raster(tile, args.tiles_m, args.tiles_n, tm, tn);
            const int nkb = nkb_of(tm);
            const bool ok = __all_sync(FULL, mbar_wait_bounded(&tfull_bar[acc], acc_phase));
            if (!ok || __any_sync(FULL, s_abort != 0)) {
                if (lane == 0) atomicOr(args.status, SFFN_STATUS_WAIT_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * CK_BN + wg * 128);
            const int row0 = tm * G_BM + ew * 32;
            const int grow = row0 + lane;
            const int gcol0 = tn * CK_BN + wg * 128;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t r[32];
                tmem_ld32(tbase + c * 32, r);
                tmem_wait_ld();
                uint32_t w[16];
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    w[q] = nkb ? pack_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1])) : 0u;
                if (args.vec_out) {
                    stage_store32(&tmC, sbuf, lane, w, gcol0 + c * 32, row0);
                } else if (grow < args.M) {
                    store_row32(args.out + (size_t)grow * args.ldc, gcol0 + c * 32, args.N, false, w);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_group0();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * CK_BN);
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

// 2-D bf16 (or float32) tensor map: `inner` contiguous elements per row,
// `outer` rows, row stride `ld` elements, box = box_inner x box_outer,
// 128-byte swizzle.
bool make_tmap(CUtensorMap* m, const void* base, long long inner, long long outer, long long ld,
               int box_inner, int box_outer,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B, bool f32 = false) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * (f32 ? 4 : 2))};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                          box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
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

// Clusters of G_CTAS that can be resident at once (each CTA fills an SM).
template <typename K>
int max_active_clusters(K kernel, int smem) {
    static int cached = 0;
    if (!cached) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(G_CTAS * 64);
        cfg.blockDim = dim3(G_THREADS);
        cfg.dynamicSmemBytes = (size_t)smem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = G_CTAS;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (void*)kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = g_num_sms() / G_CTAS;
        }
        cached = n;
    }
    return cached;
}

bool device_is_sm100() {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
    return major == 10;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool TF32 = false>
int launch_gemm(const void* A, long long lda, const void* B, long long ldb, GemmArgs args,
                cudaStream_t st, long long kmap = -1) {
    CUtensorMap ta, tb;
    // K extent of the operands' tensor maps (beyond the K blocks this launch reads)
    const long long KM = kmap > 0 ? kmap : args.K;
    // K-major operand [rows][K]: inner = K; MN-major operand [K][rows]: inner = rows.
    // TF32 (K-major only): float32 elements, 32 of them per 128-byte box row.
    constexpr int KB_ELEMS = TF32 ? G_BK / 2 : G_BK;
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
    const bool okA = A_MN ? make_tmap(&ta, A, args.M, KM, lda, 64, G_BK)
                          : make_tmap(&ta, A, KM, args.M, lda, KB_ELEMS, G_BM, sw, TF32);
    const bool okB = B_MN ? make_tmap(&tb, B, args.N, KM, ldb, 64, G_BK)
                          : make_tmap(&tb, B, KM, args.N, ldb, KB_ELEMS, BN / G_CTAS, sw, TF32);
    if (!okA || !okB) return SFFN_ERR_CUDA;
    // outputs: 32 x 32 boxes with 64-byte swizzle for the epilogue's bulk stores
    CUtensorMap tc, tc2;
    memset(&tc, 0, sizeof(tc));
    memset(&tc2, 0, sizeof(tc2));
    if (args.out_f32) {
        // plain vector stores from the epilogue; no tensor map
    } else if (args.c_trans) {
        if (!make_tmap(&tc, args.out, args.M, args.N, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
            return SFFN_ERR_CUDA;
    } else if (args.vec_out) {
        if (!make_tmap(&tc, args.out, args.N, args.M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
            return SFFN_ERR_CUDA;
        if (EPI == EPI_DGRAD && args.out2 &&
            !make_tmap(&tc2, args.out2, args.N, args.M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
            return SFFN_ERR_CUDA;
    }
    // stages + 8 epilogue warps x 2 KB staging (+ the z buffers) + alignment slack
    constexpr int smem = gemm_smem_bytes<EPI>(BN);
    auto k = gemm_kernel<BN, A_MN, B_MN, EPI, TF32>;
    SFFN_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int npairs = ((args.tiles_m + 1) / 2) * args.tiles_n;
    const int clusters = std::min(npairs, max_active_clusters(k, smem));
    if (clusters <= 0) return SFFN_OK;
    k<<<clusters * G_CTAS, G_THREADS, smem, st>>>(ta, tb, tc, tc2, args);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

template <int EPI>
int dispatch_kmap(bool a_mn, bool b_mn, const void* A, long long lda, const void* B, long long ldb,
                  GemmArgs args, long long kmap, cudaStream_t st) {
    constexpr int BN = 256;
    if (!a_mn && !b_mn) return launch_gemm<BN, false, false, EPI>(A, lda, B, ldb, args, st, kmap);
    if (!a_mn && b_mn) return launch_gemm<BN, false, true, EPI>(A, lda, B, ldb, args, st, kmap);
    if (a_mn && b_mn) return launch_gemm<BN, true, true, EPI>(A, lda, B, ldb, args, st, kmap);
    return launch_gemm<BN, true, false, EPI>(A, lda, B, ldb, args, st, kmap);
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
int check_operands(DeviceScope& scope, const void* A, long long lda, bool a_mn, const void* B, long long ldb,
                   bool b_mn, long long M, long long N, long long K) {
    if (M <= 0 || N <= 0 || K <= 0) return SFFN_ERR_ARG;
    if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return SFFN_ERR_ARG;
    if (!A || !B) return SFFN_ERR_ARG;
    if (!aligned16(A) || !aligned16(B) || (lda * 2) % 16 || (ldb * 2) % 16) return SFFN_ERR_ALIGN;
    if (lda < (a_mn ? M : K) || ldb < (b_mn ? N : K)) return SFFN_ERR_ARG;
    if (int rc = scope.bind_same(A, {B})) return rc;
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

template <bool B_MN>
int launch_sp24(const void* vals, const uint32_t* meta, long long M, long long K, const void* B, long long ldb,
                void* C, long long ldc, long long N, const Sp24Epi& epi, uint32_t* status, cudaStream_t st) {
    CUtensorMap ta, tb, tc;
    if (!make_tmap(&ta, vals, K / 2, M, K / 2, 64, 128)) return SFFN_ERR_CUDA;
    const bool okB = B_MN ? make_tmap(&tb, B, N, K, ldb, 64, 128) : make_tmap(&tb, B, K, N, ldb, 64, 128);
    if (!okB) return SFFN_ERR_CUDA;
    const bool okC = epi.c_trans ? make_tmap(&tc, C, M, N, ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)
                                 : make_tmap(&tc, C, N, M, ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    if (!okC) return SFFN_ERR_CUDA;
    // metadata: rows of 16 bytes (4 uint32), 128-row boxes, no swizzle
    CUtensorMap te;
    {
        auto fn = encode_fn();
        if (!fn) return SFFN_ERR_CUDA;
        cuuint64_t dims[2] = {4, (cuuint64_t)((M / 128) * (K / 128) * 128)};
        cuuint64_t strides[1] = {16};
        cuuint32_t box[2] = {4, 128};
        cuuint32_t estr[2] = {1, 1};
        const CUresult r = fn(&te, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(meta), dims, strides,
                              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            set_error_text("cuTensorMapEncodeTiled failed for the 2:4 metadata");
            return SFFN_ERR_CUDA;
        }
    }
    constexpr int smem = S_STAGES * (G_BM * (S_BK / 2) * 2 + 2 * 128 * 64 * 2 + 128 * 16) + 8 * 2048 + 1024;
    auto k = gemm_sp24_kernel<B_MN>;
    SFFN_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    static int cached[2] = {0, 0};
    int& maxc = cached[B_MN ? 1 : 0];
    if (!maxc) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(G_CTAS * 64);
        cfg.blockDim = dim3(S_THREADS);
        cfg.dynamicSmemBytes = (size_t)smem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = G_CTAS;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (void*)k, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = g_num_sms() / G_CTAS;
        }
        maxc = n;
    }
    const long long tiles_m = M / G_BM, tiles_n = (N + 255) / 256;
    const int npairs = (int)(((tiles_m + 1) / 2) * tiles_n);
    const int clusters = std::min(npairs, maxc);
    k<<<clusters * G_CTAS, S_THREADS, smem, st>>>(ta, tb, tc, te, (int)M, (int)N, (int)K, epi, status);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

// The compacted-K GEMM: tensor maps (Ac tiles, one-row gather boxes of B, C
// store boxes) and a persistent grid of one CTA per SM.
int launch_gemm_ck(const void* A, long long lda, long long kmax, const void* B, long long ldb, long long krows,
                   CkArgs args, cudaStream_t st) {
    CUtensorMap ta, tb, tbt, tc;
    if (!make_tmap(&ta, A, kmax, args.M, lda, G_BK, G_BM)) return SFFN_ERR_CUDA;
    if (!make_tmap(&tb, B, args.N, krows, ldb, 64, 1)) return SFFN_ERR_CUDA;     // one-row gather boxes
    if (!make_tmap(&tbt, B, args.N, krows, ldb, 64, G_BK)) return SFFN_ERR_CUDA;  // runs of 64 rows
    memset(&tc, 0, sizeof(tc));
    if (args.vec_out && !make_tmap(&tc, args.out, args.N, args.M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return SFFN_ERR_CUDA;
    SFFN_CUDA_TRY(cudaFuncSetAttribute(gemm_ck_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_SMEM));
    const int ntiles = args.tiles_m * args.tiles_n;
    const int grid = std::min(ntiles, g_num_sms());
    if (grid <= 0) return SFFN_OK;
    gemm_ck_kernel<<<grid, CK_THREADS, CK_SMEM, st>>>(ta, tb, tbt, tc, args);
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" int sffn_gemm_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                              void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                              const int32_t* kb_list, const int32_t* kb_count, int kb_stride,
                              uint32_t* status_dev, void* stream) {
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, A, lda, a_mn, B, ldb, b_mn, M, N, K);
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

extern "C" int sffn_gemm_relu(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                              void* C, int out_f32, int64_t ldc, int64_t M, int64_t N, int64_t K,
                              const int32_t* kb_list, const int32_t* kb_count, int kb_stride,
                              uint32_t* status_dev, void* stream) {
    // C = max(A @ B, 0), bf16 operands as sffn_gemm_bf16 takes them, C bf16
    // (out_f32 == 0) or float32, the ReLU applied by the epilogue.
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, A, lda, a_mn, B, ldb, b_mn, M, N, K);
    if (rc) return rc;
    if (!C || ldc < N || !status_dev) return SFFN_ERR_ARG;
    if ((kb_list == nullptr) != (kb_count == nullptr)) return SFFN_ERR_ARG;
    GemmArgs a = base_args(M, N, K, out_f32 ? nullptr : C, ldc);
    if (out_f32) {
        a.out_f32 = static_cast<float*>(C);
        a.vec_out = aligned16(C) && (ldc * 4) % 16 == 0;
    }
    a.relu_out = 1;
    a.kb_list = kb_list;
    a.kb_count = kb_count;
    a.kb_stride = kb_stride;
    a.status = status_dev;
    return dispatch<EPI_STORE>(a_mn != 0, b_mn != 0, A, lda, B, ldb, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sffn_gemm_bf16_ct(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                                 void* Ct, int64_t ldct, int64_t M, int64_t N, int64_t K, const int32_t* kb_list,
                                 const int32_t* kb_count, int kb_stride, uint32_t* status_dev, void* stream) {
    // C = A @ B computed as sffn_gemm_bf16 does, stored transposed: Ct[n][m].
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, A, lda, a_mn, B, ldb, b_mn, M, N, K);
    if (rc) return rc;
    if (!Ct || ldct < M || !status_dev) return SFFN_ERR_ARG;
    if (!aligned16(Ct) || (ldct * 2) % 16) return SFFN_ERR_ALIGN;
    if ((kb_list == nullptr) != (kb_count == nullptr)) return SFFN_ERR_ARG;
    GemmArgs a = base_args(M, N, K, Ct, ldct);
    a.c_trans = 1;
    a.vec_out = 0;
    a.kb_list = kb_list;
    a.kb_count = kb_count;
    a.kb_stride = kb_stride;
    a.status = status_dev;
    return dispatch<EPI_STORE>(a_mn != 0, b_mn != 0, A, lda, B, ldb, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sffn_gemm_bf16_f32out(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                                     float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int relu,
                                     uint32_t* status_dev, void* stream) {
    // C (float32) = A @ B, bf16 operands as sffn_gemm_bf16 takes them.
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, A, lda, a_mn, B, ldb, b_mn, M, N, K);
    if (rc) return rc;
    if (!C || ldc < N || !status_dev) return SFFN_ERR_ARG;
    // The tensor cores' float32 accumulation does not round to nearest: over
    // K of 18k (six split terms of 3072) its error grew to ~5e-5.  K runs in
    // chunks of kFp32ChunkK (at most 64 MMA steps each), each chunk's sum
    // added into C by the epilogue in float32 with round to nearest.
    constexpr long long kFp32ChunkK = 1024;
    for (long long k0 = 0; k0 < K; k0 += kFp32ChunkK) {
        const long long kc = std::min(kFp32ChunkK, K - k0);
        GemmArgs a = base_args(M, N, k0 + kc, nullptr, ldc);  // the maps cover K columns up to this chunk's end
        a.K = (int)kc;
        a.kb0 = (int)(k0 / G_BK);
        a.out_f32 = C;
        a.acc_f32 = k0 > 0;
        a.relu_out = relu != 0 && k0 + kc >= K;  // after the last chunk's sum
        a.vec_out = aligned16(C) && (ldc * 4) % 16 == 0;
        a.status = status_dev;
        if (int r2 = dispatch_kmap<EPI_STORE>(a_mn != 0, b_mn != 0, A, lda, B, ldb, a, k0 + kc,
                                              reinterpret_cast<cudaStream_t>(stream)))
            return r2;
    }
    return SFFN_OK;
}

extern "C" int sffn_gemm_tf32(const float* A, int64_t lda, const float* B, int64_t ldb, float* C, int64_t ldc,
                              int64_t M, int64_t N, int64_t K, int relu, uint32_t* status_dev, void* stream) {
    // C (float32 [M][ldc]) = A [M][lda] @ B^T with B given as [N][ldb] (both
    // row-major, K contiguous), the inputs read as TF32 by the tensor cores,
    // C = max(C, 0) with relu.
    DeviceScope dev_scope;
    if (M <= 0 || N <= 0 || K <= 0 || M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return SFFN_ERR_ARG;
    if (!A || !B || !C || !status_dev || lda < K || ldb < K || ldc < N) return SFFN_ERR_ARG;
    if (!aligned16(A) || !aligned16(B) || (lda * 4) % 16 || (ldb * 4) % 16) return SFFN_ERR_ALIGN;
    if (int rc = dev_scope.bind_same(A, {B, C})) return rc;
    if (!device_is_sm100()) return SFFN_ERR_DEVICE;
    GemmArgs a = base_args(M, N, K, nullptr, ldc);
    a.out_f32 = C;
    a.relu_out = relu != 0;
    a.vec_out = aligned16(C) && (ldc * 4) % 16 == 0;
    a.status = status_dev;
    return launch_gemm<256, false, false, EPI_STORE, true>(A, lda, B, ldb, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sffn_gemm_bf16_f32acc(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                                     float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int accumulate,
                                     uint32_t* status_dev, void* stream) {
    // C (float32) = A @ B, or C += A @ B with accumulate, in one pass over K.
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, A, lda, a_mn, B, ldb, b_mn, M, N, K);
    if (rc) return rc;
    if (!C || ldc < N || !status_dev) return SFFN_ERR_ARG;
    GemmArgs a = base_args(M, N, K, nullptr, ldc);
    a.out_f32 = C;
    a.acc_f32 = accumulate != 0;
    a.vec_out = aligned16(C) && (ldc * 4) % 16 == 0;
    a.status = status_dev;
    return dispatch<EPI_STORE>(a_mn != 0, b_mn != 0, A, lda, B, ldb, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sffn_ffn_up(const void* x, int64_t ldx, const void* w1, int64_t ldw1, const void* b1,
                           int64_t T, int64_t D, int64_t F, int act, void* act_out, int64_t ld_act,
                           uint8_t* bitmask, int32_t* tile_counts, void* slots, int32_t* slot_rows,
                           uint32_t* status_dev, void* stream) {
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, x, ldx, false, w1, ldw1, false, T, F, D);
    if (rc) return rc;
    if (act != ACT_RELU && act != ACT_RELU2) return SFFN_ERR_ARG;
    if ((act_out && ld_act < F) || !bitmask || !tile_counts || !status_dev) return SFFN_ERR_ARG;
    if (!slots) return SFFN_ERR_ARG;
    if (!aligned16(bitmask)) return SFFN_ERR_ALIGN;
    if (T * F > 0x7FFFFFFFll) return SFFN_ERR_ARG;
    GemmArgs a = base_args(T, F, D, act_out, act_out ? ld_act : F);
    if (!act_out) a.vec_out = 0;
    a.act = act;
    a.bias = static_cast<const uint16_t*>(b1);
    a.mask = bitmask;
    a.tile_counts = tile_counts;
    a.slots = static_cast<uint16_t*>(slots);
    a.slot_rows = slot_rows;
    a.status = status_dev;
    return dispatch<EPI_UP>(false, false, x, ldx, w1, ldw1, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sffn_ffn_dgrad(const void* dout, int64_t ld_dout, const void* w2, int64_t ldw2,
                              int64_t T, int64_t D, int64_t F, int act, const void* vals,
                              int64_t vals_len, const uint8_t* bitmask, const int32_t* row_offsets,
                              const int32_t* vals_offset_dev, void* dpre_out, void* act_out,
                              int64_t ld_out, float* db1_sum, uint32_t* status_dev, void* stream) {
    // dA[T, F] = dout[T, D] @ W2[D, F]: B = W2 is [K=D][N=F], N contiguous (MN-major).
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, dout, ld_dout, false, w2, ldw2, true, T, F, D);
    if (rc) return rc;
    if (act != ACT_RELU && act != ACT_RELU2) return SFFN_ERR_ARG;
    if (!vals || !bitmask || !row_offsets || !vals_offset_dev || !dpre_out || ld_out < F || !status_dev)
        return SFFN_ERR_ARG;
    if (!aligned16(bitmask)) return SFFN_ERR_ALIGN;
    if (act_out && !aligned16(dpre_out) != !aligned16(act_out)) return SFFN_ERR_ALIGN;
    GemmArgs a = base_args(T, F, D, dpre_out, ld_out);
    a.act = act;
    a.out2 = static_cast<uint16_t*>(act_out);
    a.mask = const_cast<uint8_t*>(bitmask);
    a.vals = static_cast<const uint16_t*>(vals);
    a.vals_len = vals_len;
    a.row_offsets = row_offsets;
    a.vals_offset = vals_offset_dev;
    a.colsum = db1_sum;
    a.status = status_dev;
    return dispatch<EPI_DGRAD>(false, true, dout, ld_dout, w2, ldw2, a, reinterpret_cast<cudaStream_t>(stream));
}

namespace {
// The host description of one 2:4 output, checked; rows x K of the matrix.
int sp24_out(const sffn_sp24_mat* m, long long rows, long long K, Sp24Out& o, cudaStream_t st) {
    if (!m || !m->vals || !m->meta || !m->ovf_cols || !m->ovf_vals || !m->ovf_count) return SFFN_ERR_ARG;
    if (!aligned16(m->vals) || !aligned16(m->meta)) return SFFN_ERR_ALIGN;
    o.vals = static_cast<uint16_t*>(m->vals);
    o.meta = m->meta;
    o.ocols = static_cast<uint16_t*>(m->ovf_cols);
    o.ovals = static_cast<uint16_t*>(m->ovf_vals);
    o.ocount = m->ovf_count;
    o.vals_ld = K / 2;
    o.nkb = (int)(K / 128);
    return cudaMemsetAsync(m->ovf_count, 0, (size_t)rows * sizeof(int32_t), st) == cudaSuccess ? SFFN_OK
                                                                                               : SFFN_ERR_CUDA;
}
bool sp24_dims_ok(long long T, long long F) {
    return T % 128 == 0 && F % 128 == 0 && T <= 65536 && F <= 65536;
}
}  // namespace

extern "C" int sffn_ffn_up_sp24(const void* x, int64_t ldx, const void* w1, int64_t ldw1, const void* b1,
                                int64_t T, int64_t D, int64_t F, int act, const sffn_sp24_mat* out,
                                uint8_t* bitmask, int32_t* tile_counts, void* slots, int32_t* slot_rows,
                                uint32_t* status_dev, void* stream) {
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, x, ldx, false, w1, ldw1, false, T, F, D);
    if (rc) return rc;
    if (!sp24_dims_ok(T, F)) return SFFN_ERR_UNSUPPORTED;
    if (act != ACT_RELU && act != ACT_RELU2) return SFFN_ERR_ARG;
    if (!bitmask || !tile_counts || !slots || !status_dev) return SFFN_ERR_ARG;
    if (!aligned16(bitmask)) return SFFN_ERR_ALIGN;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    GemmArgs a = base_args(T, F, D, nullptr, F);
    a.vec_out = 0;
    a.sp_on = 1;
    if ((rc = sp24_out(out, T, F, a.sp[0], st))) return rc;
    a.act = act;
    a.bias = static_cast<const uint16_t*>(b1);
    a.mask = bitmask;
    a.tile_counts = tile_counts;
    a.slots = static_cast<uint16_t*>(slots);
    a.slot_rows = slot_rows;
    a.status = status_dev;
    return dispatch<EPI_UP>(false, false, x, ldx, w1, ldw1, a, st);
}

extern "C" int sffn_ffn_dgrad_sp24(const void* dout, int64_t ld_dout, const void* w2, int64_t ldw2, int64_t T,
                                   int64_t D, int64_t F, int act, const void* vals, int64_t vals_len,
                                   const uint8_t* bitmask, const int32_t* row_offsets,
                                   const int32_t* vals_offset_dev, const sffn_sp24_mat* dpre,
                                   const sffn_sp24_mat* dpre_t, const sffn_sp24_mat* act_t, float* db1_sum,
                                   uint32_t* status_dev, void* stream) {
    DeviceScope dev_scope;
    int rc = check_operands(dev_scope, dout, ld_dout, false, w2, ldw2, true, T, F, D);
    if (rc) return rc;
    if (!sp24_dims_ok(T, F)) return SFFN_ERR_UNSUPPORTED;
    if (act != ACT_RELU && act != ACT_RELU2) return SFFN_ERR_ARG;
    if (!vals || !bitmask || !row_offsets || !vals_offset_dev || !status_dev) return SFFN_ERR_ARG;
    if (!aligned16(bitmask)) return SFFN_ERR_ALIGN;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    GemmArgs a = base_args(T, F, D, nullptr, F);
    a.vec_out = 0;
    a.sp_on = 1;
    if ((rc = sp24_out(dpre, T, F, a.sp[0], st)) || (rc = sp24_out(dpre_t, F, T, a.sp[1], st)) ||
        (rc = sp24_out(act_t, F, T, a.sp[2], st)))
        return rc;
    a.act = act;
    a.mask = const_cast<uint8_t*>(bitmask);
    a.vals = static_cast<const uint16_t*>(vals);
    a.vals_len = vals_len;
    a.row_offsets = row_offsets;
    a.vals_offset = vals_offset_dev;
    a.colsum = db1_sum;
    a.status = status_dev;
    return dispatch<EPI_DGRAD>(false, true, dout, ld_dout, w2, ldw2, a, st);
}

extern "C" int sffn_gemm_sp24(const void* vals, const uint32_t* meta, int64_t M, int64_t K, const void* B,
                              int64_t ldb, int b_mn, void* C, int64_t ldc, int64_t N, uint32_t* status_dev,
                              void* stream) {
    if (M <= 0 || N <= 0 || K <= 0 || M % 128 || K % 128) return SFFN_ERR_UNSUPPORTED;
    if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return SFFN_ERR_ARG;
    if (!vals || !meta || !B || !C || !status_dev) return SFFN_ERR_ARG;
    if (!aligned16(vals) || !aligned16(meta) || !aligned16(B) || !aligned16(C) || (ldb * 2) % 16 || (ldc * 2) % 16)
        return SFFN_ERR_ALIGN;
    if (ldb < (b_mn ? N : K) || ldc < N) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, vals);
    if (!device_is_sm100()) return SFFN_ERR_DEVICE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    Sp24Epi epi{};
    return b_mn ? launch_sp24<true>(vals, meta, M, K, B, ldb, C, ldc, N, epi, status_dev, st)
                : launch_sp24<false>(vals, meta, M, K, B, ldb, C, ldc, N, epi, status_dev, st);
}

extern "C" int sffn_sp24_mm(const sffn_sp24_mat* a, int64_t M, int64_t K, const void* B, int64_t ldb, int b_mn,
                            const void* bt, int64_t ldbt, void* C, int64_t ldc, int c_trans, int64_t N,
                            uint32_t* status_dev, void* stream) {
    if (M <= 0 || N <= 0 || K <= 0 || M % 128 || K % 128 || N % 32 || K > 65536) return SFFN_ERR_UNSUPPORTED;
    if (M > 0x7FFFFFFF || N > 0x7FFFFFFF) return SFFN_ERR_ARG;
    if (!a || !a->vals || !a->meta || !a->ovf_cols || !a->ovf_vals || !a->ovf_count || !B || !bt || !C ||
        !status_dev)
        return SFFN_ERR_ARG;
    if (!aligned16(a->vals) || !aligned16(a->meta) || !aligned16(B) || !aligned16(bt) || !aligned16(C) ||
        (ldb * 2) % 16 || (ldbt * 2) % 16 || (ldc * 2) % 16)
        return SFFN_ERR_ALIGN;
    if (ldb < (b_mn ? N : K) || ldbt < N || ldc < (c_trans ? M : N)) return SFFN_ERR_ARG;
    SFFN_BIND(dev_scope, a->vals);
    if (!device_is_sm100()) return SFFN_ERR_DEVICE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    Sp24Epi epi{};
    epi.ocols = static_cast<const uint16_t*>(a->ovf_cols);
    epi.ovals = static_cast<const uint16_t*>(a->ovf_vals);
    epi.ocount = a->ovf_count;
    epi.ovf_ld = K / 2;
    epi.bt = static_cast<const uint16_t*>(bt);
    epi.ldbt = ldbt;
    epi.c_trans = c_trans ? 1 : 0;
    return b_mn ? launch_sp24<true>(a->vals, a->meta, M, K, B, ldb, C, ldc, N, epi, status_dev, st)
                : launch_sp24<false>(a->vals, a->meta, M, K, B, ldb, C, ldc, N, epi, status_dev, st);
}

extern "C" int sffn_gemm_ck(const void* A, int64_t lda, int64_t kmax, const void* B, int64_t ldb, int64_t krows,
                            const int32_t* idx, int64_t ld_idx, const int32_t* kcount, void* C, int64_t ldc,
                            int64_t M, int64_t N, uint32_t* status_dev, void* stream) {
    // C[M, N] = Ac[M, :K(tm)] * B[idx[tm][:K(tm)], :] per 128-row tile tm.
    if (M <= 0 || N <= 0 || kmax <= 0 || krows <= 0 || M % 128 || N % CK_BN || kmax % 64) return SFFN_ERR_UNSUPPORTED;
    if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || kmax > 0x7FFFFFFF || krows > 0x7FFFFFFF) return SFFN_ERR_ARG;
    if (!A || !B || !C || !idx || !kcount || !status_dev || lda < kmax || ldb < N || ldc < N || ld_idx < kmax)
        return SFFN_ERR_ARG;
    if (!aligned16(A) || !aligned16(B) || !aligned16(idx) || (lda * 2) % 16 || (ldb * 2) % 16 || ld_idx % 4)
        return SFFN_ERR_ALIGN;
    DeviceScope dev_scope;
    if (int rc = dev_scope.bind_same(A, {B, C, idx, kcount, status_dev})) return rc;
    if (!device_is_sm100()) return SFFN_ERR_DEVICE;
    CkArgs a{};
    a.M = (int)M;
    a.N = (int)N;
    a.tiles_m = (int)(M / 128);
    a.tiles_n = (int)(N / CK_BN);
    a.idx = idx;
    a.ld_idx = ld_idx;
    a.kcount = kcount;
    a.out = static_cast<uint16_t*>(C);
    a.ldc = ldc;
    a.vec_out = aligned16(C) && (ldc * 2) % 16 == 0;
    a.status = status_dev;
    return launch_gemm_ck(A, lda, kmax, B, ldb, krows, a, reinterpret_cast<cudaStream_t>(stream));
}
