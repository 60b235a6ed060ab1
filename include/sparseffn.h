/*
 * sparseffn.h -- C ABI of the B200 (sm_100a) activation-sparse FFN library
 * (libsparseffn.so, sources in autoresearch2_b200/csrc/).
 *
 * Every entry point takes plain device pointers, int64 sizes, a dtype code and
 * a CUDA stream (as void*; NULL = the legacy default stream).  Nothing here
 * allocates device memory: callers pass every buffer, including scratch
 * ("workspace") whose size the *_workspace_bytes() query returns.  Work is
 * enqueued on the stream and the call returns without synchronising.
 *
 * Return value: SFFN_OK (0) or an SFFN_ERR_* code for errors found on the
 * host (bad argument, misalignment, launch failure).  Errors that only the
 * device can see (vals arena too small, a bounded wait that ran out) are
 * OR-ed into a caller-owned uint32 status word (SFFN_STATUS_* bits); read it
 * after the stream has been synchronised.
 *
 * dtype codes: SFFN_F32 = 0, SFFN_BF16 = 1, SFFN_F16 = 2.
 *
 * Each declaration names the reference function (Maccy-Z/autoresearch2,
 * path:line) whose behaviour it reproduces.
 */
#ifndef SPARSEFFN_H
#define SPARSEFFN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SFFN_F32 = 0,
    SFFN_BF16 = 1,
    SFFN_F16 = 2
};

enum {
    SFFN_OK = 0,
    SFFN_ERR_ARG = 1,         /* null pointer, negative or inconsistent size   */
    SFFN_ERR_DTYPE = 2,       /* dtype code not supported by this entry point  */
    SFFN_ERR_ALIGN = 3,       /* pointer or stride misaligned for this kernel  */
    SFFN_ERR_WORKSPACE = 4,   /* workspace smaller than *_workspace_bytes()    */
    SFFN_ERR_CUDA = 5,        /* a CUDA runtime call or kernel launch failed   */
    SFFN_ERR_UNSUPPORTED = 6, /* tile shape or GEMM layout not built           */
    SFFN_ERR_DEVICE = 7,      /* current device is not sm_100                  */
    SFFN_ERR_TOO_LARGE = 8    /* size beyond a fixed-capacity entry point      */
};

/* Bits OR-ed into the device status word. */
enum {
    SFFN_STATUS_VALS_OVERFLOW = 1u,  /* output would pass vals capacity; clipped  */
    SFFN_STATUS_WAIT_TIMEOUT = 2u,   /* a bounded spin-wait gave up               */
    SFFN_STATUS_CURSOR_OVERFLOW = 4u,/* int32 arena cursor would pass 2^31-1      */
    SFFN_STATUS_VALS_SHORT = 8u      /* mask has more set bits than vals holds    */
};

/* ---- library ----------------------------------------------------------- */

/* Version as 10000*major + 100*minor + patch. */
int sffn_version(void);

/* Static string for an SFFN_ERR_* code. */
const char* sffn_error_string(int code);

/* Text of the last CUDA error seen by this thread inside the library. */
const char* sffn_last_cuda_error(void);

/* ---- flat format --------------------------------------------------------
 * Element f of the row-major tensor -> byte f/8, bit f%8 of packed_mask (LSB
 * first; equal to bit f%32 of little-endian uint32 word f/32).  A bit is set
 * iff the element != 0 (-0.0 gives 0, NaN gives 1).  vals holds the set
 * elements in row-major order.  Tail bits of the last byte are 0.
 */

/* Scratch needed by sffn_flat_unpack for n elements: 16 bytes plus 8 per
 * 8192 elements. */
size_t sffn_flat_workspace_bytes(int64_t n);

/* Scratch needed by sffn_flat_pack (and its two halves) for n elements of
 * dtype: the unpack's tables plus a staging area of n elements rounded up
 * to 8192 (0 for a bad dtype). */
size_t sffn_flat_pack_workspace_bytes(int64_t n, int dtype);

/* bitsparse_pack(dense, block) -> (vals, packed_mask)
 *   replaces old/sparse_pack.py:66-106 (kernels :6-63) and
 *   old/bitpack/train.py:65-103 (compress_dense).
 * Two kernels: the first reads dense once, writing the mask bytes, per-tile
 * counts and each tile's set elements to its own segment of the workspace's
 * staging area; the second moves the values to their offsets.  Writes
 * ceil(n/8) bytes to packed_mask, the nonzeros to vals[0, nnz) (at most
 * vals_capacity are written; more sets SFFN_STATUS_VALS_OVERFLOW), and nnz
 * to *nnz_dev (device int64).  dense and workspace must be 16-byte aligned,
 * packed_mask 4-byte aligned; workspace_bytes >= sffn_flat_pack_workspace_bytes. */
int sffn_flat_pack(const void* dense, int dtype, int64_t n,
                   uint8_t* packed_mask, void* vals, int64_t vals_capacity,
                   int64_t* nnz_dev, void* workspace, size_t workspace_bytes,
                   uint32_t* status_dev, void* stream);

/* The two halves of sffn_flat_pack, for callers that size vals from the
 * count (as the reference does, old/sparse_pack.py:98): _count reads dense,
 * writes the mask and the staged values into the workspace and the total
 * into *nnz_dev; _values (same n, dtype and workspace, whose contents it
 * reads) writes the values to vals, as sffn_flat_pack does. */
int sffn_flat_pack_count(const void* dense, int dtype, int64_t n, uint8_t* packed_mask, int64_t* nnz_dev,
                         void* workspace, size_t workspace_bytes, void* stream);
int sffn_flat_pack_values(int dtype, int64_t n, void* vals, int64_t vals_capacity, int64_t* nnz_dev,
                          void* workspace, size_t workspace_bytes, uint32_t* status_dev, void* stream);

/* bitsparse_unpack(vals, packed_mask, shape, block) -> dense
 *   replaces old/sparse_unpack.py:57-97 (kernels :6-54) and
 *   old/bitunpack/train.py:55-90 (reconstruct_bitmask).
 * out[f] = bit f ? vals[rank(f)] : 0 for f < n.  Reads at most vals_len
 * values (a mask with more set bits sets SFFN_STATUS_VALS_SHORT).
 * out must be 16-byte aligned, packed_mask 4-byte aligned. */
int sffn_flat_unpack(const void* vals, int64_t vals_len, const uint8_t* packed_mask,
                     int dtype, int64_t n, void* out,
                     void* workspace, size_t workspace_bytes,
                     uint32_t* status_dev, void* stream);

/* sffn_flat_pack without a workspace argument, for callers that cannot
 * allocate device memory (plug-ins given only their buffers, programs whose
 * memory manager owns the device, paths that must not risk the
 * synchronisation of a cudaMalloc).  No counterpart in the reference.  Same
 * inputs, outputs and results as sffn_flat_pack; the look-back scratch is a
 * fixed 32 KB array in this library's device memory (held on every GPU that
 * loads the library until exit).  Allocates and frees nothing.  n is at most
 * 67,108,864 (bf16, fp16) or 33,554,432 (fp32); larger n returns
 * SFFN_ERR_TOO_LARGE with the limit in sffn_last_cuda_error().  The
 * first call on a device (in each CUDA context of it) looks up the array's
 * address (make it before any stream capture); calls share the array, so
 * calls that overlap on the GPU race and must be serialised by the caller.
 * The device is the one that owns dense (nnz_dev's for n == 0); every other
 * pointer must live on it (else SFFN_ERR_ARG).  The caller's current device
 * (context) is the same on return as on entry. */
int sffn_flat_pack_noalloc(const void* dense, int dtype, int64_t n,
                           uint8_t* packed_mask, void* vals, int64_t vals_capacity,
                           int64_t* nnz_dev, uint32_t* status_dev, void* stream);

/* ---- tiled format -------------------------------------------------------
 * A row-major [M, N] matrix (row stride ld elements) is cut into BM x BN tiles;
 * tile t = tm * grid_n + tn.  In-tile offset f = r*BN + c -> byte
 * t*BM*BN/8 + f/8, bit f%8.  A bit is set iff the element > 0 (negatives,
 * +-0 and NaN give 0); elements outside the matrix give 0 bits.
 * prefix[t] = number of set bits in tiles < t, prefix[num_tiles] = total.
 * Tile t's values, row-major in the tile, sit at vals[vals_offset + prefix[t]].
 * Supported (BM, BN): (32, 32), (64, 64), (128, 128), (64, 128), (128, 64).
 * Readers take the length of the vals buffer (vals_len) and never read or
 * write outside it; M*N must stay below 2^31 (int32 prefix, as in the reference).
 */

/* Scratch needed by sffn_tile_pack for an [M, N] matrix. */
size_t sffn_tile_workspace_bytes(int64_t M, int64_t N, int BM, int BN);

/* dense_to_tilesparse(dense, vals, offset, BLOCK_M, BLOCK_N) -> BitsparseTensor
 *   replaces old/lib_sparse/sparse.py:154-210 (kernels sparse_pack.py:27-92)
 *   and old/full_matmul/sparse_pack.py:95-146.
 * Three launches over independent tiles: mask words and per-tile counts
 * (into the workspace), one scan of the counts, then each tile read again
 * and its values written.  Reads the int32 arena cursor *offset_dev, writes
 * it to *vals_offset_dev, writes bitmask, prefix[num_tiles+1] and the values
 * to vals[cursor + prefix[t] ...] (never past vals_capacity), and advances
 * *offset_dev by the total -- all on the device, no host sync.  With vals
 * NULL (and vals_capacity 0) only the first two launches run: bitmask,
 * prefix and the cursor, so that a caller can size vals exactly from
 * prefix[num_tiles] and then run sffn_tile_pack_values. */
int sffn_tile_pack(const void* dense, int dtype, int64_t M, int64_t N, int64_t ld,
                   int BM, int BN, uint8_t* bitmask, int32_t* prefix,
                   void* vals, int64_t vals_capacity,
                   int32_t* offset_dev, int32_t* vals_offset_dev,
                   void* workspace, size_t workspace_bytes,
                   uint32_t* status_dev, void* stream);

/* The third launch of sffn_tile_pack alone: each tile of dense read again and
 * its values written to vals[*vals_offset_dev + prefix[t] ...] (never past
 * vals_capacity), after sffn_tile_pack with vals NULL made bitmask and
 * prefix (no counterpart in the reference, which sizes vals with a host
 * sync inside its pack, old/full_matmul/sparse_pack.py:128). */
int sffn_tile_pack_values(const void* dense, int dtype, int64_t M, int64_t N, int64_t ld,
                          int BM, int BN, const uint8_t* bitmask, const int32_t* prefix,
                          void* vals, int64_t vals_capacity, const int32_t* vals_offset_dev,
                          uint32_t* status_dev, void* stream);

/* Unpack tile rows [tile_row0, tile_row0 + tile_rows) into out (row stride
 * ld_out; out row 0 = matrix row tile_row0*BM).  `square` holds flags: bit 0
 * squares each value in the storage dtype (spAx(..., square=True)), bit 1
 * rounds float32 output values to the nearest TF32 value (ties away from
 * zero; the operand of a TF32 product).  out_dtype is dtype or SFFN_F32
 * (old/full_matmul/sparse_unpack.py:62 returns float32).
 *   replaces old/lib_sparse/sparse_unpack.py:5-55 (_unpack_batch_kernel, with
 *   column bounds added), old/full_matmul/sparse_unpack.py:6-73,
 *   old/full_matmul/train.py:89-137. */
int sffn_tile_unpack(const void* vals, int64_t vals_len, const uint8_t* bitmask,
                     const int32_t* prefix, const int32_t* vals_offset_dev, int dtype,
                     int64_t M, int64_t N, int BM, int BN,
                     int64_t tile_row0, int64_t tile_rows, int square,
                     void* out, int out_dtype, int64_t ld_out, void* stream);

/* grad[r, c] = bit ? grad[r, c] : 0, in place (ReLU backward from the mask).
 *   replaces old/lib_sparse/sparse_unpack.py:72-107 (_mask_with_bitmask_kernel). */
int sffn_tile_mask_grad(void* grad, int dtype, int64_t M, int64_t N, int64_t ld,
                        const uint8_t* bitmask, int BM, int BN, void* stream);

/* grad <- (grad * 2) * z in the storage dtype, z gathered from vals (0 off the
 * mask, so a NaN/Inf grad there gives NaN like the reference); if square,
 * vals <- z*z in place.
 *   replaces old/lib_sparse/sparse_unpack.py:110-147 (_grad_relu2_kernel). */
int sffn_tile_grad_relu2(void* grad, int dtype, int64_t M, int64_t N, int64_t ld,
                         void* vals, int64_t vals_len, const uint8_t* bitmask, const int32_t* prefix,
                         const int32_t* vals_offset_dev, int BM, int BN, int square,
                         void* stream);

/* ---- tensor-core GEMMs and the fused sparse FFN ---------------------------
 * bf16 operands, fp32 accumulation in tensor memory (tcgen05), bf16 output.
 * Operand bases and row strides must be 16-byte aligned (ld % 8 == 0).
 */

/* C[M, N] = A[M, K] @ B[N, K]^T.
 * a_mn = 0: A stored [M][lda] (K contiguous); a_mn = 1: A stored [K][lda]
 * (M contiguous, i.e. the transpose of a row-major [K, M] tensor).  Same for
 * B with N.  Optional kb_list/kb_count (both or neither): for row tile
 * m = row/256, only the kb_count[m] 64-wide K blocks listed in
 * kb_list[m*kb_stride ...] are accumulated (the others are known to be zero).
 *   replaces the torch/cuBLAS matmuls of old/lib_sparse/sparse.py:72-149 and
 *   prepare_layer.py:25-27,131-160 (x@W1.T, z@W2.T, grad@W2, grad.T@z,
 *   grad@W1, grad.T@x). */
int sffn_gemm_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                   void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                   const int32_t* kb_list, const int32_t* kb_count, int kb_stride,
                   uint32_t* status_dev, void* stream);

/* sffn_gemm_bf16 with C stored transposed: Ct[n*ldct + m] = C[m][n] (Ct
 * 16-byte aligned, ldct*2 a multiple of 16).  With kb_list/kb_count the K
 * skipping applies per 256-row tile of A as in sffn_gemm_bf16; the weight
 * gradient dW2 = dout^T @ a is computed as (a^T @ dout)^T so that the skip
 * lists of sffn_live_kblocks_t (per 256 activation columns) apply.  No
 * reference counterpart (the reference's dW2 is a dense torch matmul inside
 * spAx, old/lib_sparse/sparse.py:305-351). */
int sffn_gemm_bf16_ct(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                      void* Ct, int64_t ldct, int64_t M, int64_t N, int64_t K,
                      const int32_t* kb_list, const int32_t* kb_count, int kb_stride,
                      uint32_t* status_dev, void* stream);

/* float32 / float16 products on the bf16 tensor cores.  sffn_split_bf16x3
 * writes src (rows x cols, element (r, c) at src[r*s_row + c*s_col], dtype
 * SFFN_F32 or SFFN_F16) as six blocks of cols bf16 per row of dst (ld_dst >=
 * 6*cols): x = hi + mid + lo (hi = bf16(x), mid = bf16(x - hi), lo =
 * bf16(x - hi - mid)), the blocks ordered hi hi mid hi lo mid (b_order 0,
 * for A [M][K]) or hi mid hi lo hi mid (b_order 1, for B^T [N][K]).
 * sffn_gemm_bf16_f32out multiplies such an A by such a B over 6*cols (C in
 * float32): hi*hi + hi*mid + mid*hi + hi*lo + lo*hi + mid*mid, the float32
 * product up to terms of relative size 2^-24, accumulated in float32.  They
 * replace the float32 torch matmuls of old/lib_sparse/sparse.py:72-75,
 * 92,106-107,116-118,132,148-149 and spAx's (sparse.py:305-351). */
int sffn_split_bf16x3(const void* src, int dtype, int64_t rows, int64_t cols, int64_t s_row, int64_t s_col,
                      void* dst, int64_t ld_dst, int b_order, void* stream);
int sffn_gemm_bf16_f32out(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                          float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int relu,
                          uint32_t* status_dev, void* stream);

/* C = max(A @ B, 0): bf16 operands and optional K-block lists as
 * sffn_gemm_bf16 takes them, C bf16 (out_f32 == 0) or float32 [M][ldc], the
 * ReLU applied by the epilogue.  The products of relu_spAx
 * (old/full_matmul/train.py:140-184: F.relu(F.linear(unpacked rows, W2)))
 * and relu_sparse_Ax (old/sparse_matmul/train.py:56-76: relu(A @ x) stored
 * in float32). */
int sffn_gemm_relu(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                   void* C, int out_f32, int64_t ldc, int64_t M, int64_t N, int64_t K,
                   const int32_t* kb_list, const int32_t* kb_count, int kb_stride,
                   uint32_t* status_dev, void* stream);

/* C (float32, [M][ldc]) = A @ B, or C += A @ B with accumulate != 0 (the
 * epilogue adds into C in float32, round to nearest), bf16 operands as
 * sffn_gemm_bf16 takes them, in one pass over K: spAx's row batches
 * accumulate into one float32 result this way (old/lib_sparse/sparse.py:
 * 321-351 accumulates them in the storage dtype with a separate add). */
int sffn_gemm_bf16_f32acc(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                          float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int accumulate,
                          uint32_t* status_dev, void* stream);

/* C (float32, [M][ldc]) = A @ B^T, A [M][lda] and B [N][ldb] float32
 * row-major (16-byte aligned bases, lda and ldb multiples of 4), read as
 * TF32 by the tensor cores (tcgen05 kind::tf32), float32 accumulation;
 * relu != 0 stores max(C, 0).  The float32 product of sparse_relu_Ax at its
 * default input_precision "tf32" (old/matmul_bitsparse/train.py:45-52,
 * tl.dot(..., input_precision="tf32") then tl.maximum(acc, 0)). */
int sffn_gemm_tf32(const float* A, int64_t lda, const float* B, int64_t ldb, float* C, int64_t ldc,
                   int64_t M, int64_t N, int64_t K, int relu, uint32_t* status_dev, void* stream);

/* dst[i] = src[i] rounded to the nearest TF32 value (ties away from zero),
 * as float32 (in place when dst == src).  The tensor cores' kind::tf32 read
 * keeps the top 19 bits of each operand (truncation, as Triton's tl.dot at
 * input_precision "tf32"); operands rounded first give the products of
 * cuBLAS's TF32 GEMMs behind F.linear under set_float32_matmul_precision
 * ("high") (old/full_matmul/train.py:35,177-178). */
int sffn_round_tf32(const float* src, float* dst, int64_t n, void* stream);

/* Fused up-projection: pre = bf16(x @ W1^T [+ b1]), z = relu(pre).
 * Writes act_out = z*z (act = 1, ReLU^2) or z (act = 0, ReLU) densely
 * (unless act_out is NULL: the compacted-K down-projection needs none), the
 * tiled 128x128 bitmask of z > 0 (ceil(T/128)*ceil(F/128) tiles of 2048 B),
 * four partial counts per tile (tile_counts[t*4 .. t*4+3]) and z's values:
 *  - slot_rows NULL: row r of tile t in order at slots[t*16384 + r*128 ...];
 *    finish the BitsparseTensor with sffn_tile_scan_counts (parts = 4) and
 *    sffn_tile_gather_slots;
 *  - slot_rows given (warp-packed): rows 32w .. 32w+31 of tile t in the order
 *    of the arena (row-major) at slots[t*16384 + w*4096 ...] (their count is
 *    tile_counts[t*4 + w]), and slot_rows[t*128 + r] = the values in the rows
 *    of r's group of 32 before r; finish with sffn_tile_scan_counts and
 *    sffn_tile_copy_slots (one contiguous copy per group), passing slot_rows
 *    there as row_offsets.
 *   replaces old/lib_sparse/sparse.py:72-77,116-120 (matmul, relu, square,
 *   dense_to_tilesparse) and old/matmul_bitsparse/train.py:11-116
 *   (_matmul_sparse_kernel + compaction). */
int sffn_ffn_up(const void* x, int64_t ldx, const void* w1, int64_t ldw1, const void* b1,
                int64_t T, int64_t D, int64_t F, int act, void* act_out, int64_t ld_act,
                uint8_t* bitmask, int32_t* tile_counts, void* slots, int32_t* slot_rows,
                uint32_t* status_dev, void* stream);

/* prefix[t] = sum over tiles < t of (tile_counts[t*parts] + ... + [t*parts+parts-1]),
 * prefix[ntiles] = total; *vals_offset_dev = *offset_dev; *offset_dev += total.
 *   replaces old/lib_sparse/sparse.py:181-186,200-204 (cumsum, cursor). */
int sffn_tile_scan_counts(const int32_t* tile_counts, int parts, int64_t ntiles, int32_t* prefix,
                          int32_t* offset_dev, int32_t* vals_offset_dev, uint32_t* status_dev,
                          void* stream);

/* For 128x128 tiles: moves row r of tile t from slots[t*16384 + r*128 ...]
 * (count = popcount of the row's mask) to
 * vals[*vals_offset_dev + prefix[t] + values in rows < r ...] (16-bit
 * dtypes; never past vals_capacity) and, if row_offsets is not NULL, writes
 * row_offsets[t*128 + r] = prefix[t] + values in rows < r.  If colmask is
 * not NULL (16-byte aligned, 4 uint32 per tile), colmask[t*4 .. t*4+3] =
 * the OR of tile t's 128 rows of mask words: its live columns.
 *   replaces old/lib_sparse/sparse_pack.py:65-92 (_compact_vals_kernel). */
int sffn_tile_gather_slots(const void* slots, const uint8_t* bitmask, const int32_t* prefix,
                           const int32_t* vals_offset_dev, int64_t ntiles, void* vals,
                           int64_t vals_capacity, int dtype, int32_t* row_offsets,
                           uint32_t* colmask, uint32_t* status_dev, void* stream);

/* For 128x128 tiles and the warp-packed slots of sffn_ffn_up: for each group
 * w = 0..3 of 32 rows of tile t, copies tile_counts[t*4 + w] values from
 * slots[t*16384 + w*4096 ...] to vals[*vals_offset_dev + prefix[t] + the
 * counts of the groups before w ...] (16-bit dtypes; never past
 * vals_capacity) and adds prefix[t] plus those counts to the group's
 * row_offsets (the offsets in the group's run sffn_ffn_up wrote), which then
 * hold what sffn_tile_gather_slots writes there.  tile_counts 16-byte
 * aligned.  colmask (optional) as in sffn_tile_gather_slots, read from
 * bitmask (which may be NULL without it).
 *   replaces old/lib_sparse/sparse_pack.py:65-92 (_compact_vals_kernel). */
int sffn_tile_copy_slots(const void* slots, const int32_t* tile_counts, const int32_t* prefix,
                         const int32_t* vals_offset_dev, int64_t ntiles, void* vals, int64_t vals_capacity,
                         int32_t* row_offsets, const uint8_t* bitmask, uint32_t* colmask,
                         uint32_t* status_dev, void* stream);

/* row_offsets[t*128 + r] = prefix[t] + number of values in rows < r of tile t,
 * for a tiled 128x128 bitmask (the per-row index sffn_ffn_dgrad reads; the
 * reference recomputes ranks with tl.cumsum in every kernel,
 * old/lib_sparse/sparse_unpack.py:142,237); colmask (optional) as in
 * sffn_tile_gather_slots.  Either output may be NULL, not both. */
int sffn_tile_row_offsets(const uint8_t* bitmask, const int32_t* prefix, int64_t ntiles,
                          int32_t* row_offsets, uint32_t* colmask, void* stream);

/* For a tiled 128x128 bitmask of an [M, N] matrix: kb_count[m] and the
 * ascending list kb_list[m*ceil(N/64) ...] of 64-column blocks of 256-row
 * tile m (rows 256m .. 256m+255) that hold any set bit -- the K-skip lists
 * sffn_gemm_bf16 takes (no reference counterpart: the reference's
 * down-projection is dense, sparse.py:75,118). */
int sffn_live_kblocks(const uint8_t* bitmask, int64_t M, int64_t N, int32_t* kb_list,
                      int32_t* kb_count, void* stream);

/* The transposed lists, for the weight gradients (contractions over the M
 * rows of the activation): for each 256-column tile p of the [M, N] tiled
 * bitmask, kb_count[p] and the ascending list kb_list[p*ceil(M/64) ...] of
 * 64-row blocks holding any set bit.  Used by dW1 = dpre^T @ x and
 * dW2 = (a^T @ dout)^T (no reference counterpart, as above). */
int sffn_live_kblocks_t(const uint8_t* bitmask, int64_t M, int64_t N, int32_t* kb_list,
                        int32_t* kb_count, void* stream);

/* ---- compacted-K down-projection -----------------------------------------
 * The bitmask-sparse down-projection out = act(z) @ W2^T (and dX = dpre @ W1)
 * over each 128-row tile's live columns only.  The reference's forward is a
 * dense z @ W2.T (old/lib_sparse/sparse.py:75,118) and its sparse-operand
 * product unpacks to dense first (spAx, sparse.py:305-351); these replace
 * both with a contraction over the compacted K.  T % 128 == 0, F % 64 == 0,
 * F <= 65536; the live columns of format tile t come from the colmask of
 * sffn_tile_gather_slots / sffn_tile_row_offsets. */

/* Per 128-row tile tm of a [T, F] 128x128-tiled activation: kcount[tm] =
 * live columns K, idx[tm*ld_idx + j] (j < K) = the live columns in ascending
 * order, padded up to a multiple of 64 with a column that is zero in every
 * row of the tile, and colpref[tm*ceil(F/128) + n] = live columns of the
 * tile's blocks before block n (where block n's live columns start in the
 * list).  With idx NULL only kcount is written (colpref must then be NULL). */
int sffn_ck_lists(const uint32_t* colmask, int64_t T, int64_t F, int32_t* idx, int64_t ld_idx,
                  int32_t* kcount, int32_t* colpref, void* stream);

/* The compacted activation from the packed z (tiled 128x128 vals, bitmask,
 * prefix, row_offsets, *vals_offset_dev): ac[row*ld_ac + j] = act(z[row][idx[tm][j]])
 * for j < kcount[tm] (act = 1: bf16(z*z), ReLU^2; act = 0: z) -- zero where
 * the row's bit is clear -- and zeros from kcount[tm] up to the padded
 * count.  No dense activation is formed. */
int sffn_ck_gather_packed(const void* vals, int64_t vals_len, const uint8_t* bitmask,
                          const int32_t* prefix, const int32_t* row_offsets, const int32_t* vals_offset_dev,
                          const uint32_t* colmask, const int32_t* colpref, const int32_t* kcount,
                          int64_t T, int64_t F, int act, void* ac, int64_t ld_ac, uint32_t* status_dev,
                          void* stream);

/* In place: x[row][j] = x[row][idx[tm][j]] for j below tile tm's padded
 * count (16-bit elements, [T, ld]); rows of tiles with every column live are
 * left as they are.  Compacts a dense activation gradient whose zeros follow
 * the activation's (dpre of the ReLU / ReLU^2 backward). */
int sffn_ck_compact_rows(void* x, int64_t ld, int64_t T, int64_t F, const int32_t* idx, int64_t ld_idx,
                         const int32_t* kcount, void* stream);

/* C[M, N] (bf16, fp32 accumulation) = for each 128-row tile tm,
 * A[rows, 0:Kp] @ B[idx[tm][0:Kp], :], Kp = kcount[tm] rounded up to 64:
 * A [M][lda] K-major (the compacted activation, kmax >= every Kp columns
 * addressable), B [krows][ldb] with rows = the contraction index (W2^T for
 * the down-projection, W1 for dX), gathered by TMA.  M % 128 == 0,
 * N % 256 == 0, kmax % 64 == 0. */
int sffn_gemm_ck(const void* A, int64_t lda, int64_t kmax, const void* B, int64_t ldb, int64_t krows,
                 const int32_t* idx, int64_t ld_idx, const int32_t* kcount, void* C, int64_t ldc,
                 int64_t M, int64_t N, uint32_t* status_dev, void* stream);

/* Fused activation gradient: g = bf16(dout @ W2) ([T, F]; W2 is [D, F]).
 * ReLU^2 (act = 1): dpre = bf16((g*2) * z) and act_out = bf16(z*z); ReLU
 * (act = 0): dpre = bit ? g : 0 and act_out = z -- z gathered from the
 * tiled 128x128 BitsparseTensor (vals, bitmask, *vals_offset_dev) at the
 * row offsets of sffn_tile_row_offsets.  act_out may be NULL (no second
 * output: a caller that rebuilt the activation already).
 * If db1_sum is not NULL, the column sums of dpre (the bias gradient, over
 * the T rows) are added into db1_sum[F] in fp32 (zero it first; the order of
 * the additions is not fixed).
 *   replaces old/lib_sparse/sparse.py:92-102,132-145 (grad_output @ W2 with
 *   _mask_with_bitmask_kernel / _grad_relu2_kernel) and the unpack inside spAx
 *   (sparse.py:305-351). */
int sffn_ffn_dgrad(const void* dout, int64_t ld_dout, const void* w2, int64_t ldw2,
                   int64_t T, int64_t D, int64_t F, int act, const void* vals, int64_t vals_len,
                   const uint8_t* bitmask, const int32_t* row_offsets, const int32_t* vals_offset_dev,
                   void* dpre_out, void* act_out, int64_t ld_out, float* db1_sum, uint32_t* status_dev,
                   void* stream);

/* ---- 2:4 structured form for the sparse tensor-core GEMMs -------------------
 * No counterpart in the reference, whose products are dense cuBLAS matmuls
 * (old/lib_sparse/sparse.py:75,95-100,118,136-139); the sparse path is
 * checked end to end against dense products.  A [M, K] (M, K multiples of
 * 128, K <= 65536) splits into its 2:4 part -- per group of 4 consecutive K
 * elements the first two non-zeros: vals [M, K/2] bf16 and meta
 * [M/128][K/128][128 lanes][4] uint32, index nibbles in tensor-memory lane
 * order (lane dp = m0 + 8*k1 + 16*m2: K-half k1 of 32-wide step j, rows
 * 16*m2+m0 in bits 0-15 and 16*m2+m0+8 in bits 16-31) -- and its overflow,
 * the 3rd and 4th non-zero of a group, per row r at ovf_cols/ovf_vals
 * [r*(K/2) ...], ovf_count[r] entries (in no fixed order). */

/* Compress A (trans = 0: src is A [M][ld]; trans = 1: src is X [K][ld] and
 * A = X^T) into the 2:4 form.  16-bit dtypes. */
int sffn_sp24_compress(const void* src, int64_t ld, int trans, int64_t M, int64_t K, void* vals,
                       uint32_t* meta, void* ovf_cols, void* ovf_vals, int32_t* ovf_count, void* stream);

/* C[M, N] (bf16, row stride ldc) = A24 @ B for the 2:4 part of A, where B is
 * [K, N]: b_mn = 1 for B stored [K][ldb] (N contiguous), 0 for B stored
 * [N][ldb] (K contiguous).  bf16 in, fp32 accumulation. */
int sffn_gemm_sp24(const void* vals, const uint32_t* meta, int64_t M, int64_t K, const void* B, int64_t ldb,
                   int b_mn, void* C, int64_t ldc, int64_t N, uint32_t* status_dev, void* stream);

/* C[r, :] += sum over row r's overflow entries (k, v) of v * Bt[k, :]
 * (Bt = B as [K][ldb] row-major, N % 16 == 0), accumulated in fp32
 * and rounded once to bf16. */
int sffn_sp24_overflow_add(const void* ovf_cols, const void* ovf_vals, const int32_t* ovf_count, int64_t M,
                           int64_t K, const void* bt, int64_t ldb, int64_t N, void* C, int64_t ldc,
                           void* stream);

/* dst[c][r] = src[r][c] for a 16-bit [rows][ld_src] matrix (rows and cols
 * multiples of 8, 16-byte aligned rows): B^T for sffn_sp24_mm's bt when B is
 * a transposed view. */
int sffn_transpose16(const void* src, int64_t ld_src, int64_t rows, int64_t cols, void* dst, int64_t ld_dst,
                     void* stream);

/* One matrix in the 2:4 form above: vals [M, K/2], meta, overflow columns
 * (uint16), values and per-row counts. */
typedef struct sffn_sp24_mat {
    void* vals;
    uint32_t* meta;
    void* ovf_cols;
    void* ovf_vals;
    int32_t* ovf_count;
} sffn_sp24_mat;

/* The full product of a 2:4 matrix A (a, [M, K]) with B [K, N] (B as in
 * sffn_gemm_sp24): the 2:4 part on the sparse tensor cores and the overflow
 * added in the same kernel from bt, B as row-major [K][ldbt] (bt may be B
 * itself when b_mn = 1).  The 2:4 part is rounded to bf16, the overflow added
 * in fp32 and the sum rounded to bf16.  c_trans = 0: C is [M][ldc]; 1: C^T
 * is stored, [N][ldc].  M, K multiples of 128 (K <= 65536), N of 32. */
int sffn_sp24_mm(const sffn_sp24_mat* a, int64_t M, int64_t K, const void* B, int64_t ldb, int b_mn,
                 const void* bt, int64_t ldbt, void* C, int64_t ldc, int c_trans, int64_t N,
                 uint32_t* status_dev, void* stream);

/* sffn_ffn_up with the activation a written in the 2:4 form (out, K = F)
 * instead of dense; bitmask, tile counts, slots and slot_rows (NULL: per-row
 * slots; given: warp-packed) as there.  T and F multiples of 128,
 * F <= 65536.  The 2:4 form is bit-identical to sffn_sp24_compress of the
 * dense a (overflow order aside). */
int sffn_ffn_up_sp24(const void* x, int64_t ldx, const void* w1, int64_t ldw1, const void* b1, int64_t T,
                     int64_t D, int64_t F, int act, const sffn_sp24_mat* out, uint8_t* bitmask,
                     int32_t* tile_counts, void* slots, int32_t* slot_rows, uint32_t* status_dev,
                     void* stream);

/* sffn_ffn_dgrad with its outputs in the 2:4 form instead of dense:
 * dpre [T, F] (K = F, for dX = dpre @ W1), dpre^T [F, T] and act^T [F, T]
 * (K = T, for dW1 = dpre^T @ x and dW2^T = act^T @ dout); db1_sum as there.
 * T and F multiples of 128, both <= 65536. */
int sffn_ffn_dgrad_sp24(const void* dout, int64_t ld_dout, const void* w2, int64_t ldw2, int64_t T, int64_t D,
                        int64_t F, int act, const void* vals, int64_t vals_len, const uint8_t* bitmask,
                        const int32_t* row_offsets, const int32_t* vals_offset_dev, const sffn_sp24_mat* dpre,
                        const sffn_sp24_mat* dpre_t, const sffn_sp24_mat* act_t, float* db1_sum,
                        uint32_t* status_dev, void* stream);

/* ---- 15-bit sign-strip codec --------------------------------------------
 * n 16-bit words (bf16 / fp16 bit patterns of non-negative values) <-> a byte
 * stream of ceil(15 n / 8) bytes, value i at stream bits [15 i, 15 i + 15),
 * little-endian.  The bytes are the reference's for every input: a set sign
 * bit of word i is OR-ed into stream bit 15 (i + 1) unless i % 8 == 7, as
 * its byte formula does (bitshifting/code.py:39-69).  Word and byte buffers
 * must not overlap; words are 2-byte aligned.  Sizes up to 2^40 words.
 */

/* ceil(15 n / 8): packed bytes of n words (bitshifting/code.py:135); -1 for n < 0. */
int64_t sffn_codec15_bytes(int64_t n);

/* compress_fn(data) (bitshifting/code.py:129-160): writes exactly
 * sffn_codec15_bytes(n) bytes of dst (dst_bytes may be larger; the rest is
 * left as it is -- the reference leaves its 8-9 padding bytes unset too). */
int sffn_codec15_compress(const void* src, int64_t n, uint8_t* dst, int64_t dst_bytes, void* stream);

/* uncompress_fn(compressed, shape, dtype) (bitshifting/code.py:163-177):
 * dst[i] = field i (sign bit 0).  Reads only the first sffn_codec15_bytes(n)
 * of src's src_bytes. */
int sffn_codec15_uncompress(const uint8_t* src, int64_t src_bytes, int64_t n, void* dst, void* stream);

/* ---- bounded waits ------------------------------------------------------ */

/* Test hook, no counterpart in the reference.  Runs one of this library's
 * bounded device waits on a condition that never comes true, giving up after
 * limit_ns (0 < limit_ns <= 100 ms) instead of the 500 ms the kernels use:
 * kind 0 waits on an mbarrier that nothing arrives on (the GEMM and pack
 * pipelines' wait), kind 1 is a decoupled look-back over predecessors that
 * never publish (the tiled and flat packs' wait) and needs 64 uint64 of
 * device memory in `states` (cleared by the call).  The wait records
 * SFFN_STATUS_WAIT_TIMEOUT in *status_dev and the kernel returns; when
 * elapsed_ns_dev is non-null it receives the wait's duration (%globaltimer). */
int sffn_wait_probe(int kind, int64_t limit_ns, uint64_t* states, uint64_t* elapsed_ns_dev,
                    uint32_t* status_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSEFFN_H */
