/*
 * CPU oracle for the bitmask-sparse formats (test infrastructure only).
 *
 * This file restates, in plain C, the algorithms of the reference's Triton
 * kernels for the two bitmask formats.  It is the checker for the CUDA
 * library and the timed CPU baseline; nothing in the product links it.
 *
 * Flat format (old/sparse_pack.py:6-106, old/sparse_unpack.py:6-97,
 * golden packer old/bitpack/prepare.py:6-23):
 *   element f of the row-major flattened tensor -> byte f/8, bit f%8 of the
 *   uint8 mask (LSB first); the bit is set iff x != 0 (old/sparse_pack.py:21),
 *   so -0.0 gives 0 and NaN gives 1.  vals = the set elements in row-major
 *   order.  Tail bits of the last byte are 0.
 *
 * Tiled format (old/lib_sparse/sparse_pack.py:27-92, sparse.py:154-210):
 *   tile t = tm * grid_n + tn of BM x BN elements; in-tile offset
 *   f = r * BN + c -> byte t*BM*BN/8 + f/8, bit f%8.  The bit is set iff
 *   x > 0 (sparse_pack.py:48,88): negatives, +-0 and NaN give 0.  Elements
 *   outside the matrix give 0 bits.  prefix[t] = sum of counts of tiles < t,
 *   prefix[num_tiles] = total; tile t's values are written in row-major in-tile
 *   order to vals[offset + prefix[t] + rank] (sparse_pack.py:75-92), and the
 *   cursor advances by the total (sparse.py:200-204).
 *   Unpack (sparse_unpack.py:5-55): dense[r,c] = bit ? vals[offset+prefix[t]+rank] : 0.
 *
 * Comparisons are done on bit patterns, which matches IEEE float compares:
 *   x != 0  <=>  (bits & ~sign) != 0
 *   x >  0  <=>  sign == 0 && (bits & ~sign) != 0 && (bits & ~sign) <= +inf
 *
 * dtype codes: 0 = float32, 1 = bfloat16, 2 = float16.
 * Build: oracle/Makefile (gcc -O3 -pthread -shared).  The flat routines split
 * the tensor into 8192-element chunks handled by `nthreads` POSIX threads
 * (count pass, serial exclusive scan, scatter pass).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* Minimal parallel-for over [0, n) in contiguous slices, one per thread. */
typedef void (*range_fn)(void* ctx, int64_t lo, int64_t hi);
typedef struct { range_fn fn; void* ctx; int64_t lo, hi; } slice_t;

static void* run_slice(void* p) {
    slice_t* s = (slice_t*)p;
    s->fn(s->ctx, s->lo, s->hi);
    return NULL;
}

static void parallel_for(int64_t n, int nthreads, range_fn fn, void* ctx) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > n) nthreads = n > 0 ? (int)n : 1;
    pthread_t th[256];
    slice_t sl[256];
    int started[256];
    for (int i = 0; i < nthreads; ++i) {
        sl[i].fn = fn; sl[i].ctx = ctx;
        sl[i].lo = n * i / nthreads; sl[i].hi = n * (i + 1) / nthreads;
        started[i] = 0;
        if (i > 0) started[i] = pthread_create(&th[i], NULL, run_slice, &sl[i]) == 0;
        if (i > 0 && !started[i]) run_slice(&sl[i]);
    }
    run_slice(&sl[0]);
    for (int i = 1; i < nthreads; ++i) if (started[i]) pthread_join(th[i], NULL);
}

static inline uint32_t load_bits(const void* p, int dtype, int64_t i) {
    if (dtype == 0) return ((const uint32_t*)p)[i];
    return ((const uint16_t*)p)[i];
}

static inline void store_bits(void* p, int dtype, int64_t i, uint32_t v) {
    if (dtype == 0) ((uint32_t*)p)[i] = v;
    else ((uint16_t*)p)[i] = (uint16_t)v;
}

static inline int is_nonzero(uint32_t b, int dtype) {
    uint32_t mag = dtype == 0 ? (b & 0x7FFFFFFFu) : (b & 0x7FFFu);
    return mag != 0;
}

static inline int is_positive(uint32_t b, int dtype) {
    uint32_t sign, mag, inf;
    if (dtype == 0) { sign = b >> 31; mag = b & 0x7FFFFFFFu; inf = 0x7F800000u; }
    else if (dtype == 1) { sign = b >> 15; mag = b & 0x7FFFu; inf = 0x7F80u; }
    else { sign = b >> 15; mag = b & 0x7FFFu; inf = 0x7C00u; }
    return sign == 0 && mag != 0 && mag <= inf;
}

int orc_num_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

#define CH 8192
typedef struct {
    const void* src; void* dst; const uint8_t* mask_in; uint8_t* mask_out;
    int dtype; int64_t n; int64_t* cnt;
} flat_ctx;

static void flat_pack_count(void* p, int64_t c0, int64_t c1) {
    flat_ctx* x = (flat_ctx*)p;
    for (int64_t c = c0; c < c1; ++c) {
        int64_t lo = c * CH, hi = lo + CH < x->n ? lo + CH : x->n, k = 0;
        for (int64_t byte = lo / 8; byte * 8 < hi; ++byte) {
            uint8_t v = 0;
            for (int j = 0; j < 8; ++j) {
                int64_t f = byte * 8 + j;
                if (f < x->n && is_nonzero(load_bits(x->src, x->dtype, f), x->dtype)) {
                    v |= (uint8_t)(1u << j);
                    ++k;
                }
            }
            x->mask_out[byte] = v;
        }
        x->cnt[c + 1] = k;
    }
}

static void flat_pack_scatter(void* p, int64_t c0, int64_t c1) {
    flat_ctx* x = (flat_ctx*)p;
    for (int64_t c = c0; c < c1; ++c) {
        int64_t lo = c * CH, hi = lo + CH < x->n ? lo + CH : x->n, o = x->cnt[c];
        for (int64_t f = lo; f < hi; ++f) {
            uint32_t b = load_bits(x->src, x->dtype, f);
            if (is_nonzero(b, x->dtype)) store_bits(x->dst, x->dtype, o++, b);
        }
    }
}

static void flat_unpack_count(void* p, int64_t c0, int64_t c1) {
    flat_ctx* x = (flat_ctx*)p;
    for (int64_t c = c0; c < c1; ++c) {
        int64_t lo = c * CH, hi = lo + CH < x->n ? lo + CH : x->n, k = 0;
        for (int64_t f = lo; f < hi; ++f) k += (x->mask_in[f >> 3] >> (f & 7)) & 1;
        x->cnt[c + 1] = k;
    }
}

static void flat_unpack_scatter(void* p, int64_t c0, int64_t c1) {
    flat_ctx* x = (flat_ctx*)p;
    for (int64_t c = c0; c < c1; ++c) {
        int64_t lo = c * CH, hi = lo + CH < x->n ? lo + CH : x->n, o = x->cnt[c];
        for (int64_t f = lo; f < hi; ++f) {
            if ((x->mask_in[f >> 3] >> (f & 7)) & 1)
                store_bits(x->dst, x->dtype, f, load_bits(x->src, x->dtype, o++));
            else
                store_bits(x->dst, x->dtype, f, 0);
        }
    }
}

/* Flat pack.  Writes ceil(n/8) mask bytes and the nonzeros to vals
 * (capacity vals_cap).  Returns nnz, or -1 if vals_cap is too small. */
int64_t orc_flat_pack(const void* dense, int dtype, int64_t n, uint8_t* mask,
                      void* vals, int64_t vals_cap, int nthreads) {
    int64_t nch = (n + CH - 1) / CH;
    int64_t* cnt = (int64_t*)calloc((size_t)(nch + 1), sizeof(int64_t));
    if (!cnt) return -2;
    flat_ctx x = {dense, vals, NULL, mask, dtype, n, cnt};
    parallel_for(nch, nthreads, flat_pack_count, &x);
    for (int64_t c = 0; c < nch; ++c) cnt[c + 1] += cnt[c];
    int64_t nnz = cnt[nch];
    if (nnz > vals_cap) { free(cnt); return -1; }
    parallel_for(nch, nthreads, flat_pack_scatter, &x);
    free(cnt);
    return nnz;
}

/* Flat unpack: out[f] = bit(f) ? vals[rank(f)] : 0.  Returns the number of
 * set bits consumed, or -1 if it exceeds vals_len. */
int64_t orc_flat_unpack(const void* vals, int64_t vals_len, const uint8_t* mask, int dtype,
                        int64_t n, void* out, int nthreads) {
    int64_t nch = (n + CH - 1) / CH;
    int64_t* cnt = (int64_t*)calloc((size_t)(nch + 1), sizeof(int64_t));
    if (!cnt) return -2;
    flat_ctx x = {vals, out, mask, NULL, dtype, n, cnt};
    parallel_for(nch, nthreads, flat_unpack_count, &x);
    for (int64_t c = 0; c < nch; ++c) cnt[c + 1] += cnt[c];
    int64_t total = cnt[nch];
    if (total > vals_len) { free(cnt); return -1; }
    parallel_for(nch, nthreads, flat_unpack_scatter, &x);
    free(cnt);
    return total;
}

/* Tiled pack of a row-major [M, N] matrix (row stride ld elements).
 * bitmask: num_tiles * BM*BN/8 bytes; prefix: num_tiles + 1 int32;
 * vals written from vals[offset + prefix[t]].  Returns the total nnz, or -1
 * if offset + total exceeds vals_cap. */
int64_t orc_tile_pack(const void* dense, int dtype, int64_t M, int64_t N, int64_t ld,
                      int BM, int BN, uint8_t* bitmask, int32_t* prefix,
                      void* vals, int64_t vals_cap, int64_t offset) {
    int64_t gm = (M + BM - 1) / BM, gn = (N + BN - 1) / BN, nt = gm * gn;
    int64_t tb = (int64_t)BM * BN / 8;
    memset(bitmask, 0, (size_t)(nt * tb));
    int64_t run = 0;
    for (int64_t t = 0; t < nt; ++t) {
        int64_t tm = t / gn, tn = t % gn;
        prefix[t] = (int32_t)run;
        for (int r = 0; r < BM; ++r) {
            for (int c = 0; c < BN; ++c) {
                int64_t gr = tm * BM + r, gc = tn * BN + c;
                if (gr >= M || gc >= N) continue;
                uint32_t b = load_bits(dense, dtype, gr * ld + gc);
                if (is_positive(b, dtype)) {
                    int64_t f = (int64_t)r * BN + c;
                    bitmask[t * tb + f / 8] |= (uint8_t)(1u << (f % 8));
                    if (offset + run >= vals_cap) return -1;
                    store_bits(vals, dtype, offset + run, b);
                    ++run;
                }
            }
        }
    }
    prefix[nt] = (int32_t)run;
    return run;
}

/* Tiled unpack of rows [row0, row0 + rows) into out (row stride ld_out),
 * as _unpack_batch_kernel does for one row batch (sparse_unpack.py:5-55),
 * but with column bounds. */
void orc_tile_unpack(const void* vals, const uint8_t* bitmask, const int32_t* prefix,
                     int64_t offset, int dtype, int64_t M, int64_t N, int BM, int BN,
                     int64_t row0, int64_t rows, void* out, int64_t ld_out) {
    int64_t gn = (N + BN - 1) / BN, tb = (int64_t)BM * BN / 8;
    for (int64_t r = row0; r < row0 + rows && r < M; ++r) {
        int64_t tm = r / BM, rr = r % BM;
        for (int64_t tn = 0; tn < gn; ++tn) {
            int64_t t = tm * gn + tn;
            const uint8_t* m = bitmask + t * tb;
            int64_t rank = 0;
            for (int64_t f = 0; f < rr * BN; ++f) rank += (m[f / 8] >> (f % 8)) & 1;
            for (int c = 0; c < BN; ++c) {
                int64_t gc = tn * BN + c, f = rr * BN + c;
                int bit = (m[f / 8] >> (f % 8)) & 1;
                if (gc < N) {
                    uint32_t v = bit ? load_bits(vals, dtype, offset + prefix[t] + rank) : 0;
                    store_bits(out, dtype, (r - row0) * ld_out + gc, v);
                }
                rank += bit;
            }
        }
    }
}
