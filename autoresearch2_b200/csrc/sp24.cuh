// 2:4 compression of one 32-element chunk (shared by the standalone
// compression kernel and the fused GEMM epilogues, so both follow the same
// rule).  Per group of 4 consecutive elements: the first two non-zeros by
// position (non-zero: magnitude bits != 0); fewer than two keep zero slots
// with idx0 < idx1 (one non-zero at f: f and 3, or 2 and 3 when f == 3; none:
// 0 and 1); the 3rd and 4th non-zero are overflow.  A slot holds the bits of
// the element at its index (a kept zero keeps its sign).
#pragma once
#include <stdint.h>

namespace sffn {

// Tables over the 16 non-zero patterns p of a group (bit i: element i).
__host__ __device__ constexpr int sp24_i0(int p) {
    return p == 0 ? 0 : ((p & (p - 1)) == 0 ? ((p == 8) ? 2 : (p == 1 ? 0 : p == 2 ? 1 : 2)) : (p & 1 ? 0 : p & 2 ? 1 : 2));
}
__host__ __device__ constexpr int sp24_first_two_second(int p) {  // index of the second non-zero (p has >= 2)
    return (p & 1) ? ((p & 2) ? 1 : (p & 4) ? 2 : 3) : (p & 2) ? ((p & 4) ? 2 : 3) : 3;
}
__host__ __device__ constexpr int sp24_i1(int p) {
    return p == 0 ? 1 : ((p & (p - 1)) == 0 ? 3 : sp24_first_two_second(p));
}
__host__ __device__ constexpr int sp24_ov(int p) {  // bits beyond the second non-zero
    return (p & (p - 1)) & ((p & (p - 1)) - 1);
}
__host__ __device__ constexpr uint64_t sp24_lut_nib() {  // idx0 | idx1 << 2 per pattern
    uint64_t v = 0;
    for (int p = 0; p < 16; ++p) v |= (uint64_t)(sp24_i0(p) | (sp24_i1(p) << 2)) << (4 * p);
    return v;
}
__host__ __device__ constexpr uint64_t sp24_lut_ov() {
    uint64_t v = 0;
    for (int p = 0; p < 16; ++p) v |= (uint64_t)sp24_ov(p) << (4 * p);
    return v;
}
constexpr uint64_t SP24_LUT_NIB = sp24_lut_nib();
constexpr uint64_t SP24_LUT_OV = sp24_lut_ov();
static_assert(sp24_i0(1) == 0 && sp24_i1(1) == 3 && sp24_i0(8) == 2 && sp24_i1(8) == 3, "single non-zero");
static_assert(sp24_i0(0) == 0 && sp24_i1(0) == 1 && sp24_i0(12) == 2 && sp24_i1(12) == 3, "pairs");
static_assert(sp24_i0(15) == 0 && sp24_i1(15) == 1 && sp24_ov(15) == 12 && sp24_ov(7) == 4, "overflow");
static_assert(sp24_i0(14) == 1 && sp24_i1(14) == 2 && sp24_ov(14) == 8, "three");

// w: 32 bf16 values, two per word in element order (element 2q in the low
// half of w[q]).  cw: the 16 kept values, two per word (group g -> cw[g]);
// nib: the 8 index nibbles (group g at bits 4g); ov: overflow positions
// (bit e for element e).
__device__ __forceinline__ void sp24_chunk(const uint32_t (&w)[16], uint32_t (&cw)[8], uint32_t& nib,
                                           uint32_t& ov) {
    nib = 0;
    ov = 0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const uint32_t w0 = w[2 * g], w1 = w[2 * g + 1];
        const uint32_t t0 = (w0 & 0x7FFF7FFFu) + 0x7FFF7FFFu, t1 = (w1 & 0x7FFF7FFFu) + 0x7FFF7FFFu;
        const uint32_t p = ((t0 >> 15) & 1u) | ((t0 >> 30) & 2u) | ((t1 >> 13) & 4u) | ((t1 >> 28) & 8u);
        const uint32_t n = (uint32_t)(SP24_LUT_NIB >> (4 * p)) & 15u;
        const uint32_t o = (uint32_t)(SP24_LUT_OV >> (4 * p)) & 15u;
        // element h of the group is bytes 2h, 2h+1 of (w1:w0): one byte permute
        // puts element idx0 in the low half and idx1 in the high half
        cw[g] = __byte_perm(w0, w1, 0x1010u + 0x22u * ((n & 3u) + ((n >> 2) << 8)));
        nib |= n << (4 * g);
        ov |= o << (4 * g);
    }
}

// Visit the overflow elements of a chunk in element order without indexing
// the register array: f(e, value) for every set bit e of ov.
template <typename Fn>
__device__ __forceinline__ void sp24_for_overflow(const uint32_t (&w)[16], uint32_t ov, Fn&& f) {
#pragma unroll
    for (int e = 0; e < 32; ++e)
        if ((ov >> e) & 1u) f(e, (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
}

// Lane-order metadata word for lane l of a warp whose 32 lanes hold 32
// consecutive rows of a 128-row tile, from each row's nibble word (K-half 0
// in bits 0-15, K-half 1 in bits 16-31): tensor-memory lane
// dp = m0 + 8*k1 + 16*m2 gets K-half k1 of rows 16*m2 + m0 (low) and
// 16*m2 + m0 + 8 (high).
__device__ __forceinline__ uint32_t sp24_lane_word(uint32_t rowword, int lane) {
    const int k1 = (lane >> 3) & 1;
    const int la = 16 * (lane >> 4) + (lane & 7);
    const uint32_t a = __shfl_sync(0xFFFFFFFFu, rowword, la);
    const uint32_t b = __shfl_sync(0xFFFFFFFFu, rowword, la + 8);
    return ((a >> (16 * k1)) & 0xFFFFu) | (((b >> (16 * k1)) & 0xFFFFu) << 16);
}

}  // namespace sffn
