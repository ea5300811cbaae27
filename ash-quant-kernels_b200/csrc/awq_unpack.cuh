// int4 -> fp16 unpacking of AWQ words into mma.sync A fragments.
//
// AWQ nibble order (ashqk/ref.py:20-21): nibble i of a word holds column
// AWQ_ORDER[i] = (0,2,4,6,1,3,5,7)[i]. Byte-permuting two rows' words with
// prmt selector 0x6420 gives a word whose nibbles are
//   [r0c0, r0c2, r0c1, r0c3, r1c0, r1c2, r1c1, r1c3]
// (0x7531 gives the same for columns 4..7), so each LOP3 below extracts one
// column at two consecutive k as a half2 -- the K-pair layout of an mma.sync
// A-fragment register.
#pragma once

#include "common.cuh"

namespace ashqk {

constexpr uint32_t kSixteenthX2 = 0x2C002C00u;     // half2(1/16, 1/16)
constexpr uint32_t kOneX2 = 0x3C003C00u;           // half2(1, 1)
// Nibble of a packed AWQ word holding column c (inverse of AWQ_ORDER, ashqk/ref.py:20-22).
__device__ constexpr int kAwqNibbleOfCol[8] = {0, 4, 1, 5, 2, 6, 3, 7};
constexpr uint32_t kNegSixteenthX2 = 0xAC00AC00u;  // half2(-1/16, -1/16)

// 1024+q (low nibble) or 1024+16q (high nibble) -> q - z, exact in fp16.
__device__ __forceinline__ void unpack_pairs(uint32_t T, const uint32_t (&zz)[4], uint32_t (&o)[4]) {
  const uint32_t T8 = T >> 8;
  o[0] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(T, kLoNibbles, kMagic1024x2)), u32_as_h2(zz[0])));
  o[1] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(T, kHiNibbles, kMagic1024x2)), u32_as_h2(kSixteenthX2),
                           u32_as_h2(zz[1])));
  o[2] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(T8, kLoNibbles, kMagic1024x2)), u32_as_h2(zz[2])));
  o[3] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(T8, kHiNibbles, kMagic1024x2)), u32_as_h2(kSixteenthX2),
                           u32_as_h2(zz[3])));
}

// Zero-point constants for one packed qzeros word, in the order unpack_pairs
// consumes them: [0..3] for columns (0,2,1,3), [4..7] for columns (4,6,5,7).
// Low-nibble slots hold 1024+z (subtracted); high-nibble slots hold -(64+z)
// (added after scaling 1024+16q by 1/16).
__device__ __forceinline__ void zero_consts(uint32_t zw, uint32_t (&zc)[8]) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t T = prmt(zw, zw, half ? 0x3131u : 0x2020u);
    const uint32_t T8 = T >> 8;
    zc[4 * half + 0] = lop3_and_or(T, kLoNibbles, kMagic1024x2);
    zc[4 * half + 1] =
        h2_as_u32(__hmul2(u32_as_h2(lop3_and_or(T, kHiNibbles, kMagic1024x2)), u32_as_h2(kNegSixteenthX2)));
    zc[4 * half + 2] = lop3_and_or(T8, kLoNibbles, kMagic1024x2);
    zc[4 * half + 3] =
        h2_as_u32(__hmul2(u32_as_h2(lop3_and_or(T8, kHiNibbles, kMagic1024x2)), u32_as_h2(kNegSixteenthX2)));
  }
}

// Magic-number halves without the zero-point subtraction: slots 0 and 2 hold
// 1024 + q (low nibbles), slots 1 and 3 hold 1024 + 16 q (high nibbles). Dot
// products of these with x are corrected once per group (the RAW variant of
// the column-strip GEMV).
__device__ __forceinline__ void unpack_raw(uint32_t T, uint32_t (&o)[4]) {
  const uint32_t T8 = T >> 8;
  o[0] = lop3_and_or(T, kLoNibbles, kMagic1024x2);
  o[1] = lop3_and_or(T, kHiNibbles, kMagic1024x2);
  o[2] = lop3_and_or(T8, kLoNibbles, kMagic1024x2);
  o[3] = lop3_and_or(T8, kHiNibbles, kMagic1024x2);
}

// ---- dequantisation of one packed word into 8 fp16 weights (GEMM operand tiles) ----
//
// Word w holds columns (0,2,4,6,1,3,5,7) in nibbles 0..7, so masking nibbles
// {0,4}, {1,5} of w and of w >> 8 yields the column pairs (0,1), (2,3), (4,5),
// (6,7) as half2 -- a row of 8 consecutive columns. Low nibbles give 1024 + q,
// from which 1024 + z is subtracted; high nibbles give 1024 + 16 q, scaled by
// 1/16 and offset by -(64 + z) in one fma. Both give q - z exactly; the product
// with the fp16 scale is then rounded once, which is the fp32 (q - z) * s of
// ashqk/ref.py:78-86 rounded to fp16, bit for bit.

// Zero-point constants of one packed qzeros word, for dequant_word.
__device__ __forceinline__ void word_zero_consts(uint32_t zw, uint32_t (&zc)[4]) {
  const uint32_t z8 = zw >> 8;
  zc[0] = lop3_and_or(zw, kLoNibbles, kMagic1024x2);
  zc[1] = h2_as_u32(__hmul2(u32_as_h2(lop3_and_or(zw, kHiNibbles, kMagic1024x2)), u32_as_h2(kNegSixteenthX2)));
  zc[2] = lop3_and_or(z8, kLoNibbles, kMagic1024x2);
  zc[3] = h2_as_u32(__hmul2(u32_as_h2(lop3_and_or(z8, kHiNibbles, kMagic1024x2)), u32_as_h2(kNegSixteenthX2)));
}

// 8 fp16 weights (q - z) * s of columns 0..7 of packed word w, as 4 half2.
// sc: the 8 columns' scales as 4 half2 (one 16-byte load of the scale row).
__device__ __forceinline__ void dequant_word(uint32_t w, const uint32_t (&zc)[4], const uint32_t (&sc)[4],
                                             uint32_t (&h)[4]) {
  const uint32_t w8 = w >> 8;
  const __half2 d0 = __hsub2(u32_as_h2(lop3_and_or(w, kLoNibbles, kMagic1024x2)), u32_as_h2(zc[0]));
  const __half2 d1 = __hfma2(u32_as_h2(lop3_and_or(w, kHiNibbles, kMagic1024x2)), u32_as_h2(kSixteenthX2),
                             u32_as_h2(zc[1]));
  const __half2 d2 = __hsub2(u32_as_h2(lop3_and_or(w8, kLoNibbles, kMagic1024x2)), u32_as_h2(zc[2]));
  const __half2 d3 = __hfma2(u32_as_h2(lop3_and_or(w8, kHiNibbles, kMagic1024x2)), u32_as_h2(kSixteenthX2),
                             u32_as_h2(zc[3]));
  h[0] = h2_as_u32(__hmul2(d0, u32_as_h2(sc[0])));
  h[1] = h2_as_u32(__hmul2(d1, u32_as_h2(sc[1])));
  h[2] = h2_as_u32(__hmul2(d2, u32_as_h2(sc[2])));
  h[3] = h2_as_u32(__hmul2(d3, u32_as_h2(sc[3])));
}

// Slot of column j (0..7 of a word) in the unpack_pairs output of T_a / T_b.
__device__ __forceinline__ constexpr int col_slot(int j) { return 4 * (j >> 2) + (((j & 1) << 1) | ((j >> 1) & 1)); }

}  // namespace ashqk
