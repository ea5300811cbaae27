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
// products of these with x are corrected once per group (see gemv_tma.cu).
__device__ __forceinline__ void unpack_raw(uint32_t T, uint32_t (&o)[4]) {
  const uint32_t T8 = T >> 8;
  o[0] = lop3_and_or(T, kLoNibbles, kMagic1024x2);
  o[1] = lop3_and_or(T, kHiNibbles, kMagic1024x2);
  o[2] = lop3_and_or(T8, kLoNibbles, kMagic1024x2);
  o[3] = lop3_and_or(T8, kHiNibbles, kMagic1024x2);
}

// Slot of column j (0..7 of a word) in the unpack_pairs output of T_a / T_b.
__device__ __forceinline__ constexpr int col_slot(int j) { return 4 * (j >> 2) + (((j & 1) << 1) | ((j >> 1) & 1)); }

}  // namespace ashqk
