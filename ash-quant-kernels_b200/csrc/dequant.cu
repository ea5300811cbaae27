// Dequantisation of AWQ int4 weights to a dense fp16 / fp32 [K, N] matrix.
//
// Follows ashqk/ref.py:78-86 (dequantize_awq): W = (q - z) * s computed in fp32,
// then cast. (q - z) is a small integer and s an fp16 value, so the fp32 product
// is exact and the single fp32 -> fp16 rounding reproduces the reference bit for
// bit. One thread handles one packed word (8 columns of one row); the kernel is
// HBM-bound (0.5 B read + 2 or 4 B written per weight).
#include "common.cuh"

namespace ashqk {
namespace {

template <typename OutT>
struct Store8;

template <>
struct Store8<__half> {
  static __device__ __forceinline__ void store(__half* dst, const float (&v)[8], bool vec) {
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    if (vec) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(h);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = __float2half_rn(v[i]);
    }
  }
};

template <>
struct Store8<float> {
  static __device__ __forceinline__ void store(float* dst, const float (&v)[8], bool vec) {
    if (vec) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = v[i];
    }
  }
};

template <typename OutT>
__global__ void __launch_bounds__(256) dequant_awq_kernel(const int32_t* __restrict__ qweight, int64_t qw_ld,
                                                          const int32_t* __restrict__ qzeros, int64_t qz_ld,
                                                          const __half* __restrict__ scales, int64_t s_ld,
                                                          OutT* __restrict__ w, int64_t w_ld, int words_per_row,
                                                          int K, int group_size, bool vec_scales, bool vec_out) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(K) * words_per_row;
  if (idx >= total) return;
  const int k = static_cast<int>(idx / words_per_row);
  const int wd = static_cast<int>(idx % words_per_row);
  const int grp = k / group_size;
  const uint32_t q = static_cast<uint32_t>(qweight[k * qw_ld + wd]);
  const uint32_t z = static_cast<uint32_t>(qzeros[grp * qz_ld + wd]);
  const __half* srow = scales + grp * s_ld + 8 * wd;
  float s[8];
  if (vec_scales) {
    uint4 raw = *reinterpret_cast<const uint4*>(srow);
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      s[2 * i] = f.x;
      s[2 * i + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = __half2float(srow[i]);
  }
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    // Column j of the block lives in nibble (j % 2) * 4 + j / 2.
    const int shift = 4 * ((j & 1) * 4 + (j >> 1));
    const int qj = static_cast<int>((q >> shift) & 0xF);
    const int zj = static_cast<int>((z >> shift) & 0xF);
    v[j] = static_cast<float>(qj - zj) * s[j];
  }
  Store8<OutT>::store(w + k * w_ld + 8 * wd, v, vec_out);
}

template <typename OutT>
int launch_dequant(const int32_t* qweight, int64_t qw_ld, const int32_t* qzeros, int64_t qz_ld, const void* scales,
                   int64_t s_ld, OutT* w, int64_t w_ld, int N, int K, int group_size, void* stream) {
  if (!qweight || !qzeros || !scales || !w) return ASHQK_ERR_INVALID_ARGUMENT;
  if (N <= 0 || K <= 0 || group_size <= 0 || N % 8 || K % group_size) return ASHQK_ERR_INVALID_ARGUMENT;
  const int words = N / 8;
  if (qw_ld < words || qz_ld < words || s_ld < N || w_ld < N) return ASHQK_ERR_INVALID_ARGUMENT;
  if (!aligned(qweight, 4) || !aligned(qzeros, 4) || !aligned(scales, 2) || !aligned(w, sizeof(OutT)))
    return ASHQK_ERR_INVALID_ARGUMENT;
  const bool vec_scales = aligned(scales, 16) && (s_ld % 8 == 0);
  const bool vec_out = aligned(w, 16) && ((w_ld * sizeof(OutT)) % 16 == 0);
  const int64_t total = static_cast<int64_t>(K) * words;
  const int threads = 256;
  const int64_t blocks = ceil_div64(total, threads);
  if (blocks > 0x7fffffff) return ASHQK_ERR_UNSUPPORTED;
  dequant_awq_kernel<OutT><<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      qweight, qw_ld, qzeros, qz_ld, static_cast<const __half*>(scales), s_ld, w, w_ld, words, K, group_size,
      vec_scales, vec_out);
  return launch_status();
}

}  // namespace
}  // namespace ashqk

extern "C" int ashqk_dequantize_awq_f16(const int32_t* qweight, int64_t qw_ld, const int32_t* qzeros, int64_t qz_ld,
                                        const void* scales, int64_t s_ld, void* w, int64_t w_ld, int N, int K,
                                        int group_size, void* stream) {
  return ashqk::launch_dequant<__half>(qweight, qw_ld, qzeros, qz_ld, scales, s_ld, static_cast<__half*>(w), w_ld,
                                       N, K, group_size, stream);
}

extern "C" int ashqk_dequantize_awq_f32(const int32_t* qweight, int64_t qw_ld, const int32_t* qzeros, int64_t qz_ld,
                                        const void* scales, int64_t s_ld, float* w, int64_t w_ld, int N, int K,
                                        int group_size, void* stream) {
  return ashqk::launch_dequant<float>(qweight, qw_ld, qzeros, qz_ld, scales, s_ld, w, w_ld, N, K, group_size,
                                      stream);
}
