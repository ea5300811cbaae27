// Prefill GEMM entry point. The tcgen05 kernel (gemm_tc.cu) takes every
// problem whose shapes and alignments it supports; anything else runs the
// decode GEMV over 16-row chunks, which accepts every valid AWQ layer.
#include "common.cuh"

namespace ashqk {
int gemv_workspace_bytes(int M, int N, int K, int G, int split_k, size_t* bytes);
bool gemm_tc_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld,
                      const void* s, int64_t s_ld, const void* y, int64_t y_ld, int N, int K, int G);
int gemm_tc_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld,
                   const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G, int sm_count,
                   cudaStream_t stream);
int gemm_impl();

// The chunked-GEMV fallback's workspace (the tcgen05 kernel needs none).
int gemm_workspace_bytes(int M, int N, int K, int G, size_t* bytes) {
  return gemv_workspace_bytes(M < 16 ? M : 16, N, K, G, 0, bytes);
}
}  // namespace ashqk

extern "C" int ashqk_gemm_workspace_size(int M, int N, int K, int group_size, size_t* bytes) {
  if (!bytes || M <= 0 || N <= 0 || K <= 0 || group_size <= 0 || N % 8 || K % group_size)
    return ASHQK_ERR_INVALID_ARGUMENT;
  return ashqk::gemm_workspace_bytes(M, N, K, group_size, bytes);
}

extern "C" int ashqk_w4a16_gemm(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                                const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld, void* y,
                                int64_t y_ld, int M, int N, int K, int group_size, void* workspace,
                                size_t workspace_bytes, void* stream) {
  int rc = ashqk::check_awq_args(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size);
  if (rc) return rc;
  const int impl = ashqk::gemm_impl();
  const bool tc_ok =
      ashqk::gemm_tc_eligible(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, N, K, group_size);
  if (impl >= 2 && !tc_ok) return ASHQK_ERR_UNSUPPORTED;
  if (tc_ok && impl != 1) {
    ashqk::DeviceInfo info;
    rc = ashqk::device_info(&info);
    if (rc) return rc;
    return ashqk::gemm_tc_launch(static_cast<const __half*>(x), x_ld, qweight, qw_ld, qzeros, qz_ld,
                                 static_cast<const __half*>(scales), s_ld, static_cast<__half*>(y), y_ld, M, N, K,
                                 group_size, info.sm_count, static_cast<cudaStream_t>(stream));
  }
  return ashqk_w4a16_gemv(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size, 0,
                          workspace, workspace_bytes, stream);
}
