// Prefill GEMM entry point (M > 16). Interim: runs the decode GEMV over 16-row
// chunks until the tcgen05 kernel lands.
#include "common.cuh"

namespace ashqk {
int gemv_workspace_bytes(int M, int N, int K, int G, int split_k, size_t* bytes);

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
  return ashqk_w4a16_gemv(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size, 0,
                          workspace, workspace_bytes, stream);
}
