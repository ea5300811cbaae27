// C-ABI plumbing: status strings, version, device queries, argument checks and
// the M-based dispatcher (ashqk/ops.py:18-26).
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace ashqk {

int gemv_workspace_bytes(int M, int N, int K, int G, int split_k, size_t* bytes);
int gemm_workspace_bytes(int M, int N, int K, int G, size_t* bytes);
int gemv_max_m();

namespace {
constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::mutex g_info_mu;
}  // namespace

int device_info(DeviceInfo* out) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    cudaGetLastError();  // clear the sticky-free error so later calls start clean
    return ASHQK_ERR_NO_DEVICE;
  }
  if (e != cudaSuccess) return ASHQK_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return ASHQK_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_info_mu);
  DeviceInfo& d = g_info[dev];
  if (d.device != dev) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return ASHQK_ERR_CUDA;
    d.sm_count = prop.multiProcessorCount;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.max_smem_optin = prop.sharedMemPerBlockOptin;
    d.device = dev;
  }
  *out = d;
  if (d.cc_major != 10) return ASHQK_ERR_NO_DEVICE;  // built for sm_100a only
  return ASHQK_OK;
}

int check_awq_args(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld, const int32_t* qzeros,
                   int64_t qz_ld, const void* scales, int64_t s_ld, const void* y, int64_t y_ld, int M, int N, int K,
                   int group_size) {
  if (!x || !qweight || !qzeros || !scales || !y) return ASHQK_ERR_INVALID_ARGUMENT;
  if (M <= 0 || N <= 0 || K <= 0 || group_size <= 0) return ASHQK_ERR_INVALID_ARGUMENT;
  if (N % 8 || K % group_size) return ASHQK_ERR_INVALID_ARGUMENT;
  const int64_t words = N / 8;
  if (x_ld < K || qw_ld < words || qz_ld < words || s_ld < N || y_ld < N) return ASHQK_ERR_INVALID_ARGUMENT;
  if (!aligned(x, 2) || !aligned(qweight, 4) || !aligned(qzeros, 4) || !aligned(scales, 2) || !aligned(y, 2))
    return ASHQK_ERR_INVALID_ARGUMENT;
  return ASHQK_OK;
}

}  // namespace ashqk

extern "C" const char* ashqk_status_string(int status) {
  switch (status) {
    case ASHQK_OK:
      return "ok";
    case ASHQK_ERR_INVALID_ARGUMENT:
      return "invalid argument (null pointer, size, stride or alignment)";
    case ASHQK_ERR_UNSUPPORTED:
      return "unsupported problem for this build";
    case ASHQK_ERR_WORKSPACE:
      return "workspace missing, misaligned or too small";
    case ASHQK_ERR_CUDA:
      return "CUDA runtime error";
    case ASHQK_ERR_NO_DEVICE:
      return "current device is not an sm_100 (B200-class) GPU";
    default:
      return "unknown status";
  }
}

extern "C" const char* ashqk_version(void) { return "0.1.0"; }

extern "C" int ashqk_linear_workspace_size(int M, int N, int K, int group_size, size_t* bytes) {
  if (!bytes || M <= 0 || N <= 0 || K <= 0 || group_size <= 0 || N % 8 || K % group_size)
    return ASHQK_ERR_INVALID_ARGUMENT;
  if (M <= ashqk::gemv_max_m()) return ashqk::gemv_workspace_bytes(M, N, K, group_size, 0, bytes);
  return ashqk::gemm_workspace_bytes(M, N, K, group_size, bytes);
}

extern "C" int ashqk_w4a16_linear(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                                  const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld, void* y,
                                  int64_t y_ld, int M, int N, int K, int group_size, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (M > 0 && M <= ashqk::gemv_max_m())
    return ashqk_w4a16_gemv(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size, 0,
                            workspace, workspace_bytes, stream);
  return ashqk_w4a16_gemm(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size,
                          workspace, workspace_bytes, stream);
}
