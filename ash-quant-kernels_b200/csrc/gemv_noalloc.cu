// Decode GEMV entry point that allocates nothing.
//
// ashqk_w4a16_gemv needs a caller-owned split-K workspace. Some callers cannot
// provide one: code that owns no allocator (a plugin handed only the tensors'
// device pointers by its host framework), or code that must not call
// cudaMalloc at all (it can synchronise the device, and some hosts forbid it
// on their hot path). For them this file keeps the scratch in a fixed-size
// device array that the library itself holds, and exposes one entry point
// that uses it.
//
// The array lives for as long as the library is loaded, on every GPU that
// loads it (kScratchBytes each). All calls share it, so calls that can overlap
// on the GPU (different streams, different host threads) race on it; order
// them on one stream. Each call clears the arrival counters at the start of
// the array before its kernel runs, so contents left by an earlier call (or by
// a kernel that gave up) never leak into the next one.
#include <mutex>

#include "common.cuh"

namespace ashqk {

int gemv_call_workspace_bytes(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                              int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int K, int G, int split_k,
                              size_t* bytes);
int gemv_launch_rows(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                     int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K,
                     int G, int split_k, void* workspace, size_t ws_bytes, cudaStream_t stream);

namespace {

// Largest split-K workspace the no-allocation path serves: 64 KiB of arrival
// counters followed by the fp32 partial-sum slots.
constexpr size_t kScratchBytes = 8u << 20;
constexpr size_t kCounterBytes = 64u << 10;  // the counter region every GEMV kernel uses

static __device__ __align__(256) unsigned char g_gemv_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_gemv_scratch on the current device, looked up once per
// device (the host-side symbol is only a handle, never a device pointer).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ASHQK_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return ASHQK_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemv_scratch) != cudaSuccess || p == nullptr) return ASHQK_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return ASHQK_OK;
}

}  // namespace
}  // namespace ashqk

extern "C" int ashqk_w4a16_gemv_noalloc(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                                        const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                                        void* y, int64_t y_ld, int M, int N, int K, int group_size, int split_k,
                                        void* stream) {
  int rc = ashqk::check_awq_args(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size);
  if (rc) return rc;
  const int rows = M < 16 ? M : 16;
  // The kernel chosen for these operands decides whether any scratch is used:
  // the cluster-split strip kernel (the default for aligned operands) needs
  // none, so it is neither capped nor preceded by a counter clear.
  size_t need = 0;
  rc = ashqk::gemv_call_workspace_bytes(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, rows, N, K, group_size,
                                        split_k, &need);
  if (rc) return rc;
  if (need > ashqk::kScratchBytes) return ASHQK_ERR_WORKSPACE;  // problem too large for the fixed scratch
  void* scratch = nullptr;
  if (need > 0) {
    rc = ashqk::scratch_address(&scratch);
    if (rc) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < M; m0 += 16) {
    const int mc = M - m0 < 16 ? M - m0 : 16;
    // The counters must start at zero; the partial-sum slots are fully
    // overwritten before they are read.
    if (need > 0 && cudaMemsetAsync(scratch, 0, ashqk::kCounterBytes, st) != cudaSuccess) return ASHQK_ERR_CUDA;
    rc = ashqk::gemv_launch_rows(static_cast<const __half*>(x) + m0 * x_ld, x_ld, qweight, qw_ld, qzeros, qz_ld,
                                 static_cast<const __half*>(scales), s_ld, static_cast<__half*>(y) + m0 * y_ld, y_ld,
                                 mc, N, K, group_size, split_k, scratch, need > 0 ? ashqk::kScratchBytes : 0, st);
    if (rc) return rc;
  }
  return ASHQK_OK;
}
