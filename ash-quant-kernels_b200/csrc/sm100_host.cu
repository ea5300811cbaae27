// Host-side helpers for the sm_100a kernels: tensor-map encoding, PDL switch,
// and the device error word.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "sm100.cuh"

namespace ashqk {

__device__ unsigned int g_device_errors = 0;
__device__ unsigned int* g_error_mirror = nullptr;

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t inner_elems,
                         uint64_t outer_elems, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return ASHQK_ERR_CUDA;
  if (!aligned(base, 16) || row_stride_bytes % 16) return ASHQK_ERR_INVALID_ARGUMENT;
  const cuuint64_t dims[2] = {inner_elems, outer_elems};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ASHQK_OK : ASHQK_ERR_INVALID_ARGUMENT;
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return ASHQK_ERR_CUDA;
  if (rank < 1 || rank > 5 || !aligned(base, 16)) return ASHQK_ERR_INVALID_ARGUMENT;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) {
      if (strides_bytes[i] % 16) return ASHQK_ERR_INVALID_ARGUMENT;
      st[i] = strides_bytes[i];
    }
  }
  CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank), base, d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ASHQK_OK : ASHQK_ERR_INVALID_ARGUMENT;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ASHQK_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

}  // namespace ashqk

extern "C" int ashqk_get_device_errors(unsigned int* bits, int clear) {
  if (!bits) return ASHQK_ERR_INVALID_ARGUMENT;
  if (cudaDeviceSynchronize() != cudaSuccess) return ASHQK_ERR_CUDA;
  if (cudaMemcpyFromSymbol(bits, ashqk::g_device_errors, sizeof(unsigned int)) != cudaSuccess) return ASHQK_ERR_CUDA;
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(ashqk::g_device_errors, &zero, sizeof(zero)) != cudaSuccess) return ASHQK_ERR_CUDA;
  }
  return ASHQK_OK;
}

extern "C" int ashqk_set_error_mirror(unsigned int* host_pinned) {
  unsigned int* dev_ptr = nullptr;
  if (host_pinned != nullptr &&
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev_ptr), host_pinned, 0) != cudaSuccess) {
    cudaGetLastError();
    return ASHQK_ERR_INVALID_ARGUMENT;  // not page-locked, mapped host memory
  }
  if (cudaMemcpyToSymbol(ashqk::g_error_mirror, &dev_ptr, sizeof(dev_ptr)) != cudaSuccess) return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}
