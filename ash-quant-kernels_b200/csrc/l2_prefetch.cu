// L2 prefetch of a decode layer's weights, launched just before its GEMV.
//
// A decode step is a chain of short launches (2-20 us each), and each one
// spends its first microseconds waiting for the first bytes from HBM and its
// last ones draining -- time during which HBM idles. The weights of a layer do
// not depend on the previous layer's output, so they can be fetched while that
// layer still runs. This kernel does exactly that: with programmatic dependent
// launch it starts as soon as the previous kernel (the GEMV of the layer
// before) has started, needs one warp and no shared memory per CTA (so it
// fits beside that kernel's CTAs), issues bulk L2 prefetches of the packed
// weights, zeros and scales, and then waits for the previous kernel to finish
// before it exits. The GEMV launched after it therefore still sees the
// previous layer's output complete (its griddepcontrol.wait covers this
// kernel, which covered the previous one), and its TMA loads hit L2.
#include <cstdlib>

#include "common.cuh"
#include "sm100.cuh"

namespace ashqk {
namespace {

constexpr int kPrefetchCtas = 64;
constexpr uint32_t kChunkBytes = 16384;  // bytes per prefetch instruction

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
               : "memory");
}

struct Region {
  const unsigned char* base;
  int64_t ld_bytes;   // row stride
  int64_t row_bytes;  // bytes used per row (multiple of 16)
  int rows;
};

// Prefetch a 2-D region in 16-byte aligned pieces of at most kChunkBytes,
// spread over all lanes of all CTAs. Contiguous regions are one long range.
__device__ void prefetch_region(const Region& r, int worker, int workers) {
  if (r.rows <= 0 || r.row_bytes <= 0) return;
  if (r.ld_bytes == r.row_bytes) {
    const int64_t total = r.row_bytes * r.rows;
    const int64_t pieces = (total + kChunkBytes - 1) / kChunkBytes;
    for (int64_t i = worker; i < pieces; i += workers) {
      const int64_t off = i * kChunkBytes;
      const int64_t n = total - off < kChunkBytes ? total - off : kChunkBytes;
      prefetch_l2(r.base + off, static_cast<uint32_t>(n));
    }
    return;
  }
  const int64_t per_row = (r.row_bytes + kChunkBytes - 1) / kChunkBytes;
  const int64_t pieces = per_row * r.rows;
  for (int64_t i = worker; i < pieces; i += workers) {
    const int64_t row = i / per_row, off = (i % per_row) * kChunkBytes;
    const int64_t n = r.row_bytes - off < kChunkBytes ? r.row_bytes - off : kChunkBytes;
    prefetch_l2(r.base + row * r.ld_bytes + off, static_cast<uint32_t>(n));
  }
}

__global__ void __launch_bounds__(32) l2_prefetch_kernel(Region qw, Region qz, Region s) {
  pdl_launch_dependents();
  const int worker = blockIdx.x * 32 + threadIdx.x, workers = gridDim.x * 32;
  prefetch_region(qw, worker, workers);
  prefetch_region(qz, worker, workers);
  prefetch_region(s, worker, workers);
  pdl_wait();  // complete only after the kernel before it: the next launch relies on that
}

}  // namespace

bool l2_prefetch_enabled() {
  static const bool on = [] {  // read once (thread-safe static initialisation)
    const char* e = std::getenv("ASHQK_L2_PREFETCH");
    return e && e[0] == '1';
  }();
  return on;
}

// Launch the prefetch of one layer's AWQ tensors on `stream` (programmatic
// dependent launch). Rows whose byte length is not a multiple of 16 are
// rounded down (prefetching is only a hint).
int l2_prefetch_launch(const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld, const __half* s,
                       int64_t s_ld, int N, int K, int G, cudaStream_t stream) {
  if (!aligned(qw, 16) || !aligned(qz, 16) || !aligned(s, 16)) return ASHQK_OK;  // nothing to do
  Region rq{reinterpret_cast<const unsigned char*>(qw), qw_ld * 4, (static_cast<int64_t>(N) / 2) & ~int64_t(15), K};
  Region rz{reinterpret_cast<const unsigned char*>(qz), qz_ld * 4, (static_cast<int64_t>(N) / 2) & ~int64_t(15),
            K / G};
  Region rs{reinterpret_cast<const unsigned char*>(s), s_ld * 2, (static_cast<int64_t>(N) * 2) & ~int64_t(15), K / G};
  if (rq.ld_bytes % 16 || rz.ld_bytes % 16 || rs.ld_bytes % 16) return ASHQK_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kPrefetchCtas);
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, l2_prefetch_kernel, rq, rz, rs) != cudaSuccess) return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}

}  // namespace ashqk
