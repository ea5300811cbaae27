// One-shot all-reduce of small fp16 tensors over NVLink peer memory.
//
// The tensor-parallel decode path reduces an [M, N] fp16 partial per
// row-parallel layer (8-128 KB at M <= 16). NCCL spends 10-20 us on such a
// message; here one CTA per rank does it in one pass over peer memory:
//
//   region of each rank (one cudaMalloc, shared with the peers by CUDA IPC):
//     [0, 4)     epoch counter (this rank's calls so far)
//     [64, 96)   flags[8]: flags[q] = last epoch rank q has published to us
//     [256, ...) two slots of slot_bytes, alternating by epoch parity
//
//   a call: epoch = ++counter; copy the local partial into slot (epoch & 1);
//   publish epoch into every peer's flags[rank] (system-scope release after a
//   system fence); wait until our flags[q] >= epoch for every peer q (bounded);
//   sum slot (epoch & 1) of every rank in rank order (fp32) and write the fp16
//   result.
//
// A rank starts epoch e + 2 -- and overwrites slot e & 1 -- only after every
// peer has published e + 1, which each does after finishing its reads of e,
// so no slot is overwritten while a peer still reads it. The wait gives up
// after ~2 s instead of hanging when a peer never arrives: it sets
// kDevErrPeer in the device error word and leaves the output unwritten, and
// every later call returns at once while that bit is set (the peers time out
// in turn), so a lost rank costs each survivor one bounded wait. The object is
// unusable afterwards. Plain loads and stores only: no multicast, no library
// kernel touches peer memory.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "ll_lines.cuh"
#include "sm100.cuh"

namespace ashqk {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 512;
constexpr size_t kHeaderBytes = 256;

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) allreduce_oneshot_kernel(const __half* in, __half* out, int n,
                                                                     unsigned char* const* regions, int rank,
                                                                     int world, long long slot_bytes) {
  __shared__ unsigned int epoch_s;
  __shared__ int failed_s;
  unsigned char* mine = regions[rank];
  // The next kernel (the next layer's GEMV) may launch now and stream its
  // weights while this one waits for the peers; it reads our output only after
  // its own griddepcontrol.wait, i.e. after this grid has completed.
  pdl_launch_dependents();
  pdl_wait();  // the partial is the previous kernel's output
  if (threadIdx.x == 0) {
    failed_s = (atomicOr(&g_device_errors, 0u) & kDevErrPeer) != 0;
    if (!failed_s) epoch_s = atomicAdd(reinterpret_cast<unsigned int*>(mine), 1u) + 1u;
  }
  __syncthreads();
  if (failed_s) return;
  const unsigned int epoch = epoch_s;
  const long long slot_off = static_cast<long long>(kHeaderBytes) + (epoch & 1u) * slot_bytes;

  // 1. Stage the local partial (16-byte pieces; n is a multiple of 8).
  const uint4* src = reinterpret_cast<const uint4*>(in);
  uint4* dst = reinterpret_cast<uint4*>(mine + slot_off);
  for (int i = threadIdx.x; i < n / 8; i += kThreads) dst[i] = src[i];
  __syncthreads();

  // 2. Publish, 3. wait for the peers (thread q handles peer q).
  const int q = threadIdx.x;
  if (q < world && q != rank) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned int*>(regions[q] + 64) + rank, epoch);
    const unsigned int* flag = reinterpret_cast<const unsigned int*>(mine + 64) + q;
    const long long t0 = clock64();
    while (static_cast<int>(ld_acquire_sys(flag) - epoch) < 0) {
      if (clock64() - t0 > kWaitLimitCycles) {
        failed_s = 1;
        raise_device_error(kDevErrPeer);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (failed_s) return;

  // 4. Sum every rank's slot in rank order.
  for (int i = threadIdx.x; i < n / 8; i += kThreads) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < world; ++r) {
      const uint4 v = reinterpret_cast<const uint4*>(regions[r] + slot_off)[i];
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) oh[j] = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

// ---- low-latency variant: the epoch travels with the data --------------------
//
// Region layout and protocol: ll_lines.cuh. CTA b handles pairs
// [b * kLLPairsPerCta, ...): pushes each of them to every peer as one 8-byte
// line, then sums the peers' lines of the same pairs from its own inbox.
constexpr int kLLThreads = 256;
constexpr int kLLPairsPerThread = 2;
constexpr int kLLPairsPerCta = kLLThreads * kLLPairsPerThread;
constexpr int kLLMaxCtas = 64;

__global__ void __launch_bounds__(kLLThreads) allreduce_ll_kernel(const __half* in, __half* out, int npairs,
                                                               const LLPeers peers) {
  __shared__ unsigned int epoch_s;
  __shared__ int failed_s;
  pdl_launch_dependents();
  pdl_wait();  // the partial is the previous kernel's output; the call counter is final
  if (threadIdx.x == 0) {
    failed_s = ll_sticky_failure();
    epoch_s = ll_call_epoch(peers);
  }
  __syncthreads();
  if (failed_s) return;
  const unsigned int epoch = epoch_s;
  const unsigned int* src = reinterpret_cast<const unsigned int*>(in);
  unsigned int own[kLLPairsPerThread];
  int pair[kLLPairsPerThread];
#pragma unroll
  for (int u = 0; u < kLLPairsPerThread; ++u) {
    pair[u] = blockIdx.x * kLLPairsPerCta + u * kLLThreads + threadIdx.x;
    own[u] = pair[u] < npairs ? src[pair[u]] : 0u;
    if (pair[u] < npairs) ll_push(peers, epoch, pair[u], own[u]);
  }
  bool failed = false;
#pragma unroll
  for (int u = 0; u < kLLPairsPerThread; ++u) {
    if (pair[u] >= npairs) continue;
    const float2 v = ll_pull_sum(peers, epoch, pair[u], own[u], failed);
    if (failed) break;
    reinterpret_cast<__half2*>(out)[pair[u]] = __floats2half2_rn(v.x, v.y);
  }
  __syncthreads();
  if (threadIdx.x == 0) ll_cta_done(peers, gridDim.x);
}

}  // namespace
}  // namespace ashqk

extern "C" int ashqk_p2p_ll_region_bytes(int64_t max_elems, size_t* bytes) {
  if (!bytes || max_elems <= 0 || max_elems % 8 ||
      max_elems > static_cast<int64_t>(ashqk::kLLMaxCtas) * ashqk::kLLPairsPerCta * 2)
    return ASHQK_ERR_INVALID_ARGUMENT;
  *bytes = ashqk::kLLHeaderBytes + 2ull * ashqk::kLLMaxRanks * static_cast<size_t>(max_elems / 2) * 8;
  return ASHQK_OK;
}

extern "C" int ashqk_allreduce_f16_ll(const void* in, void* out, int64_t n, const void* regions_dev, int rank,
                                      int world, int64_t max_elems, void* stream) {
  size_t region = 0;
  if (!in || !out || !regions_dev || n <= 0 || n % 8 || n > max_elems || world < 1 ||
      world > ashqk::kMaxRanks || rank < 0 || rank >= world || ashqk_p2p_ll_region_bytes(max_elems, &region))
    return ASHQK_ERR_INVALID_ARGUMENT;
  if (!ashqk::aligned(in, 16) || !ashqk::aligned(out, 16)) return ASHQK_ERR_INVALID_ARGUMENT;
  const int npairs = static_cast<int>(n / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((npairs + ashqk::kLLPairsPerCta - 1) / ashqk::kLLPairsPerCta);
  cfg.blockDim = dim3(ashqk::kLLThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ashqk::pdl_enabled() ? 1 : 0;
  ashqk::LLPeers peers;
  peers.regions = static_cast<unsigned char* const*>(regions_dev);
  peers.rank = rank;
  peers.world = world;
  peers.inbox_pairs = static_cast<long long>(max_elems / 2);
  if (cudaLaunchKernelEx(&cfg, ashqk::allreduce_ll_kernel, static_cast<const __half*>(in), static_cast<__half*>(out),
                         npairs, peers) != cudaSuccess)
    return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}

extern "C" int ashqk_p2p_region_bytes(int64_t max_elems, size_t* bytes) {
  if (!bytes || max_elems <= 0 || max_elems % 8) return ASHQK_ERR_INVALID_ARGUMENT;
  const size_t slot = (static_cast<size_t>(max_elems) * 2 + 255) / 256 * 256;
  *bytes = ashqk::kHeaderBytes + 2 * slot;
  return ASHQK_OK;
}

extern "C" int ashqk_p2p_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return ASHQK_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return ASHQK_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return ASHQK_ERR_CUDA;
  }
  *ptr = p;
  return ASHQK_OK;
}

extern "C" int ashqk_p2p_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? ASHQK_OK : ASHQK_ERR_CUDA; }

extern "C" int ashqk_p2p_export(void* ptr, void* handle) {
  if (!ptr || !handle) return ASHQK_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return ASHQK_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return ASHQK_OK;
}

extern "C" int ashqk_p2p_import(const void* handle, void** ptr) {
  if (!handle || !ptr) return ASHQK_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return ASHQK_ERR_CUDA;
  *ptr = p;
  return ASHQK_OK;
}

extern "C" int ashqk_p2p_close(void* ptr) {
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? ASHQK_OK : ASHQK_ERR_CUDA;
}

extern "C" int ashqk_allreduce_f16_oneshot(const void* in, void* out, int64_t n, const void* regions_dev, int rank,
                                           int world, int64_t max_elems, void* stream) {
  if (!in || !out || !regions_dev || n <= 0 || n % 8 || n > max_elems || world < 1 ||
      world > ashqk::kMaxRanks || rank < 0 || rank >= world)
    return ASHQK_ERR_INVALID_ARGUMENT;
  if (!ashqk::aligned(in, 16) || !ashqk::aligned(out, 16)) return ASHQK_ERR_INVALID_ARGUMENT;
  size_t region = 0;
  ashqk_p2p_region_bytes(max_elems, &region);
  const long long slot_bytes = static_cast<long long>((region - ashqk::kHeaderBytes) / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(ashqk::kThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ashqk::pdl_enabled() ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, ashqk::allreduce_oneshot_kernel, static_cast<const __half*>(in),
                         static_cast<__half*>(out), static_cast<int>(n),
                         static_cast<unsigned char* const*>(regions_dev), rank, world, slot_bytes) != cudaSuccess)
    return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}
