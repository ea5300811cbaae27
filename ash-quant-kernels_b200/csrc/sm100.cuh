// sm_100a building blocks: mbarriers with bounded waits, TMA tensor loads,
// programmatic dependent launch, tcgen05 (TMEM + UMMA) wrappers, and the host
// helpers that encode tensor maps and launch with PDL.
//
// Every wait on an mbarrier is bounded: after kWaitLimitCycles SM clocks it
// records ASHQK_DEVERR_TIMEOUT in the device error word (readable through
// ashqk_get_device_errors) and gives up, so a logic error ends the kernel with
// a status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace ashqk {

// Device error word shared by all kernels of the library (bit flags).
enum DeviceError : unsigned int {
  kDevErrTimeout = 1u,       // a pipeline wait ran past its limit
  kDevErrBadLaunch = 2u,     // kernel found launch parameters it cannot handle
};
extern __device__ unsigned int g_device_errors;

constexpr long long kWaitLimitCycles = 4ll * 1000 * 1000 * 1000;  // ~2 s at 1.9 GHz

__device__ __forceinline__ void raise_device_error(unsigned int bits) { atomicOr(&g_device_errors, bits); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the warp sleeps in hardware until the
// phase completes (or the hint, in ns, runs out) instead of spinning, so
// waiting warps put no load on shared memory or the issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false (and flags
// the device error word) if the limit ran out, or if `abort` was already set by
// another thread of the CTA; on false the caller must stop its pipeline work.
// `spin` polls without the suspend hint: lower wake-up latency, for the single
// producer thread whose refills gate the pipeline.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, bool spin = false) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (spin ? mbar_try_wait(bar, parity) : mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort = 1;
      raise_device_error(kDevErrTimeout);
      return false;
    }
  }
}

// Make generic-proxy shared-memory writes visible to the async proxy (TMA, UMMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA ----------------------------------------------------------------------

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load, no multicast: box at (x = inner coordinate, y) -> dst.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> shared, completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16). No multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ---- explicit shared-memory loads (32-bit shared-window addresses) ---------------

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// ---- thread-block clusters ---------------------------------------------------

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Full cluster barrier (release / acquire): every thread of every CTA arrives.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_shared_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Not volatile and no memory clobber: callers order these reads with
// cluster_sync(), so independent remote loads can be in flight together.
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// ---- programmatic dependent launch -------------------------------------------

// Block until the grid this launch depends on has completed and its writes are
// visible. A no-op when the kernel was launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allow the next kernel in the stream (launched with PDL) to be scheduled.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- named barriers -----------------------------------------------------------

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- host helpers -------------------------------------------------------------

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda
// link dependency). Returns ASHQK_OK or ASHQK_ERR_CUDA / ASHQK_ERR_INVALID_ARGUMENT.
int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t inner_elems,
                         uint64_t outer_elems, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

// Whether launches use programmatic dependent launch (env ASHQK_PDL=0 disables).
bool pdl_enabled();

}  // namespace ashqk
