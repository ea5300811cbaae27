// Low-latency exchange lines over NVLink peer memory, shared by the LL
// all-reduce (p2p_allreduce.cu) and the row-parallel GEMV with a fused
// all-reduce epilogue (gemv_strip.cu).
//
// Each rank owns one region (cudaMalloc, shared with the peers by CUDA IPC):
//   [0, 4)    call counter: calls completed on this region
//   [4, 8)    CTAs of the running call that have finished (reset by the last)
//   [256, ..) inbox[parity][source rank][pair]: 8-byte lines
//             {two fp16 of the source's partial, call epoch}
//
// A call's epoch is counter + 1, read by every CTA after griddepcontrol.wait
// (the previous call has completed, counter included); the last CTA of the
// call to finish bumps the counter. A rank pushes its pair p of call e into
// inbox[e & 1][rank][p] of every peer with one 64-bit store (single-copy
// atomic: a reader that sees the epoch sees the data) and polls its own inbox
// for the peers' lines. A line of parity e & 1 is overwritten at call e + 2
// only after this rank has read, in call e + 1, lines that every peer wrote in
// its call e + 1 -- which each peer began after its call e had completed -- so
// no line is overwritten before it is read, whatever pairs each call covers.
// Waits are bounded (~2 s): on expiry the device error word gets kDevErrPeer,
// which is sticky (later calls skip the exchange) until the host clears it.
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace ashqk {

constexpr size_t kLLHeaderBytes = 256;
constexpr int kLLMaxRanks = 8;

struct LLPeers {
  unsigned char* const* regions;  // device array: world region pointers, own at [rank]
  int rank, world;
  long long inbox_pairs;          // pairs per (parity, source) inbox: max_elems / 2
};

__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_volatile_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool ll_sticky_failure() { return (atomicOr(&g_device_errors, 0u) & kDevErrPeer) != 0; }

// This call's epoch; call after griddepcontrol.wait.
__device__ __forceinline__ unsigned int ll_call_epoch(const LLPeers& p) {
  return ld_volatile_u32(reinterpret_cast<const unsigned int*>(p.regions[p.rank])) + 1u;
}

__device__ __forceinline__ unsigned long long* ll_inbox(const LLPeers& p, int dst, unsigned int epoch, int src) {
  return reinterpret_cast<unsigned long long*>(p.regions[dst] + kLLHeaderBytes) +
         (static_cast<long long>(epoch & 1u) * kLLMaxRanks + src) * p.inbox_pairs;
}

// Push pair `pair` of this rank's partial (two fp16 in `data`) to every peer.
__device__ __forceinline__ void ll_push(const LLPeers& p, unsigned int epoch, long long pair, unsigned int data) {
  const unsigned long long line = (static_cast<unsigned long long>(epoch) << 32) | data;
  for (int q = 0; q < p.world; ++q)
    if (q != p.rank) st_volatile_u64(ll_inbox(p, q, epoch, p.rank) + pair, line);
}

// Sum pair `pair` over all ranks in rank order (fp32): the own value `data`
// and every peer's line of this epoch. `failed` is set, and the sum left
// incomplete, when a peer's line does not arrive within the time limit.
__device__ __forceinline__ float2 ll_pull_sum(const LLPeers& p, unsigned int epoch, long long pair, unsigned int data,
                                              bool& failed) {
  float a0 = 0.f, a1 = 0.f;
  for (int r = 0; r < p.world; ++r) {
    unsigned int v = data;
    if (r != p.rank) {
      if (failed) break;
      const unsigned long long* line = ll_inbox(p, p.rank, epoch, r) + pair;
      unsigned long long w = ld_volatile_u64(line);
      if (static_cast<unsigned int>(w >> 32) != epoch) {
        const long long t0 = clock64();
        do {
          if (clock64() - t0 > kWaitLimitCycles) {
            failed = true;
            raise_device_error(kDevErrPeer);
            break;
          }
          __nanosleep(32);
          w = ld_volatile_u64(line);
        } while (static_cast<unsigned int>(w >> 32) != epoch);
        if (failed) break;
      }
      v = static_cast<unsigned int>(w);
    }
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v));
    a0 += f.x;
    a1 += f.y;
  }
  return make_float2(a0, a1);
}

// End of a CTA's part of the call (one thread, after the CTA's exchange): the
// last of the grid's `ctas` CTAs resets the finish count and bumps the counter.
__device__ __forceinline__ void ll_cta_done(const LLPeers& p, unsigned int ctas) {
  unsigned int* hdr = reinterpret_cast<unsigned int*>(p.regions[p.rank]);
  __threadfence();
  if (atomicAdd(hdr + 1, 1u) == ctas - 1u) {
    atomicExch(hdr + 1, 0u);
    __threadfence();
    atomicAdd(hdr, 1u);
  }
}

}  // namespace ashqk
