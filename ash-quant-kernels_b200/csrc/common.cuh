// Shared helpers for the sm_100a AWQ W4A16 kernels: status plumbing, device
// queries, and the small inline-PTX building blocks (int4 -> fp16 unpack,
// byte permutes, streaming loads, mma.sync).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ashqk_b200.h"

namespace ashqk {

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  size_t max_smem_optin = 0;
};

// Cached per device (first call on a device queries the runtime).
int device_info(DeviceInfo* out);

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Checks shared by every linear-layer entry point. Returns ASHQK_OK or an error.
int check_awq_args(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                   const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                   const void* y, int64_t y_ld, int M, int N, int K, int group_size);

// Launch-error check after a kernel launch.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ASHQK_OK : ASHQK_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Device side
// ---------------------------------------------------------------------------

// fp16 bit patterns used by the magic-exponent int4 -> fp16 conversion:
// OR-ing a nibble into the mantissa of 1024.0 gives 1024 + q exactly; a nibble in
// mantissa bits 4..7 gives 1024 + 16 q.
constexpr uint32_t kMagic1024x2 = 0x64006400u;
constexpr uint32_t kLoNibbles = 0x000F000Fu;  // nibbles 0 and 4 of a word
constexpr uint32_t kHiNibbles = 0x00F000F0u;  // nibbles 1 and 5 of a word

// (a & b) | c in one LOP3.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Byte permute: result byte i = byte sel[4i+3:4i] of {b, a} (a = bytes 0-3).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Streaming loads for data read exactly once (packed weights): no L1 allocation.
__device__ __forceinline__ uint32_t ld_stream_u32(const int32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream_v2(const int32_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// D = A(16x16, row) * B(16x8, col), fp16 inputs, fp32 result (no accumulator input).
__device__ __forceinline__ void mma_16816_first(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

// D = A(16x16, row) * B(16x8, col) + C, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace ashqk
