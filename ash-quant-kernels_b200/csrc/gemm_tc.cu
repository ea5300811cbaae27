// Prefill GEMM on the 5th-generation tensor cores: tcgen05.mma with the
// accumulator in tensor memory (TMEM), operands staged by TMA, int4 weights
// dequantised on the fly into shared memory.
//
// y[M,N] = x[M,K] @ W[K,N], W = (q - z) * s from AWQ tensors -- the contraction
// ashqk/kernels/w4a16_gemm_v3.py:20-105 runs as a Triton dot over a dequantised
// fp16 tile. Here, per CTA (one per SM, persistent over output tiles):
//
//   warp 0        TMA producer: x tile [128 x 64] (128-byte swizzle, the K-major
//                 A operand as the MMA reads it), packed weights [64 x BN/8] words,
//                 the scale and zero rows of the stage's groups.
//   warps 6..21   dequantisers, 4 k rows of each stage per warp: int4 -> fp16,
//                 W = (q - z) * s with an exact q - z and one rounding of the
//                 product (bit-exact with ashqk/ref.py:78-86, awq_unpack.cuh),
//                 written as the MN-major B operand in the 128-byte-swizzled
//                 canonical layout (8 k-rows x 64 columns per 1 KB atom).
//   warp 1        one thread issues tcgen05.mma (M=128, N=BN, K=16) x 4 per stage
//                 into one of two TMEM accumulators, and commits stage releases
//                 and tile completion to mbarriers.
//   warps 2..5    epilogue: tcgen05.ld of the finished accumulator (one lane
//                 quadrant per warp), fp32 -> fp16, stores to y; the other
//                 accumulator is meanwhile filled by the next tile's MMAs.
//
// Every mbarrier wait is bounded (sm100.cuh); on a timeout the CTA records the
// device error, all roles stop, and TMEM is released before the kernel exits.
#include <atomic>
#include <algorithm>

#include "awq_unpack.cuh"
#include "sm100.cuh"

namespace ashqk {
namespace {

constexpr int kBM = 128;   // tokens per tile = MMA M = TMEM lanes
constexpr int kBK = 64;    // K per stage: one 128-byte swizzle row of x
constexpr int kStagesA = 5;
constexpr int kStagesB = 2;
constexpr int kDeqWarps = 16;  // each owns 64 / 16 = 4 k rows of every stage
constexpr int kEpiWarps = 4;
constexpr int kFirstEpiWarp = 2;
constexpr int kFirstDeqWarp = kFirstEpiWarp + kEpiWarps;
constexpr int kThreads = 32 * (kFirstDeqWarp + kDeqWarps);
constexpr int kMaxGps = 4;  // scale / zero rows per stage (group size >= 16)

struct GemmMaps {
  CUtensorMap x, qw, s, z;
};

struct GemmArgs {
  __half* y;
  int64_t y_ld;
  int M, N, K, G;
  int tiles_m, tiles_n, num_kb, gps;
  int n_fastest;  // tile order: 1 = consecutive tiles walk N (x block stays in L2), 0 = walk M
  int ksplit;  // > 1: a cluster of ksplit CTAs shares one tile's K range (one tile per cluster)
};

template <int BN>
struct Smem {
  static constexpr int kWC = BN / 8;  // packed words per weight row of a tile
  static constexpr uint32_t kX = kBM * kBK * 2;
  static constexpr uint32_t kB = kBK * BN * 2;
  static constexpr uint32_t kQ = kBK * kWC * 4;
  static constexpr uint32_t kS = kMaxGps * BN * 2;
  static constexpr uint32_t kZ = kMaxGps * kWC * 4;
  static constexpr uint32_t kSbo = (BN / 64) * 1024;  // byte stride of 8-row k groups in the B tile
  static constexpr uint32_t off_x = 0;
  static constexpr uint32_t off_b = off_x + kStagesA * kX;
  static constexpr uint32_t off_q = off_b + kStagesB * kB;
  static constexpr uint32_t off_s = off_q + kStagesA * kQ;
  static constexpr uint32_t off_z = off_s + kStagesA * kS;
  static constexpr uint32_t off_bar = off_z + kStagesA * kZ;
  static constexpr int kBars = 2 * kStagesA + 2 * kStagesB + 5;
  static constexpr uint32_t off_misc = off_bar + kBars * 8;
  static constexpr uint32_t bytes = off_misc + 16;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static_assert(off_b % 1024 == 0 && kX % 1024 == 0 && kB % 1024 == 0, "swizzle atoms need 1 KB alignment");
  static_assert(off_bar % 8 == 0, "mbarriers need 8-byte alignment");
};

// Tile t -> (row block, column block). Tiles that run at the same time share
// their row block of x when N is walked first (x larger than the weights: the
// weights stay in L2 and x is read once), or their weight columns otherwise.
__device__ __forceinline__ int tile_m(const GemmArgs& a, int t) { return a.n_fastest ? t / a.tiles_n : t % a.tiles_m; }
__device__ __forceinline__ int tile_n(const GemmArgs& a, int t) { return a.n_fastest ? t % a.tiles_n : t / a.tiles_m; }

__device__ __forceinline__ void sts_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ GemmMaps maps, const GemmArgs a) {
  using L = Smem<BN>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  unsigned char* smem = smem_raw + pad;
  const uint32_t sbase = smem_u32(smem);

  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* empty_a = full_a + kStagesA;
  uint64_t* full_b = empty_a + kStagesA;
  uint64_t* empty_b = full_b + kStagesB;
  uint64_t* acc_full = empty_b + kStagesB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::off_misc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::off_misc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesA; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kStagesB; ++s) {
      mbar_init(&full_b[s], kDeqWarps);
      mbar_init(&empty_b[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    fence_mbarrier_init();
    prefetch_tensormap(&maps.x);
    prefetch_tensormap(&maps.qw);
    prefetch_tensormap(&maps.s);
    prefetch_tensormap(&maps.z);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish_alloc_permit();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  // x is the previous kernel's output and y may be its input.
  pdl_wait();
  pdl_launch_dependents();

  const int tiles = a.tiles_m * a.tiles_n;
  // With a K split, cluster (blockIdx.x / ksplit) owns one tile and its CTA of
  // rank `split` the k blocks [kb0, kb1); otherwise CTAs stride over tiles.
  const int ks = a.ksplit;
  const int split = ks > 1 ? static_cast<int>(cluster_rank()) : 0;
  const int t_first = ks > 1 ? static_cast<int>(blockIdx.x) / ks : static_cast<int>(blockIdx.x);
  const int t_step = ks > 1 ? tiles : static_cast<int>(gridDim.x);
  const int kb0 = split * a.num_kb / ks, kb1 = (split + 1) * a.num_kb / ks;
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint32_t tx = L::kX + L::kQ + static_cast<uint32_t>(a.gps) * (BN * 2 + L::kWC * 4);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = t_first; t < tiles; t += t_step) {
        const int mb = tile_m(a, t), nb = tile_n(a, t);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_a[stage], phase ^ 1u, abort, true)) break;
          mbar_arrive_expect_tx(&full_a[stage], tx);
          const int k0 = kb * kBK;
          const int g0 = k0 / a.G;
          tma_load_2d(smem + L::off_x + stage * L::kX, &maps.x, k0, mb * kBM, &full_a[stage]);
          tma_load_2d(smem + L::off_q + stage * L::kQ, &maps.qw, nb * L::kWC, k0, &full_a[stage]);
          tma_load_2d(smem + L::off_s + stage * L::kS, &maps.s, nb * BN, g0, &full_a[stage]);
          tma_load_2d(smem + L::off_z + stage * L::kZ, &maps.z, nb * L::kWC, g0, &full_a[stage]);
          ++issued;
          if (++stage == kStagesA) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (*abort) break;
      }
      // Let the last fill of every stage land before the CTA can exit (they all
      // have landed already unless the pipeline gave up).
      for (int i = 1; i <= kStagesA && i <= issued; ++i) {
        const int f = issued - i;  // fill number
        mbar_drain(&full_a[f % kStagesA], static_cast<uint32_t>(f / kStagesA) & 1u);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_f32(kBM, BN, false, true);
      int sa = 0, sb = 0, acc = 0;
      uint32_t pa = 0, pb = 0, pacc = 0;
      for (int t = t_first; t < tiles && !*abort; t += t_step) {
        if (!mbar_wait(&acc_empty[acc], pacc ^ 1u, abort)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_a[sa], pa, abort, true) || !mbar_wait(&full_b[sb], pb, abort, true)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t xa = sbase + L::off_x + sa * L::kX;
          const uint32_t ba = sbase + L::off_b + sb * L::kB;
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            // A: K-major, advance 16 halves (32 B) inside the swizzle row.
            // B: MN-major, advance two 8-row k groups.
            umma_f16_ss(d_tmem, umma_desc_sw128(xa + 32u * j, 16u, 1024u),
                        umma_desc_sw128(ba + 2u * L::kSbo * j, 1024u, L::kSbo), idesc, (kb != kb0) || (j != 0));
          }
          umma_commit(&empty_a[sa]);
          umma_commit(&empty_b[sb]);
          if (++sa == kStagesA) {
            sa = 0;
            pa ^= 1u;
          }
          if (++sb == kStagesB) {
            sb = 0;
            pb ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) pacc ^= 1u;
      }
      // Every MMA this thread issued completes before TMEM is released.
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else if (warp < kFirstDeqWarp) {
    // ---------------- epilogue ----------------
    const int quad = warp & 3;  // the TMEM lane quadrant this warp may read
    int acc = 0;
    uint32_t pacc = 0;
    for (int t = t_first; t < tiles; t += t_step) {
      const int mb = tile_m(a, t), nb = tile_n(a, t);
      if (!mbar_wait(&acc_full[acc], pacc, abort)) break;
      tc_fence_after_sync();
      const int row = mb * kBM + 32 * quad + lane;
      __half* yrow = a.y + static_cast<int64_t>(row) * a.y_ld + nb * BN;
      // K split: this CTA's fp32 partial goes to its own shared memory (over the
      // drained ring), row stride BN + 4 floats; the cluster sums it below.
      float* prow = reinterpret_cast<float*>(smem) + (32 * quad + lane) * (BN + 4);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * quad) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c, r);
        tmem_wait_ld();
        if (ks > 1) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(prow + c + 4 * i) = make_float4(
                __uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                __uint_as_float(r[4 * i + 3]));
        } else if (row < a.M) {
          uint32_t h[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            h[i] = h2_as_u32(__floats2half2_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])));
          uint4* dst = reinterpret_cast<uint4*>(yrow + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) pacc ^= 1u;
    }
  } else {
    // ---------------- dequantisers ----------------
    constexpr int WC = L::kWC;                      // packed words per row of this CTA's columns
    constexpr int kRowsPerWarp = kBK / kDeqWarps;     // k rows of a stage per warp
    constexpr int kRowStep = 32 / WC;                 // rows covered by one pass of the warp's lanes
    constexpr int kRowsPerThread = kRowsPerWarp / kRowStep;
    static_assert(kRowsPerThread >= 1 && kRowsPerWarp % kRowStep == 0, "dequantiser tiling");
    const int d = warp - kFirstDeqWarp;               // rows kRowsPerWarp*d .. of every stage
    const int c = lane % WC;                          // packed word column (8 weight columns)
    const int r0 = kRowsPerWarp * d + lane / WC;
    const int grp_row = a.G >= kBK ? 0 : (kRowsPerWarp * d) / a.G;  // group >= 16 >= kRowsPerWarp
    int sa = 0, sb = 0;
    uint32_t pa = 0, pb = 0;
    for (int t = t_first; t < tiles; t += t_step) {
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_a[sa], pa, abort) || !mbar_wait(&empty_b[sb], pb ^ 1u, abort)) {
          ok = false;
          break;
        }
        const uint32_t qa = sbase + L::off_q + sa * L::kQ;
        const uint32_t sa_addr = sbase + L::off_s + sa * L::kS + grp_row * (BN * 2) + c * 16;
        const uint32_t za = sbase + L::off_z + sa * L::kZ + grp_row * (WC * 4) + c * 4;
        const uint32_t ba = sbase + L::off_b + sb * L::kB + (c >> 3) * 1024u;
        const uint32_t zw = lds_u32(za);
        const uint4 sv = lds_v4(sa_addr);
        const uint32_t sc[4] = {sv.x, sv.y, sv.z, sv.w};
        uint32_t zc[4];
        word_zero_consts(zw, zc);
        uint32_t wv[kRowsPerThread];
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) wv[i] = lds_u32(qa + (r0 + i * kRowStep) * (WC * 4) + c * 4);
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
          const int kr = r0 + i * kRowStep;
          uint32_t h[4];
          dequant_word(wv[i], zc, sc, h);
          const uint32_t addr =
              ba + (kr >> 3) * L::kSbo + (kr & 7) * 128u + ((static_cast<uint32_t>(c & 7) ^ (kr & 7)) << 4);
          sts_v4(addr, h[0], h[1], h[2], h[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_b[sb]);
        if (++sa == kStagesA) {
          sa = 0;
          pa ^= 1u;
        }
        if (++sb == kStagesB) {
          sb = 0;
          pb ^= 1u;
        }
      }
      if (!ok) break;
    }
  }

  // Teardown: every role has finished (or given up); release TMEM.
  tc_fence_before_sync();
  __syncthreads();
  if (ks > 1) {
    // Sum the cluster's partial tiles: CTA `split` owns rows [r0, r1) of the
    // tile and adds the ranks' partials in fixed order (deterministic).
    cluster_sync();
    if (!*abort) {
      const int mb = tile_m(a, t_first), nb = tile_n(a, t_first);
      const int r0 = split * kBM / ks, r1 = (split + 1) * kBM / ks;
      constexpr int kQuads = BN / 4;
      const float* part = reinterpret_cast<const float*>(smem);
      for (int i = threadIdx.x; i < (r1 - r0) * kQuads; i += kThreads) {
        const int rr = r0 + i / kQuads, c4 = (i % kQuads) * 4;
        const int row = mb * kBM + rr;
        const float* src = part + rr * (BN + 4) + c4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < ks; ++q) {
          const float4 v = ld_shared_cluster_v4(map_shared_rank(src, static_cast<uint32_t>(q)));
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        if (row < a.M) {
          const __half2 h0 = __floats2half2_rn(acc.x, acc.y), h1 = __floats2half2_rn(acc.z, acc.w);
          *reinterpret_cast<uint2*>(a.y + static_cast<int64_t>(row) * a.y_ld + nb * BN + c4) =
              make_uint2(h2_as_u32(h0), h2_as_u32(h1));
        }
      }
    }
    cluster_sync();  // keep every CTA's partial alive until all remote reads are done
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

int g_gemm_impl = 0;  // 0 auto, 1 chunked decode GEMV, 2 tcgen05, 3 tcgen05 one CTA, 4 tcgen05 CTA pairs

template <int BN>
int launch_gemm_tc(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld,
                   const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G, int sm_count,
                   int ksplit, cudaStream_t stream) {
  using L = Smem<BN>;
  GemmArgs a;
  a.y = y;
  a.y_ld = y_ld;
  a.M = M;
  a.N = N;
  a.K = K;
  a.G = G;
  a.tiles_m = ceil_div(M, kBM);
  a.tiles_n = N / BN;
  a.num_kb = K / kBK;
  a.gps = G >= kBK ? 1 : kBK / G;
  // x bytes vs packed weight bytes: keep the smaller operand resident in L2.
  a.n_fastest = static_cast<int64_t>(M) * K * 2 > static_cast<int64_t>(K) * N / 2 ? 1 : 0;
  a.ksplit = ksplit;
  GemmMaps maps;
  int rc = encode_tensor_map_2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(x), K, M,
                                static_cast<uint64_t>(x_ld) * 2, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.qw, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<int32_t*>(qw), N / 8, K,
                              static_cast<uint64_t>(qw_ld) * 4, L::kWC, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(s), N, K / G,
                              static_cast<uint64_t>(s_ld) * 2, BN, a.gps, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.z, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<int32_t*>(qz), N / 8, K / G,
                              static_cast<uint64_t>(qz_ld) * 4, L::kWC, a.gps, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;

  const size_t smem = L::bytes + 1024;  // + alignment slack
  static std::atomic<bool> configured[64];  // zero-initialised (static storage)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ASHQK_ERR_CUDA;
  auto kernel = gemm_tc_kernel<BN>;
  if (!configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return ASHQK_ERR_CUDA;
    configured[dev].store(true, std::memory_order_release);
  }
  const int tiles = a.tiles_m * a.tiles_n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ksplit > 1 ? tiles * ksplit : std::min(tiles, sm_count));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (ksplit > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = ksplit;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (cudaLaunchKernelEx(&cfg, kernel, maps, a) != cudaSuccess) return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}

}  // namespace

bool gemm_tc_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld,
                      const void* s, int64_t s_ld, const void* y, int64_t y_ld, int N, int K, int G) {
  return N % 128 == 0 && K % kBK == 0 && G >= 16 && G % 16 == 0 && (G % kBK == 0 || kBK % G == 0) &&
         aligned(x, 16) && x_ld % 8 == 0 && aligned(qw, 16) && qw_ld % 4 == 0 && aligned(qz, 16) &&
         qz_ld % 4 == 0 && aligned(s, 16) && s_ld % 8 == 0 && aligned(y, 16) && y_ld % 8 == 0;
}

bool gemm_tc_pair_eligible(int M, int N);
int gemm_tc_pair_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                        int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K,
                        int G, int sm_count, cudaStream_t stream);

int gemm_tc_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld,
                   const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G, int sm_count,
                   cudaStream_t stream) {
  // CTA pairs (cta_group::2) once M spans two 128-row tiles, N % 256 == 0,
  // the pair tiles occupy at least ~0.6 of the SM pairs and padding M to 256
  // rows wastes at most 1/8 of them: each SM then writes and feeds the tensor
  // core half as much of the fp16 weight tile, which bounds the one-CTA kernel
  // (shared-memory bandwidth). Measured crossover on the Qwen3-8B shapes: pairs
  // win from 48 tiles (o, qkv, down at M = 768; qkv at 512), the one-CTA
  // kernel below that and when M is an odd number of 128-row tiles (384).
  const bool pair_ok = gemm_tc_pair_eligible(M, N);
  const int pair_tiles = pair_ok ? ceil_div(M, 2 * kBM) * (N / 256) : 0;
  const bool pair_fill = 10 * 2 * pair_tiles >= 6 * sm_count;
  const bool pair_pad = 8 * ceil_div(M, 2 * kBM) * (2 * kBM) <= 9 * M;
  if (g_gemm_impl == 4 && !pair_ok) return ASHQK_ERR_UNSUPPORTED;
  if (g_gemm_impl == 4 || (pair_ok && g_gemm_impl != 3 && pair_fill && pair_pad))
    return gemm_tc_pair_launch(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, y, y_ld, M, N, K, G, sm_count, stream);
  // One CTA per tile: 256-column tiles unless that leaves most SMs idle and 128
  // columns divide N; with fewer tiles than half the SMs, split K over a
  // cluster (at most 8 CTAs, at least 4 k blocks each).
  const int tiles256 = N % 256 == 0 ? ceil_div(M, kBM) * (N / 256) : 0;
  const bool wide = tiles256 > 0 && (tiles256 >= sm_count || N % 128 != 0);
  const int tiles = wide ? tiles256 : ceil_div(M, kBM) * (N / 128);
  int ks = 1;
  if (2 * tiles <= sm_count) ks = std::max(1, std::min({8, sm_count / tiles, (K / kBK) / 4}));
  if (wide)
    return launch_gemm_tc<256>(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, y, y_ld, M, N, K, G, sm_count, ks, stream);
  return launch_gemm_tc<128>(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, y, y_ld, M, N, K, G, sm_count, ks, stream);
}

int gemm_impl() { return g_gemm_impl; }

}  // namespace ashqk

extern "C" int ashqk_set_gemm_kernel(int which) {
  if (which < 0 || which > 4) return ASHQK_ERR_INVALID_ARGUMENT;
  ashqk::g_gemm_impl = which;
  return ASHQK_OK;
}
