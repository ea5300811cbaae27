// Prefill GEMM on a CTA pair: tcgen05.mma.cta_group::2 with M = 256 tokens
// and N = 256 weight columns per instruction, the two SMs of a cluster
// sharing the operands.
//
// Same contraction as gemm_tc.cu (ashqk/kernels/w4a16_gemm_v3.py:20-105), but
// each CTA of the pair holds only half of each operand: its own 128 rows of x
// and its own 128 of the tile's 256 weight columns. So per SM and per stage the
// dequantisers write half as much fp16 and the tensor core reads half as much B
// from shared memory as with one CTA -- the two costs that bound gemm_tc.cu.
//
//   both CTAs   warp 0: TMA of its x rows, packed weights, scales, zeros (plain
//               loads into its own shared memory, completing on its own barrier);
//               warps 6..21: dequantise its 128 columns, fence the stores to the
//               async proxy, then arrive on the even CTA's "B ready" barrier;
//               warps 2..5: epilogue of its 128 rows from its own TMEM.
//   even CTA    warp 1, one thread: the pair MMAs, commits multicast to both
//               CTAs' "stage free" and "accumulator full" barriers.
//
// Both CTAs allocate TMEM together (cta_group::2) and meet at a cluster barrier
// before releasing it, after every MMA has completed. All waits are bounded.
#include <atomic>
#include <algorithm>

#include "awq_unpack.cuh"
#include "sm100.cuh"

namespace ashqk {
namespace {

constexpr int kBM = 128;     // rows per CTA (256 per pair)
constexpr int kBN = 256;     // columns per pair tile (MMA N)
constexpr int kHalfN = 128;  // columns staged per CTA
constexpr int kBK = 64;
constexpr int kStagesA = 6;
constexpr int kStagesB = 3;
constexpr int kDeqWarps = 16;  // each owns 64 / 16 = 4 k rows of every stage
constexpr int kEpiWarps = 4;
constexpr int kFirstEpiWarp = 2;
constexpr int kFirstDeqWarp = kFirstEpiWarp + kEpiWarps;
constexpr int kThreads = 32 * (kFirstDeqWarp + kDeqWarps);
constexpr int kMaxGps = 4;

struct PairMaps {
  CUtensorMap x, qw, s, z;
};

struct PairArgs {
  __half* y;
  int64_t y_ld;
  int M, N, K, G;
  int tiles_m, tiles_n, num_kb, gps;  // tiles_m counts 256-row pair tiles
  int n_fastest;  // tile order: 1 = consecutive tiles walk N (x block stays in L2), 0 = walk M
};

struct PairSmem {
  static constexpr int kWC = kHalfN / 8;
  static constexpr uint32_t kX = kBM * kBK * 2;
  static constexpr uint32_t kB = kBK * kHalfN * 2;
  static constexpr uint32_t kQ = kBK * kWC * 4;
  static constexpr uint32_t kS = kMaxGps * kHalfN * 2;
  static constexpr uint32_t kZ = kMaxGps * kWC * 4;
  static constexpr uint32_t kSbo = (kHalfN / 64) * 1024;
  static constexpr uint32_t off_x = 0;
  static constexpr uint32_t off_b = off_x + kStagesA * kX;
  static constexpr uint32_t off_q = off_b + kStagesB * kB;
  static constexpr uint32_t off_s = off_q + kStagesA * kQ;
  static constexpr uint32_t off_z = off_s + kStagesA * kS;
  static constexpr uint32_t off_bar = off_z + kStagesA * kZ;
  static constexpr int kBars = 2 * kStagesA + 2 * kStagesB + 5;
  static constexpr uint32_t off_misc = off_bar + kBars * 8;
  static constexpr uint32_t bytes = off_misc + 16;
  static constexpr uint32_t kTmemCols = 2 * kBN;  // two accumulators of 128 lanes x 256 fp32 columns
  static_assert(off_b % 1024 == 0 && kX % 1024 == 0 && kB % 1024 == 0, "swizzle atoms need 1 KB alignment");
  static_assert(off_q % 128 == 0 && off_s % 128 == 0 && off_z % 128 == 0, "TMA destinations need 128 B alignment");
};

// Tile t -> (row block, column block). Tiles that run at the same time share
// their row block of x when N is walked first (x larger than the weights: the
// weights stay in L2 and x is read once), or their weight columns otherwise.
__device__ __forceinline__ int tile_m(const PairArgs& a, int t) { return a.n_fastest ? t / a.tiles_n : t % a.tiles_m; }
__device__ __forceinline__ int tile_n(const PairArgs& a, int t) { return a.n_fastest ? t % a.tiles_n : t / a.tiles_m; }

__device__ __forceinline__ void sts_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ PairMaps maps, const PairArgs a) {
  using L = PairSmem;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  unsigned char* smem = smem_raw + pad;
  const uint32_t sbase = smem_u32(smem);

  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* empty_a = full_a + kStagesA;
  uint64_t* full_b = empty_a + kStagesA;  // used in the even CTA: both CTAs' dequantisers arrive
  uint64_t* empty_b = full_b + kStagesB;
  uint64_t* acc_full = empty_b + kStagesB;
  uint64_t* acc_empty = acc_full + 2;     // used in the even CTA: both CTAs' epilogues arrive
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::off_misc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::off_misc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: issues the MMAs

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesA; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kStagesB; ++s) {
      mbar_init(&full_b[s], 2 * kDeqWarps);
      mbar_init(&empty_b[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);
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
    tmem_alloc_pair(tmem_slot, L::kTmemCols);
    tmem_relinquish_alloc_permit_pair();
  }
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before anyone arrives on them
  tc_fence_after_sync();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  pdl_wait();
  pdl_launch_dependents();

  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);
  const int tiles = a.tiles_m * a.tiles_n;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      const uint32_t tx = L::kX + L::kQ + static_cast<uint32_t>(a.gps) * (kHalfN * 2 + L::kWC * 4);
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = pair; t < tiles && !*abort; t += pairs) {
        const int mp = tile_m(a, t), nb = tile_n(a, t);
        const int row0 = mp * (2 * kBM) + static_cast<int>(rank) * kBM;
        const int col0 = nb * kBN + static_cast<int>(rank) * kHalfN;
        for (int kb = 0; kb < a.num_kb; ++kb) {
          if (!mbar_wait(&empty_a[stage], phase ^ 1u, abort, true)) break;
          mbar_arrive_expect_tx(&full_a[stage], tx);
          const int k0 = kb * kBK;
          const int g0 = k0 / a.G;
          tma_load_2d(smem + L::off_x + stage * L::kX, &maps.x, k0, row0, &full_a[stage]);
          tma_load_2d(smem + L::off_q + stage * L::kQ, &maps.qw, col0 / 8, k0, &full_a[stage]);
          tma_load_2d(smem + L::off_s + stage * L::kS, &maps.s, col0, g0, &full_a[stage]);
          tma_load_2d(smem + L::off_z + stage * L::kZ, &maps.z, col0 / 8, g0, &full_a[stage]);
          ++issued;
          if (++stage == kStagesA) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int i = 1; i <= kStagesA && i <= issued; ++i) {
        const int f = issued - i;
        mbar_drain(&full_a[f % kStagesA], static_cast<uint32_t>(f / kStagesA) & 1u);
      }
    }
  } else if (warp == 1) {
    // ---------------- pair MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_f32(2 * kBM, kBN, false, true);
      int sa = 0, sb = 0, acc = 0;
      uint32_t pb = 0, pacc = 0;
      for (int t = pair; t < tiles && !*abort; t += pairs) {
        if (!mbar_wait(&acc_empty[acc], pacc ^ 1u, abort)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        bool ok = true;
        for (int kb = 0; kb < a.num_kb; ++kb) {
          // Both CTAs' dequantisers arrive here after their own x, int4 and
          // fp16 tiles of this stage are in place.
          if (!mbar_wait(&full_b[sb], pb, abort, true)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t xa = sbase + L::off_x + sa * L::kX;
          const uint32_t ba = sbase + L::off_b + sb * L::kB;
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            umma_f16_ss_pair(d_tmem, umma_desc_sw128(xa + 32u * j, 16u, 1024u),
                             umma_desc_sw128(ba + 2u * L::kSbo * j, 1024u, L::kSbo), idesc, (kb | j) != 0);
          }
          umma_commit_pair_mc(&empty_a[sa], 0x3);
          umma_commit_pair_mc(&empty_b[sb], 0x3);
          if (++sa == kStagesA) sa = 0;
          if (++sb == kStagesB) {
            sb = 0;
            pb ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(&acc_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) pacc ^= 1u;
      }
      umma_commit_pair(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else if (warp < kFirstDeqWarp) {
    // ---------------- epilogue (both CTAs) ----------------
    const int quad = warp & 3;
    const uint32_t acc_empty_lead = map_shared_rank(acc_empty, 0);
    int acc = 0;
    uint32_t pacc = 0;
    for (int t = pair; t < tiles; t += pairs) {
      const int mp = tile_m(a, t), nb = tile_n(a, t);
      if (!mbar_wait(&acc_full[acc], pacc, abort)) break;
      tc_fence_after_sync();
      const int row = mp * (2 * kBM) + static_cast<int>(rank) * kBM + 32 * quad + lane;
      __half* yrow = a.y + static_cast<int64_t>(row) * a.y_ld + nb * kBN;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * quad) << 16) + static_cast<uint32_t>(acc * kBN);
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c, r);
        tmem_wait_ld();
        if (row < a.M) {
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
      if (lane == 0) mbar_arrive_cluster(acc_empty_lead + 8u * acc);
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
    const uint32_t full_b_lead = map_shared_rank(full_b, 0);
    int sa = 0, sb = 0;
    uint32_t pa = 0, pb = 0;
    for (int t = pair; t < tiles; t += pairs) {
      bool ok = true;
      for (int kb = 0; kb < a.num_kb; ++kb) {
        if (!mbar_wait(&full_a[sa], pa, abort) || !mbar_wait(&empty_b[sb], pb ^ 1u, abort)) {
          ok = false;
          break;
        }
        const uint32_t qa = sbase + L::off_q + sa * L::kQ;
        const uint32_t s_addr = sbase + L::off_s + sa * L::kS + grp_row * (kHalfN * 2) + c * 16;
        const uint32_t za = sbase + L::off_z + sa * L::kZ + grp_row * (WC * 4) + c * 4;
        const uint32_t ba = sbase + L::off_b + sb * L::kB + (c >> 3) * 1024u;
        const uint32_t zw = lds_u32(za);
        const uint4 sv = lds_v4(s_addr);
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
        if (lane == 0) mbar_arrive_cluster(full_b_lead + 8u * sb);
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

  // Teardown: both CTAs finish (the even CTA's MMAs have completed and no
  // longer read the odd CTA's shared memory) before TMEM is released.
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
}

}  // namespace

// Pair tiles need N % 256 == 0 and are worth it once M spans more than one 128-row tile.
bool gemm_tc_pair_eligible(int M, int N) { return M > kBM && N % kBN == 0; }

int gemm_tc_pair_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                        int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K,
                        int G, int sm_count, cudaStream_t stream) {
  using L = PairSmem;
  PairArgs a;
  a.y = y;
  a.y_ld = y_ld;
  a.M = M;
  a.N = N;
  a.K = K;
  a.G = G;
  a.tiles_m = ceil_div(M, 2 * kBM);
  a.tiles_n = N / kBN;
  a.num_kb = K / kBK;
  a.gps = G >= kBK ? 1 : kBK / G;
  // x bytes vs packed weight bytes: keep the smaller operand resident in L2.
  a.n_fastest = static_cast<int64_t>(M) * K * 2 > static_cast<int64_t>(K) * N / 2 ? 1 : 0;
  PairMaps maps;
  int rc = encode_tensor_map_2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(x), K, M,
                                static_cast<uint64_t>(x_ld) * 2, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.qw, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<int32_t*>(qw), N / 8, K,
                              static_cast<uint64_t>(qw_ld) * 4, L::kWC, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(s), N, K / G,
                              static_cast<uint64_t>(s_ld) * 2, kHalfN, a.gps, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.z, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<int32_t*>(qz), N / 8, K / G,
                              static_cast<uint64_t>(qz_ld) * 4, L::kWC, a.gps, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;

  const size_t smem = L::bytes + 1024;
  static std::atomic<bool> configured[64];  // zero-initialised (static storage)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ASHQK_ERR_CUDA;
  if (!configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(gemm_tc_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return ASHQK_ERR_CUDA;
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = 2;
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  // The kernel is persistent, so every pair must be resident at once: a pair
  // left for a second wave would start its whole share of tiles late. Pairs
  // need two free SMs in one GPC, so fewer than sm_count / 2 may fit.
  static std::atomic<int> resident_pairs[64];  // zero-initialised (static storage)
  if (resident_pairs[dev].load(std::memory_order_acquire) == 0) {
    cfg.gridDim = dim3(2 * (sm_count / 2));
    cfg.attrs = attr;
    cfg.numAttrs = n;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_pair_kernel, &cfg) != cudaSuccess || clusters <= 0)
      return ASHQK_ERR_CUDA;
    resident_pairs[dev].store(std::min(clusters, sm_count / 2), std::memory_order_release);
  }
  const int tiles = a.tiles_m * a.tiles_n;
  const int pairs = std::min(tiles, resident_pairs[dev].load(std::memory_order_acquire));
  cfg.gridDim = dim3(2 * pairs);
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (cudaLaunchKernelEx(&cfg, gemm_tc_pair_kernel, maps, a) != cudaSuccess) return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}

}  // namespace ashqk
