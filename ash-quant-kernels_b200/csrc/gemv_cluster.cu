// Decode GEMV for AWQ W4A16 (M <= 16): output tiles of 256 or 512 columns,
// K streamed in 32 KB stages and split over the CTAs of a thread-block cluster.
//
// Same math as the reference's decode GEMV (ashqk/kernels/w4a16_gemv.py:28-107):
// y = x @ W, W = (q - z) * s, factored per quantization group, fp32
// accumulation:  sum_k x_k (q_kn - z_gn) s_gn = s_gn (sum_k x_k q_kn - z_gn sum_k x_k).
//
// What bounds a streaming kernel on B200 (measured here): a TMA producer's
// round -- wait for a free slot, arm its barrier, issue the copies -- costs
// about 600-700 SM cycles plus about 100 per copy while copies are in flight,
// whatever their size, and one CTA's copies land at ~45 GB/s at most even from
// L2. So every stage carries 32 KB of packed weights (a 256-column tile: one
// 256-row box; a 512-column tile: two 128-row boxes) and its x, and nothing
// else: the scale and zero rows of the CTA's whole K range come once, at the
// start, in one or two copies each.
//
// Work split. A tile's K is cut into stages; a cluster of C CTAs owns one tile
// and deals its stages out in C contiguous ranges. (tile width, C) is chosen per
// shape so that the grid has at most one CTA per SM and the busiest CTA streams
// as few stages as possible. The CTAs of a cluster sum their partial tiles
// through distributed shared memory in rank order (deterministic, no workspace).
//
// Two launches per SM (M <= 8). A CTA takes at most half of an SM's shared
// memory and registers, so the next decode launch (programmatic dependent
// launch) becomes resident beside the running one and issues its first stages
// of weights -- which no kernel writes -- while the running one finishes; only
// x (the previous layer's output) and the stores of y wait for the previous grid.
//
// Consumers: 8 warps, each owning a 64-column strip of the tile and a 128-row
// block of every stage (a 512-column tile: 8 strips x 1 block; 256 columns:
// 4 strips x 2 blocks), so every stage is consumed by all 8 warps. Per 16-row
// step a warp does:
//  * one ldmatrix.x4.trans of its strip: lane (g, t) receives half-word g of
//    rows {2t, 2t+1} (and {2t+8, 2t+9}) of words 0-3 and 4-7 -- four nibbles of
//    one half of a word at two consecutive k, i.e. four columns' mma.sync
//    A-fragment pairs. Stages arrive with the 128-byte TMA swizzle, which puts
//    the eight 16-byte rows of every matrix in distinct banks;
//  * one LOP3 per fragment register: a nibble pair becomes the fp16 pair
//    (1024 + q) or (1024 + 16 q) (the exponent of 1024 ORed over the nibble,
//    csrc/awq_unpack.cuh); the zero point is not subtracted per weight;
//  * mma.sync.m16n8k16 accumulates those against x (tokens along n), plus one
//    mma against ones for the group's sum of x (at one token: one per block,
//    its B columns the block's eight steps);
//  * once per group: sum x (q - z) = f * dot - (c + z) * sum x, with f = 1,
//    c = 1024 (low nibble of a byte) or f = 1/16, c = 64 (high nibble), times
//    the scale, into the fp32 accumulator.
// x arrives token-interleaved ([16-k pair][token][16 k], 32-byte swizzle) so
// one ldmatrix.x4 gives the B fragments of two steps for 8 tokens without bank
// conflicts. Every wait is bounded; a wait that runs out sets the device error
// word and the cluster skips its stores.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "awq_unpack.cuh"
#include "sm100.cuh"

namespace ashqk {
namespace {

constexpr int kStripCols = 64;             // columns per consumer warp
constexpr int kBlockRows = 128;            // rows per consumer warp per stage
constexpr int kStepBytes = 16 * 128;       // 16 rows of a 128-byte box row
constexpr int kStageWeightBytes = 32768;   // packed weights per stage
constexpr int kConsumers = 8;
// A consumed stage holds the partial strips of all consumer warps (16 tokens at most) before they are sent.
static_assert(kStageWeightBytes >= kConsumers * kStripCols * 16 * 4, "staging area");
constexpr int kMaxRing = 8;
constexpr int kMaxCluster = 16;

struct ClusterArgs {
  __half* y;
  int64_t y_ld;
  int M, N, K, G;
  int W;            // tile columns: 256 or 512
  int R;            // rows per stage: 65536 / W
  int tiles;        // ceil(N / W)
  int stages;       // per tile: ceil(K / R)
  int C;            // CTAs per cluster (K split), == gridDim.x
  int ring;         // stages resident in shared memory
  int stage_bytes;  // multiple of 1024
  int x_off;        // x within a stage
  // Scale / zero area: scale rows [W / 256][sz_rows][256] fp16, then zero rows [sz_rows][W / 8] int32.
  // hoisted: one area for the CTA's whole K range, loaded once (sz_off from the shared-memory base);
  // otherwise one per stage with the rows of that stage's groups (sz_off from the stage's base).
  int hoisted;
  int sz_off;
  int z_off;        // zero rows within the area
  int sz_rows;      // rows the area holds: >= the groups its K range spans
  int sz_box_rows;  // rows per copy
  int tile_off;     // byte offset of the CTA's partial tile (outside the ring)
  int presum;       // the blocks of a strip are added in the CTA before the exchange (else sent apart)
  int y_pairs;      // y rows allow 4-byte half2 stores
  uint32_t tx_bytes;     // per stage: weights, x (and the area when not hoisted)
  uint32_t sz_tx_bytes;  // a hoisted area
};

struct ClusterMaps {
  CUtensorMap qw, x, s, z;
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// Part r of n equal contiguous parts of [0, total).
__host__ __device__ __forceinline__ int part_lo(int r, int total, int n) {
  return static_cast<int>(static_cast<long long>(r) * total / n);
}

// Cluster barrier in two halves: arrive early, wait when needed.
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Stores into another CTA's shared memory that complete on that CTA's mbarrier (bytes counted).
__device__ __forceinline__ void st_async_v4(uint32_t remote_addr, uint4 v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   remote_addr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void sts_f32x2(uint32_t addr, float v0, float v1) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(v0), "f"(v1) : "memory");
}

// TOKS: 1 (M == 1), 8 (M <= 8) or 16 (M <= 16). GB: one quantization group per 128-row block
// (G % 128 == 0), so groups change only at block starts.
template <int TOKS, bool GB>
__global__ void __launch_bounds__(32 * (kConsumers + 1), TOKS > 8 ? 1 : 2)
    gemv_cluster_kernel(const __grid_constant__ ClusterMaps maps, const ClusterArgs a) {
  constexpr int MT = TOKS > 8 ? 2 : 1;  // 8-token tiles
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kMaxRing];
  __shared__ uint64_t empty[kMaxRing];
  __shared__ uint64_t sz_full;   // the CTA's scale and zero rows have landed
  __shared__ uint64_t partials;  // the other CTAs' partial strips for this CTA have arrived
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = blockIdx.x;  // == rank in the cluster (gridDim.x == C)
  const int tile = blockIdx.y;
  const int C = a.C;
  const int st0 = part_lo(rank, a.stages, C);
  const int nloc = part_lo(rank + 1, a.stages, C) - st0;
  const int M = a.M, R = a.R, G = a.G, ring = a.ring, stage_bytes = a.stage_bytes;
  const int W = a.W, strips = W / kStripCols, blocks = kConsumers / strips;
  const int my_strips = strips > rank ? (strips - rank + C - 1) / C : 0;  // strips rank, rank + C, ...
  // Partial strips per stored strip: one per CTA (presum) or one per (CTA, block) at slot rank * blocks + block.
  const int nsend = a.presum ? C : C * blocks;
  // The partial strips this CTA stores: [my_strips][nsend][64 columns][M] fp32.
  float* slots = reinterpret_cast<float*>(smem + a.tile_off);

  if (threadIdx.x == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumers);
    }
    mbar_init(&sz_full, 1);
    mbar_init(&partials, 1);
    if (C > 1 && my_strips > 0)  // what the other CTAs will store here with st.async
      mbar_arrive_expect_tx(&partials,
                            static_cast<uint32_t>(my_strips * (C - 1) * (nsend / C) * kStripCols * M * 4));
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (C > 1) cluster_arrive_release();  // the barriers above are ready before any CTA sends
  pdl_launch_dependents();

  float acc[MT][4][4];  // consumer warps: this warp's strip, fp32
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[mt][j][r] = 0.f;

  if (warp == kConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&maps.qw);
      prefetch_tensormap(&maps.x);
      prefetch_tensormap(&maps.s);
      prefetch_tensormap(&maps.z);
      const int boxes = W / 256;
      const int col_words = tile * (W / 8);
      const int x_off = a.x_off;
      const uint32_t tx = a.tx_bytes;
      // Scale and zero rows from group g0 into the area at sz, completing on bar.
      auto issue_sz = [&](unsigned char* sz, int g0, uint64_t* bar) {
        for (int r = 0; r < a.sz_rows; r += a.sz_box_rows) {
          for (int b = 0; b < boxes; ++b)
            tma_load_2d(sz + (b * a.sz_rows + r) * 512, &maps.s, 8 * col_words + 256 * b, g0 + r, bar);
          tma_load_2d(sz + a.z_off + r * (W / 2), &maps.z, col_words, g0 + r, bar);
        }
      };
      if (a.hoisted) {  // every group this CTA's stages touch, before any stage
        mbar_arrive_expect_tx(&sz_full, a.sz_tx_bytes);
        issue_sz(smem + a.sz_off, st0 * R / G, &sz_full);
      }
      auto issue_weights = [&](int li, int slot) {
        const int k0 = (st0 + li) * R;
        unsigned char* base = smem + slot * stage_bytes;
        mbar_arrive_expect_tx(&full[slot], tx);
        for (int b = 0; b < boxes; ++b) tma_load_2d(base + b * R * 128, &maps.qw, col_words + 32 * b, k0, &full[slot]);
        if (!a.hoisted) issue_sz(base + a.sz_off, k0 / G, &full[slot]);
      };
      auto issue_x = [&](int li, int slot) {
        tma_load_3d(smem + slot * stage_bytes + x_off, &maps.x, 0, 0, (st0 + li) * R / 16, &full[slot]);
      };
      const int prologue = min(nloc, ring);
      for (int li = 0; li < prologue; ++li) issue_weights(li, li);
      pdl_wait();  // x is the previous kernel's output
      for (int li = 0; li < prologue; ++li) issue_x(li, li);
      int issued = prologue;
      for (int li = prologue; li < nloc; ++li) {
        const int slot = li % ring;
        if (!mbar_wait(&empty[slot], ((li / ring) - 1) & 1, &abort_flag, true)) break;
        issue_weights(li, slot);
        issue_x(li, slot);
        ++issued;
      }
      if (abort_flag) {  // let every issued copy land before the CTA's shared memory is released
        int unused = 0;
        if (a.hoisted) mbar_wait(&sz_full, 0, &unused);
        for (int slot = 0; slot < ring && slot < issued; ++slot)
          mbar_wait(&full[slot], ((issued - 1 - slot) / ring) & 1, &unused);
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    pdl_wait();  // y may only be written after the previous kernel ends
    const int strip = warp % strips;
    const int block = warp / strips;  // 128-row block of every stage
    const int g = lane >> 2;
    const int wA = g >> 1;  // word of A-row g (columns 8 wA + 2 j + hA); A-row g + 8: word 4 + wA
    const int hA = g & 1;   // half of the word: nibbles 4 hA .. 4 hA + 3
    const uint32_t smem_s = smem_u32(smem);
    // Weights: box strip / 4 of the stage, 16-byte chunks 2 (strip % 4) and +1 of each 128-byte row.
    // ldmatrix matrix q = lane / 8: rows 8 (q / 2) + lane % 8 of the step, chunk + q % 2; the 128-byte
    // swizzle moves chunk c of row r to c ^ (r % 8), and r % 8 == lane % 8 here.
    const int lq = lane >> 3, lr = lane & 7;
    const uint32_t w_lane = static_cast<uint32_t>((strip >> 2) * R * 128 +
                                                  (block * kBlockRows + 8 * (lq >> 1) + lr) * 128 +
                                                  16 * ((2 * (strip & 3) + (lq & 1)) ^ lr));
    // x: matrix q holds 16-row pair (step) s + q / 2 of the block, k half q % 2; row r = token 8 mt + r
    // (token 0 past M: those columns of the mma are never read). Byte offset of pair p for tile mt:
    // row = p * M + token (32 bytes), chunk half ^ (row / 4 % 2) (32-byte swizzle).
    int xtok[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) xtok[mt] = (8 * mt + lr < M) ? 8 * mt + lr : 0;
    const int xq_pair = block * (kBlockRows / 16) + (lq >> 1), xq_half = lq & 1;
    auto x_addr = [&](uint32_t xbase, int s, int mt) {
      const int row = (xq_pair + s) * M + xtok[mt];
      return xbase + row * 32 + 16 * (xq_half ^ ((row >> 2) & 1));
    };
    const int x_off = a.x_off;
    // One token and whole-block groups: the block's sum of x comes from one mma per stage against
    // ones whose B column n is step n of the block (ldmatrix row n = x row n of the block, k halves
    // as matrices 0 and 1), added over the columns afterwards, instead of an mma against ones at every
    // step: a fifth of the tensor work, which bounds a stage when two CTAs share an SM. (With 2 or 4
    // tokens, M such mma per block measured slower than the per-step form.)
    constexpr bool kBlockSumX = TOKS == 1 && GB;
    const int xs_row = block * (kBlockRows / 16) + (lane & 7);
    const uint32_t xs_lane = static_cast<uint32_t>(xs_row * 32 + 16 * (((lane >> 3) & 1) ^ ((xs_row >> 2) & 1)));
    // Scale row r of this strip's box: (strip / 4) * sz_rows + r rows of 512 bytes; zero row r: W / 2 bytes.
    const uint32_t s_lane =
        static_cast<uint32_t>(a.sz_off + (strip >> 2) * a.sz_rows * 512 + (strip & 3) * 128);
    const uint32_t z_lane = static_cast<uint32_t>(a.sz_off + a.z_off + strip * 32);
    const int z_pitch = W / 2;
    uint32_t sz_base = smem_s;     // the area holding the current stage's groups
    int g_ref = st0 * R / G;       // the group in its row 0

    float part[MT][4][4], psx[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) part[mt][j][r] = 0.f;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int r = 0; r < 4; ++r) psx[mt][r] = 0.f;
    float ca[8], cb[8];  // per group: scale * f and -scale * (c + z) of A-rows g (0..3) and g + 8 (4..7)
#pragma unroll
    for (int i = 0; i < 8; ++i) ca[i] = cb[i] = 0.f;

    auto flush = [&]() {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[mt][j][0] = fmaf(ca[j], part[mt][j][0], fmaf(cb[j], psx[mt][0], acc[mt][j][0]));
          acc[mt][j][2] = fmaf(ca[4 + j], part[mt][j][2], fmaf(cb[4 + j], psx[mt][0], acc[mt][j][2]));
          if (TOKS > 1) {
            acc[mt][j][1] = fmaf(ca[j], part[mt][j][1], fmaf(cb[j], psx[mt][1], acc[mt][j][1]));
            acc[mt][j][3] = fmaf(ca[4 + j], part[mt][j][3], fmaf(cb[4 + j], psx[mt][1], acc[mt][j][3]));
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) part[mt][j][r] = 0.f;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) psx[mt][r] = 0.f;
      }
    };

    // Scale and zero point of this lane's 8 columns for group g_ref + gslot.
    auto load_group = [&](int gslot) {
      const uint32_t srow = sz_base + s_lane + gslot * 512;
      const uint4 sa = lds_v4(srow + 16 * wA);
      const uint4 sb = lds_v4(srow + 16 * (4 + wA));
      const uint32_t zrow = sz_base + z_lane + gslot * z_pitch;
      const uint32_t za = lds_u32(zrow + 4 * wA) >> (16 * hA);
      const uint32_t zb = lds_u32(zrow + 4 * (4 + wA)) >> (16 * hA);
      const uint32_t sav[4] = {sa.x, sa.y, sa.z, sa.w};
      const uint32_t sbv[4] = {sb.x, sb.y, sb.z, sb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // column 2 j + hA of the word: half hA of scale component j, nibble 4 hA + j of the zero word
        const float f = (j & 1) ? 0.0625f : 1.f;
        const float s_a = half_bits_to_float(sav[j] >> (16 * hA));
        const float s_b = half_bits_to_float(sbv[j] >> (16 * hA));
        // c + z exactly: z ORed into the mantissa of 1024.0f (unit 2^-13 there) or of 64.0f (2^-17)
        const uint32_t base_bits = (j & 1) ? 0x42800000u : 0x44800000u;
        const int sh = (j & 1) ? 17 : 13;
        const float cz_a = __uint_as_float(base_bits | (((za >> (4 * j)) & 15u) << sh));
        const float cz_b = __uint_as_float(base_bits | (((zb >> (4 * j)) & 15u) << sh));
        ca[j] = s_a * f;
        cb[j] = -s_a * cz_a;
        ca[4 + j] = s_b * f;
        cb[4 + j] = -s_b * cz_b;
      }
    };

    const uint32_t ones_a[4] = {kOneX2, kOneX2, kOneX2, kOneX2};
    // One 16-row step: the weights R4 of this lane against the x fragments b0, b1; `first`
    // starts the block's sums from zero instead of adding to them.
    auto step = [&](const uint32_t (&R4)[4], const uint32_t (&bx)[MT][4], int h, bool first) {
      uint32_t R8[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) R8[i] = R4[i] >> 8;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t mask = (j & 1) ? kHiNibbles : kLoNibbles;
        uint32_t A[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) A[i] = lop3_and_or(j < 2 ? R4[i] : R8[i], mask, kMagic1024x2);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if (first)
            mma_16816_first(part[mt][j], A, bx[mt][2 * h], bx[mt][2 * h + 1]);
          else
            mma_16816(part[mt][j], A, bx[mt][2 * h], bx[mt][2 * h + 1]);
        }
      }
      if constexpr (!kBlockSumX) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if (first)
            mma_16816_first(psx[mt], ones_a, bx[mt][2 * h], bx[mt][2 * h + 1]);
          else
            mma_16816(psx[mt], ones_a, bx[mt][2 * h], bx[mt][2 * h + 1]);
        }
      }
    };
    // Whole-block groups (G % 128 == 0): fold the block's sums into acc with its group's scale and
    // zero point, read from the stage now (nothing to zero: the next block starts from zero).
    auto fold_block = [&](int gslot) {
      load_group(gslot);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[mt][j][0] = fmaf(ca[j], part[mt][j][0], fmaf(cb[j], psx[mt][0], acc[mt][j][0]));
          acc[mt][j][2] = fmaf(ca[4 + j], part[mt][j][2], fmaf(cb[4 + j], psx[mt][0], acc[mt][j][2]));
          if (TOKS > 1) {
            acc[mt][j][1] = fmaf(ca[j], part[mt][j][1], fmaf(cb[j], psx[mt][1], acc[mt][j][1]));
            acc[mt][j][3] = fmaf(ca[4 + j], part[mt][j][3], fmaf(cb[4 + j], psx[mt][1], acc[mt][j][3]));
          }
        }
    };

    int cur_grp = -1;
    int grp_end = -1;
    auto enter_group = [&](int k) {
      if (k >= grp_end) {  // a new quantization group (rows past K read zero scales: no effect)
        if (cur_grp >= 0) flush();
        cur_grp = k / G;
        grp_end = (cur_grp + 1) * G;
        load_group(cur_grp - g_ref);
      }
    };
    // A hoisted scale / zero area is complete before the first group is read.
    const bool sz_ok = !a.hoisted || mbar_wait(&sz_full, 0, &abort_flag, true);
    for (int li = 0; sz_ok && li < nloc; ++li) {
      const int slot = li % ring;
      if (!mbar_wait(&full[slot], (li / ring) & 1, &abort_flag, true)) break;
      const uint32_t base = smem_s + slot * stage_bytes;
      const int k0 = (st0 + li) * R;
      const int kb = k0 + block * kBlockRows;
      if (!a.hoisted) {
        sz_base = base;
        g_ref = k0 / G;
      }
      const uint32_t wbase = base + w_lane;
      const uint32_t xbase = base + x_off;
      // Loads run one step pair ahead of the arithmetic; the block's x rows for its sum of x load with
      // the first pair and their mma follows that pair's steps.
      uint32_t bx[MT][4], Ra[4], Rb[4], bs[2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) ldsm_x4(x_addr(xbase, 0, mt), bx[mt]);
      ldsm_x4_trans(wbase, Ra);
      ldsm_x4_trans(wbase + kStepBytes, Rb);
      if constexpr (kBlockSumX) ldsm_x2(xbase + xs_lane, bs);
#pragma unroll
      for (int s = 0; s < kBlockRows / 16; s += 2) {
        uint32_t bxn[MT][4], Ran[4], Rbn[4];
        if (s + 2 < kBlockRows / 16) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) ldsm_x4(x_addr(xbase, s + 2, mt), bxn[mt]);
          ldsm_x4_trans(wbase + (s + 2) * kStepBytes, Ran);
          ldsm_x4_trans(wbase + (s + 3) * kStepBytes, Rbn);
        }
        if (!GB) enter_group(kb + 16 * s);
        step(Ra, bx, 0, GB && s == 0);
        if (!GB) enter_group(kb + 16 * (s + 1));
        step(Rb, bx, 1, false);
        if (kBlockSumX && s == 0) mma_16816_first(psx[0], ones_a, bs[0], bs[1]);  // column n: step n's sum
        if (s + 2 < kBlockRows / 16) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            Ra[i] = Ran[i];
            Rb[i] = Rbn[i];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) bx[mt][i] = bxn[mt][i];
          }
        }
      }
      if constexpr (kBlockSumX) {  // lane (g, t) holds steps 2t and 2t + 1
        float v = psx[0][0] + psx[0][1];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        psx[0][0] = v;
      }
      if (GB) fold_block(kb / G - g_ref);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (!GB && cur_grp >= 0) flush();
  }

  // ---------------- the cluster's sum ----------------
  // Strip s of the tile is stored by CTA s % C of the cluster. The consumer warps lay their partial
  // strips out in this CTA's consumed ring ([64 columns][M tokens] fp32 each) and hand them to the
  // owner's slots in 16-byte st.async pieces that complete on the owner's `partials` barrier (plain
  // stores when the owner is this CTA). With presum (M > 4, where the slots would crowd out the ring)
  // the blocks of each strip are first added here, in block order, and the CTA sends one partial per
  // strip to slot [rank]; otherwise warp (strip, block) sends its own to slot [rank * blocks + block].
  // The owner adds its slots in that fixed order (deterministic) and stores y.
  if (C > 1) cluster_wait_acquire();  // every CTA's `partials` barrier is armed
  if (warp < kConsumers) {
    const int strip = warp % strips, block = warp / strips;
    const int g = lane >> 2, t = lane & 3, wA = g >> 1, hA = g & 1;
    const int owner = strip % C;
    const bool remote = owner != rank;
    const uint32_t strip_bytes = static_cast<uint32_t>(kStripCols * M * 4);
    const bool presum = a.presum != 0;
    // Every consumer warp is past its last stage before any of them reuses the ring.
    if (presum || C > 1) asm volatile("bar.sync 1, %0;" ::"r"(32 * kConsumers) : "memory");
    const uint32_t stg = smem_u32(smem);  // warp w's partial strip at stg + w * strip_bytes
    // Without presum a strip owned here goes straight into its slot.
    const uint32_t direct_slot = static_cast<uint32_t>((strip / C) * nsend + rank * blocks + block) * strip_bytes;
    const uint32_t dst = (presum || remote) ? stg + static_cast<uint32_t>(warp) * strip_bytes
                                            : smem_u32(slots) + direct_slot;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {  // column c (rows g) or c + 32 (rows g + 8)
          const int c = 8 * wA + 2 * j + hA + 32 * hh;
          const int m0 = 8 * mt + 2 * t;
          const uint32_t addr = dst + static_cast<uint32_t>((c * M + m0) * 4);
          const float v0 = acc[mt][j][2 * hh], v1 = acc[mt][j][2 * hh + 1];
          if (TOKS > 1 && m0 + 1 < M && (M & 1) == 0) {  // an 8-byte aligned pair of tokens
            sts_f32x2(addr, v0, v1);
          } else {
            if (m0 < M) sts_f32(addr, v0);
            if (TOKS > 1 && m0 + 1 < M) sts_f32(addr + 4, v1);
          }
        }
    const int pieces = kStripCols * M / 4;
    if (presum) {
      asm volatile("bar.sync 1, %0;" ::"r"(32 * kConsumers) : "memory");  // every block's strip is laid out
      // The warps of strip s share its 16-byte pieces: warp (s, b) adds and sends part b of blocks.
      const int lo = part_lo(block, pieces, blocks), hi = part_lo(block + 1, pieces, blocks);
      const uint32_t slot = static_cast<uint32_t>((strip / C) * nsend + rank) * strip_bytes;
      const uint32_t out = remote ? map_shared_rank(slots, owner) + slot : smem_u32(slots) + slot;
      const uint32_t bar = remote ? map_shared_rank(&partials, owner) : 0u;
      for (int i = lo + lane; i < hi; i += 32) {
        float4 v = lds_f4(stg + static_cast<uint32_t>(strip) * strip_bytes + 16 * i);
        for (int b = 1; b < blocks; ++b) {
          const float4 u = lds_f4(stg + static_cast<uint32_t>(b * strips + strip) * strip_bytes + 16 * i);
          v.x += u.x;
          v.y += u.y;
          v.z += u.z;
          v.w += u.w;
        }
        const uint4 bits = make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z),
                                      __float_as_uint(v.w));
        if (remote)
          st_async_v4(out + 16 * i, bits, bar);
        else
          sts_v4(out + 16 * i, bits);
      }
    } else if (remote) {
      __syncwarp();
      const uint32_t rdst = map_shared_rank(slots, owner) + direct_slot;
      const uint32_t bar = map_shared_rank(&partials, owner);
      for (int i = lane; i < pieces; i += 32) st_async_v4(rdst + 16 * i, lds_v4(dst + 16 * i), bar);
    }
  }
  __syncthreads();  // this CTA's own strips are in its slots
  bool failed = abort_flag != 0;
  if (my_strips > 0) {
    if (C > 1) {
      int unused = 0;
      failed |= !mbar_wait(&partials, 0, &unused);
    }
    const int nthreads = 32 * (kConsumers + 1);
    for (int i = threadIdx.x; i < my_strips * kStripCols * M; i += nthreads) {
      const int os = i / (kStripCols * M), rem = i % (kStripCols * M);  // rem = c * M + m
      const float* src = slots + os * nsend * kStripCols * M + rem;
      float v = 0.f;
      for (int sdr = 0; sdr < nsend; ++sdr) v += src[sdr * kStripCols * M];
      const int c = rem / M, m = rem % M;
      const int col = tile * W + (os * C + rank) * kStripCols + c;
      if (!failed && col < a.N) a.y[m * a.y_ld + col] = __float2half_rn(v);
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side: plan, tensor maps, launch.
// ---------------------------------------------------------------------------

struct ClusterPlan {
  int W, R, tiles, stages, C, ctas, per, ring, stage_bytes, x_off, hoisted, sz_off, z_off, sz_rows, sz_box_rows,
      tile_off, toks;
  uint32_t tx, sz_tx;
  size_t smem;
};

namespace {

// Process-wide tuning of the plan (0 = automatic), set by ashqk_gemv_set_tuning.
std::atomic<int> g_smem_kb{0};
std::atomic<int> g_force_c{0};
std::atomic<int> g_force_w{0};
std::atomic<int> g_max_ctas{0};

int align_to(int v, int a) { return (v + a - 1) / a * a; }

// Quantization groups that `stages` consecutive stages of R rows (starting on a stage boundary) span.
int groups_spanned(int stages, int R, int G) {
  if (R % G == 0) return stages * R / G;
  if (stages == 1 && G % R == 0) return 1;
  return (stages * R + G - 1) / G + 1;
}

}  // namespace

// split > 0: the caller's K split (the reference's split_k): that many CTAs per cluster, at most 16 and
// at most the tile's stages.
bool plan_cluster(int M, int N, int K, int G, int sm_count, ClusterPlan* p, int split) {
  if (M < 1 || M > 16 || N % 32 || G % 16 || sm_count < 1) return false;
  const int toks = M == 1 ? 1 : (M <= 8 ? 8 : 16);
  const int smem_kb = g_smem_kb.load(std::memory_order_relaxed);
  // M <= 8: two CTAs (this launch's and the next one's) per SM, 2 x (dynamic + ~0.5 KB static + 1 KB
  // reserved) within the SM's 228 KB; M > 8 needs the register file of a whole SM.
  // Small quantization groups make the scale / zero area large: when nothing fits two per SM, one per SM.
  const size_t budget0 = smem_kb > 0 ? static_cast<size_t>(smem_kb) * 1024 : (M <= 8 ? 112 : 200) * 1024;
  // Grid cap (measured on B200). M <= 8: up to ~1.65 CTAs per SM -- an SM that holds two CTAs of the
  // launch runs 16 consumer warps and gets through its stages ~1.7x faster than with one, while more
  // than ~1.65 per SM leaves clusters that cannot be placed with the others (a second wave). M > 8:
  // one CTA per SM at most (the 16-token variant needs an SM's register file), and only ~0.65 of
  // the SMs, so that the next launch finds free SMs to start streaming on. A tuning cap overrides.
  const int max_ctas = g_max_ctas.load(std::memory_order_relaxed) > 0
                           ? std::min(g_max_ctas.load(std::memory_order_relaxed), 2 * sm_count)
                           : (M <= 8 ? sm_count * 33 / 20 : sm_count * 13 / 20);
  const int force_c = split > 0 ? std::min(split, kMaxCluster) : g_force_c.load(std::memory_order_relaxed);
  const int force_w = g_force_w.load(std::memory_order_relaxed);

  // Estimated time in stage units (measured on B200, decode shapes): the busiest CTA's stages, x1.18
  // when some SMs hold two CTAs (each then runs at ~0.85 of its speed alone); clusters cost a
  // partial-strip exchange that grows with C and M: +0.5 stage past 8 CTAs for M <= 8, +1 stage per
  // CTA for M > 8 (16 tokens of partials per column).
  bool found = false;
  double best_cost = 0.0;
  int best_key[3] = {0, 0, 0};
  auto search = [&](size_t budget, int cta_cap) {
    for (int W : {256, 512}) {
      if (force_w && W != force_w) continue;
      for (int hoisted = 1; hoisted >= 0; --hoisted) {
        ClusterPlan q;
        q.toks = toks;
        q.W = W;
        q.R = kStageWeightBytes * 2 / W;
        q.tiles = ceil_div(N, W);
        q.stages = ceil_div(K, q.R);
        q.x_off = kStageWeightBytes;
        q.hoisted = hoisted;
        const int sz_row_bytes = (W / 256) * 512 + W / 2;
        const int fc = split > 0 ? std::min(force_c, q.stages) : force_c;
        for (int C = 1; C <= kMaxCluster; ++C) {
          if (fc && C != fc) continue;
          if (C > q.stages) break;
          q.C = C;
          q.ctas = q.tiles * C;
          if (q.ctas > cta_cap && !(fc || (C == 1 && q.tiles > cta_cap))) continue;
          q.per = ceil_div(q.stages, C);
          // The partial strips this CTA stores: [ceil(strips / C)][C * blocks][64][M] fp32.
          const int strips = W / kStripCols, blocks = kConsumers / strips;
          // presum (M > 4): one partial per CTA and strip; else one per CTA, strip and block.
          const size_t slots =
              static_cast<size_t>(ceil_div(strips, C)) * C * (M > 4 ? 1 : blocks) * kStripCols * M * 4;
          // The scale / zero area: the groups of the longest stage range (hoisted) or of one stage, in
          // copies of at most 256 rows.
          const int span = groups_spanned(hoisted ? q.per : 1, q.R, G);
          const int nbox = ceil_div(span, 256);
          q.sz_box_rows = ceil_div(span, nbox);
          q.sz_rows = nbox * q.sz_box_rows;
          q.z_off = (W / 256) * q.sz_rows * 512;
          const int sz_bytes = q.sz_rows * sz_row_bytes;
          size_t hoisted_bytes = 0;
          if (hoisted) {
            q.stage_bytes = align_to(q.x_off + align_to(2 * q.R * M, 128), 1024);
            q.tx = static_cast<uint32_t>(kStageWeightBytes + 2 * q.R * M);
            q.sz_tx = static_cast<uint32_t>(sz_bytes);
            hoisted_bytes = static_cast<size_t>(align_to(sz_bytes, 1024));
          } else {
            q.sz_off = q.x_off + align_to(2 * q.R * M, 128);
            q.stage_bytes = align_to(q.sz_off + sz_bytes, 1024);
            q.tx = static_cast<uint32_t>(kStageWeightBytes + 2 * q.R * M + sz_bytes);
            q.sz_tx = 0;
          }
          if (slots + hoisted_bytes + 1024 + q.stage_bytes > budget) continue;
          int ring = static_cast<int>((budget - 1024 - slots - hoisted_bytes) / q.stage_bytes);
          ring = std::min(std::min(ring, kMaxRing), q.per);
          if (ring < 1 || (ring < 2 && q.per > 1)) continue;
          q.ring = ring;
          if (hoisted) q.sz_off = ring * q.stage_bytes;
          q.tile_off = ring * q.stage_bytes + static_cast<int>(hoisted_bytes);
          q.smem = 1024 + static_cast<size_t>(q.tile_off) + slots;
          // Per-stage scale / zero copies cost ~3% over a hoisted area (measured on the decode shapes).
          const double cost = (M <= 8 ? q.per * (q.ctas > sm_count ? 1.18 : 1.0) + (C > 8 ? 0.5 : 0.0)
                                      : static_cast<double>(q.per + C)) *
                              (hoisted ? 1.0 : 1.03);
          // ties: the 256-column tile (fewer copies per stage), then smaller clusters
          const int key[3] = {W == 256 ? 0 : 1, C, 0};
          if (!found || cost < best_cost - 1e-9 ||
              (cost < best_cost + 1e-9 && std::lexicographical_compare(key, key + 3, best_key, best_key + 3))) {
            found = true;
            best_cost = cost;
            std::copy(key, key + 3, best_key);
            *p = q;
          }
        }
      }
    }
  };
  search(budget0, max_ctas);
  if (!found && smem_kb == 0 && budget0 < 200 * 1024) search(200 * 1024, std::min(max_ctas, sm_count));
  if (!found && smem_kb == 0 && budget0 < 200 * 1024) search(200 * 1024, max_ctas);
  return found;
}

namespace {

template <int TOKS, bool GB>
int launch_cluster_t(const ClusterMaps& maps, const ClusterArgs& args, size_t smem, cudaStream_t stream) {
  static std::atomic<bool> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ASHQK_ERR_CUDA;
  auto kernel = gemv_cluster_kernel<TOKS, GB>;
  if (!configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
        cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      return ASHQK_ERR_CUDA;
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(args.C, args.tiles);
  cfg.blockDim = dim3(32 * (kConsumers + 1));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (args.C > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = args.C;
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
  if (cudaLaunchKernelEx(&cfg, kernel, maps, args) != cudaSuccess) return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}

}  // namespace

bool gemv_cluster_plannable(int M, int N, int K, int G, int sm_count, int split) {
  ClusterPlan p;
  return plan_cluster(M, N, K, G, sm_count, &p, split);
}

bool gemv_cluster_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                           int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int G) {
  return M >= 1 && M <= 16 && N % 32 == 0 && G % 16 == 0 && aligned(qw, 16) && qw_ld % 4 == 0 && aligned(qz, 16) &&
         qz_ld % 4 == 0 && aligned(s, 16) && s_ld % 8 == 0 && aligned(x, 16) && x_ld % 8 == 0;
}

int gemv_cluster_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                        int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K,
                        int G, int split, int sm_count, cudaStream_t stream) {
  ClusterPlan p;
  if (!plan_cluster(M, N, K, G, sm_count, &p, split)) return ASHQK_ERR_UNSUPPORTED;
  ClusterMaps maps;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N / 8), static_cast<uint64_t>(K)};
    const uint64_t strides[1] = {static_cast<uint64_t>(qw_ld) * 4};
    const uint32_t box[2] = {32, static_cast<uint32_t>(p.R)};
    int rc = encode_tensor_map(&maps.qw, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qw), dims, strides,
                               box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    // x as [K / 16 pairs][M tokens][16 values]: pairs are 32 bytes apart, tokens x_ld apart.
    const uint64_t dims[3] = {16, static_cast<uint64_t>(M), static_cast<uint64_t>(K / 16)};
    const uint64_t strides[2] = {static_cast<uint64_t>(x_ld) * 2, 32};
    const uint32_t box[3] = {16, static_cast<uint32_t>(M), static_cast<uint32_t>(p.R / 16)};
    int rc = encode_tensor_map(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(x), dims, strides,
                               box, CU_TENSOR_MAP_SWIZZLE_32B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K / G)};
    const uint64_t strides[1] = {static_cast<uint64_t>(s_ld) * 2};
    const uint32_t box[2] = {256, static_cast<uint32_t>(p.sz_box_rows)};
    int rc = encode_tensor_map(&maps.s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(s), dims, strides,
                               box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N / 8), static_cast<uint64_t>(K / G)};
    const uint64_t strides[1] = {static_cast<uint64_t>(qz_ld) * 4};
    const uint32_t box[2] = {static_cast<uint32_t>(p.W / 8), static_cast<uint32_t>(p.sz_box_rows)};
    int rc = encode_tensor_map(&maps.z, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qz), dims, strides,
                               box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  ClusterArgs a = {};
  a.y = y;
  a.y_ld = y_ld;
  a.M = M;
  a.N = N;
  a.K = K;
  a.G = G;
  a.W = p.W;
  a.R = p.R;
  a.tiles = p.tiles;
  a.stages = p.stages;
  a.C = p.C;
  a.ring = p.ring;
  a.stage_bytes = p.stage_bytes;
  a.x_off = p.x_off;
  a.hoisted = p.hoisted;
  a.sz_off = p.sz_off;
  a.z_off = p.z_off;
  a.sz_rows = p.sz_rows;
  a.sz_box_rows = p.sz_box_rows;
  a.tile_off = p.tile_off;
  a.y_pairs = aligned(y, 4) && (y_ld % 2 == 0);
  a.presum = M > 4 ? 1 : 0;
  a.tx_bytes = p.tx;
  a.sz_tx_bytes = p.sz_tx;
  const bool gb = G % kBlockRows == 0;
  switch (p.toks) {
    case 1:
      return gb ? launch_cluster_t<1, true>(maps, a, p.smem, stream) : launch_cluster_t<1, false>(maps, a, p.smem, stream);
    case 8:
      return gb ? launch_cluster_t<8, true>(maps, a, p.smem, stream) : launch_cluster_t<8, false>(maps, a, p.smem, stream);
    default:
      return gb ? launch_cluster_t<16, true>(maps, a, p.smem, stream)
                : launch_cluster_t<16, false>(maps, a, p.smem, stream);
  }
}

}  // namespace ashqk

extern "C" int ashqk_gemv_set_tuning(int smem_kb, int cluster_ctas, int tile_cols, int max_ctas) {
  if (smem_kb < 0 || smem_kb > 200 || cluster_ctas < 0 || cluster_ctas > ashqk::kMaxCluster ||
      (tile_cols != 0 && tile_cols != 256 && tile_cols != 512) || max_ctas < 0)
    return ASHQK_ERR_INVALID_ARGUMENT;
  ashqk::g_smem_kb.store(smem_kb);
  ashqk::g_force_c.store(cluster_ctas);
  ashqk::g_force_w.store(tile_cols);
  ashqk::g_max_ctas.store(max_ctas);
  return ASHQK_OK;
}

extern "C" int ashqk_gemv_cluster_plan(int M, int N, int K, int group_size, int sm_count, ashqk_cluster_plan* plan) {
  if (!plan || M <= 0 || N <= 0 || K <= 0 || group_size <= 0 || N % 8 || K % group_size || sm_count < 0)
    return ASHQK_ERR_INVALID_ARGUMENT;
  if (M > 16 || N % 32 || group_size % 16) return ASHQK_ERR_UNSUPPORTED;
  if (sm_count == 0) {
    ashqk::DeviceInfo info;
    const int rc = ashqk::device_info(&info);
    if (rc) return rc;
    sm_count = info.sm_count;
  }
  ashqk::ClusterPlan p;
  if (!ashqk::plan_cluster(M, N, K, group_size, sm_count, &p, 0)) return ASHQK_ERR_UNSUPPORTED;
  plan->tile_cols = p.W;
  plan->stage_rows = p.R;
  plan->tiles = p.tiles;
  plan->stages_per_tile = p.stages;
  plan->cluster_ctas = p.C;
  plan->ctas = p.ctas;
  plan->max_stages_per_cta = p.per;
  plan->threads = 32 * (ashqk::kConsumers + 1);
  plan->ring_stages = p.ring;
  plan->stage_bytes = p.stage_bytes;
  plan->smem_bytes = static_cast<int>(p.smem);
  return ASHQK_OK;
}
