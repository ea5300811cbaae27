// Decode GEMV for AWQ W4A16 (M <= 16): column strips with the whole K per CTA.
//
// Same math as the other decode kernels (reference ashqk/kernels/w4a16_gemv.py:28-107):
// y = x @ W, W = (q - z) * s, factored per quantization group, fp32 accumulation.
//
// Why this shape: on 2-10 us layers the split-K variants spend as long in their
// prologue (staging x, scales, zeros) and their split-K tail (partial sums to
// global memory, fence, arrival counter, a last CTA re-reading them) as in
// streaming weights. Here a CTA owns 64 output columns over all of K, so there
// is no split-K tail at all, and everything a stage needs -- 256 rows of packed
// weights (a 32-byte wide TMA box), the matching 256 columns of x, and the
// scale / zero rows of the groups it spans -- arrives with one mbarrier phase,
// so there is no prologue either. Many stages (up to ~200 KB) are kept in
// flight per SM: a 64 KB ring lets one SM stream ~49 GB/s, and layers with few
// column strips need more than that per SM.
//
// Warps: one producer (lane 0 issues all TMA loads) and C consumer warps. Ring
// slot j belongs to consumer warp j % C, which consumes every stage that lands
// in it, in order -- so no warp waits on a slot whose previous fill belongs to
// another warp (mbarrier phase parities never alias) -- and runs all 16 of a
// stage's 16-row steps with no further synchronisation, keeping one
// quantization group for G/16 steps.
// A lane unpacks one word (8 columns) of rows {2t, 2t+1, 2t+8, 2t+9} per step
// -- the k order of an mma.sync A fragment -- with the prmt / LOP3 / HSUB2 code
// of csrc/awq_unpack.cuh, and mma.sync.m16n8k16 accumulates sum x (q - z) per
// group in fp32; the scale is applied once per group. At the end the C warps'
// partial tiles are summed in shared memory and y is stored.
//
// Programmatic dependent launch: weights, scales and zeros of the first ring
// stages are requested before griddepcontrol.wait; x (the previous kernel's
// output) after it; y is written only after it.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "awq_unpack.cuh"
#include "ll_lines.cuh"
#include "sm100.cuh"

namespace ashqk {
namespace {

constexpr int kStripCols = 64;
constexpr int kStripWords = kStripCols / 8;
constexpr int kBoxRows = 256;                            // rows per stage (TMA box height limit)
constexpr int kWeightBytes = kBoxRows * kStripWords * 4;  // 8 KB
constexpr int kXRowBytes = kBoxRows * 2;                  // one token's 256 x values
constexpr int kMaxStages = 24;

struct StripArgs {
  __half* y;
  int64_t y_ld;
  int M, N, K, G;
  int stages_total;  // ceil(K / 256)
  int ksplit;        // CTAs (one thread-block cluster) sharing a strip's K range
  int ring;          // stages resident in shared memory
  int gps;           // scale / zero rows loaded per stage
  int stage_bytes;   // bytes of one ring slot (multiple of 128)
  int x_off, s_off, z_off;  // byte offsets of x, scales, zeros inside a slot
  uint32_t tx_bytes;        // transaction bytes per stage
  LLPeers ll;               // regions != nullptr: sum y over the ranks before storing it
};

struct StripMaps {
  CUtensorMap qw, x, s, z;
};

// Sum over the S CTAs of the cluster (fixed rank order; S == 1: the own tile)
// of column c of token m's partial tile.
__device__ __forceinline__ float strip_tile_value(const float* tile_sum, int m, int c, int S) {
  if (S == 1) return tile_sum[m * kStripCols + c];
  float pq[4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
    pq[q] = q < S ? ld_shared_cluster_f32(map_shared_rank(const_cast<float*>(tile_sum) + m * kStripCols + c, q)) : 0.f;
  return ((pq[0] + pq[1]) + pq[2]) + pq[3];
}

// Row-parallel epilogue: this rank's fp16 partial of columns [c_lo, c_hi) of
// the strip (pairs) goes to every peer as low-latency lines (ll_lines.cuh);
// the stored y is the fp32 sum of all ranks' fp16 partials in rank order,
// rounded once -- the same value an unfused GEMV followed by the LL or one-shot
// all-reduce produces.
template <typename Args>
__device__ void strip_allreduce_store(const Args& a, const float* tile_sum, int col0, int c_lo, int c_hi, int S,
                                      unsigned int epoch, int nthreads) {
  const int pairs_per_row = (c_hi - c_lo) / 2;
  const int total = a.M * pairs_per_row;
  for (int i = threadIdx.x; i < total; i += nthreads) {
    const int m = i / pairs_per_row, c = c_lo + 2 * (i % pairs_per_row);
    if (col0 + c >= a.N) continue;
    const __half2 h = __floats2half2_rn(strip_tile_value(tile_sum, m, c, S), strip_tile_value(tile_sum, m, c + 1, S));
    ll_push(a.ll, epoch, static_cast<long long>(m) * (a.N / 2) + (col0 + c) / 2, *reinterpret_cast<const unsigned int*>(&h));
  }
  bool failed = false;
  for (int i = threadIdx.x; i < total && !failed; i += nthreads) {
    const int m = i / pairs_per_row, c = c_lo + 2 * (i % pairs_per_row);
    if (col0 + c >= a.N) continue;
    const __half2 h = __floats2half2_rn(strip_tile_value(tile_sum, m, c, S), strip_tile_value(tile_sum, m, c + 1, S));
    const float2 v = ll_pull_sum(a.ll, epoch, static_cast<long long>(m) * (a.N / 2) + (col0 + c) / 2,
                                 *reinterpret_cast<const unsigned int*>(&h), failed);
    if (!failed) *reinterpret_cast<__half2*>(a.y + m * a.y_ld + col0 + c) = __floats2half2_rn(v.x, v.y);
  }
}

// FUSED: row-parallel tensor parallelism -- y is this rank's partial over its K
// shard, summed over the ranks in the epilogue (strip_allreduce_store) before
// it is stored.
template <int MT, int C, bool FUSED>
__global__ void __launch_bounds__(32 * (C + 1)) gemv_strip_kernel(const __grid_constant__ StripMaps maps,
                                                                  const StripArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kMaxStages];
  __shared__ uint64_t empty[kMaxStages];
  __shared__ int abort_flag;
  __shared__ unsigned int ll_epoch;
  __shared__ int ll_skip;

  const int strip = blockIdx.x;
  const int col0 = strip * kStripCols;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // This CTA's stages of the strip's K range (blockIdx.y of a.ksplit).
  const int sb = static_cast<int>(static_cast<int64_t>(blockIdx.y) * a.stages_total / a.ksplit);
  const int se = static_cast<int>(static_cast<int64_t>(blockIdx.y + 1) * a.stages_total / a.ksplit);
  const int nloc = se - sb;

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[mt][j][r] = 0.f;

  if (warp == C) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&maps.qw);
      prefetch_tensormap(&maps.x);
      prefetch_tensormap(&maps.s);
      prefetch_tensormap(&maps.z);
      auto issue_weights = [&](int i, int slot) {
        unsigned char* base = smem + slot * a.stage_bytes;
        const int k0 = i * kBoxRows;
        mbar_arrive_expect_tx(&full[slot], a.tx_bytes);
        tma_load_2d(base, &maps.qw, strip * kStripWords, k0, &full[slot]);
        tma_load_2d(base + a.s_off, &maps.s, col0, k0 / a.G, &full[slot]);
        tma_load_2d(base + a.z_off, &maps.z, strip * kStripWords, k0 / a.G, &full[slot]);
      };
      auto issue_x = [&](int i, int slot) {
        tma_load_2d(smem + slot * a.stage_bytes + a.x_off, &maps.x, i * kBoxRows, 0, &full[slot]);
      };
      const int prologue = min(nloc, a.ring);
      for (int li = 0; li < prologue; ++li) issue_weights(sb + li, li);
      pdl_wait();  // x is the previous kernel's output
      for (int li = 0; li < prologue; ++li) issue_x(sb + li, li);
      int issued = prologue;
      for (int li = prologue; li < nloc; ++li) {
        const int slot = li % a.ring;
        if (!mbar_wait(&empty[slot], ((li / a.ring) - 1) & 1, &abort_flag)) break;
        issue_weights(sb + li, slot);
        issue_x(sb + li, slot);
        ++issued;
      }
      if (abort_flag) {
        int unused = 0;
        for (int slot = 0; slot < a.ring && slot < issued; ++slot)
          mbar_wait(&full[slot], ((issued - 1 - slot) / a.ring) & 1, &unused);
      }
    }
  } else {
    // ---------------- consumers ----------------
    pdl_wait();  // y may only be written after the previous kernel ends
    const int g = lane >> 2;
    const int t = lane & 3;
    const uint32_t smem_s = smem_u32(smem);
    // Row offsets (bytes) of rows {2t, 2t+1, 2t+8, 2t+9} of step 0, word g.
    uint32_t roff[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      roff[q] = (2 * t + (q & 1) + 8 * (q >> 1)) * (kStripWords * 4) + 4 * g;
    bool xok[MT];
    uint32_t xrow[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      xok[mt] = 8 * mt + g < a.M;
      xrow[mt] = (xok[mt] ? 8 * mt + g : 0) * kXRowBytes + 4 * t;
    }
    float part[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) part[mt][j][r] = 0.f;
    uint32_t zc[8];  // zero-point constants
    uint32_t sh[4];
    int cur_grp = -1;

    auto flush = [&]() {
      float sc[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(u32_as_h2(sh[i]));
        sc[2 * i] = f.x;
        sc[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[mt][j][0] = fmaf(sc[j], part[mt][j][0], acc[mt][j][0]);
          acc[mt][j][1] = fmaf(sc[j], part[mt][j][1], acc[mt][j][1]);
          acc[mt][j][2] = fmaf(sc[4 + j], part[mt][j][2], acc[mt][j][2]);
          acc[mt][j][3] = fmaf(sc[4 + j], part[mt][j][3], acc[mt][j][3]);
#pragma unroll
          for (int r = 0; r < 4; ++r) part[mt][j][r] = 0.f;
        }
      }
    };

    int grp_end = -1;
    // Warp w consumes every fill of the ring slots j with j % C == w, in stage
    // order, so it never waits on a slot whose previous fill belongs to
    // another warp and may not have landed (phase parity would alias).
    for (int li = warp < a.ring ? warp : nloc, round = 0; li < nloc;) {  // a warp past the ring owns no slot
      const int slot = li - round;  // round = the first stage of this pass over the ring
      if (!mbar_wait(&full[slot], (li / a.ring) & 1, &abort_flag)) break;
      const uint32_t base = smem_s + slot * a.stage_bytes;
      const int k0 = (sb + li) * kBoxRows;
      const int gbase = k0 / a.G;
      const int steps = min(kBoxRows, a.K - k0) / 16;  // K is a multiple of 16
#pragma unroll 2
      for (int s = 0; s < steps; ++s) {
        const int k = k0 + 16 * s;
        if (k >= grp_end || k < grp_end - a.G) {  // a new quantization group (no division per step)
          if (cur_grp >= 0) flush();
          const int grp = k / a.G;
          grp_end = (grp + 1) * a.G;
          const uint32_t gslot = static_cast<uint32_t>(grp - gbase);
          const uint32_t zw = lds_u32(base + a.z_off + gslot * (kStripWords * 4) + 4 * g);
          zero_consts(zw, zc);
          const uint4 sv = lds_v4(base + a.s_off + gslot * (kStripCols * 2) + 16 * g);
          sh[0] = sv.x;
          sh[1] = sv.y;
          sh[2] = sv.z;
          sh[3] = sv.w;
          cur_grp = grp;
        }
        const uint32_t wrow = base + s * 16 * (kStripWords * 4);
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = lds_u32(wrow + roff[q]);
        uint32_t oa[4], ob[4], oc[4], od[4];
        const uint32_t za[4] = {zc[0], zc[1], zc[2], zc[3]};
        const uint32_t zb[4] = {zc[4], zc[5], zc[6], zc[7]};
        unpack_pairs(prmt(w[0], w[1], 0x6420u), za, oa);
        unpack_pairs(prmt(w[0], w[1], 0x7531u), zb, ob);
        unpack_pairs(prmt(w[2], w[3], 0x6420u), za, oc);
        unpack_pairs(prmt(w[2], w[3], 0x7531u), zb, od);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint32_t b0 = 0u, b1 = 0u;
          if (xok[mt]) {
            const uint32_t xa = base + a.x_off + xrow[mt] + s * 32;
            b0 = lds_u32(xa);
            b1 = lds_u32(xa + 16);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int sl = ((j & 1) << 1) | (j >> 1);
            const uint32_t A[4] = {oa[sl], ob[sl], oc[sl], od[sl]};
            mma_16816(part[mt][j], A, b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      // Next slot of this warp (j += C); past the ring's end, the next pass.
      li += C;
      if (li - round >= a.ring) {
        round += a.ring;
        li = round + warp;
      }
    }
    if (cur_grp >= 0) flush();
  }

  // ---------------- sum the C warps' partial tiles ----------------
  __syncthreads();  // every stage consumed: reuse the ring
  float* red = reinterpret_cast<float*>(smem);  // [C][MT*8 tokens][64 columns + 4 pad]
  constexpr int kTok = MT * 8;
  constexpr int kRow = kStripCols + 4;
  if (warp < C) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float* r0 = red + (warp * kTok + 8 * mt + 2 * t) * kRow + 8 * g;
        r0[j] = acc[mt][j][0];
        r0[kRow + j] = acc[mt][j][1];
        r0[4 + j] = acc[mt][j][2];
        r0[kRow + 4 + j] = acc[mt][j][3];
      }
  }
  __syncthreads();
  const bool failed = abort_flag != 0;
  // The CTA's partial tile [M][64] goes to row 0.. of the reduction area.
  float* tile_sum = red + C * kTok * kRow;
  for (int i = threadIdx.x; i < a.M * kStripCols; i += 32 * (C + 1)) {
    const int m = i / kStripCols, c = i % kStripCols;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < C; ++w) v += red[(w * kTok + m) * kRow + c];
    tile_sum[m * kStripCols + c] = v;
  }
  constexpr bool fused = FUSED;
  if (fused && threadIdx.x == 0) {  // a consumer thread: past griddepcontrol.wait
    ll_skip = ll_sticky_failure();
    ll_epoch = ll_call_epoch(a.ll);
  }
  // A fused call counts every CTA as done, even one whose pipeline gave up,
  // so that the region's call counter stays in step with the peers'.
  if (a.ksplit == 1) {
    __syncthreads();
    if (fused) {
      if (ll_skip) return;
      if (!failed) strip_allreduce_store(a, tile_sum, col0, 0, kStripCols, 1, ll_epoch, 32 * (C + 1));
      __syncthreads();
      if (threadIdx.x == 0) ll_cta_done(a.ll, gridDim.x * gridDim.y);
      return;
    }
    if (failed) return;
    for (int i = threadIdx.x; i < a.M * kStripCols; i += 32 * (C + 1)) {
      const int m = i / kStripCols, c = i % kStripCols;
      if (col0 + c < a.N) a.y[m * a.y_ld + col0 + c] = __float2half_rn(tile_sum[m * kStripCols + c]);
    }
    return;
  }
  // K split across the CTAs of a cluster: CTA r sums column slice r of every
  // CTA's tile through distributed shared memory, in fixed rank order.
  cluster_sync();
  if (fused) {
    if (!failed && !ll_skip) {
      // Pair-aligned column slices, so that every exchanged line is one CTA's.
      const int S = a.ksplit;
      const int c_lo = (static_cast<int>(blockIdx.y) * (kStripCols / 2)) / S * 2;
      const int c_hi = ((static_cast<int>(blockIdx.y) + 1) * (kStripCols / 2)) / S * 2;
      strip_allreduce_store(a, tile_sum, col0, c_lo, c_hi, S, ll_epoch, 32 * (C + 1));
    }
    cluster_sync();  // keep shared memory alive until every remote read is done
    if (!ll_skip && threadIdx.x == 0) ll_cta_done(a.ll, gridDim.x * gridDim.y);
    return;
  }
  if (!failed) {
    const int S = a.ksplit;
    const int c_lo = (static_cast<int>(blockIdx.y) * kStripCols) / S;
    const int c_hi = ((static_cast<int>(blockIdx.y) + 1) * kStripCols) / S;
    const int width = c_hi - c_lo;
    for (int i = threadIdx.x; i < a.M * width; i += 32 * (C + 1)) {
      const int m = i / width, c = c_lo + i % width;
      float pq[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) pq[q] = q < S ? ld_shared_cluster_f32(map_shared_rank(tile_sum + m * kStripCols + c, q)) : 0.f;
      const float v = ((pq[0] + pq[1]) + pq[2]) + pq[3];
      if (col0 + c < a.N) a.y[m * a.y_ld + col0 + c] = __float2half_rn(v);
    }
  }
  cluster_sync();  // keep shared memory alive until every remote read is done
}

struct StripPlan {
  int tiles, stages_total, ksplit, ring, gps, stage_bytes, x_off, s_off, z_off, consumers;
  uint32_t tx;
  size_t smem;
};

int align128(int v) { return (v + 127) / 128 * 128; }

// CTAs per SM a K split may reach: 3 for deep layers at M <= 8 (>= 32 stages,
// K >= 8192: measured 14.1 -> 13.6 us on 4096 x 12288 at M=1), else 1
// (shallower layers, and M > 8 with its twice larger stages, lose more to
// sharing SMs than they gain).
int split_limit(int M, int stages_total) { return (M <= 8 && stages_total >= 32) ? 3 : 1; }

// CTAs of each kernel variant that one SM holds by registers and threads alone
// ([M > 8][C = 4, 8, 16]; 0 = unknown: no cap). Measured on the device with
// cudaOccupancyMaxActiveBlocksPerMultiprocessor at the first launch.
struct StripCaps {
  int cap[2][3];
};

int consumer_index(int c) { return c == 4 ? 0 : (c == 8 ? 1 : 2); }

bool plan_strip(int M, int N, int K, int G, int sm_count, StripPlan* p, const StripCaps* caps = nullptr) {
  p->tiles = ceil_div(N, kStripCols);
  p->stages_total = ceil_div(K, kBoxRows);
  p->gps = (kBoxRows % G == 0) ? kBoxRows / G : kBoxRows / G + 2;
  if (p->gps > 256) return false;
  p->x_off = kWeightBytes;
  p->s_off = p->x_off + align128(M * kXRowBytes);
  p->z_off = p->s_off + align128(p->gps * kStripCols * 2);
  p->stage_bytes = p->z_off + align128(p->gps * kStripWords * 4);
  p->tx = static_cast<uint32_t>(kWeightBytes + M * kXRowBytes + p->gps * kStripCols * 2 + p->gps * kStripWords * 4);
  // Split K (one cluster of up to 4 CTAs per strip) only while the CTAs stay
  // within split_limit per SM; wide layers (more strips than SMs) are not split.
  p->ksplit = 1;
  for (int ks = 4; ks >= 2; --ks)
    if (p->tiles * ks <= split_limit(M, p->stages_total) * sm_count && ks <= p->stages_total) {
      p->ksplit = ks;
      break;
    }
  // CTAs that share an SM so that every CTA is resident at once.
  int per_sm = std::max(1, ceil_div(p->tiles * p->ksplit, sm_count));
  // Consumer warps per CTA within the SM's register file (one CTA per SM and
  // M <= 8 affords 16).
  if (per_sm >= 3 || (M > 8 && per_sm >= 2))
    p->consumers = 4;
  else if (per_sm == 1 && M <= 8)
    p->consumers = 16;
  else
    p->consumers = 8;
  const size_t cap = 224 * 1024;
  // More CTAs than the register file holds run in waves: size the ring for the
  // CTAs that are resident together, not for the whole grid.
  if (caps) {
    const int c = caps->cap[M > 8 ? 1 : 0][consumer_index(p->consumers)];
    if (c > 0 && per_sm > c) per_sm = c;
  }
  const size_t budget = std::min<size_t>(cap, (228 * 1024) / per_sm - 2048) - 1024;
  int ring = static_cast<int>(budget / p->stage_bytes);
  ring = std::min(ring, kMaxStages);
  const int local = ceil_div(p->stages_total, p->ksplit);
  ring = std::min(ring, std::max(local, 1));
  // Slots are owned by warps (slot j by warp j % C); with fewer slots than
  // warps the extra warps would idle, so shrink C first.
  while (p->consumers > 4 && ring < p->consumers) p->consumers /= 2;
  p->ring = std::max(ring, 1);
  const size_t red = static_cast<size_t>(p->consumers) * (M > 8 ? 16 : 8) * (kStripCols + 4) * 4 +
                     static_cast<size_t>(M) * kStripCols * 4;
  p->smem = 1024 + std::max(static_cast<size_t>(p->ring) * p->stage_bytes, red);
  return true;
}

template <int MT, int C, bool FUSED>
int launch_strip_t(const StripMaps& maps, const StripArgs& args, int tiles, size_t smem, cudaStream_t stream) {
  const int ks = args.ksplit;
  static std::atomic<bool> configured[64];  // zero-initialised (static storage)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ASHQK_ERR_CUDA;
  auto kernel = gemv_strip_kernel<MT, C, FUSED>;
  if (!configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return ASHQK_ERR_CUDA;
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, ks);
  cfg.blockDim = dim3(32 * (C + 1));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (ks > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = ks;
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
  if (FUSED) {
    // A CTA waits for the same CTA of every peer: all CTAs of the grid must be
    // resident at once, or a peer's CTA could queue behind CTAs that wait.
    int resident = 0;
    if (ks > 1) {
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) return ASHQK_ERR_CUDA;
      resident = clusters * ks;
    } else {
      int per_sm = 0, sms = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 32 * (C + 1), smem) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return ASHQK_ERR_CUDA;
      resident = per_sm * sms;
    }
    if (resident < tiles * ks) return ASHQK_ERR_UNSUPPORTED;
  }
  if (cudaLaunchKernelEx(&cfg, kernel, maps, args) != cudaSuccess) return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}

template <int MT, int C>
int launch_strip(const StripMaps& maps, const StripArgs& args, int tiles, size_t smem, cudaStream_t stream) {
  if (args.ll.regions != nullptr) return launch_strip_t<MT, C, true>(maps, args, tiles, smem, stream);
  return launch_strip_t<MT, C, false>(maps, args, tiles, smem, stream);
}

}  // namespace

bool gemv_strip_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                         int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int G) {
  return M >= 1 && M <= 16 && N % 32 == 0 && G % 16 == 0 && aligned(qw, 16) && qw_ld % 4 == 0 && aligned(qz, 16) &&
         qz_ld % 4 == 0 && aligned(s, 16) && s_ld % 8 == 0 && aligned(x, 16) && x_ld % 8 == 0;
}

namespace {

template <int MT, int C, bool FUSED>
int occupancy_cap() {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_strip_kernel<MT, C, FUSED>, 32 * (C + 1), 0) !=
      cudaSuccess)
    return 0;
  return n;
}

template <bool FUSED>
void fill_caps(StripCaps* c) {
  c->cap[0][0] = occupancy_cap<1, 4, FUSED>();
  c->cap[0][1] = occupancy_cap<1, 8, FUSED>();
  c->cap[0][2] = occupancy_cap<1, 16, FUSED>();
  c->cap[1][0] = occupancy_cap<2, 4, FUSED>();
  c->cap[1][1] = occupancy_cap<2, 8, FUSED>();
  c->cap[1][2] = 0;  // M > 8 never plans 16 consumer warps
}

// Register-file residency of the kernel variant this process launches, per
// device (measured once).
const StripCaps* strip_caps(bool fused) {
  static StripCaps caps[64][2];
  static std::atomic<bool> ready[64][2];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  const int f = fused ? 1 : 0;
  if (!ready[dev][f].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (!ready[dev][f].load(std::memory_order_relaxed)) {
      StripCaps c = {};
      if (fused)
        fill_caps<true>(&c);
      else
        fill_caps<false>(&c);
      caps[dev][f] = c;
      ready[dev][f].store(true, std::memory_order_release);
    }
  }
  return &caps[dev][f];
}

int strip_launch_impl(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                      int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G,
                      int sm_count, const LLPeers* ll, cudaStream_t stream) {
  StripPlan p;
  if (!plan_strip(M, N, K, G, sm_count, &p, strip_caps(ll != nullptr))) return ASHQK_ERR_UNSUPPORTED;
  StripMaps maps;
  int rc = encode_tensor_map_2d(&maps.qw, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<int32_t*>(qw), N / 8, K,
                                static_cast<uint64_t>(qw_ld) * 4, kStripWords, kBoxRows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(x), K, M,
                              static_cast<uint64_t>(x_ld) * 2, kBoxRows, M, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(s), N, K / G,
                              static_cast<uint64_t>(s_ld) * 2, kStripCols, p.gps, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = encode_tensor_map_2d(&maps.z, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<int32_t*>(qz), N / 8, K / G,
                              static_cast<uint64_t>(qz_ld) * 4, kStripWords, p.gps, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  StripArgs a = {};
  if (ll) a.ll = *ll;
  a.y = y;
  a.y_ld = y_ld;
  a.M = M;
  a.N = N;
  a.K = K;
  a.G = G;
  a.stages_total = p.stages_total;
  a.ksplit = p.ksplit;
  a.ring = p.ring;
  a.gps = p.gps;
  a.stage_bytes = p.stage_bytes;
  a.x_off = p.x_off;
  a.s_off = p.s_off;
  a.z_off = p.z_off;
  a.tx_bytes = p.tx;
  if (M > 8) {
    return p.consumers == 4 ? launch_strip<2, 4>(maps, a, p.tiles, p.smem, stream)
                            : launch_strip<2, 8>(maps, a, p.tiles, p.smem, stream);
  }
  if (p.consumers == 16) return launch_strip<1, 16>(maps, a, p.tiles, p.smem, stream);
  return p.consumers == 4 ? launch_strip<1, 4>(maps, a, p.tiles, p.smem, stream)
                          : launch_strip<1, 8>(maps, a, p.tiles, p.smem, stream);
}

}  // namespace

int gemv_strip_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                      int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G,
                      int sm_count, cudaStream_t stream) {
  return strip_launch_impl(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, y, y_ld, M, N, K, G, sm_count, nullptr, stream);
}

}  // namespace ashqk

extern "C" int ashqk_w4a16_gemv_allreduce(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                                          const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                                          void* y, int64_t y_ld, int M, int N, int K, int group_size,
                                          const void* regions_dev, int rank, int world, int64_t max_elems,
                                          void* stream) {
  int rc = ashqk::check_awq_args(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size);
  if (rc) return rc;
  size_t region = 0;
  if (!regions_dev || world < 1 || world > ashqk::kLLMaxRanks || rank < 0 || rank >= world ||
      ashqk_p2p_ll_region_bytes(max_elems, &region) || static_cast<int64_t>(M) * N > max_elems)
    return ASHQK_ERR_INVALID_ARGUMENT;
  // The epilogue stores y as fp16 pairs.
  if (!ashqk::gemv_strip_eligible(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, M, N, group_size) ||
      !ashqk::aligned(y, 4) || y_ld % 2)
    return ASHQK_ERR_UNSUPPORTED;
  ashqk::DeviceInfo info;
  rc = ashqk::device_info(&info);
  if (rc) return rc;
  ashqk::LLPeers ll;
  ll.regions = static_cast<unsigned char* const*>(regions_dev);
  ll.rank = rank;
  ll.world = world;
  ll.inbox_pairs = max_elems / 2;
  return ashqk::strip_launch_impl(static_cast<const __half*>(x), x_ld, qweight, qw_ld, qzeros, qz_ld,
                                  static_cast<const __half*>(scales), s_ld, static_cast<__half*>(y), y_ld, M, N, K,
                                  group_size, info.sm_count, &ll, static_cast<cudaStream_t>(stream));
}

extern "C" int ashqk_gemv_strip_plan(int M, int N, int K, int group_size, int sm_count, ashqk_strip_plan* plan) {
  if (!plan || M <= 0 || N <= 0 || K <= 0 || group_size <= 0 || N % 8 || K % group_size || sm_count < 0)
    return ASHQK_ERR_INVALID_ARGUMENT;
  if (M > 16 || N % 32 || group_size % 16) return ASHQK_ERR_UNSUPPORTED;
  const bool on_device = sm_count == 0;
  if (on_device) {
    ashqk::DeviceInfo info;
    const int rc = ashqk::device_info(&info);
    if (rc) return rc;
    sm_count = info.sm_count;
  }
  ashqk::StripPlan p;
  if (!ashqk::plan_strip(M, N, K, group_size, sm_count, &p, on_device ? ashqk::strip_caps(false) : nullptr))
    return ASHQK_ERR_UNSUPPORTED;
  plan->grid_x = p.tiles;
  plan->grid_y = p.ksplit;
  // The launch instantiates 4 or 8 consumer warps when M > 8 (16 is planned only for M <= 8).
  plan->consumer_warps = p.consumers;
  plan->threads = 32 * (p.consumers + 1);
  plan->ring_stages = p.ring;
  plan->stages_total = p.stages_total;
  plan->stage_bytes = p.stage_bytes;
  plan->smem_bytes = static_cast<int>(p.smem);
  return ASHQK_OK;
}
