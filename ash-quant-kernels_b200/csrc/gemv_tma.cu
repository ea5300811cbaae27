// Decode GEMV for AWQ W4A16 (M <= 16), TMA-pipelined variant for sm_100a.
//
// Same math as csrc/gemv.cu (and the reference's ashqk/kernels/w4a16_gemv.py:28-107):
// y = x @ W with W = (q - z) * s factored per group and fp32 accumulation;
// split-K partial sums are reduced inside the same launch.
//
// Structure (one CTA per column tile of 256 outputs and one K slice):
//  * warp 8, lane 0 is the producer. At kernel start it issues bulk copies of
//    the slice's scales and zeros and TMA loads of the first weight stages
//    (64 rows x 128 bytes = 8 KB each, 128-byte swizzle, 8-stage ring); then it
//    waits for the previous kernel (griddepcontrol.wait), bulk-copies the x
//    slice, and keeps the weight ring full. Everything the CTA reads from HBM
//    is in flight before the first consumer instruction needs it.
//  * warps 0-7 are consumers: 4 column groups of 64 outputs x 2 halves of every
//    stage's four 16-row steps. A lane reads one word (8 columns) of rows
//    {2t, 2t+1, 2t+8, 2t+9}: with the 128-byte swizzle the four lanes t of a
//    column group land on distinct banks, and those rows are the k order of an
//    mma.sync A fragment, so x needs no permutation. Unpacking (prmt + LOP3
//    magic exponent + HSUB2/HFMA2) and mma.sync m16n8k16 are shared with
//    csrc/gemv.cu (csrc/awq_unpack.cuh).
//  * split-K (the caller's split_k, or about one CTA per SM): each CTA writes
//    its partial tile to an fp32 workspace slot; the last CTA to arrive on the
//    tile's counter sums the slots in split order (deterministic), stores y and
//    resets the counter.
//  * programmatic dependent launch: dependents may launch at once; only x (the
//    previous kernel's output), y and the workspace are touched after
//    griddepcontrol.wait, so the next layer's weights stream during this
//    layer's tail.
#include <atomic>
#include <algorithm>
#include <cstdlib>

#include "awq_unpack.cuh"
#include "sm100.cuh"

namespace ashqk {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kThreads = kConsumers + 32;
constexpr int kTileWords = 32;  // one 128-byte TMA row
constexpr int kTileCols = kTileWords * 8;
// A stage is kBoxes TMA boxes of 64 rows x 128 bytes behind one mbarrier phase:
// the barrier round trip is paid once per kBoxes x 8 KB of weights.
#ifndef ASHQK_GEMV_BOXES
#define ASHQK_GEMV_BOXES 2
#endif
#ifndef ASHQK_GEMV_STAGES
#define ASHQK_GEMV_STAGES 6
#endif
constexpr int kBoxRows = 64;
constexpr int kBoxBytes = kBoxRows * kTileWords * 4;
constexpr int kBoxes = ASHQK_GEMV_BOXES;
constexpr int kStageRows = kBoxRows * kBoxes;
constexpr int kStageBytes = kBoxBytes * kBoxes;
constexpr int kStages = ASHQK_GEMV_STAGES;
static_assert(kBoxes == 1 || kBoxes % 2 == 0, "stages hold one box or an even number of boxes");
constexpr int kMaxTiles = 16384;
constexpr size_t kCounterBytes = kMaxTiles * sizeof(int);
constexpr size_t kSmemLimitTwoCtas = 112 * 1024;  // M <= 8: two CTAs per SM
constexpr size_t kSmemLimitOneCta = 220 * 1024;   // M > 8: one CTA per SM (register bound)

struct TmaGemvArgs {
  const __half* x;
  const int32_t* qz;
  const __half* s;
  __half* y;
  float* ws;
  int* counters;
  int64_t x_ld, qz_ld, s_ld, y_ld;
  int M, N, K, G;
  int words;
  int stages_total;  // ceil(K / 64)
  int splits;
  int x_stride;      // halves; == 8 mod 64 for conflict-free fragment reads
  int max_groups;
};

template <int MT>
__global__ void __launch_bounds__(kThreads) __maxnreg__(MT == 1 ? 112 : 168) gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap,
                                                               const TmaGemvArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* ring = smem;
  __half* xs = reinterpret_cast<__half*>(ring + kStages * kStageBytes);
  __half* ss = xs + a.M * a.x_stride;
  uint32_t* zs = reinterpret_cast<uint32_t*>(ss + a.max_groups * kTileCols);
  uint64_t* full = reinterpret_cast<uint64_t*>(zs + a.max_groups * kTileWords);
  uint64_t* empty = full + kStages;
  uint64_t* aux_bar = empty + kStages;  // scales + zeros
  uint64_t* x_bar = aux_bar + 1;
  __shared__ int abort_flag;
  __shared__ int is_last;

  const int tile = blockIdx.x;
  const int split = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int st0 = static_cast<int>(static_cast<int64_t>(split) * a.stages_total / a.splits);
  const int st1 = static_cast<int>(static_cast<int64_t>(split + 1) * a.stages_total / a.splits);
  const int nst = st1 - st0;
  const int k_begin = st0 * kStageRows;
  const int k_end = min(st1 * kStageRows, a.K);
  const int krows = k_end - k_begin;
  const int col0 = tile * kTileCols;
  const int cols_valid = min(kTileCols, a.N - col0);  // multiple of 32
  const int g0 = k_begin / a.G;
  const int ngrp = krows > 0 ? (k_end - 1) / a.G + 1 - g0 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    mbar_init(aux_bar, 1);
    mbar_init(x_bar, 1);
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

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmap);
      // Scales and zeros are weights: independent of the previous kernel.
      mbar_arrive_expect_tx(aux_bar, static_cast<uint32_t>(ngrp) * (cols_valid * 2 + cols_valid / 2));
      for (int gi = 0; gi < ngrp; ++gi) {
        bulk_load(ss + gi * kTileCols, a.s + static_cast<int64_t>(g0 + gi) * a.s_ld + col0, cols_valid * 2, aux_bar);
        bulk_load(zs + gi * kTileWords, a.qz + static_cast<int64_t>(g0 + gi) * a.qz_ld + tile * kTileWords,
                  cols_valid / 2, aux_bar);
      }
      auto issue = [&](int i, int slot) {
        mbar_arrive_expect_tx(&full[slot], kStageBytes);
#pragma unroll
        for (int b = 0; b < kBoxes; ++b)
          tma_load_2d(ring + slot * kStageBytes + b * kBoxBytes, &tmap, tile * kTileWords,
                      (st0 + i) * kStageRows + b * kBoxRows, &full[slot]);
      };
      const int prologue = min(nst, kStages);
      for (int i = 0; i < prologue; ++i) issue(i, i);
      // x is the previous kernel's output.
      pdl_wait();
      mbar_arrive_expect_tx(x_bar, static_cast<uint32_t>(a.M) * krows * 2);
      for (int m = 0; m < a.M; ++m)
        bulk_load(xs + m * a.x_stride, a.x + m * a.x_ld + k_begin, krows * 2, x_bar);
      int issued = prologue;
      for (int i = prologue; i < nst; ++i) {
        const int slot = i % kStages;
        if (!mbar_wait(&empty[slot], ((i / kStages) - 1) & 1, &abort_flag, true)) break;
        issue(i, slot);
        ++issued;
      }
      if (abort_flag) {
        // Let every issued copy land before the CTA's shared memory goes away.
        int unused = 0;
        mbar_wait(aux_bar, 0, &unused);
        mbar_wait(x_bar, 0, &unused);
        for (int slot = 0; slot < kStages && slot < issued; ++slot) {
          const int last_round = (issued - 1 - slot) / kStages;
          mbar_wait(&full[slot], last_round & 1, &unused);
        }
      }
    }
  } else {
    // ---------------- consumers ----------------
    const int cw = warp & 3;   // column group: 64 outputs = 8 words
    const int kh = warp >> 2;  // steps {2kh, 2kh+1} of each stage's four 16-row steps
    const int g = lane >> 2;
    const int t = lane & 3;
    // y and the workspace may only be written after the previous kernel ends.
    pdl_wait();
    // Columns past N in a partial tile: zero scales and zeros (never stored).
    if (cols_valid < kTileCols) {
      for (int i = threadIdx.x; i < ngrp * kTileCols; i += kConsumers) {
        const int gi = i / kTileCols, c = i % kTileCols;
        if (c >= cols_valid) ss[gi * kTileCols + c] = __float2half_rn(0.f);
        if (c < kTileWords && c >= cols_valid / 8) zs[gi * kTileWords + c] = 0u;
      }
    }
    bool ok = mbar_wait(aux_bar, 0, &abort_flag) && mbar_wait(x_bar, 0, &abort_flag);

    named_barrier_sync(1, kConsumers);

    float part[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) part[mt][j][r] = 0.f;
    uint32_t zc[8];                        // zero-point constants of this lane's word (current group)
    uint32_t sh[4];                        // its 8 scales, as half2
    const int wcol = cw * 8 + g;           // the word (8 columns) of the tile this lane unpacks
    const int chunk = wcol >> 2;           // its 16-byte chunk in a 128-byte row
    const int in_chunk = (wcol & 3) * 4;
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t ss_s = smem_u32(ss);
    const uint32_t zs_s = smem_u32(zs);
    // Byte offsets within a stage of rows {2t, 2t+1, 2t+8, 2t+9} of step 2kh; the
    // second step is 16 rows (2 KB) further and keeps the same swizzle phase.
    // With the 128-byte swizzle the four lanes t of a column group use distinct banks.
    uint32_t roff[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = 32 * kh + 2 * t + (q & 1) + 8 * (q >> 1);
      roff[q] = r * 128 + ((chunk ^ (r & 7)) << 4) + in_chunk;
    }
    // x fragments: token g (+8 for the second n8 tile), k = step + 2t (and +8).
    uint32_t xa[MT];
    bool xok[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      xok[mt] = 8 * mt + g < a.M;
      xa[mt] = smem_u32(xs + (xok[mt] ? (8 * mt + g) * a.x_stride : 0) + 32 * kh + 2 * t);
    }
    int grp = -1, grp_end = -1;

    // part accumulates sum_k x_k (q_k - z) over the current group; the scale is
    // applied once per group in fp32.
    auto flush = [&](int) {
      float sc[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(u32_as_h2(sh[i]));
        sc[2 * i] = f.x;
        sc[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[mt][j][0] = fmaf(sc[j], part[mt][j][0], acc[mt][j][0]);
          acc[mt][j][1] = fmaf(sc[j], part[mt][j][1], acc[mt][j][1]);
          acc[mt][j][2] = fmaf(sc[4 + j], part[mt][j][2], acc[mt][j][2]);
          acc[mt][j][3] = fmaf(sc[4 + j], part[mt][j][3], acc[mt][j][3]);
#pragma unroll
          for (int r = 0; r < 4; ++r) part[mt][j][r] = 0.f;
        }
    };
    auto load_group = [&](int gi) {
      zero_consts(lds_u32(zs_s + (gi * kTileWords + wcol) * 4), zc);
      const uint4 sv = lds_v4(ss_s + (gi * kTileCols + wcol * 8) * 2);
      sh[0] = sv.x;
      sh[1] = sv.y;
      sh[2] = sv.z;
      sh[3] = sv.w;
    };

    // One 16-row step: unpack 4 rows x 8 columns and feed 4 (x MT) mma.sync.
    auto step = [&](const uint32_t (&w)[4], const uint32_t (&b)[MT][2]) {
      const uint32_t za[4] = {zc[0], zc[1], zc[2], zc[3]};
      const uint32_t zb[4] = {zc[4], zc[5], zc[6], zc[7]};
      uint32_t oa[4], ob[4], oc[4], od[4];
      unpack_pairs(prmt(w[0], w[1], 0x6420u), za, oa);
      unpack_pairs(prmt(w[0], w[1], 0x7531u), zb, ob);
      unpack_pairs(prmt(w[2], w[3], 0x6420u), za, oc);
      unpack_pairs(prmt(w[2], w[3], 0x7531u), zb, od);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int sl = ((j & 1) << 1) | (j >> 1);
          const uint32_t A[4] = {oa[sl], ob[sl], oc[sl], od[sl]};
          mma_16816(part[mt][j], A, b[mt][0], b[mt][1]);
        }
    };
    auto load_x = [&](uint32_t off, uint32_t (&b)[MT][2]) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        b[mt][0] = xok[mt] ? lds_u32(xa[mt] + off) : 0u;
        b[mt][1] = xok[mt] ? lds_u32(xa[mt] + off + 16) : 0u;
      }
    };
    auto enter_group = [&](int k0) {
      if (k0 >= grp_end) {
        if (grp >= 0) flush(grp - g0);
        grp = k0 / a.G;
        grp_end = (grp + 1) * a.G;
        load_group(grp - g0);
      }
    };
    // The warp's two steps share one quantization group whenever G % 32 == 0.
    const bool pair_groups = (a.G % 32) == 0;

    for (int i = 0; ok && i < nst; ++i) {
      const int slot = i % kStages;
      if (!mbar_wait(&full[slot], (i / kStages) & 1, &abort_flag)) break;
      const int k_stage = k_begin + kStageRows * i;
      if (pair_groups && k_stage + kStageRows <= k_end) {
        // Fast path (every box of the stage valid): shared loads are issued two
        // boxes at a time ahead of their unpack / mma chains, so one wait on the
        // stage covers the latency of the next loads (the barrier's memory
        // clobber would otherwise serialise them box by box).
        constexpr int kBatch = kBoxes >= 2 ? 2 : 1;
#pragma unroll
        for (int bp = 0; bp < kBoxes; bp += kBatch) {
          uint32_t w[kBatch][2][4], b[kBatch][2][MT][2];
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const uint32_t st = ring_s + slot * kStageBytes + (bp + u) * kBoxBytes;
            const uint32_t xoff = static_cast<uint32_t>(i * kStageRows + (bp + u) * kBoxRows) * 2;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              w[u][0][q] = lds_u32(st + roff[q]);
              w[u][1][q] = lds_u32(st + roff[q] + 2048);
            }
            load_x(xoff, b[u][0]);
            load_x(xoff + 32, b[u][1]);
          }
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            enter_group(k_stage + (bp + u) * kBoxRows + 32 * kh);
            step(w[u][0], b[u][0]);
            step(w[u][1], b[u][1]);
          }
        }
      } else {
        // Ragged tail, or G not a multiple of 32: one step at a time.
#pragma unroll 1
        for (int bx = 0; bx < kBoxes; ++bx) {
          const uint32_t st = ring_s + slot * kStageBytes + bx * kBoxBytes;
          const uint32_t xoff = static_cast<uint32_t>(i * kStageRows + bx * kBoxRows) * 2;
          const int kb = k_stage + kBoxRows * bx + 32 * kh;
#pragma unroll
          for (int s2 = 0; s2 < 2; ++s2) {
            const int k0 = kb + 16 * s2;
            if (k0 < k_end) {
              enter_group(k0);
              uint32_t w[4], b[MT][2];
#pragma unroll
              for (int q = 0; q < 4; ++q) w[q] = lds_u32(st + roff[q] + s2 * 2048);
              load_x(xoff + s2 * 32, b);
              step(w, b);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (grp >= 0) flush(grp - g0);
  }

  // ---------------- CTA partial tile ----------------
  __syncthreads();  // ring drained: reuse it
  float* red = reinterpret_cast<float*>(ring);  // [2][MT*8][256], then [M][256] in place
  constexpr int kTok = MT * 8;
  if (warp < kConsumerWarps) {
    const int cw = warp & 3, kh = warp >> 2, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float* r0 = red + (kh * kTok + 8 * mt + 2 * t) * kTileCols + cw * 64 + 8 * g;
        r0[j] = acc[mt][j][0];
        r0[kTileCols + j] = acc[mt][j][1];
        r0[4 + j] = acc[mt][j][2];
        r0[kTileCols + 4 + j] = acc[mt][j][3];
      }
  }
  __syncthreads();
  if (threadIdx.x < kTileCols) {
    for (int m = 0; m < a.M; ++m) red[m * kTileCols + threadIdx.x] += red[(kTok + m) * kTileCols + threadIdx.x];
  }
  const bool failed = abort_flag != 0;

  __syncthreads();
  if (threadIdx.x >= kTileCols) return;
  const int col = threadIdx.x;
  const bool col_ok = col < cols_valid;
  if (a.splits == 1) {
    if (failed) return;
    for (int m = 0; m < a.M; ++m)
      if (col_ok) a.y[m * a.y_ld + col0 + col] = __float2half_rn(red[m * kTileCols + col]);
    return;
  }
  // ---------------- split-K through workspace slots ----------------
  // A CTA whose pipeline gave up still takes its turn on the tile's arrival
  // counter, so that the last arrival resets it and the workspace stays
  // zeroed for the next call; a last arrival that itself gave up stores nothing.
  float* slot = a.ws + (static_cast<int64_t>(tile) * a.splits + split) * a.M * kTileCols;
  for (int m = 0; m < a.M; ++m) slot[m * kTileCols + col] = red[m * kTileCols + col];
  named_barrier_sync(1, kTileCols);
  // One fence after the barrier publishes the whole CTA's slot (cumulativity).
  if (threadIdx.x == 0) {
    __threadfence();
    is_last = (atomicAdd(a.counters + tile, 1) == a.splits - 1);
  }
  named_barrier_sync(1, kTileCols);
  if (!is_last) return;
  __threadfence();
  const float* tile_ws = a.ws + static_cast<int64_t>(tile) * a.splits * a.M * kTileCols;
  if (!failed) {
    for (int m = 0; m < a.M; ++m) {
      float v = 0.f;
      for (int s = 0; s < a.splits; ++s) v += __ldcg(tile_ws + (s * a.M + m) * kTileCols + col);
      if (col_ok) a.y[m * a.y_ld + col0 + col] = __float2half_rn(v);
    }
  }
  if (threadIdx.x == 0) a.counters[tile] = 0;
}

struct TmaPlan {
  int tiles, stages_total, splits, ks_max, x_stride, max_groups;
  size_t smem, ws_bytes;
};

void plan_tma(int M, int N, int K, int G, int split_req, int sm_count, TmaPlan* p) {
  p->tiles = ceil_div(N, kTileCols);
  p->stages_total = ceil_div(K, kStageRows);
  // Without a requested split: about one CTA per SM.
  int splits = split_req > 0 ? split_req : std::max(1, (sm_count + p->tiles / 2) / p->tiles);
  splits = std::min(std::max(splits, 1), p->stages_total);
  // The split is a hint: raise it until the staged slice fits in shared memory.
  for (;; ++splits) {
    p->splits = splits;
    p->ks_max = ceil_div(p->stages_total, splits) * kStageRows;
    p->x_stride = ((p->ks_max + 63) / 64) * 64 + 8;
    p->max_groups = p->ks_max / G + 2;
    p->smem = 1024 /* alignment slack */ + static_cast<size_t>(kStages) * kStageBytes +
              static_cast<size_t>(M) * p->x_stride * 2 + static_cast<size_t>(p->max_groups) * kTileCols * 2 +
              static_cast<size_t>(p->max_groups) * kTileWords * 4 + (2 * kStages + 2) * 8;
    if (p->smem <= (M > 8 ? kSmemLimitOneCta : kSmemLimitTwoCtas) || splits >= p->stages_total) break;
  }
  p->ws_bytes = p->splits > 1
                    ? kCounterBytes + static_cast<size_t>(p->tiles) * p->splits * M * kTileCols * 4
                    : 0;
}

template <int MT>
int launch_tma(const CUtensorMap& map, const TmaGemvArgs& args, const TmaPlan& p, cudaStream_t stream) {
  static std::atomic<bool> configured[64];  // zero-initialised (static storage)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ASHQK_ERR_CUDA;
  auto kernel = gemv_tma_kernel<MT>;
  if (!configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimitOneCta) != cudaSuccess ||
        cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return ASHQK_ERR_CUDA;
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.tiles, p.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (cudaLaunchKernelEx(&cfg, kernel, map, args) != cudaSuccess) return ASHQK_ERR_CUDA;
  return ASHQK_OK;
}

}  // namespace

bool gemv_tma_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                       int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int G) {
  return M >= 1 && M <= 16 && N % 32 == 0 && G % 16 == 0 && aligned(qw, 16) && qw_ld % 4 == 0 &&
         aligned(qz, 16) && qz_ld % 4 == 0 && aligned(s, 16) && s_ld % 8 == 0 && aligned(x, 16) && x_ld % 8 == 0;
}

size_t gemv_tma_workspace_bytes(int M, int N, int K, int G, int split_k, int sm_count) {
  TmaPlan p;
  plan_tma(M, N, K, G, split_k, sm_count, &p);
  return p.ws_bytes;
}

int gemv_tma_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld,
                    const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G, int split_k,
                    void* workspace, size_t ws_bytes, int sm_count, cudaStream_t stream) {
  TmaPlan p;
  plan_tma(M, N, K, G, split_k, sm_count, &p);
  if (p.smem > (M > 8 ? kSmemLimitOneCta : kSmemLimitTwoCtas) || p.tiles > kMaxTiles) return ASHQK_ERR_UNSUPPORTED;
  if (p.ws_bytes > 0 && (workspace == nullptr || ws_bytes < p.ws_bytes || !aligned(workspace, 256)))
    return ASHQK_ERR_WORKSPACE;
  CUtensorMap map;
  int rc = encode_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<int32_t*>(qw), N / 8, K,
                                static_cast<uint64_t>(qw_ld) * 4, kTileWords, kBoxRows,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  TmaGemvArgs a;
  a.x = x;
  a.qz = qz;
  a.s = s;
  a.y = y;
  a.x_ld = x_ld;
  a.qz_ld = qz_ld;
  a.s_ld = s_ld;
  a.y_ld = y_ld;
  a.M = M;
  a.N = N;
  a.K = K;
  a.G = G;
  a.words = N / 8;
  a.stages_total = p.stages_total;
  a.splits = p.splits;
  a.x_stride = p.x_stride;
  a.max_groups = p.max_groups;
  if (p.ws_bytes > 0) {
    a.counters = static_cast<int*>(workspace);
    a.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  } else {
    a.counters = nullptr;
    a.ws = nullptr;
  }
  return M > 8 ? launch_tma<2>(map, a, p, stream) : launch_tma<1>(map, a, p, stream);
}

}  // namespace ashqk
