// Decode GEMV for AWQ W4A16, M <= 16 (sm_100a).
//
// Replaces the reference's Triton decode kernel (ashqk/kernels/w4a16_gemv.py:28-107)
// with the same math: y = x @ W, W = (q - z) * s, the per-group factorisation
//     sum_{k in g} x_k (q_kn - z_gn) s_gn = s_gn * sum_{k in g} x_k (q_kn - z_gn)
// and a single-launch split-K whose last-arriving CTA finishes the tile and
// leaves the workspace as it found it (ashqk/kernels/w4a16_gemv.py:93-107).
//
// How the work maps to the hardware:
//  * A CTA owns 128 output columns (16 packed words per row) and one K slice;
//    its 4 warps split that slice again. Each lane owns 16 columns (2 words)
//    of 4 consecutive rows per 16-row step; packed words stream from HBM
//    straight into registers (no L1 allocation, kDepth steps in flight).
//  * Two rows of a word are byte-permuted (prmt) so that one LOP3 against the
//    fp16 exponent of 1024 yields a half2 of one column at two consecutive k:
//    exactly the K-pair layout of an mma.sync A fragment. One HSUB2 (or HFMA2
//    for the high nibble) turns 1024 + q into the exact small integer q - z.
//  * The dot products run on the tensor cores (mma.sync m16n8k16, fp32
//    accumulate): the 16 mma rows are weight columns, the 8 mma columns are
//    tokens. The scale is applied once per group in fp32 on the accumulator.
//    CUDA-core FMAs would need ~3 instructions per weight, more than the issue
//    rate allows at HBM speed; this path needs ~1.25 (unpack) per weight.
//  * x, scales and zeros for the CTA's slice are staged in shared memory once.
//  * Split-K partials go to fp32 slots of a caller-owned workspace; the last
//    CTA of a column tile sums the slots in fixed order (deterministic), writes
//    fp16 y and resets the tile's arrival counter.
#include <atomic>
#include <algorithm>

#include "awq_unpack.cuh"

namespace ashqk {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kBlockCols = 128;
constexpr int kBlockWords = kBlockCols / 8;
constexpr int kDepth = 4;       // 16-row steps of packed words in flight per warp
constexpr int kMaxM = 16;
// Split-K workspace layout: [arrival counters: kMaxTiles ints][partial slots].
constexpr int kMaxTiles = 16384;  // N <= 2,097,152
constexpr size_t kCounterBytes = kMaxTiles * sizeof(int);

struct GemvArgs {
  const __half* x;
  const int32_t* qw;
  const int32_t* qz;
  const __half* s;
  __half* y;
  float* ws;
  int* counters;
  int64_t x_ld, qw_ld, qz_ld, s_ld, y_ld;
  int M, N, K, G;
  int words;       // N / 8
  int steps;       // K / 16
  int splits;
  int x_stride;    // shared-memory row stride of the x slice, in halves
  int max_groups;  // shared-memory rows reserved for scales / zeros
  bool x_vec;      // x rows are 16-byte aligned
  bool s_vec;      // scale rows are 16-byte aligned
};

template <bool VEC>
__device__ __forceinline__ void load_step(uint32_t (&dst)[8], const int32_t* qp, int64_t qw_ld, int step, int t,
                                          bool v0, bool v1) {
  const int64_t row0 = static_cast<int64_t>(step) * 16 + 4 * t;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int32_t* p = qp + (row0 + i) * qw_ld;
    if (VEC) {
      if (v0) {
        const uint2 w = ld_stream_v2(p);
        dst[2 * i] = w.x;
        dst[2 * i + 1] = w.y;
      } else {
        dst[2 * i] = 0u;
        dst[2 * i + 1] = 0u;
      }
    } else {
      dst[2 * i] = v0 ? ld_stream_u32(p) : 0u;
      dst[2 * i + 1] = v1 ? ld_stream_u32(p + 1) : 0u;
    }
  }
}

template <int MT, bool VEC>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int tile = blockIdx.x;
  const int split = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;

  const int cs0 = static_cast<int>(static_cast<int64_t>(split) * a.steps / a.splits);
  const int cs1 = static_cast<int>(static_cast<int64_t>(split + 1) * a.steps / a.splits);
  const int ws0 = cs0 + (warp * (cs1 - cs0)) / kWarps;
  const int ws1 = cs0 + ((warp + 1) * (cs1 - cs0)) / kWarps;

  const int wbase = tile * kBlockWords + 2 * g;
  const bool v0 = wbase < a.words;
  const bool v1 = wbase + 1 < a.words;
  const int32_t* qp = a.qw + wbase;

  // 1. Put the first kDepth steps of packed weights in flight.
  uint32_t buf[kDepth][8];
#pragma unroll
  for (int p = 0; p < kDepth; ++p) {
    if (ws0 + p < ws1) load_step<VEC>(buf[p], qp, a.qw_ld, ws0 + p, t, v0, v1);
  }

  // 2. Stage x, scales and zeros of this CTA's K slice in shared memory.
  const int krow0 = cs0 * 16;
  const int krows = (cs1 - cs0) * 16;
  const int grp0 = krow0 / a.G;
  const int ngrp = krows > 0 ? (krow0 + krows - 1) / a.G + 1 - grp0 : 0;
  __half* xs = reinterpret_cast<__half*>(smem);
  __half* ss = xs + a.M * a.x_stride;
  uint32_t* zs = reinterpret_cast<uint32_t*>(ss + a.max_groups * kBlockCols);
  if (a.x_vec) {
    const int chunks = krows / 8;
    for (int i = threadIdx.x; i < a.M * chunks; i += kThreads) {
      const int m = i / chunks, c = i % chunks;
      *reinterpret_cast<uint4*>(xs + m * a.x_stride + 8 * c) =
          *reinterpret_cast<const uint4*>(a.x + m * a.x_ld + krow0 + 8 * c);
    }
  } else {
    for (int i = threadIdx.x; i < a.M * krows; i += kThreads) {
      const int m = i / krows, c = i % krows;
      xs[m * a.x_stride + c] = a.x[m * a.x_ld + krow0 + c];
    }
  }
  const int col0 = tile * kBlockCols;
  for (int i = threadIdx.x; i < ngrp * (kBlockCols / 8); i += kThreads) {
    const int gi = i / (kBlockCols / 8), c8 = i % (kBlockCols / 8);
    const int col = col0 + 8 * c8;
    const __half* src = a.s + static_cast<int64_t>(grp0 + gi) * a.s_ld + col;
    __half* dst = ss + gi * kBlockCols + 8 * c8;
    if (col < a.N) {
      if (a.s_vec) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[e] = src[e];
      }
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  for (int i = threadIdx.x; i < ngrp * kBlockWords; i += kThreads) {
    const int gi = i / kBlockWords, w = i % kBlockWords;
    const int word = tile * kBlockWords + w;
    zs[gi * kBlockWords + w] =
        word < a.words ? static_cast<uint32_t>(a.qz[static_cast<int64_t>(grp0 + gi) * a.qz_ld + word]) : 0u;
  }
  __syncthreads();

  // 3. Main loop over this warp's 16-row steps.
  float acc[MT][8][4];
  float part[MT][8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        acc[mt][j][r] = 0.f;
        part[mt][j][r] = 0.f;
      }
  uint32_t zc[2][8];
  float sc[16];
  int cur_grp = -1;

  auto flush = [&]() {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc[mt][j][0] = fmaf(sc[j], part[mt][j][0], acc[mt][j][0]);
        acc[mt][j][1] = fmaf(sc[j], part[mt][j][1], acc[mt][j][1]);
        acc[mt][j][2] = fmaf(sc[8 + j], part[mt][j][2], acc[mt][j][2]);
        acc[mt][j][3] = fmaf(sc[8 + j], part[mt][j][3], acc[mt][j][3]);
#pragma unroll
        for (int r = 0; r < 4; ++r) part[mt][j][r] = 0.f;
      }
  };
  auto load_group = [&](int grp) {
    const int gi = grp - grp0;
    const uint2 zw = *reinterpret_cast<const uint2*>(zs + gi * kBlockWords + 2 * g);
    zero_consts(zw.x, zc[0]);
    zero_consts(zw.y, zc[1]);
    const uint4 s0 = *reinterpret_cast<const uint4*>(ss + gi * kBlockCols + 16 * g);
    const uint4 s1 = *reinterpret_cast<const uint4*>(ss + gi * kBlockCols + 16 * g + 8);
    const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = __half22float2(u32_as_h2(sw[i]));
      sc[2 * i] = f.x;
      sc[2 * i + 1] = f.y;
    }
  };

  auto process = [&](const uint32_t (&w)[8], int step) {
    const int grp = (step * 16) / a.G;
    if (grp != cur_grp) {
      if (cur_grp >= 0) flush();
      load_group(grp);
      cur_grp = grp;
    }
    // A fragments: tile j <- columns (j, 8+j) of this lane's 16; regs
    // {rows 0-1 word 0, rows 0-1 word 1, rows 2-3 word 0, rows 2-3 word 1}.
    uint32_t A[8][4];
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t r0 = w[2 * (2 * pr) + c];
        const uint32_t r1 = w[2 * (2 * pr + 1) + c];
        uint32_t oa[4], ob[4];
        const uint32_t za[4] = {zc[c][0], zc[c][1], zc[c][2], zc[c][3]};
        const uint32_t zb[4] = {zc[c][4], zc[c][5], zc[c][6], zc[c][7]};
        unpack_pairs(prmt(r0, r1, 0x6420u), za, oa);
        unpack_pairs(prmt(r0, r1, 0x7531u), zb, ob);
        const int reg = 2 * pr + c;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int slot = col_slot(j);
          A[j][reg] = slot < 4 ? oa[slot] : ob[slot - 4];
        }
      }
    }
    const int kl = (step - cs0) * 16 + 4 * t;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int tok = 8 * mt + g;
      uint2 b = make_uint2(0u, 0u);
      if (tok < a.M) b = *reinterpret_cast<const uint2*>(xs + tok * a.x_stride + kl);
#pragma unroll
      for (int j = 0; j < 8; ++j) mma_16816(part[mt][j], A[j], b.x, b.y);
    }
  };

  for (int base = ws0; base < ws1; base += kDepth) {
#pragma unroll
    for (int p = 0; p < kDepth; ++p) {
      const int step = base + p;
      if (step < ws1) {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = buf[p][i];
        if (step + kDepth < ws1) load_step<VEC>(buf[p], qp, a.qw_ld, step + kDepth, t, v0, v1);
        process(w, step);
      }
    }
  }
  if (cur_grp >= 0) flush();

  // 4. Reduce the 4 warps' partial tiles through shared memory.
  __syncthreads();  // everyone is done reading the staged x / scales / zeros
  float* red = reinterpret_cast<float*>(smem);  // [kWarps][MT*8][128]
  constexpr int kTok = MT * 8;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float* r0 = red + (warp * kTok + 8 * mt + 2 * t) * kBlockCols;
      r0[16 * g + j] = acc[mt][j][0];
      r0[kBlockCols + 16 * g + j] = acc[mt][j][1];
      r0[16 * g + 8 + j] = acc[mt][j][2];
      r0[kBlockCols + 16 * g + 8 + j] = acc[mt][j][3];
    }
  __syncthreads();

  const int col = threadIdx.x;  // kThreads == kBlockCols
  const int n = col0 + col;
  const bool col_ok = n < a.N;
  if (a.splits == 1) {
    for (int m = 0; m < a.M; ++m) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += red[(w * kTok + m) * kBlockCols + col];
      if (col_ok) a.y[m * a.y_ld + n] = __float2half_rn(v);
    }
    return;
  }

  float* slot = a.ws + (static_cast<int64_t>(tile) * a.splits + split) * a.M * kBlockCols;
  for (int m = 0; m < a.M; ++m) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[(w * kTok + m) * kBlockCols + col];
    slot[m * kBlockCols + col] = v;
  }
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = (atomicAdd(a.counters + tile, 1) == a.splits - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* tile_ws = a.ws + static_cast<int64_t>(tile) * a.splits * a.M * kBlockCols;
  for (int m = 0; m < a.M; ++m) {
    float v = 0.f;
    for (int s = 0; s < a.splits; ++s) v += __ldcg(tile_ws + (s * a.M + m) * kBlockCols + col);
    if (col_ok) a.y[m * a.y_ld + n] = __float2half_rn(v);
  }
  if (threadIdx.x == 0) a.counters[tile] = 0;
}

struct Plan {
  int tiles, steps, splits, ks_max, x_stride, max_groups;
  size_t smem, ws_bytes;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int plan_gemv(int M, int N, int K, int G, int split_req, int sm_count, Plan* p) {
  p->tiles = ceil_div(N, kBlockCols);
  p->steps = K / 16;
  int splits;
  if (split_req > 0) {
    splits = split_req;
  } else {
    // About four resident CTAs per SM, in whole waves of column tiles.
    const int target = 4 * sm_count;
    splits = std::max(1, (target + p->tiles / 2) / p->tiles);
  }
  splits = std::min(splits, p->steps);
  // Keep the staged x slice within 64 KB of shared memory.
  const int max_rows = std::max(16, (32768 / std::max(M, 1)) / 16 * 16);
  splits = std::max(splits, ceil_div(K, max_rows));
  splits = std::min(std::max(splits, 1), p->steps);
  const int mt = M > 8 ? 2 : 1;
  // The split is a hint: raise it until the staged slice fits in shared memory.
  for (;; ++splits) {
    p->splits = splits;
    p->ks_max = ceil_div(p->steps, splits) * 16;
    p->x_stride = static_cast<int>(align_up(p->ks_max, 64)) + 16;  // row stride = 32 mod 128 bytes
    p->max_groups = p->ks_max / G + 2;
    const size_t stage = static_cast<size_t>(M) * p->x_stride * 2 +
                         static_cast<size_t>(p->max_groups) * kBlockCols * 2 +
                         static_cast<size_t>(p->max_groups) * kBlockWords * 4;
    const size_t red = static_cast<size_t>(kWarps) * mt * 8 * kBlockCols * 4;
    p->smem = align_up(std::max(stage, red), 16);
    if (p->smem <= 200 * 1024 || splits >= p->steps) break;
  }
  p->ws_bytes = splits > 1 ? kCounterBytes + static_cast<size_t>(p->tiles) * splits * M * kBlockCols * 4 : 0;
  return ASHQK_OK;
}

template <int MT, bool VEC>
int launch_instance(const GemvArgs& args, const Plan& p, cudaStream_t stream) {
  static std::atomic<bool> configured[64];  // zero-initialised (static storage)  // per template instance and device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ASHQK_ERR_CUDA;
  if (!configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(gemv_kernel<MT, VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
        cudaSuccess)
      return ASHQK_ERR_CUDA;
    configured[dev].store(true, std::memory_order_release);
  }
  gemv_kernel<MT, VEC><<<dim3(p.tiles, p.splits), kThreads, p.smem, stream>>>(args);
  return launch_status();
}

}  // namespace

bool gemv_tma_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                       int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int G);
size_t gemv_tma_workspace_bytes(int M, int N, int K, int G, int split_k, int sm_count);
int gemv_tma_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz, int64_t qz_ld,
                    const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G, int split_k,
                    void* workspace, size_t ws_bytes, int sm_count, cudaStream_t stream);

bool gemv_strip_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                         int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int G);
int gemv_strip_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                      int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K, int G,
                      int sm_count, cudaStream_t stream);

bool gemv_cluster_eligible(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                           int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int G);
int gemv_cluster_launch(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                        int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K,
                        int G, int split, int sm_count, cudaStream_t stream);

namespace {
// 0 auto (cluster-split strips, then split-K TMA, then register streaming),
// 1 register-streaming, 2 split-K TMA, 3 column strips (whole K per CTA),
// 4 cluster-split strips.
int g_gemv_impl = 0;
}

int gemv_workspace_bytes(int M, int N, int K, int G, int split_k, size_t* bytes) {
  DeviceInfo info;
  int rc = device_info(&info);
  if (rc) return rc;
  Plan p;
  const int m = std::min(M, kMaxM);
  plan_gemv(m, N, K, G, split_k, info.sm_count, &p);
  *bytes = std::max(p.ws_bytes, gemv_tma_workspace_bytes(m, N, K, G, split_k, info.sm_count));
  return ASHQK_OK;
}

bool gemv_cluster_plannable(int M, int N, int K, int G, int sm_count, int split);

// Workspace bytes the call below will use with these operands: 0 when it takes
// the cluster-split kernel (which needs none, whatever the split), else the
// split-K kernels' need for this problem.
int gemv_call_workspace_bytes(const void* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                              int64_t qz_ld, const void* s, int64_t s_ld, int M, int N, int K, int G, int split_k,
                              size_t* bytes) {
  DeviceInfo info;
  int rc = device_info(&info);
  if (rc) return rc;
  const bool cluster_ok = gemv_cluster_eligible(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, M, N, G);
  if (cluster_ok && (g_gemv_impl == 4 || g_gemv_impl == 0) &&
      gemv_cluster_plannable(M, N, K, G, info.sm_count, split_k)) {
    *bytes = 0;
    return ASHQK_OK;
  }
  return gemv_workspace_bytes(M, N, K, G, split_k, bytes);
}

// M <= 16 rows, already validated.
int gemv_launch_rows(const __half* x, int64_t x_ld, const int32_t* qw, int64_t qw_ld, const int32_t* qz,
                     int64_t qz_ld, const __half* s, int64_t s_ld, __half* y, int64_t y_ld, int M, int N, int K,
                     int G, int split_k, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  DeviceInfo info;
  int rc = device_info(&info);
  if (rc) return rc;
  if (G % 16) return ASHQK_ERR_UNSUPPORTED;
  // The cluster-split kernel takes a caller's split_k as its K split (CTAs per
  // cluster) and needs no workspace. Column strips split K their own way, so a
  // forced split_k that the cluster kernel cannot plan goes to the split-K kernels.
  const bool cluster_ok = gemv_cluster_eligible(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, M, N, G);
  if (g_gemv_impl == 4 && !cluster_ok) return ASHQK_ERR_UNSUPPORTED;
  if (cluster_ok && (g_gemv_impl == 4 || g_gemv_impl == 0)) {
    const int rc_cl = gemv_cluster_launch(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, y, y_ld, M, N, K, G, split_k,
                                          info.sm_count, stream);
    if (!(rc_cl == ASHQK_ERR_UNSUPPORTED && g_gemv_impl == 0)) return rc_cl;
  }
  const bool strip_ok = gemv_strip_eligible(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, M, N, G);
  if (g_gemv_impl == 3 && !strip_ok) return ASHQK_ERR_UNSUPPORTED;
  if (strip_ok && (g_gemv_impl == 3 || (g_gemv_impl == 0 && split_k <= 0))) {
    const int rc_strip = gemv_strip_launch(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, y, y_ld, M, N, K, G,
                                           info.sm_count, stream);
    if (!(rc_strip == ASHQK_ERR_UNSUPPORTED && g_gemv_impl == 0)) return rc_strip;
  }
  const bool tma_ok = gemv_tma_eligible(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, M, N, G);
  if (g_gemv_impl == 2 && !tma_ok) return ASHQK_ERR_UNSUPPORTED;
  if (tma_ok && g_gemv_impl != 1) {
    const int rc_tma = gemv_tma_launch(x, x_ld, qw, qw_ld, qz, qz_ld, s, s_ld, y, y_ld, M, N, K, G, split_k, workspace,
                                       ws_bytes, info.sm_count, stream);
    // A slice that cannot fit the TMA kernel's shared memory (tiny groups with a
    // forced small split) falls back to the register-streaming kernel.
    if (!(rc_tma == ASHQK_ERR_UNSUPPORTED && g_gemv_impl == 0)) return rc_tma;
  }
  Plan p;
  plan_gemv(M, N, K, G, split_k, info.sm_count, &p);
  if (p.smem > 200 * 1024 || p.tiles > kMaxTiles) return ASHQK_ERR_UNSUPPORTED;
  if (p.splits > 1 && (workspace == nullptr || ws_bytes < p.ws_bytes || !aligned(workspace, 256)))
    return ASHQK_ERR_WORKSPACE;
  GemvArgs a;
  a.x = x;
  a.qw = qw;
  a.qz = qz;
  a.s = s;
  a.y = y;
  a.x_ld = x_ld;
  a.qw_ld = qw_ld;
  a.qz_ld = qz_ld;
  a.s_ld = s_ld;
  a.y_ld = y_ld;
  a.M = M;
  a.N = N;
  a.K = K;
  a.G = G;
  a.words = N / 8;
  a.steps = p.steps;
  a.splits = p.splits;
  a.x_stride = p.x_stride;
  a.max_groups = p.max_groups;
  a.x_vec = aligned(x, 16) && (x_ld % 8 == 0);
  a.s_vec = aligned(s, 16) && (s_ld % 8 == 0);
  if (p.splits > 1) {
    // Counters first, at a fixed offset: every problem that shares the
    // workspace sees them zero, whatever it left in the partial-sum slots.
    a.counters = static_cast<int*>(workspace);
    a.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  } else {
    a.ws = nullptr;
    a.counters = nullptr;
  }
  const bool vec = (a.words % 2 == 0) && (qw_ld % 2 == 0) && aligned(qw, 8);
  if (M > 8) return vec ? launch_instance<2, true>(a, p, stream) : launch_instance<2, false>(a, p, stream);
  return vec ? launch_instance<1, true>(a, p, stream) : launch_instance<1, false>(a, p, stream);
}

int gemv_max_m() { return kMaxM; }

}  // namespace ashqk

extern "C" int ashqk_gemv_max_m(void) { return ashqk::kMaxM; }

extern "C" int ashqk_set_gemv_kernel(int which) {
  if (which < 0 || which > 4) return ASHQK_ERR_INVALID_ARGUMENT;
  ashqk::g_gemv_impl = which;
  return ASHQK_OK;
}

extern "C" int ashqk_gemv_workspace_size(int M, int N, int K, int group_size, int split_k, size_t* bytes) {
  if (!bytes || M <= 0 || N <= 0 || K <= 0 || group_size <= 0 || N % 8 || K % group_size)
    return ASHQK_ERR_INVALID_ARGUMENT;
  return ashqk::gemv_workspace_bytes(M, N, K, group_size, split_k, bytes);
}

extern "C" int ashqk_w4a16_gemv(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                                const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld, void* y,
                                int64_t y_ld, int M, int N, int K, int group_size, int split_k, void* workspace,
                                size_t workspace_bytes, void* stream) {
  int rc = ashqk::check_awq_args(x, x_ld, qweight, qw_ld, qzeros, qz_ld, scales, s_ld, y, y_ld, M, N, K, group_size);
  if (rc) return rc;
  // Rows beyond 16 are processed 16 at a time (each chunk re-reads the weights).
  for (int m0 = 0; m0 < M; m0 += ashqk::kMaxM) {
    const int mc = std::min(ashqk::kMaxM, M - m0);
    rc = ashqk::gemv_launch_rows(static_cast<const __half*>(x) + m0 * x_ld, x_ld, qweight, qw_ld, qzeros, qz_ld,
                                 static_cast<const __half*>(scales), s_ld, static_cast<__half*>(y) + m0 * y_ld, y_ld,
                                 mc, N, K, group_size, split_k, workspace, workspace_bytes,
                                 static_cast<cudaStream_t>(stream));
    if (rc) return rc;
  }
  return ASHQK_OK;
}
