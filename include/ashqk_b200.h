/*
 * ashqk_b200.h -- C ABI of the B200 (sm_100a) AWQ W4A16 linear-layer kernels.
 *
 * Drop-in for the hot path of MMMchou/ash-quant-kernels (`ashqk`): the same
 * AutoAWQ "GEMM" tensors, the same math, called with plain pointers and sizes.
 *
 *   x        fp16  [M, K]      row stride x_ld (elements), unit column stride
 *   qweight  int32 [K, N/8]    row stride qw_ld (words); 8 uint4 per word, packed
 *                              along N in nibble order [0,2,4,6,1,3,5,7]
 *   qzeros   int32 [K/G, N/8]  row stride qz_ld (words), same packing
 *   scales   fp16  [K/G, N]    row stride s_ld (elements)
 *   y        fp16  [M, N]      row stride y_ld (elements), written, never read
 *   W[k, n] = (q[k, n] - z[k/G, n]) * s[k/G, n];   y = x @ W
 *
 * Conventions shared by every entry point:
 *   - fp16 buffers are passed as `void*` holding IEEE binary16 values;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 *     asynchronous on it and never synchronises the device;
 *   - all pointers are device pointers on the current CUDA device;
 *   - the return value is an ashqk_status; ashqk_status_string() names it.
 *     On error nothing was launched, except ASHQK_ERR_CUDA, which reports a
 *     launch failure from the CUDA runtime.
 *
 * Workspace. The split-K kernels reduce partial sums through a caller-owned
 * device workspace of ashqk_*_workspace_size() bytes. It must be zero-filled
 * once when allocated; every call leaves it zeroed again on exit (the same
 * self-resetting contract as the reference, ashqk/kernels/w4a16_gemv.py:110-120).
 * Calls that share a workspace must be ordered on one stream.
 */
#ifndef ASHQK_B200_H_
#define ASHQK_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ASHQK_API __attribute__((visibility("default")))
#else
#define ASHQK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ashqk_status {
  ASHQK_OK = 0,
  ASHQK_ERR_INVALID_ARGUMENT = 1, /* a null pointer, a bad size, stride or alignment */
  ASHQK_ERR_UNSUPPORTED = 2,      /* legal for the format, not handled by this build */
  ASHQK_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required */
  ASHQK_ERR_CUDA = 4,             /* the CUDA runtime reported an error */
  ASHQK_ERR_NO_DEVICE = 5         /* the current device is not an sm_100 GPU */
} ashqk_status;

/* Static string naming a status code. */
ASHQK_API const char* ashqk_status_string(int status);

/* Library version, "major.minor.patch". */
ASHQK_API const char* ashqk_version(void);

/* Largest M the decode GEMV accepts (the dispatcher's GEMV_MAX_M). */
ASHQK_API int ashqk_gemv_max_m(void);

/*
 * Bytes of workspace ashqk_w4a16_gemv needs for this problem and split count
 * (split_k <= 0 picks the default). Replaces the workspace sizing of
 * ashqk/kernels/w4a16_gemv.py:110-120.
 */
ASHQK_API int ashqk_gemv_workspace_size(int M, int N, int K, int group_size, int split_k, size_t* bytes);

/*
 * Decode GEMV, 1 <= M <= ashqk_gemv_max_m(): y = x @ deq(qweight, qzeros, scales).
 * Tensor-core (mma.sync m16n8k16) dot products on int4 unpacked in registers,
 * per-group factored scales and zero points, split-K reduced in the same launch.
 * split_k <= 0 picks the split from the problem size and SM count; split_k > 0
 * is the number of CTAs that share each output tile's K (at most 16), which
 * needs no workspace when the default kernel takes the problem.
 * Replaces ashqk/kernels/w4a16_gemv.py:132-167 (w4a16_gemv).
 */
ASHQK_API int ashqk_w4a16_gemv(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                     const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                     void* y, int64_t y_ld, int M, int N, int K, int group_size, int split_k,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Decode GEMV that allocates nothing: same arguments and result as
 * ashqk_w4a16_gemv, but without a workspace. It is meant for callers that
 * cannot allocate device memory (a plugin that is handed only device pointers
 * by its host framework, or a caller that must not call cudaMalloc on its hot
 * path). Calls that take the default cluster-split kernel (16-byte aligned
 * operands, N % 32 == 0, group_size % 16 == 0) use no scratch at all. The split-K kernels the other calls take use a fixed 8 MiB array inside
 * this library, held on every GPU that loads it until the process exits;
 * those whose scratch need exceeds it return ASHQK_ERR_WORKSPACE without
 * launching anything. The first such call on a device looks up that array's
 * device address, so make it before any stream capture. All calls share the
 * array: calls that may overlap on the GPU (other streams, other threads)
 * race, so order them on one stream. Each such call clears the part that must
 * start at zero. This entry point has no counterpart in the reference.
 */
ASHQK_API int ashqk_w4a16_gemv_noalloc(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                                       const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                                       void* y, int64_t y_ld, int M, int N, int K, int group_size, int split_k,
                                       void* stream);

/*
 * Selects the decode GEMV kernel for later calls in this process: 0 = automatic
 * (cluster-split tiles when N % 32 == 0, group_size % 16 == 0, rows are
 * 16-byte aligned and a plan fits; else column strips when no split_k is
 * requested; else the split-K TMA kernel when eligible; else the
 * register-streaming kernel), 1 = always
 * register-streaming, 2 = always split-K TMA, 3 = always column strips over
 * the whole K per CTA, 4 = always cluster-split tiles (ineligible
 * problems then return ASHQK_ERR_UNSUPPORTED). No reference counterpart: a
 * test and tuning switch.
 */
ASHQK_API int ashqk_set_gemv_kernel(int which);

/*
 * Selects the prefill GEMM kernel for later calls in this process: 0 = automatic
 * (tcgen05 when the problem is eligible -- on CTA pairs, cta_group::2 with
 * M = 256 per instruction, when M > 128, N % 256 == 0, the 256-row tiles fill
 * at least ~0.6 of the SM pairs and pad M by at most 1/8, else one CTA per
 * output tile -- otherwise the chunked GEMV), 1 = always the chunked GEMV,
 * 2 = always tcgen05 (automatic variant), 3 = tcgen05 on one CTA per tile,
 * 4 = tcgen05 on CTA pairs. Forced choices return ASHQK_ERR_UNSUPPORTED for
 * problems they do not take. No reference counterpart: a test and tuning
 * switch.
 */
ASHQK_API int ashqk_set_gemm_kernel(int which);

/*
 * Reads (and with clear != 0 resets) the device error word of the current
 * device after synchronising it. Bit 1: a pipeline wait inside a kernel ran
 * past its time limit and the kernel gave up (its output and any split-K
 * workspace it used are then invalid; re-zero the workspace). Bit 2: a kernel
 * rejected its launch parameters. Bit 3: a peer rank never arrived at
 * ashqk_allreduce_f16_oneshot. No reference counterpart.
 */
ASHQK_API int ashqk_get_device_errors(unsigned int* bits, int clear);

/*
 * Registers, for the current device, a page-locked host word (e.g. a pinned
 * torch tensor) that receives the device error word whenever a kernel raises
 * a bit in it -- only then, so calls that succeed pay nothing. A host can poll
 * it before its next call instead of synchronising. NULL unregisters. Returns
 * ASHQK_ERR_INVALID_ARGUMENT for memory the device cannot map. No reference
 * counterpart.
 */
ASHQK_API int ashqk_set_error_mirror(unsigned int* host_pinned);

/*
 * Bytes of workspace ashqk_w4a16_gemm may need: 0 for the tcgen05 kernel; the
 * chunked-GEMV fallback (shapes the tcgen05 kernel does not take) needs the
 * decode GEMV's split-K workspace. Replaces the sizing of
 * ashqk/kernels/w4a16_gemm_v3.py:108-119.
 */
ASHQK_API int ashqk_gemm_workspace_size(int M, int N, int K, int group_size, size_t* bytes);

/*
 * Prefill GEMM, any M >= 1: y = x @ deq(...). int4 is dequantised into shared
 * memory and fed to tcgen05.mma with the accumulator in tensor memory, for
 * N % 128 == 0, K % 64 == 0, group size 16, 32 or a multiple of 64, 16-byte
 * aligned bases and leading dimensions (x, scales, y in multiples of 8 halves;
 * qweight, qzeros in multiples of 4 words). Other valid problems run the decode
 * GEMV over 16-row chunks. Replaces ashqk/kernels/w4a16_gemm_v3.py:131-171
 * (w4a16_gemm_v3).
 */
ASHQK_API int ashqk_w4a16_gemm(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                     const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                     void* y, int64_t y_ld, int M, int N, int K, int group_size,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Workspace for ashqk_w4a16_linear: the larger of the two paths' needs.
 */
ASHQK_API int ashqk_linear_workspace_size(int M, int N, int K, int group_size, size_t* bytes);

/*
 * Dispatcher: M <= ashqk_gemv_max_m() runs the GEMV, larger M the GEMM.
 * Replaces ashqk/ops.py:18-26 (w4a16_linear) for a 2-D x.
 */
ASHQK_API int ashqk_w4a16_linear(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                       const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                       void* y, int64_t y_ld, int M, int N, int K, int group_size,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * W = (q - z) * s written as fp16 [K, N] (row stride w_ld), bit-identical to
 * dequantize_awq(qweight, qzeros, scales, torch.float16) of ashqk/ref.py:78-86.
 */
ASHQK_API int ashqk_dequantize_awq_f16(const int32_t* qweight, int64_t qw_ld, const int32_t* qzeros,
                             int64_t qz_ld, const void* scales, int64_t s_ld, void* w, int64_t w_ld,
                             int N, int K, int group_size, void* stream);

/*
 * Same, written as fp32 [K, N]: dequantize_awq(..., torch.float32) of ashqk/ref.py:78-86.
 */
ASHQK_API int ashqk_dequantize_awq_f32(const int32_t* qweight, int64_t qw_ld, const int32_t* qzeros,
                             int64_t qz_ld, const void* scales, int64_t s_ld, float* w, int64_t w_ld,
                             int N, int K, int group_size, void* stream);

/*
 * Launch plan of the column-strip decode GEMV (the default kernel for M <= 16
 * on 16-byte aligned operands) for an M x N x K problem with the given group
 * size on sm_count SMs (0: the current device's, and the plan the library
 * launches there, which also caps CTAs per SM at what the register file holds
 * for grids larger than that). Host arithmetic only: with sm_count > 0 it
 * needs no GPU. The counterpart of the reference's launch
 * configuration choice, _default_config (ashqk/kernels/w4a16_gemv.py:123-129).
 * Returns ASHQK_ERR_UNSUPPORTED for problems the strip kernel does not take
 * (M > 16, N % 32, group_size % 16).
 */
typedef struct {
  int grid_x;          /* column strips of 64 outputs */
  int grid_y;          /* CTAs sharing a strip's K range (one cluster along y when > 1) */
  int threads;         /* per CTA: one producer warp + the consumer warps */
  int consumer_warps;  /* 4, 8 or 16 */
  int ring_stages;     /* 256-row stages resident in shared memory */
  int stages_total;    /* ceil(K / 256) */
  int stage_bytes;     /* bytes of one stage: weights, x, scale and zero rows */
  int smem_bytes;      /* dynamic shared memory per CTA */
} ashqk_strip_plan;
ASHQK_API int ashqk_gemv_strip_plan(int M, int N, int K, int group_size, int sm_count, ashqk_strip_plan* plan);

/*
 * Launch plan of the cluster-split decode GEMV (the default kernel for M <= 16
 * on 16-byte aligned operands with N % 32 == 0 and group_size % 16 == 0) on
 * sm_count SMs (0: the current device's). Output tiles of 256 or 512 columns;
 * each tile's K in stages of 32 KB of packed weights (256 or 128 rows); a
 * cluster of cluster_ctas CTAs shares a tile, dealing its stages out in equal
 * contiguous ranges. Host arithmetic only: with sm_count > 0 it needs no GPU.
 * The counterpart of the reference's launch configuration choice,
 * _default_config (ashqk/kernels/w4a16_gemv.py:123-129). Returns
 * ASHQK_ERR_UNSUPPORTED for problems the kernel does not take.
 */
typedef struct {
  int tile_cols;           /* 256 or 512 */
  int stage_rows;          /* 256 or 128: 32 KB of packed weights per stage */
  int tiles;               /* ceil(N / tile_cols) */
  int stages_per_tile;     /* ceil(K / stage_rows) */
  int cluster_ctas;        /* CTAs per thread-block cluster sharing a tile's K (1: no cluster) */
  int ctas;                /* grid size */
  int max_stages_per_cta;  /* the busiest CTA's stages */
  int threads;             /* per CTA: one producer warp + 8 consumer warps */
  int ring_stages;         /* stages resident in shared memory */
  int stage_bytes;
  int smem_bytes;          /* dynamic shared memory per CTA */
} ashqk_cluster_plan;
ASHQK_API int ashqk_gemv_cluster_plan(int M, int N, int K, int group_size, int sm_count, ashqk_cluster_plan* plan);

/*
 * Tuning of the cluster-split decode GEMV's plan for later calls in this
 * process (0 = automatic for each): shared-memory budget per CTA in KiB
 * (32-200), CTAs per cluster (1-16), tile columns (256 or 512) and a cap on
 * the grid's CTAs. No reference counterpart: a benchmark sweep switch.
 */
ASHQK_API int ashqk_gemv_set_tuning(int smem_kb, int cluster_ctas, int tile_cols, int max_ctas);

/*
 * One-shot all-reduce of fp16 tensors over NVLink peer memory, for the
 * tensor-parallel decode path (row-parallel partials of 8-128 KB, where NCCL's
 * per-call cost dominates). No reference counterpart: the reference has no
 * multi-GPU code. Usage, per rank (one process per GPU, same order everywhere):
 * size a region for the largest tensor (ashqk_p2p_region_bytes), allocate it
 * (ashqk_p2p_alloc, zeroed), exchange ashqk_p2p_export handles (64 bytes) with
 * the peers, open theirs (ashqk_p2p_import), put the world's region pointers
 * (own one at index rank) in a device array, and call
 * ashqk_allreduce_f16_oneshot. Every rank must make the same sequence of calls;
 * a rank that does not arrive within ~2 s makes the others give up (device
 * error bit 3, output not written) rather than hang, and while that bit is set
 * every later call returns at once; the regions are unusable after it.
 * n: a multiple of 8 elements, <= max_elems;
 * in/out 16-byte aligned (in == out allowed). Sum in fp32 over ranks in rank
 * order, one rounding to fp16.
 */
ASHQK_API int ashqk_p2p_region_bytes(int64_t max_elems, size_t* bytes);
ASHQK_API int ashqk_p2p_alloc(size_t bytes, void** ptr);
ASHQK_API int ashqk_p2p_free(void* ptr);
ASHQK_API int ashqk_p2p_export(void* ptr, void* handle64);
ASHQK_API int ashqk_p2p_import(const void* handle64, void** ptr);
ASHQK_API int ashqk_p2p_close(void* ptr);
ASHQK_API int ashqk_allreduce_f16_oneshot(const void* in, void* out, int64_t n, const void* regions_dev, int rank,
                                          int world, int64_t max_elems, void* stream);

/*
 * Low-latency variant of the same all-reduce: every rank pushes each pair of
 * fp16 values into every peer's region as one 8-byte line together with the
 * call's epoch (no fence, no peer-load round trip) and polls its own region;
 * one CTA per 1024 elements (at most 64 CTAs). Regions are sized by
 * ashqk_p2p_ll_region_bytes (max_elems <= 65536) and set up exactly as for
 * ashqk_allreduce_f16_oneshot (allocate, export, import, pointer array); an
 * LL region serves this call and ashqk_w4a16_gemv_allreduce, not the one-shot
 * call. Same sum (fp32, rank order, one rounding), same ~2 s peer limit and
 * sticky device error bit 3.
 */
ASHQK_API int ashqk_p2p_ll_region_bytes(int64_t max_elems, size_t* bytes);
ASHQK_API int ashqk_allreduce_f16_ll(const void* in, void* out, int64_t n, const void* regions_dev, int rank,
                                     int world, int64_t max_elems, void* stream);

/*
 * Row-parallel decode layer with the all-reduce fused into the GEMV: every rank
 * passes its K shard (x columns, qweight / qzeros / scales rows on group
 * boundaries) and gets in y the sum over the ranks of the fp16 partials, in
 * fp32, rank order, rounded once -- bit for bit what ashqk_w4a16_gemv followed
 * by ashqk_allreduce_f16_ll gives. The partial never reaches HBM: the
 * column-strip GEMV's epilogue pushes it to the peers as low-latency lines and
 * sums theirs. Regions as for ashqk_allreduce_f16_ll (the two share a region
 * and its call counter); M * N <= max_elems. Returns ASHQK_ERR_UNSUPPORTED
 * (nothing launched) when the column-strip kernel does not take the problem
 * or cannot keep its whole grid resident; the caller then runs the two steps.
 * No reference counterpart: the reference has no multi-GPU code.
 */
ASHQK_API int ashqk_w4a16_gemv_allreduce(const void* x, int64_t x_ld, const int32_t* qweight, int64_t qw_ld,
                                         const int32_t* qzeros, int64_t qz_ld, const void* scales, int64_t s_ld,
                                         void* y, int64_t y_ld, int M, int N, int K, int group_size,
                                         const void* regions_dev, int rank, int world, int64_t max_elems,
                                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ASHQK_B200_H_ */
