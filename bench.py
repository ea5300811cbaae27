"""Benchmark of the W4A16 decode hot path on B200 (one JSON line on rank 0).

Workload: all linear layers of one decoded token of a
Qwen3-8B-shaped model -- 36 decoder layers x {qkv 4096->6144, o 4096->4096,
gate_up 4096->24576, down 12288->4096}, int4 AWQ, G=128, with distinct weight
buffers per layer (3.6 GB, far beyond the 126 MB L2, so no flush is needed).
Within a layer the calls are chained (qkv -> o -> gate_up -> down) through
row-strided views, as a real decoder would feed them. A step = one token (M=1)
through all 144 layers, captured once in a CUDA graph and replayed.

Metric: us/token (lower is better). The M=4 figure, per-layer GEMV bandwidth and
roofline fractions are reported alongside. ``e2e`` repeats the M=1 step through
the public API with the input copied from pinned host memory and the result
read back every step.

Multi-GPU (torchrun, N ranks): the same model under tensor parallelism --
qkv / gate_up column-parallel (N sharded) and o / down row-parallel (K sharded,
NCCL all-reduce of the partial sums); strong scaling of the same token.

``--impl reference`` times the reference algorithm on the host cores instead
(the oracle's C restatement of ashqk/ref.py: dequantise in fp32, then the
GEMM), on a bounded sample extrapolated to the whole token.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "ash-quant-kernels_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "us/token all linear layers at M=1,4; GEMV HBM GB/s vs peak; GEMM TFLOPS"
UNIT = "us/token"
LAYERS = (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 24576, 4096), ("down", 4096, 12288))
N_LAYERS = 36
GROUP = 128
FALLBACK_HBM_GBS = 6650.0


def w4a16_bytes(m, n, k, g):
    """Algorithmic bytes of one call (bench/bench_gemm.py:45-46 of the reference)."""
    return m * k * 2 + k * n // 2 + (k // g) * n * 2 + (k // g) * n // 2 + m * n * 2


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# CPU reference arm / baseline: the reference's algorithm on the host cores.
# ---------------------------------------------------------------------------

def _cpu_layer_set(seed_base=0):
    """One decoder layer's four AWQ problems at M=1 (uniform 4-bit q and z in random words,
    scales ~ U(0.002, 0.02), x ~ N(0, 1)), as numpy arrays."""
    import numpy as np

    probs = []
    for i, (_, n, k) in enumerate(LAYERS):
        rng = np.random.default_rng(seed_base + i)
        x = rng.standard_normal((1, k), dtype=np.float32).astype(np.float16)
        qw = rng.integers(0, 2 ** 32, size=(k, n // 8), dtype=np.uint32).view(np.int32)
        qz = rng.integers(0, 2 ** 32, size=(k // GROUP, n // 8), dtype=np.uint32).view(np.int32)
        s = rng.uniform(0.002, 0.02, size=(k // GROUP, n)).astype(np.float16)
        probs.append((x, qw, qz, s))
    return probs


def cpu_reference_sample(steps: int, warmup: int, budget_s: float | None = None):
    """Time one decoder layer's four linear calls at M=1 per step on the host (all threads), with the
    oracle's C restatement of ashqk/ref.py (fp32 dequantisation, fp64-accumulated GEMM).

    Returns (us_per_token, threads, sample_description, per_step_seconds list).
    """
    from oracle import awq_oracle as O

    threads = O.c_oracle().awq_oracle_threads()
    probs = _cpu_layer_set()

    def one_layer_set():
        t0 = time.perf_counter()
        for x, qw, qz, s in probs:
            O.c_gemm(x, qw, qz, s, out_fp16=True)
        return time.perf_counter() - t0

    for _ in range(warmup):
        one_layer_set()
    times = []
    t_start = time.perf_counter()
    for i in range(max(steps, 1)):
        times.append(one_layer_set())
        if budget_s is not None and time.perf_counter() - t_start > budget_s and i >= 2:
            break
    desc = (f"each step: one decoder layer's 4 linear calls (qkv, o, gate_up, down) at M=1, G=128, via the C "
            f"restatement of ashqk/ref.py (fp32 dequant + fp64 GEMM, OpenMP {threads} threads); "
            f"us/token = 36 x median step; {len(times)} steps; CPU {cpu_model()}, "
            f"os.cpu_count()={os.cpu_count()}")
    return statistics.median(times) * N_LAYERS * 1e6, threads, desc, times


def torch_ref_sample():
    """The reference's own CPU path, ashqk/ref.py's w4a16_gemm_ref (dequantise to fp16, then x @ W)
    and w4a16_gemm_fp32 (the fp32 truth), with torch.set_num_threads(os.cpu_count()): each of one
    decoder layer's four calls at M=1 timed once after one untimed call; per-token figures = 36 x the
    layer sum. The package's ashqk.ref is the same code path (no native extension is loaded)."""
    import torch

    from ashqk import ref as R

    torch.set_num_threads(os.cpu_count() or 1)
    res = {"threads": torch.get_num_threads(), "per_layer_ms": {}}
    tot = {"w4a16_gemm_ref": 0.0, "w4a16_gemm_fp32": 0.0}
    for (name, _, _), (x, qw, qz, s) in zip(LAYERS, _cpu_layer_set(100)):
        xt, qwt, qzt, st = (torch.from_numpy(a) for a in (x, qw, qz, s))
        entry = {}
        for fn_name in tot:
            fn = getattr(R, fn_name)
            fn(xt, qwt, qzt, st)
            t0 = time.perf_counter()
            fn(xt, qwt, qzt, st)
            dt = time.perf_counter() - t0
            entry[fn_name] = round(dt * 1e3, 1)
            tot[fn_name] += dt
        res["per_layer_ms"][name] = entry
    res["us_per_token"] = {k: round(v * N_LAYERS * 1e6, 1) for k, v in tot.items()}
    res["config1_qkv_m1_ms"] = res["per_layer_ms"]["qkv"]
    return res


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    warmup = max(args.warmup, 1)
    value, threads, desc, times = cpu_reference_sample(args.steps, warmup)
    ms_per_step = statistics.mean(times) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT,
        "n_gpus": args.gpus, "steps": len(times), "warmup": warmup, "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (fp16 in/out)",
        "data": "synthetic", "config": workload_config(args.gpus),  # the same workload keys as our arm
        "step": "one decoder layer (4 linear calls) of the 36-layer token; value = 36 x median step",
        "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_torch_ref:
        line["ref_py"] = torch_ref_sample()
    print(json.dumps(line), flush=True)


def default_tp_allreduce(world):
    """The row-parallel reduction bench.py uses without ASHQK_TP_ALLREDUCE: NVLink lines up to 4 ranks."""
    return "ll" if world <= 4 else "nccl"


def workload_config(world, n_layers=N_LAYERS):
    cfg = {
        "workload": "BASELINE config 3: 36-layer Qwen3-8B-shape linear stack (qkv 4096->6144, o 4096->4096, "
                    "gate_up 4096->24576, down 12288->4096), M=1 (M=4 reported too), int4 AWQ G=128, "
                    "CUDA-graph replay",
        "model": "qwen3-8b linear layers (random AWQ weights)",
        "global_batch": 1, "seq_len": 1,
        "parallelism": f"tp{world}" if world > 1 else "none",
        "tp_allreduce": os.environ.get("ASHQK_TP_ALLREDUCE", default_tp_allreduce(world)) if world > 1 else None,
        "l2": "inputs larger than L2: 3.6 GB of distinct per-layer weights per step",
    }
    if n_layers != N_LAYERS:  # a reduced stack (profiling runs), not the benchmark workload
        cfg["decoder_layers"] = n_layers
        cfg["l2"] = f"{n_layers} layers x 96.5 MB of distinct weights per step"
    return cfg


# ---------------------------------------------------------------------------
# Clock sampling during the timed region (NVML, read-only).
# ---------------------------------------------------------------------------

class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = None
            try:
                import torch

                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM))
                self.reasons |= int(n.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [k for k, bit in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def make_stack(world, rank, device, n_layers=N_LAYERS):
    """Random AWQ weights for 36 layers; TP-sharded when world > 1.

    q, z are uniform over 0..15 (random 32-bit words), scales ~ U(0.002, 0.02),
    generated on the device from a per-layer seed.
    """
    import torch

    gen = torch.Generator(device=device)
    stack = []
    for li in range(n_layers):
        layer = {}
        for j, (name, n, k) in enumerate(LAYERS):
            gen.manual_seed(1000 * li + j)
            col_parallel = name in ("qkv", "gate_up")
            n_loc = n // world if col_parallel else n
            k_loc = k // world if not col_parallel else k
            qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (k_loc, n_loc // 8), dtype=torch.int32, device=device,
                               generator=gen)
            qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (k_loc // GROUP, n_loc // 8), dtype=torch.int32,
                               device=device, generator=gen)
            s = (torch.rand((k_loc // GROUP, n_loc), device=device, generator=gen) * 0.018 + 0.002).half()
            layer[name] = (qw, qz, s)
        stack.append(layer)
    return stack


def stack_step(stack, h, world, group, allreduce=None, fused=False):
    """One token through every linear layer (public API calls). The row-parallel partials are summed
    with NCCL, or with ``allreduce`` (an ``ashqk.tp.P2PAllReduce``) when given; with ``fused`` the
    row-parallel layers run as one GEMV + all-reduce kernel each where it takes them."""
    import torch.distributed as dist

    from ashqk import w4a16_linear

    def row_parallel(x, weights):
        if world > 1 and fused:
            y = allreduce.fused_linear(x, *weights)
            if y is not None:
                return y
        y = w4a16_linear(x, *weights)                           # partial [M, 4096]
        if world > 1:
            if allreduce is not None:
                allreduce(y, out=y)
            else:
                dist.all_reduce(y, group=group)
        return y

    out = None
    for layer in stack:
        a = w4a16_linear(h, *layer["qkv"])                      # [M, 6144/P]
        # Attention output stands in as the first columns of qkv (o input: 4096/P per rank).
        o_in = a[:, : 4096 // world]
        b = row_parallel(o_in, layer["o"])                      # [M, 4096], summed over ranks
        c = w4a16_linear(b, *layer["gate_up"])                  # [M, 24576/P]
        d_in = c[:, : 12288 // world]
        out = row_parallel(d_in, layer["down"])                 # [M, 4096], summed over ranks
    return out


def time_graph(graph, steps, warmup, torch, dist, world):
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def per_layer_gemv(stack, m, torch, reps=3):
    """Average device time of one GEMV launch per layer type (graph of 36 launches
    over the 36 distinct weight sets, so every launch streams its weights from HBM),
    and the same with all 36 launches on layer 0's weights (resident in L2 after the
    first): equal times mean the kernel is not bound by DRAM."""
    from ashqk import w4a16_linear

    def graph_us(calls):
        calls[0]()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for c in calls:
                c()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
        del g
        return start.elapsed_time(end) * 1e3 / (reps * len(calls))

    res = {}
    for name, n, k in LAYERS:
        x = torch.randn(m, k, device="cuda").half()
        us = graph_us([lambda w=layer[name]: w4a16_linear(x, *w) for layer in stack])
        us_l2 = graph_us([lambda w=stack[0][name]: w4a16_linear(x, *w) for _ in stack])
        nbytes = w4a16_bytes(m, n, k, GROUP)
        res[name] = {"us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1), "l2_resident_us": round(us_l2, 2),
                     "launch": cluster_plan(m, n, k)}
    return res


DECODE_M = (1, 2, 4, 8, 16)


def decode_sweep(stack, torch, hbm_peak, reps=5):
    """M in {1, 2, 4, 8, 16} x {qkv, o, gate_up, down}. Per layer type and M, the
    mean device time of one launch in a CUDA graph of 36 launches over the 36 distinct weight sets
    (every launch streams its weights from HBM), for the W4A16 GEMV and for cuBLAS fp16 on the
    dequantised weights (x @ W_fp16, the reference's yardstick); GB/s of the algorithmic bytes and the
    fraction of the measured HBM peak for the sum of the four layers."""
    from ashqk import _ext

    def graph_us(calls):
        calls[0]()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for c in calls:
                c()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        del g
        return a.elapsed_time(b) * 1e3 / (reps * len(calls))

    from ashqk import w4a16_linear

    res = {m: {"us": [], "cublas_us": []} for m in DECODE_M}
    for name, n, k in LAYERS:
        w16 = [_ext.ops().dequantize_awq(*layer[name], torch.float16) for layer in stack]
        for m in DECODE_M:
            x = torch.randn(m, k, device="cuda").half()
            res[m]["us"].append(round(graph_us([lambda w=layer[name]: w4a16_linear(x, *w) for layer in stack]), 2))
            res[m]["cublas_us"].append(round(graph_us([lambda w=w: x @ w for w in w16]), 2))
        del w16
        torch.cuda.empty_cache()
    out = {}
    for m in DECODE_M:
        nbytes = sum(w4a16_bytes(m, n, k, GROUP) for _, n, k in LAYERS)
        gbs = nbytes / sum(res[m]["us"]) / 1e3
        out[f"m{m}"] = {"us": res[m]["us"], "cublas_us": res[m]["cublas_us"], "gbs": round(gbs, 1),
                        "frac": round(gbs / hbm_peak, 3),
                        "vs_cublas": round(sum(res[m]["cublas_us"]) / sum(res[m]["us"]), 2)}
    return out


def cluster_plan(m, n, k):
    """The cluster-split GEMV's launch shape for this layer on this device (ashqk_gemv_cluster_plan)."""
    import ctypes

    from ashqk import _ext

    class Plan(ctypes.Structure):
        _fields_ = [(f, ctypes.c_int) for f in ("tile_cols", "stage_rows", "tiles", "stages_per_tile", "cluster_ctas",
                                                "ctas", "max_stages_per_cta", "threads", "ring_stages",
                                                "stage_bytes", "smem_bytes")]

    lib = ctypes.CDLL(_ext.C_LIBRARY)
    lib.ashqk_gemv_cluster_plan.argtypes = [ctypes.c_int] * 5 + [ctypes.POINTER(Plan)]
    p = Plan()
    if lib.ashqk_gemv_cluster_plan(m, n, k, GROUP, 0, ctypes.byref(p)) != 0:
        return None
    return {"tile_cols": p.tile_cols, "cluster": p.cluster_ctas, "ctas": p.ctas,
            "stages_per_cta": p.max_stages_per_cta, "ring": p.ring_stages, "smem_kb": round(p.smem_bytes / 1024, 1)}


def cublas_fp16_stack(stack, steps, warmup, torch):
    """us per step of the same stack with fp16 weights through cuBLAS (x @ W), at M=1 and M=4.

    The yardstick the reference compares against: dequantise once (bit-exact
    kernel), then plain fp16 GEMMs, chained and graph-replayed like the W4A16 stack.
    """
    from ashqk import _ext

    deq = [{nm: _ext.ops().dequantize_awq(*layer[nm], torch.float16) for nm, _, _ in LAYERS} for layer in stack]
    res = {}
    for m in (1, 4):
        h = torch.randn(m, 4096, device="cuda").half()

        def step():
            for w in deq:
                a = h @ w["qkv"]
                b = a[:, :4096] @ w["o"]
                c = b @ w["gate_up"]
                out = c[:, :12288] @ w["down"]
            return out

        step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        res[m] = time_graph(g, max(steps // 2, 10), warmup, torch, None, 1) * 1e3
        del g
    del deq
    torch.cuda.empty_cache()
    return res


PREFILL_M = (128, 512, 2048, 8192)
PREFILL_LAYERS = (("gate_up", 24576, 4096), ("down", 4096, 12288))
TP_MLP = (("gate_up", 57344, 8192), ("down", 8192, 28672))
TP_M = (1, 16, 4096)


def random_awq(n, k, seed, device, torch):
    """Random AWQ tensors for an [K, N] layer: q, z uniform over 0..15, scales ~ U(0.002, 0.02)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (k, n // 8), dtype=torch.int32, device=device, generator=gen)
    qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (k // GROUP, n // 8), dtype=torch.int32, device=device, generator=gen)
    s = (torch.rand((k // GROUP, n), device=device, generator=gen) * 0.018 + 0.002).half()
    return qw, qz, s


def time_flushed(fn, reps, warmup, torch, flush):
    """Median CUDA-event time (us) of fn() with the L2 flushed (a 256 MB write) before every rep."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    times.sort()
    return times[len(times) // 2]


def prefill_gemm(ms, reps, warmup, torch, tensor_peak):
    """the prefill GEMM (tcgen05 kernel) on gate_up and down, TFLOP/s = 2MNK / time,
    beside cuBLAS fp16 on the dequantised weights (x @ W_fp16); SM clocks sampled over the section
    (the GEMM is compute-bound, so its throughput follows the clock)."""
    from ashqk import _ext, w4a16_linear

    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    res = {}
    with ClockSampler(torch.cuda.current_device()) as sampler:
        for j, (name, n, k) in enumerate(PREFILL_LAYERS):
            qw, qz, s = random_awq(n, k, 77 + j, "cuda", torch)
            w16 = _ext.ops().dequantize_awq(qw, qz, s, torch.float16)
            for m in ms:
                x = torch.randn(m, k, device="cuda").half()
                us = time_flushed(lambda: w4a16_linear(x, qw, qz, s), reps, warmup, torch, flush)
                us_cb = time_flushed(lambda: x @ w16, reps, warmup, torch, flush)
                tf = 2.0 * m * n * k / us / 1e6
                res[f"{name}_m{m}"] = {"us": round(us, 1), "tflops": round(tf, 1),
                                       "frac_of_peak": round(tf / tensor_peak, 3),
                                       "cublas_fp16_us": round(us_cb, 1),
                                       "cublas_fp16_tflops": round(2.0 * m * n * k / us_cb / 1e6, 1)}
                del x
            del qw, qz, s, w16
    res["clocks"] = sampler.summary()
    del flush
    torch.cuda.empty_cache()
    return res


# The reference's default benchmark model (its bench/shapes.py): Qwen3.5-9B, 32 decoder layers in a
# 3:1 pattern of linear-attention and full-attention layers (name, N, K, layer count).
QWEN35_LAYERS = (("in_proj_qkvz", 12288, 4096, 24), ("in_proj_ba", 64, 4096, 24), ("out_proj", 4096, 4096, 24),
                 ("qkv_proj", 10240, 4096, 8), ("o_proj", 4096, 4096, 8), ("gate_up_proj", 24576, 4096, 32),
                 ("down_proj", 4096, 12288, 32))


def qwen35_stack(torch, steps, warmup):
    """All linear layers of one Qwen3.5-9B token at M=1 (distinct weights per layer, one CUDA graph,
    each call fed a fixed input of its K); us/token and algorithmic GB/s."""
    from ashqk import w4a16_linear

    dev = torch.device("cuda", torch.cuda.current_device())
    layers = []
    for j, (name, n, k, count) in enumerate(QWEN35_LAYERS):
        for i in range(count):
            layers.append((n, k) + random_awq(n, k, 2000 + 100 * j + i, dev, torch))
    res = {"model": "qwen3.5-9b linear layers (random AWQ weights, G=128)",
           "launches": sum(c for *_, c in QWEN35_LAYERS),
           "reference_h200_published_us_per_token": {"m1": {"ashqk": 3325, "marlin": 1990, "fp16": 3886},
                                                     "m4": {"ashqk": 5580, "marlin": 2002, "fp16": 3899}}}
    for m in (1, 4):
        xs = {k: torch.randn(m, k, device=dev).half() for _, _, k, _ in QWEN35_LAYERS}

        def step():
            for n, k, qw, qz, s in layers:
                w4a16_linear(xs[k], qw, qz, s)

        step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        ms = time_graph(g, steps, warmup, torch, None, 1)
        nbytes = sum(w4a16_bytes(m, n, k, GROUP) for n, k, _, _, _ in layers)
        res[f"m{m}"] = {"us_per_step": round(ms * 1e3, 1), "hbm_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1)}
        del g
    del layers
    torch.cuda.empty_cache()
    return res


def marlin_compare(torch, reps=3):
    """The reference's real bar (its results/v0.2-vs-marlin-findings.md): vLLM's AWQ-Marlin
    kernel on the same B200, as a black box through vLLM's own conversion helpers. Per layer
    type: a CUDA graph of 36 launches over 36 distinct converted weight sets at M=1, like the
    per-layer GEMV timing; prefill gate_up / down at M=2048 with the L2 flushed; and the
    relative difference of Marlin's output from ours on one layer (both fp32-accumulated)."""
    try:
        from vllm import _custom_ops as vops
        from vllm.model_executor.layers.quantization.utils import marlin_utils as mu
        from vllm.scalar_type import scalar_types
    except Exception as e:  # vLLM absent or unusable here
        return {"unavailable": f"vllm import failed: {type(e).__name__}: {e}"[:300]}
    from ashqk import w4a16_linear

    dev = torch.device("cuda", torch.cuda.current_device())

    def convert(qw, qz, s, n, k):
        return (vops.awq_marlin_repack(qw, size_k=k, size_n=n, num_bits=4),
                mu.marlin_permute_scales(s, size_k=k, size_n=n, group_size=GROUP),
                mu.awq_to_marlin_zero_points(qz, size_k=k // GROUP, size_n=n, num_bits=4))

    g_idx = mu.marlin_make_empty_g_idx(dev)
    perm = mu.marlin_make_empty_g_idx(dev)
    ws = mu.marlin_make_workspace_new(dev)

    def marlin(x, w, n, k):
        return mu.apply_awq_marlin_linear(x, w[0], w[1], w[2], g_idx, perm, ws, scalar_types.uint4, n, k)

    res = {"kernel": "vLLM awq_marlin (marlin_gemm), weights converted with vLLM's helpers", "per_layer_m1_us": {}}
    try:
        for j, (name, n, k) in enumerate(LAYERS):
            sets = [convert(*random_awq(n, k, 500 + 10 * j + i, dev, torch), n, k) for i in range(N_LAYERS)]
            x = torch.randn(1, k, device=dev).half()
            marlin(x, sets[0], n, k)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for w in sets:
                    marlin(x, w, n, k)
            for _ in range(2):
                g.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(reps):
                g.replay()
            b.record()
            torch.cuda.synchronize()
            res["per_layer_m1_us"][name] = round(a.elapsed_time(b) * 1e3 / (reps * N_LAYERS), 2)
            del g, sets
        res["stack_us_per_token_est"] = round(N_LAYERS * sum(res["per_layer_m1_us"].values()), 1)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        res["prefill_m2048"] = {}
        for j, (name, n, k) in enumerate(PREFILL_LAYERS):
            qw, qz, s = random_awq(n, k, 900 + j, dev, torch)
            w = convert(qw, qz, s, n, k)
            x = torch.randn(2048, k, device=dev).half()
            us = time_flushed(lambda: marlin(x, w, n, k), 10, 3, torch, flush)
            res["prefill_m2048"][name] = {"us": round(us, 1), "tflops": round(2.0 * 2048 * n * k / us / 1e6, 1)}
            if j == 0:
                y_ref = w4a16_linear(x, qw, qz, s).float()
                y_m = marlin(x, w, n, k).float()
                res["rel_diff_vs_ours_gate_up_m2048"] = float((y_m - y_ref).norm() / y_ref.norm())
        del flush
    except Exception as e:
        res["error"] = f"{type(e).__name__}: {e}"[:300]
    torch.cuda.empty_cache()
    return res


def tp_mlp(world, rank, group, reps, warmup, torch, dist, hbm_peak, tensor_peak):
    """a large dense MLP under tensor parallelism (gate_up K=8192 N=57344
    column-parallel + NCCL all-gather; down K=28672 N=8192 row-parallel + all-reduce), per M:
    device time of the two layers with their collectives, max over ranks, and the fraction of the
    per-rank roofline -- HBM (algorithmic bytes of the rank's shards) at M <= 16, tensor (the rank's
    share of 2MNK) at M = 4096."""
    from ashqk import tp

    layers = {}
    for j, (name, n, k) in enumerate(TP_MLP):
        if name == "gate_up":
            layers[name] = random_awq(n // world, k, 300 + 10 * rank + j, "cuda", torch)
        else:
            layers[name] = random_awq(n, k // world, 300 + 10 * rank + j, "cuda", torch)
    res = {}
    for m in TP_M:
        x = torch.randn(m, TP_MLP[0][2], device="cuda").half()
        xd = torch.randn(m, TP_MLP[1][2] // world, device="cuda").half()

        def step():
            tp.column_parallel_linear(x, *layers["gate_up"], group=group)
            tp.row_parallel_linear(xd, *layers["down"], group=group)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            step()
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / reps
        if world > 1:
            t = torch.tensor([us], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        flops = sum(2.0 * m * n * k for _, n, k in TP_MLP)
        rank_bytes = (w4a16_bytes(m, TP_MLP[0][1] // world, TP_MLP[0][2], GROUP) +
                      w4a16_bytes(m, TP_MLP[1][1], TP_MLP[1][2] // world, GROUP))
        entry = {"us": round(us, 1), "tflops_total": round(flops / us / 1e6, 1)}
        if m <= 16:
            gbs = rank_bytes / us / 1e3
            entry.update(bound="hbm", gbs_per_rank=round(gbs, 1), frac=round(gbs / hbm_peak, 3))
        else:
            tf = flops / world / us / 1e6
            entry.update(bound="tensor", tflops_per_rank=round(tf, 1), frac=round(tf / tensor_peak, 3))
        res[f"m{m}"] = entry
    del layers
    torch.cuda.empty_cache()
    return res


def run_gpu(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
        group = dist.group.WORLD
    warmup = max(args.warmup, 3)

    from ashqk import w4a16_linear  # noqa: F401  (loads the extension)

    hbm_peak, peak_kind = load_peaks()
    tensor_peak, tensor_kind = load_tensor_peak()
    if args.only == "prefill":  # profiling runs of the prefill GEMM alone
        res = prefill_gemm(args.prefill_m or PREFILL_M, args.steps, warmup, torch, tensor_peak)
        if rank == 0:
            print(json.dumps({"prefill": res}), flush=True)
        return
    stack = make_stack(world, rank, device, args.layers)
    # Tensor-parallel reductions: the NVLink low-latency-line all-reduce by default up to 4 ranks
    # (fastest on B200: tp2 1272 us/token against 1405 fused, 1471 one-shot p2p and 1828 NCCL; tp4
    # 1243 against 1830 NCCL), NCCL beyond (the line protocol has not run on 8 GPUs here);
    # ASHQK_TP_ALLREDUCE=nccl, =ll, =p2p (one-shot) or =fused (the row-parallel GEMV and its
    # all-reduce as one kernel, low-latency lines) selects one.
    p2p = None
    tp_reduce = os.environ.get("ASHQK_TP_ALLREDUCE", default_tp_allreduce(world))
    if tp_reduce not in ("nccl", "p2p", "ll", "fused"):
        raise SystemExit(f"ASHQK_TP_ALLREDUCE={tp_reduce!r}: expected nccl, p2p, ll or fused")
    fused = world > 1 and tp_reduce == "fused"
    if world > 1 and tp_reduce in ("p2p", "ll", "fused"):
        from ashqk import tp

        p2p = tp.P2PAllReduce(group=group, max_elems=4 * 4096, protocol="oneshot" if tp_reduce == "p2p" else "ll")
    results = {}
    graphs = {}
    for m in (1, 4):
        h = torch.randn(m, 4096, device=device).half()
        stack_step(stack, h, world, group, p2p, fused)  # warm-up outside capture (workspaces, NCCL comms)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = stack_step(stack, h, world, group, p2p, fused)
        graphs[m] = (g, h, out)
        del g  # the dict holds the only reference (graphs with NCCL calls must be freed before teardown)

    g1, h1, out1 = graphs[1]
    with ClockSampler(local) as clocks:
        ms1 = time_graph(g1, args.steps, warmup, torch, dist, world)
    ms4 = time_graph(graphs[4][0], max(args.steps // 2, 1), warmup, torch, dist, world)

    # End to end through the public API: pinned host input in, result out, every step.
    h_host = torch.randn(1, 4096).half().pin_memory()
    y_host = torch.empty(out1.shape, dtype=out1.dtype).pin_memory()
    for _ in range(warmup):
        h1.copy_(h_host, non_blocking=True)
        g1.replay()
        y_host.copy_(out1, non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        h1.copy_(h_host, non_blocking=True)
        g1.replay()
        y_host.copy_(out1, non_blocking=True)
    end.record()
    torch.cuda.synchronize()
    e2e_ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    d2h_bytes = int(out1.numel()) * out1.element_size()
    layer_bw = per_layer_gemv(stack, 1, torch) if world == 1 else None
    sweep = decode_sweep(stack, torch, hbm_peak) if world == 1 and args.only == "all" else None
    cublas_us = cublas_fp16_stack(stack, args.steps, warmup, torch) if world == 1 else None
    n_layers = len(stack)
    del stack
    torch.cuda.empty_cache()
    prefill = prefill_gemm(PREFILL_M, 10, warmup, torch, tensor_peak) if world == 1 and args.only == "all" else None
    tp_res = (tp_mlp(world, rank, group, 10, warmup, torch, dist, hbm_peak, tensor_peak)
              if args.only == "all" else None)
    q35 = qwen35_stack(torch, max(args.steps // 2, 10), warmup) if world == 1 and args.only == "all" else None
    marlin_res = marlin_compare(torch) if world == 1 and args.only == "all" and not args.no_marlin else None

    # Every CUDA graph that captured NCCL calls is released before the process
    # group is destroyed; a live one makes destroy_process_group wait forever.
    del g1, h1, out1
    graphs.clear()
    torch.cuda.synchronize()
    if p2p is not None:
        p2p.check()  # a timed-out peer wait would have made the timed calls no-ops
        p2p.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    per_rank_bytes = sum(w4a16_bytes(1, n // (world if nm in ("qkv", "gate_up") else 1),
                                     k // (world if nm in ("o", "down") else 1), GROUP)
                         for nm, n, k in LAYERS) * n_layers
    stack_gbs = per_rank_bytes / (ms1 * 1e-3) / 1e9
    # The one JSON line (stdout) stays short (~1.5 KB) and ends with the figures a reader of the log's
    # tail needs (cuBLAS and prefill comparisons, the M=4 step); the detail (launch shapes, per-layer
    # and per-shape breakdowns, Marlin and Qwen3.5 figures) goes to stderr.
    line = {
        "metric": METRIC, "value": round(ms1 * 1e3, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": warmup, "ms_per_step": round(ms1, 4), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16 x int4 (AWQ), fp32 accumulate", "data": "synthetic",
        "config": workload_config(world, n_layers),
        "stack_hbm_frac": round(stack_gbs / hbm_peak, 3),
        "gpu_launches": args.steps * len(LAYERS) * n_layers,
        "clocks": clocks.summary(),
        "e2e": {"value": round(e2e_ms * 1e3, 1), "unit": UNIT, "h2d_bytes_per_step": 4096 * 2,
                "d2h_bytes_per_step": d2h_bytes},
    }
    detail = {"device": {"name": torch.cuda.get_device_name(device),
                         "sm_count": torch.cuda.get_device_properties(device).multi_processor_count},
              "stack_hbm_gbs_per_gpu": round(stack_gbs, 1),
              "e2e_how": "pinned H2D of the hidden state + graph replay of the 144 w4a16_linear calls + D2H "
                         "of the output, every step, CUDA events"}
    if tp_res is not None:
        detail["tp_mlp"] = tp_res
        line["tp_mlp"] = {k: [v["us"], v["frac"]] for k, v in tp_res.items()}
    if q35 is not None:
        detail["qwen35_9b_stack"] = q35
        line["qwen35_9b_us"] = [q35["m1"]["us_per_step"], q35["m4"]["us_per_step"]]
    if marlin_res is not None:
        detail["marlin_vllm"] = marlin_res
        if "stack_us_per_token_est" in marlin_res:
            line["marlin_vllm_us"] = marlin_res["stack_us_per_token_est"]
    if layer_bw is not None and args.cpu_seconds > 0:
        value, threads, desc, _ = cpu_reference_sample(1000, 1, budget_s=args.cpu_seconds)
        detail["cpu_baseline_sample"] = desc
        line["cpu_baseline"] = {"value": round(value, 1), "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": "one decoder layer's 4 calls at M=1 via the C port of ref.py, x36"}
    if layer_bw is not None:
        tot_bytes = sum(w4a16_bytes(1, n, k, GROUP) for _, n, k in LAYERS)
        tot_us = sum(layer_bw[nm]["us"] for nm, _, _ in LAYERS)
        achieved = tot_bytes / tot_us / 1e3
        detail["per_layer_gemv"] = layer_bw
        detail["roofline_detail"] = {"algorithmic_bytes": tot_bytes, "peak_kind": peak_kind,
                                     "per_layer_us": [layer_bw[nm]["us"] for nm, _, _ in LAYERS],
                                     "kernel": "gemv_cluster_kernel, M=1, one launch of each layer type"}
        line["roofline"] = {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 3), "traffic": load_traffic(), "kernel": "gemv_cluster_kernel",
        }
    if sweep is not None:
        detail["decode_sweep"] = sweep
        line["decode_sweep"] = {k: [round(sum(v["us"]), 1), v["vs_cublas"], v["frac"]] for k, v in sweep.items()}
    if prefill is not None:
        detail["prefill_gemm"] = prefill
        line["prefill_gemm"] = {"m": list(PREFILL_M)}
        for nm, _, _ in PREFILL_LAYERS:
            line["prefill_gemm"][f"{nm}_frac"] = [prefill[f"{nm}_m{m}"]["frac_of_peak"] for m in PREFILL_M]
            line["prefill_gemm"][f"{nm}_cublas_frac"] = [
                round(prefill[f"{nm}_m{m}"]["cublas_fp16_tflops"] / tensor_peak, 3) for m in PREFILL_M]
    if cublas_us is not None:
        line["cublas_fp16"] = {
            "us_per_token": round(cublas_us[1], 1), "m4_us_per_step": round(cublas_us[4], 1),
            "speedup_m1": round(cublas_us[1] / (ms1 * 1e3), 2), "speedup_m4": round(cublas_us[4] / (ms4 * 1e3), 2)}
        detail["cublas_fp16_how"] = ("x @ W_fp16 (torch.matmul -> cuBLAS) on the dequantised weights of the same "
                                     "stack, same chaining, CUDA graph, CUDA events")
    line["m4_us_per_token"] = round(ms4 * 1e3 / 4, 1)
    line["m4_us_per_step"] = round(ms4 * 1e3, 1)
    print(json.dumps(detail), file=sys.stderr, flush=True)
    print(json.dumps(line), flush=True)


def load_tensor_peak():
    """Dense fp16/bf16 tensor peak (TFLOP/s): the measured burst cuBLAS figure, else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def load_traffic():
    """DRAM bytes (read + write) of one launch of each layer type at M=1, summed,
    from the committed ncu capture summary, if one exists."""
    path = os.path.join(ROOT, "profiles", "gemv_decode_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_layer_set")
    except Exception:
        return None


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="budget of the CPU baseline sample (0 skips it)")
    ap.add_argument("--only", choices=["all", "decode", "prefill"], default="all",
                    help="decode: the decode stack alone; prefill: only the prefill GEMM (profiling runs)")
    ap.add_argument("--prefill-m", type=int, nargs="*", default=None, help="M values for --only prefill")
    ap.add_argument("--no-marlin", action="store_true", help="skip the vLLM Marlin comparison")
    ap.add_argument("--no-torch-ref", action="store_true",
                    help="reference arm: skip the torch timing of ashqk/ref.py beside the C port")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="decoder layers in the stack (36 is the benchmark; fewer for profiling runs)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
