"""bench.py's measurement helpers and its CPU reference arm (no GPU needed)."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    sys.path.insert(0, ROOT)
    import bench

    return bench


def test_bytes_model_matches_the_worked_figures():
    """The reference's bytes model (bench/bench_gemm.py:45-46 there): M*K*2 + K*N/2 + (K/G)*N*2.5 + M*N*2."""
    b = _bench()
    assert b.w4a16_bytes(1, 6144, 4096, 128) == 1 * 4096 * 2 + 4096 * 6144 // 2 + 32 * 6144 * 2 + 32 * 6144 // 2 + 6144 * 2
    mb = {name: b.w4a16_bytes(1, n, k, 128) / 1e6 for name, n, k in b.LAYERS}
    assert round(mb["qkv"], 2) == 13.09 and round(mb["o"], 2) == 8.73
    assert round(mb["gate_up"], 2) == 52.36 and round(mb["down"], 2) == 26.18
    stack = 36 * sum(b.w4a16_bytes(1, n, k, 128) for _, n, k in b.LAYERS)
    assert abs(stack / 1e9 - 3.613) < 0.001  # the 36-layer stack moves 3.613 GB per token


def test_workload_config_names_the_baseline_config():
    b = _bench()
    cfg = b.workload_config(1)
    assert "config 3" in cfg["workload"] and cfg["parallelism"] == "none"
    assert b.workload_config(4)["parallelism"] == "tp4"
    assert b.workload_config(1, 2)["decoder_layers"] == 2


def test_multi_gpu_default_reduction():
    """The low-latency NVLink all-reduce where it has run on this pool's boxes (2 and 4 ranks), NCCL
    beyond; the workload config echoes the choice."""
    b = _bench()
    assert [b.default_tp_allreduce(n) for n in (2, 4, 8)] == ["ll", "ll", "nccl"]
    if "ASHQK_TP_ALLREDUCE" not in os.environ:
        assert b.workload_config(2)["tp_allreduce"] == "ll" and b.workload_config(8)["tp_allreduce"] == "nccl"
        assert b.workload_config(1)["tp_allreduce"] is None


def test_qwen35_shapes_are_the_references():
    b = _bench()
    names = {n: (nn, k, c) for n, nn, k, c in b.QWEN35_LAYERS}
    assert names["in_proj_ba"] == (64, 4096, 24) and names["qkv_proj"] == (10240, 4096, 8)
    assert sum(c for *_, c in b.QWEN35_LAYERS) == 152


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_build", "libawq_oracle.so")),
                    reason="C oracle not built")
def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "us/token" and line["higher_is_better"] is False
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
