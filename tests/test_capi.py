"""The C-ABI library (include/ashqk_b200.h) loads and exports every declared symbol.

CPU-only: no call here launches a kernel. Argument validation that happens
before any CUDA call is checked through ctypes.
"""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ashqk_b200.h")
LIB = os.path.join(ROOT, "ash-quant-kernels_b200", "ashqk", "libashqk_b200.so")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"ASHQK_API\s+[\w\s\*]+?\b(ashqk_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} not built; run python ash-quant-kernels_b200/build.py")
    return ctypes.CDLL(LIB)


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("ashqk_w4a16_linear", "ashqk_w4a16_gemv", "ashqk_w4a16_gemm", "ashqk_dequantize_awq_f16",
                     "ashqk_dequantize_awq_f32", "ashqk_status_string"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings_and_version(lib):
    lib.ashqk_status_string.restype = ctypes.c_char_p
    lib.ashqk_version.restype = ctypes.c_char_p
    assert lib.ashqk_status_string(0) == b"ok"
    assert b"invalid" in lib.ashqk_status_string(1)
    assert b"unknown" in lib.ashqk_status_string(999)
    assert re.fullmatch(rb"\d+\.\d+\.\d+", lib.ashqk_version())
    assert lib.ashqk_gemv_max_m() == 16


def test_invalid_arguments_rejected_before_launch(lib):
    f = lib.ashqk_w4a16_linear
    vp, i64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    f.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, i64, ci, ci, ci, ci, vp, ctypes.c_size_t, vp]
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
    # null x
    assert f(None, 256, fake, 8, fake, 8, fake, 64, fake, 64, 1, 64, 256, 128, None, 0, None) == 1
    # N not a multiple of 8
    assert f(fake, 256, fake, 8, fake, 8, fake, 60, fake, 60, 1, 60, 256, 128, None, 0, None) == 1
    # K not a multiple of the group size
    assert f(fake, 250, fake, 8, fake, 8, fake, 64, fake, 64, 1, 64, 250, 128, None, 0, None) == 1
    # leading dimension smaller than the row
    assert f(fake, 100, fake, 8, fake, 8, fake, 64, fake, 64, 1, 64, 256, 128, None, 0, None) == 1
    sz = ctypes.c_size_t(0)
    assert lib.ashqk_linear_workspace_size(1, 60, 256, 128, ctypes.byref(sz)) == 1


def test_kernel_switches_validate_their_argument(lib):
    """Test and tuning switches: out-of-range choices are refused, valid ones accepted (no GPU touched)."""
    for which in (0, 1, 2, 3, 4):
        assert lib.ashqk_set_gemv_kernel(which) == 0
    assert lib.ashqk_set_gemv_kernel(5) == 1 and lib.ashqk_set_gemv_kernel(-1) == 1
    assert lib.ashqk_gemv_set_tuning(0, 0, 0, 0) == 0 and lib.ashqk_gemv_set_tuning(96, 3, 512, 140) == 0
    assert lib.ashqk_gemv_set_tuning(-1, 0, 0, 0) == 1 and lib.ashqk_gemv_set_tuning(0, 17, 0, 0) == 1
    assert lib.ashqk_gemv_set_tuning(0, 0, 128, 0) == 1 and lib.ashqk_gemv_set_tuning(0, 0, 0, -1) == 1
    assert lib.ashqk_gemv_set_tuning(0, 0, 0, 0) == 0
    for which in (0, 1, 2, 3, 4):
        assert lib.ashqk_set_gemm_kernel(which) == 0
    assert lib.ashqk_set_gemm_kernel(5) == 1 and lib.ashqk_set_gemm_kernel(-1) == 1
    assert lib.ashqk_set_gemv_kernel(0) == 0 and lib.ashqk_set_gemm_kernel(0) == 0


def test_workspace_size_queries(lib):
    """Malformed problems are refused before the device is consulted; a well-formed query needs the
    GPU's SM count, so without a B200 it reports ASHQK_ERR_NO_DEVICE (5), never a size."""
    sz = ctypes.c_size_t(123)
    lib.ashqk_gemm_workspace_size.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_size_t)]
    assert lib.ashqk_gemm_workspace_size(0, 24576, 4096, 128, ctypes.byref(sz)) == 1
    assert lib.ashqk_gemm_workspace_size(16, 24576, 4000, 128, ctypes.byref(sz)) == 1
    lib.ashqk_gemv_workspace_size.argtypes = [ctypes.c_int] * 5 + [ctypes.POINTER(ctypes.c_size_t)]
    assert lib.ashqk_gemv_workspace_size(1, 6140, 4096, 128, 0, ctypes.byref(sz)) == 1  # N % 8 != 0
    import torch

    if not torch.cuda.is_available():
        assert lib.ashqk_gemm_workspace_size(2048, 24576, 4096, 128, ctypes.byref(sz)) == 5
        assert lib.ashqk_gemv_workspace_size(1, 6144, 4096, 128, 0, ctypes.byref(sz)) == 5


class StripPlan(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in ("grid_x", "grid_y", "threads", "consumer_warps", "ring_stages",
                                                 "stages_total", "stage_bytes", "smem_bytes")]


def _strip_plan(lib, m, n, k, g, sms):
    lib.ashqk_gemv_strip_plan.argtypes = [ctypes.c_int] * 5 + [ctypes.POINTER(StripPlan)]
    p = StripPlan()
    return lib.ashqk_gemv_strip_plan(m, n, k, g, sms, ctypes.byref(p)), p


# Qwen3-8B decode layers, the config-5 TP shards, Qwen3.5 skinny layers, and small / ragged ones.
_SHAPES = [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288), (57344 // 8, 8192), (8192, 28672 // 8),
           (64, 4096), (96, 4096), (160, 256), (32, 128), (4096, 128), (28672, 8192)]


@pytest.mark.parametrize("sms", [148, 132, 8])
def test_strip_plan_invariants(lib, sms):
    """The column-strip GEMV's launch plan, over decode shapes and every M it takes: the shared
    memory fits one CTA of an SM (225 KB dynamic), every CTA of the grid is resident at once
    (unless even one-stage rings cannot make that so, which only an 8-SM part reaches),
    ring slots hold whole stages, the warp count matches a compiled variant, and a K split is a
    cluster of at most 4 CTAs that each own at least one stage."""
    for n, k in _SHAPES:
        for g in (32, 64, 128):
            if k % g:
                continue
            for m in range(1, 17):
                rc, p = _strip_plan(lib, m, n, k, g, sms)
                assert rc == 0, (m, n, k, g, rc)
                where = (m, n, k, g, sms)
                assert p.grid_x == -(-n // 64) and p.stages_total == -(-k // 256), where
                assert 1 <= p.grid_y <= 4 and p.grid_y <= p.stages_total, where
                assert p.consumer_warps in ((4, 8, 16) if m <= 8 else (4, 8)), where
                assert p.threads == 32 * (p.consumer_warps + 1) <= 1024, where
                assert 1 <= p.ring_stages <= 24, where
                assert p.ring_stages <= -(-p.stages_total // p.grid_y), where  # no idle slot
                assert p.stage_bytes % 128 == 0 and p.ring_stages * p.stage_bytes + 1024 <= p.smem_bytes, where
                assert p.smem_bytes <= 225 * 1024, where
                per_sm = -(-(p.grid_x * p.grid_y) // sms)
                if p.ring_stages > 1:  # a one-stage ring is the floor; below it CTAs take turns
                    assert per_sm * (p.smem_bytes + 1024) <= 228 * 1024, where
                # more consumer warps than slots only at the 4-warp floor (the extra warps idle)
                assert p.consumer_warps <= max(p.ring_stages, 4), where


def test_strip_plan_rejects(lib):
    assert _strip_plan(lib, 17, 4096, 4096, 128, 148)[0] == 2     # M > 16: the chunked path
    assert _strip_plan(lib, 1, 4104, 4096, 128, 148)[0] == 2      # N % 32
    assert _strip_plan(lib, 1, 4096, 4096, 8, 148)[0] == 2        # G % 16
    assert _strip_plan(lib, 1, 4096, 4000, 128, 148)[0] == 1      # K % G
    assert _strip_plan(lib, 0, 4096, 4096, 128, 148)[0] == 1
    assert _strip_plan(lib, 1, 4096, 4096, 128, -1)[0] == 1
    import torch

    if not torch.cuda.is_available():
        assert _strip_plan(lib, 1, 4096, 4096, 128, 0)[0] == 5      # SM count of a missing device


def test_strip_plan_of_the_measured_layers(lib):
    """At M=1 on 148 SMs the planner picks the launch shapes the committed strip-GEMV profile
    measured for the Qwen3-8B layers (grid, cluster split, warps per CTA)."""
    want = {(6144, 4096): (96, 1, 544), (4096, 4096): (64, 2, 288), (24576, 4096): (384, 1, 160),
            (4096, 12288): (64, 4, 288)}
    for (n, k), (gx, gy, threads) in want.items():
        rc, p = _strip_plan(lib, 1, n, k, 128, 148)
        assert rc == 0 and (p.grid_x, p.grid_y, p.threads) == (gx, gy, threads), (n, k, p.grid_x, p.grid_y, p.threads)


def test_fused_epilogue_covers_every_pair_once(lib):
    """The fused row-parallel epilogue: CTA (strip, r) of a K-split cluster of S exchanges the pairs
    of columns [((r * 32) // S) * 2, (((r + 1) * 32) // S) * 2) of its 64-column strip, for every
    token. Over the planner's grids for the tensor-parallel decode shards, the CTAs' pairs cover
    y [M, N] exactly once and every line index lies inside the inbox of M * N / 2 pairs."""
    for n, k in [(4096, 2048), (4096, 6144), (4096, 512), (4096, 1024), (8192, 3584), (96, 1024)]:
        for m in (1, 4, 16):
            rc, p = _strip_plan(lib, m, n, k, 128, 148)
            assert rc == 0
            seen = {}
            for strip in range(p.grid_x):
                for r in range(p.grid_y):
                    lo, hi = (r * 32) // p.grid_y * 2, ((r + 1) * 32) // p.grid_y * 2
                    for tok in range(m):
                        for c in range(lo, hi, 2):
                            col = strip * 64 + c
                            if col >= n:
                                continue
                            pair = tok * (n // 2) + col // 2
                            assert pair not in seen, (n, k, m, strip, r, c)
                            seen[pair] = (strip, r)
            assert sorted(seen) == list(range(m * n // 2)), (n, k, m)


def test_p2p_entry_points_validate_before_the_device(lib):
    """The NVLink all-reduce and fused row-parallel entry points refuse malformed calls before any
    CUDA call (fake pointers are never dereferenced); a well-formed fused call needs the device."""
    vp, i64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    fake, regions = ctypes.c_void_p(0x10000), ctypes.c_void_p(0x20000)
    size = ctypes.c_size_t(0)
    lib.ashqk_p2p_region_bytes.argtypes = [i64, ctypes.POINTER(ctypes.c_size_t)]
    lib.ashqk_p2p_ll_region_bytes.argtypes = [i64, ctypes.POINTER(ctypes.c_size_t)]
    assert lib.ashqk_p2p_region_bytes(12, ctypes.byref(size)) == 1            # not a multiple of 8
    assert lib.ashqk_p2p_ll_region_bytes(1 << 17, ctypes.byref(size)) == 1    # above 65536
    assert lib.ashqk_p2p_ll_region_bytes(1 << 16, ctypes.byref(size)) == 0
    assert size.value == 256 + 2 * 8 * (1 << 15) * 8
    for name in ("ashqk_allreduce_f16_oneshot", "ashqk_allreduce_f16_ll"):
        f = getattr(lib, name)
        f.argtypes = [vp, vp, i64, vp, ci, ci, i64, vp]
        assert f(fake, fake, 1024, None, 0, 2, 4096, None) == 1               # no region array
        assert f(fake, fake, 1020, regions, 0, 2, 4096, None) == 1            # n % 8
        assert f(fake, fake, 8192, regions, 0, 2, 4096, None) == 1            # n > max_elems
        assert f(fake, fake, 1024, regions, 2, 2, 4096, None) == 1            # rank outside world
        assert f(fake, fake, 1024, regions, 0, 9, 4096, None) == 1            # more than 8 ranks
        assert f(ctypes.c_void_p(0x10002), fake, 1024, regions, 0, 2, 4096, None) == 1  # misaligned
    g = lib.ashqk_w4a16_gemv_allreduce
    g.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, i64, ci, ci, ci, ci, vp, ci, ci, i64, vp]
    ok = (fake, 2048, fake, 512, fake, 512, fake, 4096, fake, 4096, 1, 4096, 2048, 128)
    assert g(*ok, None, 0, 2, 1 << 16, None) == 1                             # no region array
    assert g(*ok, regions, 0, 2, 2048, None) == 1                             # M * N > max_elems
    assert g(*ok, regions, 3, 2, 1 << 16, None) == 1                          # rank outside world
    bad_n = (fake, 2048, fake, 5, fake, 5, fake, 40, fake, 40, 1, 40, 2048, 128)
    assert g(*bad_n, regions, 0, 2, 1 << 16, None) == 2                       # N % 32: not the strip kernel
    import torch

    if not torch.cuda.is_available():
        assert g(*ok, regions, 0, 2, 1 << 16, None) == 5                      # needs the device's SM count


@pytest.mark.parametrize("lang,std", [("c", "-std=c99"), ("c++", "-std=c++11")])
def test_header_compiles_standalone(lang, std, tmp_path):
    """The C ABI header is self-contained plain C (and valid C++): no CUDA or torch headers needed."""
    import shutil
    import subprocess

    cc = shutil.which("gcc" if lang == "c" else "g++")
    if cc is None:
        pytest.skip("no host compiler")
    src = tmp_path / ("use." + ("c" if lang == "c" else "cpp"))
    src.write_text('#include "ashqk_b200.h"\nint main(void) { ashqk_strip_plan p; (void)p; '
                   'return ashqk_version() == 0; }\n')
    r = subprocess.run([cc, std, "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-I", os.path.dirname(HEADER),
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


class ClusterPlan(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in ("tile_cols", "stage_rows", "tiles", "stages_per_tile", "cluster_ctas",
                                                 "ctas", "max_stages_per_cta", "threads", "ring_stages",
                                                 "stage_bytes", "smem_bytes")]


def _cluster_plan(lib, m, n, k, g, sms):
    lib.ashqk_gemv_cluster_plan.argtypes = [ctypes.c_int] * 5 + [ctypes.POINTER(ClusterPlan)]
    p = ClusterPlan()
    return lib.ashqk_gemv_cluster_plan(m, n, k, g, sms, ctypes.byref(p)), p


@pytest.mark.parametrize("sms", [148, 132, 16])
def test_cluster_plan_invariants(lib, sms):
    """The cluster-split GEMV's plan over decode shapes and every M: 32 KB of packed weights per stage,
    clusters of at most 16 CTAs, at most ~1.65 CTAs per SM for M <= 8 (~0.65 for M > 8) unless the
    tiles alone exceed that, two CTAs' shared memory within an SM for M <= 8 at the BASELINE group size
    (smaller groups may need one CTA's worth for their scale / zero rows), a ring of at least two
    stages when a CTA has two, and the busiest CTA's stages the even share of its tile."""
    for n, k in _SHAPES:
        for g in (32, 64, 128):
            if k % g:
                continue
            for m in range(1, 17):
                rc, p = _cluster_plan(lib, m, n, k, g, sms)
                where = (m, n, k, g, sms)
                if g < 128 and rc == 2:
                    # A CTA keeps the scale / zero rows of its whole K range in shared memory; deep
                    # layers with small groups on few CTAs do not fit and take the column-strip kernel.
                    assert k >= 8192 and (m > 8 or sms < 100), where
                    continue
                assert rc == 0, where
                assert p.tile_cols in (256, 512) and p.tile_cols * p.stage_rows // 2 == 32768, where
                assert p.tiles == -(-n // p.tile_cols) and p.stages_per_tile == -(-k // p.stage_rows), where
                assert 1 <= p.cluster_ctas <= min(16, p.stages_per_tile), where
                assert p.ctas == p.tiles * p.cluster_ctas, where
                cap = sms * 33 // 20 if m <= 8 else sms * 13 // 20
                assert p.ctas <= cap or p.cluster_ctas == 1, where
                assert p.max_stages_per_cta == -(-p.stages_per_tile // p.cluster_ctas), where
                assert p.threads == 288 and 1 <= p.ring_stages <= min(8, p.max_stages_per_cta), where
                assert p.ring_stages >= 2 or p.max_stages_per_cta == 1, where
                assert p.stage_bytes % 1024 == 0 and p.ring_stages * p.stage_bytes + 1024 <= p.smem_bytes, where
                assert p.smem_bytes <= 201 * 1024, where
                if m <= 8 and g == 128:
                    assert 2 * (p.smem_bytes + 516 + 1024) <= 228 * 1024, where


def test_cluster_plan_rejects(lib):
    assert _cluster_plan(lib, 17, 4096, 4096, 128, 148)[0] == 2
    assert _cluster_plan(lib, 1, 4104, 4096, 128, 148)[0] == 2
    assert _cluster_plan(lib, 1, 4096, 4096, 8, 148)[0] == 2
    assert _cluster_plan(lib, 1, 4096, 4000, 128, 148)[0] == 1
    assert _cluster_plan(lib, 0, 4096, 4096, 128, 148)[0] == 1
