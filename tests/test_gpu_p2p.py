"""One-shot NVLink all-reduce kernel (``ashqk_allreduce_f16_oneshot``) on ONE GPU, with the host
playing the peer rank: the peer's region is a second local buffer whose slot and flag the test
writes before the call, so no kernel ever waits on another kernel. Checks the epoch/slot protocol,
the fp32 rank-order sum, what the kernel publishes to the peer, and the bounded wait: a flag that
nothing sets makes the kernel give up after about 2 s with the peer bit in the device error word,
and later calls return at once until the bit is cleared. The real multi-GPU exchange is covered by
``test_gpu_tp.py::test_p2p_allreduce``."""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

HEADER = 256
PEER_BIT = 4


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from ashqk import _ext

    lib = ctypes.CDLL(_ext.C_LIBRARY)
    vp = ctypes.c_void_p
    lib.ashqk_p2p_region_bytes.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_size_t)]
    lib.ashqk_allreduce_f16_oneshot.argtypes = [vp, vp, ctypes.c_int64, vp, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int64, vp]
    lib.ashqk_get_device_errors.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
    lib.ashqk_p2p_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
    lib.ashqk_p2p_free.argtypes = [vp]
    return lib


def _errors(lib, clear=False):
    bits = ctypes.c_uint(0)
    assert lib.ashqk_get_device_errors(ctypes.byref(bits), int(clear)) == 0
    return bits.value


class _TwoRegions:
    """Rank 0's region and the host-played rank 1's region, both on this GPU."""

    def __init__(self, lib, max_elems):
        size = ctypes.c_size_t(0)
        assert lib.ashqk_p2p_region_bytes(max_elems, ctypes.byref(size)) == 0
        self.max_elems, self.size = max_elems, size.value
        self.slot_bytes = (self.size - HEADER) // 2
        self.r = [torch.zeros(self.size, dtype=torch.uint8, device="cuda") for _ in range(2)]
        self.ptrs = torch.tensor([t.data_ptr() for t in self.r], dtype=torch.int64, device="cuda")

    def flags(self, q):
        return self.r[q][64:96].view(torch.int32)

    def epoch(self, q):
        return int(self.r[q][0:4].view(torch.int32)[0])

    def slot(self, q, parity, n):
        off = HEADER + parity * self.slot_bytes
        return self.r[q][off:off + 2 * n].view(torch.float16)


def _call(lib, regs, x, out, rank=0, world=2):
    return lib.ashqk_allreduce_f16_oneshot(x.data_ptr(), out.data_ptr(), x.numel(), regs.ptrs.data_ptr(), rank,
                                           world, regs.max_elems, torch.cuda.current_stream().cuda_stream)


def test_protocol_and_sum(lib):
    assert _errors(lib, clear=True) & PEER_BIT == 0
    regs = _TwoRegions(lib, 1 << 14)
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    for epoch, shape in enumerate([(4, 4096), (1, 4096), (16, 1024), (2, 8)], start=1):
        n = shape[0] * shape[1]
        a = (torch.randn(shape, device="cuda", generator=g) * 2).half()
        b = (torch.randn(shape, device="cuda", generator=g) * 2).half()
        regs.slot(1, epoch & 1, n).copy_(b.view(-1))      # the peer's partial ...
        regs.flags(0)[1] = epoch                           # ... and its arrival
        out = torch.full_like(a, float("nan"))
        assert _call(lib, regs, a, out) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, (a.float() + b.float()).half()), epoch
        assert regs.epoch(0) == epoch
        assert int(regs.flags(1)[0]) == epoch             # published to the peer
        assert torch.equal(regs.slot(0, epoch & 1, n), a.view(-1))
    # in place, world = 1 (no peers, a copy through the slot)
    a = torch.randn(8, 512, device="cuda", generator=g).half()
    ref = a.clone()
    assert _call(lib, regs, a, a, world=1) == 0
    torch.cuda.synchronize()
    assert torch.equal(a, ref)
    assert _errors(lib) & PEER_BIT == 0


def test_rejects_bad_arguments(lib):
    regs = _TwoRegions(lib, 1024)
    a = torch.zeros(1024, dtype=torch.float16, device="cuda")
    out = torch.empty_like(a)
    bad = [
        dict(x=a[:12], out=out[:12]),                     # not a multiple of 8
        dict(x=a[1:9], out=out[:8]),                       # misaligned input
        dict(x=torch.zeros(2048, dtype=torch.float16, device="cuda"), out=torch.empty(2048, dtype=torch.float16,
                                                                                    device="cuda")),  # > max
        dict(x=a, out=out, rank=2),                        # rank outside world
        dict(x=a, out=out, world=9),                       # more ranks than supported
    ]
    for kw in bad:
        assert _call(lib, regs, **kw) == 1, kw
    p = ctypes.c_void_p()
    assert lib.ashqk_p2p_alloc(4096, ctypes.byref(p)) == 0 and p.value
    assert lib.ashqk_p2p_free(p) == 0


def test_missing_peer_times_out(lib):
    regs = _TwoRegions(lib, 1024)
    a = torch.ones(1024, dtype=torch.float16, device="cuda")
    out = torch.full_like(a, -7.0)
    _errors(lib, clear=True)
    mirror = torch.zeros(1, dtype=torch.int32).pin_memory()  # host copy of the error word
    lib.ashqk_set_error_mirror.argtypes = [ctypes.c_void_p]
    assert lib.ashqk_set_error_mirror(mirror.data_ptr()) == 0
    t0 = time.time()
    assert _call(lib, regs, a, out) == 0                   # nothing ever sets the peer's flag
    while int(mirror[0]) == 0 and time.time() - t0 < 30:  # seen on the host without a synchronisation
        time.sleep(0.01)
    torch.cuda.synchronize()
    waited = time.time() - t0
    try:
        assert int(mirror[0]) & PEER_BIT
        assert _errors(lib) & PEER_BIT
        assert 0.5 < waited < 30, waited
        assert bool((out == -7.0).all())                   # output left unwritten
        # sticky: the next call returns at once and does nothing
        regs.flags(0)[1] = 2
        t0 = time.time()
        assert _call(lib, regs, a, out) == 0
        torch.cuda.synchronize()
        assert time.time() - t0 < 0.5
        assert regs.epoch(0) == 1 and bool((out == -7.0).all())
    finally:
        _errors(lib, clear=True)
        assert lib.ashqk_set_error_mirror(None) == 0
    # cleared: the kernel runs again (the peer's flag now covers epoch 2)
    regs.slot(1, 0, 1024).fill_(3.0)
    assert _call(lib, regs, a, out) == 0
    torch.cuda.synchronize()
    assert bool((out == 4.0).all()) and _errors(lib) == 0


# ---- low-latency variant (ashqk_allreduce_f16_ll) -----------------------------------------------
MAX_RANKS = 8


class _LLRegions:
    """Rank 0's LL region and the host-played rank 1's, both on this GPU."""

    def __init__(self, lib, max_elems):
        lib.ashqk_p2p_ll_region_bytes.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_size_t)]
        lib.ashqk_allreduce_f16_ll.argtypes = lib.ashqk_allreduce_f16_oneshot.argtypes
        size = ctypes.c_size_t(0)
        assert lib.ashqk_p2p_ll_region_bytes(max_elems, ctypes.byref(size)) == 0
        self.max_elems, self.pairs = max_elems, max_elems // 2
        self.r = [torch.zeros(size.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
        self.ptrs = torch.tensor([t.data_ptr() for t in self.r], dtype=torch.int64, device="cuda")

    def lines(self, dst, parity, src):
        inbox = self.r[dst][HEADER:].view(torch.int64).view(2, MAX_RANKS, self.pairs)
        return inbox[parity, src]

    def counters(self, q):
        return self.r[q][:HEADER].view(torch.int32)


def _pack_lines(t, epoch):
    data = t.reshape(-1).view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return data | (epoch << 32)


def _call_ll(lib, regs, x, out, rank=0, world=2):
    return lib.ashqk_allreduce_f16_ll(x.data_ptr(), out.data_ptr(), x.numel(), regs.ptrs.data_ptr(), rank, world,
                                      regs.max_elems, torch.cuda.current_stream().cuda_stream)


def test_ll_protocol_and_sum(lib):
    assert _errors(lib, clear=True) & PEER_BIT == 0
    regs = _LLRegions(lib, 1 << 15)
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    for e, shape in enumerate([(4, 4096), (1, 4096), (8, 4096), (2, 8)], start=1):
        n = shape[0] * shape[1]
        a = (torch.randn(shape, device="cuda", generator=g) * 2).half()
        b = (torch.randn(shape, device="cuda", generator=g) * 2).half()
        assert regs.counters(0)[:2].tolist() == [e - 1, 0]               # calls done, CTAs finished
        regs.lines(0, e & 1, 1)[: n // 2] = _pack_lines(b, e)            # the peer's pushed lines
        out = torch.full_like(a, float("nan"))
        assert _call_ll(lib, regs, a, out) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, (a.float() + b.float()).half()), e
        assert regs.counters(0)[:2].tolist() == [e, 0]                   # the last CTA bumped it
        assert torch.equal(regs.lines(1, e & 1, 0)[: n // 2], _pack_lines(a, e))  # pushed to the peer
    a = torch.randn(8, 512, device="cuda", generator=g).half()
    ref = a.clone()
    assert _call_ll(lib, regs, a, a, world=1) == 0                       # world 1: a copy, in place
    torch.cuda.synchronize()
    assert torch.equal(a, ref) and _errors(lib) & PEER_BIT == 0


def test_ll_missing_peer_times_out(lib):
    regs = _LLRegions(lib, 1024)
    a = torch.ones(1024, dtype=torch.float16, device="cuda")
    out = torch.full_like(a, -7.0)
    _errors(lib, clear=True)
    t0 = time.time()
    assert _call_ll(lib, regs, a, out) == 0                               # no line ever arrives
    torch.cuda.synchronize()
    waited = time.time() - t0
    try:
        assert _errors(lib) & PEER_BIT and 0.5 < waited < 30, waited
        assert bool((out == -7.0).all())
        t0 = time.time()
        assert _call_ll(lib, regs, a, out) == 0                           # sticky: returns at once
        torch.cuda.synchronize()
        assert time.time() - t0 < 0.5 and regs.counters(0)[:2].tolist() == [1, 0]
    finally:
        _errors(lib, clear=True)


def _fused_call(lib, regs, x, qw, qz, s, y, rank=0, world=2):
    vp, i64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.ashqk_w4a16_gemv_allreduce.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, i64, ci, ci, ci, ci, vp, ci,
                                               ci, i64, vp]
    m, k = x.shape
    n = qw.shape[1] * 8
    return lib.ashqk_w4a16_gemv_allreduce(x.data_ptr(), x.stride(0), qw.data_ptr(), qw.stride(0), qz.data_ptr(),
                                          qz.stride(0), s.data_ptr(), s.stride(0), y.data_ptr(), y.stride(0), m, n, k,
                                          k // s.shape[0], regs.ptrs.data_ptr(), rank, world, regs.max_elems,
                                          torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m,n,k", [(1, 4096, 2048), (4, 4096, 6144), (16, 4096, 512), (2, 96, 1024)])
def test_fused_row_parallel_gemv(lib, m, n, k):
    """Rank 0 of two with the host playing rank 1: the fused kernel's y equals the unfused
    column-strip GEMV's fp16 partial plus rank 1's, summed in fp32 and rounded once; the lines it pushed carry its
    partial; the region's call counter advances once per call (shared with the LL all-reduce)."""
    import ashqk
    from tests._helpers import quantized_problem, to_cuda

    _errors(lib, clear=True)
    regs = _LLRegions(lib, 1 << 16)
    x0, qw0, qz0, s0 = to_cuda(*quantized_problem(m, n, k, 128, seed=m + 1))
    x1, qw1, qz1, s1 = to_cuda(*quantized_problem(m, n, k, 128, seed=m + 101))
    # The fused epilogue is the column-strip GEMV's (kernel 3): its partial is bitwise that kernel's.
    assert lib.ashqk_set_gemv_kernel(3) == 0
    try:
        y0 = ashqk.w4a16_linear(x0, qw0, qz0, s0)   # this rank's partial, as the unfused GEMV stores it
        y1 = ashqk.w4a16_linear(x1, qw1, qz1, s1)   # the peer's
    finally:
        assert lib.ashqk_set_gemv_kernel(0) == 0
    for e in (1, 2, 3):
        regs.lines(0, e & 1, 1)[: m * n // 2] = _pack_lines(y1, e)
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
        assert _fused_call(lib, regs, x0, qw0, qz0, s0, y) == 0
        torch.cuda.synchronize()
        assert torch.equal(y, (y0.float() + y1.float()).half()), (m, n, k, e)
        assert torch.equal(regs.lines(1, e & 1, 0)[: m * n // 2], _pack_lines(y0, e))
        assert regs.counters(0)[:2].tolist() == [e, 0]
    assert _errors(lib) == 0


def test_fused_declines_what_it_cannot_take(lib):
    regs = _LLRegions(lib, 1 << 12)
    x = torch.zeros(2, 1024, dtype=torch.float16, device="cuda")
    qw = torch.zeros(1024, 4096 // 8, dtype=torch.int32, device="cuda")
    qz = torch.zeros(8, 4096 // 8, dtype=torch.int32, device="cuda")
    s = torch.ones(8, 4096, dtype=torch.float16, device="cuda")
    y = torch.empty(2, 4096, dtype=torch.float16, device="cuda")
    assert _fused_call(lib, regs, x, qw, qz, s, y) == 1               # M * N > max_elems
    regs = _LLRegions(lib, 1 << 16)
    assert _fused_call(lib, regs, x[:, :1024], qw[:, :5], qz[:, :5], s[:, :40], y[:, :40]) == 2  # N % 32
    assert regs.counters(0)[:2].tolist() == [0, 0]                     # nothing launched
