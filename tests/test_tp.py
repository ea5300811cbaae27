"""Tensor-parallel host logic on CPU: two gloo ranks, the oracle as the local product.

Covers ashqk.tp's sharding of AWQ tensors and the collective steps around the
local product (the CUDA path runs the same functions in tests/test_gpu_tp.py):
column-parallel outputs gather to exactly the unsharded product, row-parallel
partials reduce to it within fp16 rounding, and a column -> row MLP pair
composes as the unsharded pair does.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import awq_oracle as O
from tests._helpers import quantized_problem

WORLD = 2


def oracle_linear(x, qw, qz, s):
    """The oracle's product (fp64 accumulation, one rounding to fp16) on CPU tensors."""
    x2 = x.reshape(-1, x.shape[-1])
    y = O.c_gemm(x2.numpy(), qw.numpy(), qz.numpy(), s.numpy(), out_fp16=True)
    return torch.from_numpy(y).reshape(*x.shape[:-1], y.shape[-1])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _FakeP2PLib:
    """Stands in for the C library's P2P entry points on CPU: records every call and fails the
    one named by ``fail`` on this rank."""

    def __init__(self, rank, fail=None):
        self.calls, self.open, self.freed = [], [], []

        def region_bytes(n, size_ref):
            size_ref._obj.value = 256 + 4 * n
            return 0

        def alloc(nbytes, ptr_ref):
            ptr_ref._obj.value = 0x1000 * (rank + 1)
            return 0

        def export(ptr, handle):
            self.calls.append("export")
            if fail == "export":
                return 5
            handle.raw = bytes([rank]) * 64
            return 0

        def import_(handle, ptr_ref):
            self.calls.append("import")
            if fail == "import":
                return 5
            ptr_ref._obj.value = 0x100000 + handle.raw[0]
            self.open.append(ptr_ref._obj.value)
            return 0

        def close(ptr):
            self.open.remove(ptr.value if hasattr(ptr, "value") else ptr)
            return 0

        def free(ptr):
            self.freed.append(ptr.value if hasattr(ptr, "value") else ptr)
            return 0

        def nop(*args):
            return 0

        self.ashqk_p2p_region_bytes, self.ashqk_p2p_alloc, self.ashqk_p2p_export = region_bytes, alloc, export
        self.ashqk_p2p_import, self.ashqk_p2p_close, self.ashqk_p2p_free = import_, close, free
        self.ashqk_allreduce_f16_oneshot = self.ashqk_allreduce_f16_ll = nop
        self.ashqk_w4a16_gemv_allreduce = lambda *args: 0
        self.ashqk_p2p_ll_region_bytes = region_bytes
        self.ashqk_get_device_errors = nop
        self.ashqk_set_error_mirror = nop


def _worker(rank, port, case):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from ashqk import tp

        if case == "column":
            m, n, k, g = 3, 512, 256, 64
            x, qw, qz, s = (torch.from_numpy(a) for a in quantized_problem(m, n, k, g, seed=11))
            full = oracle_linear(x, qw, qz, s)
            for contiguous in (True, False):
                shard = tp.shard_columns(qw, qz, s, rank, WORLD, contiguous=contiguous)
                assert shard[0].shape == (k, n // 8 // WORLD) and shard[2].shape == (k // g, n // WORLD)
                local = tp.column_parallel_linear(x, *shard, gather_output=False, linear=oracle_linear)
                assert torch.equal(local, full[:, rank * n // WORLD:(rank + 1) * n // WORLD])
                y = tp.column_parallel_linear(x, *shard, linear=oracle_linear)
                assert torch.equal(y, full)  # each column is computed exactly as unsharded
            y1 = tp.column_parallel_linear(x[:1], *tp.shard_columns(qw, qz, s, rank, WORLD), linear=oracle_linear)
            assert torch.equal(y1, full[:1])  # the M=1 layout needs no transpose
        elif case == "row":
            m, n, k, g = 4, 256, 512, 64
            x, qw, qz, s = (torch.from_numpy(a) for a in quantized_problem(m, n, k, g, seed=12))
            truth = O.c_gemm(x.numpy(), qw.numpy(), qz.numpy(), s.numpy())
            shard = tp.shard_rows(qw, qz, s, rank, WORLD)
            assert shard[0].shape == (k // WORLD, n // 8) and shard[1].shape == (k // g // WORLD, n // 8)
            xl = tp.shard_input(x, rank, WORLD)
            assert xl.shape == (m, k // WORLD)
            for reduce_dtype in (None, torch.float32):
                y = tp.row_parallel_linear(xl, *shard, reduce_dtype=reduce_dtype, linear=oracle_linear)
                assert y.dtype == torch.float16 and y.shape == (m, n)
                err = O.rel_err(y.float().numpy(), truth)
                assert err < 1e-3, err  # two fp16 roundings of the partials, one of the sum
        elif case == "mlp":
            m, h, f, g = 2, 256, 512, 64
            rng = np.random.default_rng(13)
            x = torch.from_numpy(rng.standard_normal((m, h), dtype=np.float32).astype(np.float16))
            w1 = O.quantize_awq((rng.standard_normal((h, f), dtype=np.float32) * 0.05).astype(np.float32), g)
            w2 = O.quantize_awq((rng.standard_normal((f, h), dtype=np.float32) * 0.05).astype(np.float32), g)
            w1, w2 = [tuple(torch.from_numpy(a) for a in w) for w in (w1, w2)]
            up = tp.ColumnParallelW4A16Linear(*w1, gather_output=False)
            down = tp.RowParallelW4A16Linear(*w2, input_is_parallel=True, reduce_dtype=torch.float32)
            a = tp.column_parallel_linear(x, up.qweight, up.qzeros, up.scales, gather_output=False,
                                          linear=oracle_linear)
            y = tp.row_parallel_linear(a, down.qweight, down.qzeros, down.scales, reduce_dtype=torch.float32,
                                       linear=oracle_linear)
            a_full = oracle_linear(x, *w1)
            truth = O.c_gemm(a_full.numpy(), *(t.numpy() for t in w2))
            assert O.rel_err(y.float().numpy(), truth) < 1e-3
            # every rank ends with the same result
            others = [torch.empty_like(y) for _ in range(WORLD)]
            dist.all_gather(others, y)
            assert all(torch.equal(o, y) for o in others)
        elif case.startswith("p2p_"):
            # A failed setup step on one rank makes every rank raise (no rank is left waiting in a
            # collective), and each releases what it had opened and allocated. On CPU even a clean
            # exchange fails at the end (no CUDA device for the pointer table): the same cleanup.
            what, where = {"p2p_export": ("export", 1), "p2p_import": ("import", 0), "p2p_ok": (None, -1)}[case]
            lib = _FakeP2PLib(rank, what if rank == where else None)
            with pytest.raises(RuntimeError) as info:
                tp.P2PAllReduce(max_elems=1024, lib=lib)
            if what is not None:
                assert f"rank {where}:" in str(info.value), str(info.value)
            assert lib.open == [] and lib.freed == [0x1000 * (rank + 1)]
            assert lib.calls.count("import") == (0 if what == "export" else 1)
        elif case == "bad_split":
            qw = torch.zeros(384, 8, dtype=torch.int32)  # K=384, G=128: 3 groups
            qz = torch.zeros(3, 8, dtype=torch.int32)
            s = torch.ones(3, 64, dtype=torch.float16)
            with pytest.raises(AssertionError):
                tp.shard_rows(qw, qz, s, rank, WORLD)
            with pytest.raises(AssertionError):
                tp.shard_columns(qw[:, :3], qz[:, :3], s[:, :24], rank, WORLD)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["column", "row", "mlp", "bad_split", "p2p_export", "p2p_import", "p2p_ok"])
def test_tensor_parallel_gloo(case):
    mp.start_processes(_worker, args=(_free_port(), case), nprocs=WORLD, start_method="spawn", join=True)


def test_single_process_is_a_plain_call():
    """Without a process group the TP functions are the local product."""
    from ashqk import tp

    x, qw, qz, s = (torch.from_numpy(a) for a in quantized_problem(2, 128, 256, 64, seed=14))
    full = oracle_linear(x, qw, qz, s)
    assert torch.equal(tp.column_parallel_linear(x, qw, qz, s, linear=oracle_linear), full)
    assert torch.equal(tp.row_parallel_linear(x, qw, qz, s, linear=oracle_linear), full)
    assert [t.shape for t in tp.shard_columns(qw, qz, s, 0, 1)] == [qw.shape, qz.shape, s.shape]
