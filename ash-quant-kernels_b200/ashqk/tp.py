"""Tensor-parallel W4A16 linear layers: one process per GPU, NCCL over NVLink.

The reference runs each layer on one GPU; its multi-GPU plan shards a dense
MLP the Megatron way, and this module is that plan on AWQ tensors:

* column-parallel (qkv, gate_up): rank r owns output columns
  [r*N/P, (r+1)*N/P) -- the matching word columns of ``qweight``/``qzeros`` and
  columns of ``scales`` -- computes ``[M, N/P]`` and, if asked, all-gathers the
  full ``[M, N]``;
* row-parallel (o, down): rank r owns input rows [r*K/P, (r+1)*K/P) on group
  boundaries (K/P a multiple of G), multiplies its slice of x and all-reduces
  the partial ``[M, N]`` sums.

Every rank must call these functions in the same order (they issue
collectives). The local product is ``ashqk.w4a16_linear`` on the shard; there is
no CPU path. ``linear`` lets a caller substitute another local product with the
same signature (the CPU tests use the oracle there).
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .ops import w4a16_linear

Linear = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


# ---------------------------------------------------------------------------
# Sharding of AWQ tensors
# ---------------------------------------------------------------------------

def shard_columns(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, rank: int, world: int,
                  contiguous: bool = True):
    """Rank ``rank``'s output-column shard of an AWQ layer (N split into ``world`` parts).

    Each shard holds N/world columns, a multiple of 8 so that no packed word is
    split. With ``contiguous=False`` the shards are strided views of the inputs
    (the kernels accept them); contiguous copies stream slightly better.
    """
    words = qweight.shape[1]
    assert words % world == 0, f"N/8={words} word columns do not split into {world} shards"
    w = words // world
    qw = qweight[:, rank * w:(rank + 1) * w]
    qz = qzeros[:, rank * w:(rank + 1) * w]
    s = scales[:, rank * w * 8:(rank + 1) * w * 8]
    if contiguous:
        qw, qz, s = qw.contiguous(), qz.contiguous(), s.contiguous()
    return qw, qz, s


def shard_rows(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, rank: int, world: int):
    """Rank ``rank``'s input-row shard of an AWQ layer (K split on quantisation-group boundaries)."""
    k, groups = qweight.shape[0], scales.shape[0]
    assert groups > 0 and k % groups == 0, "K must be a multiple of the group count"
    assert groups % world == 0, f"{groups} quantisation groups do not split into {world} shards"
    g = k // groups
    per = groups // world
    return (qweight[rank * per * g:(rank + 1) * per * g], qzeros[rank * per:(rank + 1) * per],
            scales[rank * per:(rank + 1) * per])


def shard_input(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The slice of x's last dimension a row-parallel rank multiplies (a view)."""
    k = x.shape[-1]
    assert k % world == 0
    kl = k // world
    return x[..., rank * kl:(rank + 1) * kl]


# ---------------------------------------------------------------------------
# Forward passes
# ---------------------------------------------------------------------------

def column_parallel_linear(x: torch.Tensor, qweight, qzeros, scales, group=None, gather_output: bool = True,
                           linear: Optional[Linear] = None) -> torch.Tensor:
    """y = x @ W[:, shard] on every rank; with ``gather_output`` the full [..., N].

    The local [M, N/P] result is written straight into this rank's slot of the
    gather buffer, and the all-gather runs in place on it. At M=1 the gathered
    [P, 1, N/P] buffer already is the [1, N] row; for M>1 one transpose copy
    puts the columns in order.
    """
    linear = linear or w4a16_linear
    rank, world = _world(group)
    if world == 1 or not gather_output:
        return linear(x, qweight, qzeros, scales)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    m, n_loc = x2.shape[0], qweight.shape[1] * 8
    buf = torch.empty((world, m, n_loc), dtype=torch.float16, device=x.device)
    mine = buf[rank]
    if linear is w4a16_linear and x.is_cuda:
        from .ops import w4a16_linear_into

        w4a16_linear_into(x2, qweight, qzeros, scales, mine)
    else:
        mine.copy_(linear(x2, qweight, qzeros, scales))
    dist.all_gather_into_tensor(buf.view(world * m, n_loc), mine, group=group)
    y = buf.view(m, world * n_loc) if m == 1 else buf.permute(1, 0, 2).reshape(m, world * n_loc)
    return y.reshape(*lead, world * n_loc)


def row_parallel_linear(x_local: torch.Tensor, qweight, qzeros, scales, group=None,
                        reduce_dtype: Optional[torch.dtype] = None, linear: Optional[Linear] = None,
                        allreduce: Optional["P2PAllReduce"] = None, fused: bool = False) -> torch.Tensor:
    """Partial y = x[..., shard] @ W[shard, :] on every rank, summed over ranks.

    ``reduce_dtype=torch.float32`` sums the partials in fp32 (one rounding to
    fp16 at the end instead of one per reduction step). ``allreduce`` (a
    ``P2PAllReduce`` of the same group) replaces NCCL for partials it can hold;
    it too sums in fp32 with one rounding. ``fused=True`` with a low-latency
    ``allreduce`` runs the GEMV and the all-reduce as one kernel where it takes
    the shard (the column-strip GEMV with the all-reduce in its epilogue; on
    B200 slower than the default GEMV followed by the all-reduce).
    """
    _, world = _world(group)
    if fused and world > 1 and linear is None and allreduce is not None and allreduce.protocol == "ll":
        y = allreduce.fused_linear(x_local, qweight, qzeros, scales)
        if y is not None:  # GEMV and all-reduce in one kernel
            return y
    linear = linear or w4a16_linear
    y = linear(x_local, qweight, qzeros, scales)
    if world == 1:
        return y
    if allreduce is not None and y.is_contiguous() and y.numel() % 8 == 0 and y.numel() <= allreduce.max_elems:
        return allreduce(y, out=y)
    if reduce_dtype is not None and reduce_dtype != y.dtype:
        acc = y.to(reduce_dtype)
        dist.all_reduce(acc, group=group)
        return acc.to(y.dtype)
    dist.all_reduce(y, group=group)
    return y


class ColumnParallelW4A16Linear(torch.nn.Module):
    """An AWQ linear layer whose output columns are split across the ranks of ``group``."""

    def __init__(self, qweight, qzeros, scales, group=None, gather_output: bool = True):
        super().__init__()
        rank, world = _world(group)
        qw, qz, s = shard_columns(qweight, qzeros, scales, rank, world)
        self.register_buffer("qweight", qw)
        self.register_buffer("qzeros", qz)
        self.register_buffer("scales", s)
        self.group, self.gather_output = group, gather_output

    def forward(self, x):
        return column_parallel_linear(x, self.qweight, self.qzeros, self.scales, self.group, self.gather_output)


class RowParallelW4A16Linear(torch.nn.Module):
    """An AWQ linear layer whose input rows are split across the ranks of ``group``.

    ``input_is_parallel``: x already holds only this rank's K slice (the output
    of a column-parallel layer without gather); otherwise it is sliced here.
    """

    def __init__(self, qweight, qzeros, scales, group=None, input_is_parallel: bool = True,
                 reduce_dtype: Optional[torch.dtype] = None):
        super().__init__()
        rank, world = _world(group)
        qw, qz, s = shard_rows(qweight, qzeros, scales, rank, world)
        self.register_buffer("qweight", qw.contiguous())
        self.register_buffer("qzeros", qz.contiguous())
        self.register_buffer("scales", s.contiguous())
        self.group, self.input_is_parallel, self.reduce_dtype = group, input_is_parallel, reduce_dtype
        self.rank, self.world = rank, world

    def forward(self, x):
        if not self.input_is_parallel:
            x = shard_input(x, self.rank, self.world)
        return row_parallel_linear(x, self.qweight, self.qzeros, self.scales, self.group, self.reduce_dtype)


class P2PAllReduce:
    """Sum of fp16 tensors over the ranks of ``group`` through NVLink peer memory (one CUDA IPC
    region per rank, a one-CTA kernel per call; ``ashqk_allreduce_f16_oneshot``), for the small
    row-parallel partials of tensor-parallel decode where NCCL's per-call cost dominates.

    Every rank must construct it and call it in the same order. Tensors: fp16, contiguous, at most
    ``max_elems`` elements, a multiple of 8. The sum runs in fp32 over ranks in rank order and is
    rounded once. ``close()`` (collective) releases the regions.

    Every rank must reach each call within the kernels' peer-wait limit (about 2 s of GPU time from
    the call's launch on the waiting rank). A call whose peer does not arrive in time leaves its
    output unwritten (in place: the local partial) and sets a sticky error bit; the kernels also
    store that bit into a pinned host word, so the next call on this object raises RuntimeError
    instead of summing anything, and ``check()`` raises until the error word is cleared. Under
    CUDA-graph replay no Python code runs per call: call ``check()`` after the replays.
    """

    def __init__(self, group=None, max_elems: int = 1 << 16, lib=None, protocol: str = "oneshot"):
        """``protocol``: "oneshot" (copy, fenced flag, peer loads; one CTA) or "ll" (8-byte
        data + epoch lines pushed to the peers, one CTA per 1024 elements, max_elems <= 65536).
        ``lib``: the loaded C library (default: the package's own; tests pass a fake)."""
        if protocol not in ("oneshot", "ll"):
            raise ValueError("protocol: 'oneshot' or 'll'")
        self.protocol = protocol
        import ctypes

        self._ct = ctypes
        if lib is None:
            from . import _ext

            lib = ctypes.CDLL(_ext.C_LIBRARY)
        vp = ctypes.c_void_p
        lib.ashqk_p2p_region_bytes.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_size_t)]
        lib.ashqk_p2p_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        lib.ashqk_p2p_free.argtypes = [vp]
        lib.ashqk_p2p_export.argtypes = [vp, vp]
        lib.ashqk_p2p_import.argtypes = [vp, ctypes.POINTER(vp)]
        lib.ashqk_p2p_close.argtypes = [vp]
        lib.ashqk_get_device_errors.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
        for name in ("ashqk_allreduce_f16_oneshot", "ashqk_allreduce_f16_ll"):
            getattr(lib, name).argtypes = [vp, vp, ctypes.c_int64, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int64, vp]
        i64, ci = ctypes.c_int64, ctypes.c_int
        lib.ashqk_w4a16_gemv_allreduce.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, i64, ci, ci, ci, ci, vp, ci,
                                                   ci, i64, vp]
        lib.ashqk_p2p_ll_region_bytes.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_size_t)]
        self._region_bytes = lib.ashqk_p2p_ll_region_bytes if protocol == "ll" else lib.ashqk_p2p_region_bytes
        self._reduce = lib.ashqk_allreduce_f16_ll if protocol == "ll" else lib.ashqk_allreduce_f16_oneshot
        lib.ashqk_set_error_mirror.argtypes = [vp]
        self._lib, self.group = lib, group
        self.rank, self.world = _world(group)
        self._host_err, self._mirrored = None, False
        if self.world > 8:
            raise ValueError("P2PAllReduce handles at most 8 ranks (one NVLink domain of B200s)")
        self.max_elems = int(max_elems)
        size = ctypes.c_size_t(0)
        if self._region_bytes(self.max_elems, ctypes.byref(size)) != 0:
            raise ValueError("max_elems must be a positive multiple of 8 (at most 65536 for protocol 'll')")
        region = vp()
        if lib.ashqk_p2p_alloc(size.value, ctypes.byref(region)) != 0:
            raise RuntimeError("ashqk: cannot allocate the all-reduce region")
        self._region, self._imported = region, []
        handle = ctypes.create_string_buffer(64)
        # Every rank takes part in the handle exchange even when its own export
        # failed (an empty handle), so that a local failure raises on every rank
        # instead of leaving the peers waiting in the collective.
        ok = lib.ashqk_p2p_export(region, handle) == 0
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, handle.raw if ok else b"", group=group)
        else:
            handles = [handle.raw]
        err, ptrs = None, []
        bad = [r for r, h in enumerate(handles) if len(h) != 64]
        if bad:
            err = f"ranks {bad} could not export their regions"
        else:
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(region.value)
                    continue
                p = vp()
                if lib.ashqk_p2p_import(ctypes.create_string_buffer(h, 64), ctypes.byref(p)) != 0:
                    err = f"cannot open rank {r}'s region"
                    break
                self._imported.append(p)
                ptrs.append(p.value)
        # Agree on the outcome (this exchange is also the barrier after which
        # every region is open), so that all ranks raise together or none does.
        errors = [err] * self.world
        if self.world > 1:
            dist.all_gather_object(errors, err, group=group)
        failed = [f"rank {r}: {e}" for r, e in enumerate(errors) if e]
        try:
            if failed:
                raise RuntimeError("ashqk: P2P all-reduce setup failed (" + "; ".join(failed) + ")")
            dev = torch.device("cuda", torch.cuda.current_device())
            self._regions_dev = torch.tensor(ptrs, dtype=torch.int64, device=dev)
            # Host-mapped copy of the device error word, written by a kernel only when it raises a bit.
            self._host_err = torch.zeros(1, dtype=torch.int32).pin_memory()
            self._mirrored = lib.ashqk_set_error_mirror(self._host_err.data_ptr()) == 0
        except BaseException:
            for p in self._imported:
                lib.ashqk_p2p_close(p)
            lib.ashqk_p2p_free(region)
            self._region, self._imported = None, []
            raise

    def __call__(self, t: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Return the sum over ranks of ``t`` (in place when ``out is t``)."""
        assert t.dtype == torch.float16 and t.is_cuda and t.is_contiguous(), "fp16 contiguous CUDA tensor"
        assert t.numel() % 8 == 0 and t.numel() <= self.max_elems, "numel: a multiple of 8, <= max_elems"
        assert self._region is not None, "P2PAllReduce is closed"
        self._raise_if_failed()
        if out is None:
            out = torch.empty_like(t)
        assert (out.dtype == torch.float16 and out.device == t.device and out.is_contiguous()
                and out.numel() == t.numel()), "out: fp16, contiguous, same device and size as t"
        rc = self._reduce(t.data_ptr(), out.data_ptr(), t.numel(), self._regions_dev.data_ptr(), self.rank,
                          self.world, self.max_elems, torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(f"ashqk all-reduce ({self.protocol}) failed ({rc})")
        return out

    def fused_linear(self, x, qweight, qzeros, scales) -> Optional[torch.Tensor]:
        """Row-parallel layer in one kernel (protocol "ll"): the sum over ranks of
        ``x @ W_shard``, or None when the fused kernel does not take the problem (the caller
        then runs the GEMV and this all-reduce). x: [M, K_shard] fp16, M <= 16."""
        if self.protocol != "ll" or x.dim() != 2 or x.dtype != torch.float16 or not x.is_cuda:
            return None
        m, k = x.shape
        n = qweight.shape[1] * 8
        if m > 16 or m * n > self.max_elems or x.stride(1) != 1 or any(t.stride(1) != 1 for t in
                                                                        (qweight, qzeros, scales)):
            return None
        self._raise_if_failed()
        y = torch.empty(m, n, dtype=torch.float16, device=x.device)
        rc = self._lib.ashqk_w4a16_gemv_allreduce(
            x.data_ptr(), x.stride(0), qweight.data_ptr(), qweight.stride(0), qzeros.data_ptr(), qzeros.stride(0),
            scales.data_ptr(), scales.stride(0), y.data_ptr(), y.stride(0), m, n, k, k // scales.shape[0],
            self._regions_dev.data_ptr(), self.rank, self.world, self.max_elems,
            torch.cuda.current_stream().cuda_stream)
        if rc == 2:  # ASHQK_ERR_UNSUPPORTED: nothing launched
            return None
        if rc != 0:
            raise RuntimeError(f"ashqk_w4a16_gemv_allreduce failed ({rc})")
        return y

    def _raise_if_failed(self) -> None:
        if self._mirrored and int(self._host_err[0]) & 4:
            raise RuntimeError("ashqk: an earlier P2P all-reduce gave up waiting for a peer rank; its output was "
                               "not reduced and no further calls run until the error word is cleared")

    def check(self) -> None:
        """Raise if a call on this device gave up waiting for a peer (the results since are invalid)."""
        bits = self._ct.c_uint(0)
        if self._lib.ashqk_get_device_errors(self._ct.byref(bits), 0) != 0:
            raise RuntimeError("ashqk: cannot read the device error word")
        if bits.value & 4:
            raise RuntimeError("ashqk: a peer rank never arrived at a P2P all-reduce; its results are invalid")

    def close(self) -> None:
        """Collective: wait for every rank, then release the peer mappings and the region."""
        if self._region is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._imported:
            self._lib.ashqk_p2p_close(p)
        self._lib.ashqk_p2p_free(self._region)
        self._region, self._imported = None, []
        if self._mirrored:
            self._lib.ashqk_set_error_mirror(None)
            self._mirrored = False
