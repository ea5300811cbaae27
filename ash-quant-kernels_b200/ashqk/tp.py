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
                        reduce_dtype: Optional[torch.dtype] = None, linear: Optional[Linear] = None) -> torch.Tensor:
    """Partial y = x[..., shard] @ W[shard, :] on every rank, summed over ranks.

    ``reduce_dtype=torch.float32`` sums the partials in fp32 (one rounding to
    fp16 at the end instead of one per reduction step).
    """
    linear = linear or w4a16_linear
    y = linear(x_local, qweight, qzeros, scales)
    _, world = _world(group)
    if world == 1:
        return y
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
