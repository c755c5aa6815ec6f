"""Row sharding across GPUs: one process per GPU (torch.distributed over NCCL for the plumbing),
each holding a contiguous block of rows of a 2-D tensor.

Only cross-shard reductions talk to other GPUs: a whole-tensor sum reduces each shard to one
float64 partial on its GPU (ctb_sum_partial), all-gathers the partials (8 bytes per rank) and adds
them in rank order on every GPU (ctb_sum_combine), so every rank holds the same, run-to-run
identical float32 result. Row-wise work (elementwise ops with a broadcast row, per-row argmin) needs
no communication; its outputs stay sharded. ctorch itself has no multi-GPU layer; this is the
sharded form of its whole-tensor sum (src/ops/reduction_ops_cpu.cpp:463) and row-wise ops.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch


@dataclass(frozen=True)
class RowShard:
    """Rows [start, stop) of `total` owned by `rank` of `world`: contiguous blocks, the first
    `total % world` ranks one row longer."""

    rank: int
    world: int
    total: int
    start: int
    stop: int

    @property
    def rows(self) -> int:
        return self.stop - self.start


def row_shard(total: int, rank: int, world: int) -> RowShard:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    stop = start + base + (1 if rank < rem else 0)
    return RowShard(rank, world, total, start, stop)


def _partial_sum_cuda(local: torch.Tensor, out: torch.Tensor) -> None:
    from . import _capi as C
    from .ops import _call, _scratch

    v = C.view(local)
    need = C.lib.ctb_sum_partial_scratch_bytes(v)
    scratch = _scratch(need, local.device)
    _call(C.lib.ctb_sum_partial(v, out.data_ptr(), scratch.data_ptr() if scratch is not None else None,
                                need, C.stream_handle(local.device)), "sum")


def _combine_cuda(parts: torch.Tensor, out: torch.Tensor) -> None:
    from . import _capi as C
    from .ops import _call

    _call(C.lib.ctb_sum_combine(parts.data_ptr(), parts.numel(), C.view(out),
                                C.stream_handle(parts.device)), "sum")


class ShardedSum:
    """Whole-tensor sum of a row-sharded tensor. Buffers are allocated once, so repeated calls
    allocate nothing (and can be captured in a CUDA graph together with the NCCL all-gather)."""

    def __init__(self, device: torch.device, world: int, out_dtype=torch.float32,
                 group=None,
                 partial_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None):
        self.world = world
        self.group = group
        self.partial = torch.zeros(1, dtype=torch.float64, device=device)
        self.parts = torch.zeros(world, dtype=torch.float64, device=device)
        self.out = torch.zeros((), dtype=out_dtype, device=device)
        self.partial_fn = partial_fn or _partial_sum_cuda
        self.combine_fn = combine_fn or _combine_cuda

    def __call__(self, local: torch.Tensor) -> torch.Tensor:
        self.partial_fn(local, self.partial)
        return self.combine()

    def combine(self) -> torch.Tensor:
        """All-gathers self.partial (already written by this rank) and combines in rank order."""
        if self.world > 1:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.parts, self.partial, group=self.group)
        else:
            self.parts.copy_(self.partial)
        self.combine_fn(self.parts, self.out)
        return self.out


def sharded_step(x_local: torch.Tensor, r: torch.Tensor, summer: ShardedSum):
    """One pass of the sharded workload on this rank's rows:
    Y = (X - r) * r (one fused pass, bit-identical to sub then mul), s = sum(Y) over all ranks,
    k = argmin(Y, dim=1) for the local rows."""
    from .ops import argmin, binary_chain

    y = binary_chain("sub", "mul", x_local, r, r)
    s = summer(y)
    k = argmin(y, 1)
    return y, s, k


def sharded_step_fused(x_local: torch.Tensor, r: torch.Tensor, summer: ShardedSum):
    """The same step in one pass over this rank's rows (ctb_chain_rows): Y written, the per-row
    argmin and this rank's float64 partial produced in the epilogue, then the 8-byte partials
    all-gathered and combined in rank order. Y and k are bit-identical to sharded_step; s matches
    it to float64 rounding of the partials."""
    from .ops import chain_rows

    y, k, _ = chain_rows("sub", "mul", x_local, r, r, row_op="min", out_sum=summer.partial)
    s = summer.combine()
    return y, s, k
