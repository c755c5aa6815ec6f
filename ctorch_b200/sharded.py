"""Row sharding across GPUs: one process per GPU (torch.distributed over NCCL for the plumbing),
each holding a contiguous block of rows of a 2-D tensor.

Only cross-shard reductions talk to other GPUs:
- a whole-tensor sum reduces each shard to one float64 partial on its GPU (ctb_sum_partial),
  all-gathers the partials (8 bytes per rank) and adds them in rank order on every GPU
  (ctb_sum_combine), so every rank holds the same, run-to-run identical float32 result;
- a max/min over dim 0 (the rows) reduces each shard to its per-column (value, local row) pair
  (ctb_reduce_index), all-gathers those (N values + N int64 indices per rank) and combines them in
  rank order, shifting each shard's rows by its first global row (ctb_minmax_combine): the result
  is the single-GPU reduction of the whole tensor, first NaN and first occurrence included.
Row-wise work (elementwise ops with a broadcast row, per-row argmin, inner-dim reductions) and
index_select over sharded indices need no communication; their outputs stay sharded. ctorch itself
has no multi-GPU layer; these are the sharded forms of its whole-tensor sum
(src/ops/reduction_ops_cpu.cpp:463), its max/min with indices (:236-297) and its row-wise ops.
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


def _local_minmax_cuda(op: str, local: torch.Tensor, values, indices, cache: dict) -> None:
    from . import _capi as C
    from .ops import _call, _scratch

    code = C.MAX if op == "max" else C.MIN
    vx = C.view(local)
    need = C.lib.ctb_reduce_index_scratch_bytes(vx, 0)
    if cache.get("need") != need:
        cache["need"], cache["buf"] = need, _scratch(need, local.device)
    buf = cache["buf"]
    _call(C.lib.ctb_reduce_index(code, vx, C.view(values), C.view(indices), 0,
                                 buf.data_ptr() if buf is not None else None, need,
                                 C.stream_handle(local.device)), op)


def _minmax_combine_cuda(op: str, all_values, all_indices, offsets, out_values, out_indices) -> None:
    from . import _capi as C
    from .ops import _call

    code = C.MAX if op == "max" else C.MIN
    _call(C.lib.ctb_minmax_combine(code, C.view(all_values), C.view(all_indices), offsets.data_ptr(),
                                   C.view(out_values), C.view(out_indices),
                                   C.stream_handle(all_values.device)), op)


class ShardedColumnMinMax:
    """max/min over dim 0 of a row-sharded 2-D tensor [total, N] (values and global row indices),
    the same on every rank. Every rank must hold at least one row. Buffers are allocated once."""

    def __init__(self, op: str, total: int, n_cols: int, dtype, device: torch.device, world: int,
                 group=None, local_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None):
        if op not in ("max", "min"):
            raise ValueError("op must be 'max' or 'min'")
        if total < world:
            raise ValueError("every rank needs at least one row")
        self.op, self.world, self.group = op, world, group
        self.values = torch.empty(n_cols, dtype=dtype, device=device)
        self.indices = torch.empty(n_cols, dtype=torch.int64, device=device)
        # gathered flat (rank-major), viewed [world, N] for the combine
        self._flat_values = torch.empty(world * n_cols, dtype=dtype, device=device)
        self._flat_indices = torch.empty(world * n_cols, dtype=torch.int64, device=device)
        self.all_values = self._flat_values.view(world, n_cols)
        self.all_indices = self._flat_indices.view(world, n_cols)
        self.offsets = torch.tensor([row_shard(total, r, world).start for r in range(world)],
                                    dtype=torch.int64, device=device)
        self.out_values = torch.empty(n_cols, dtype=dtype, device=device)
        self.out_indices = torch.empty(n_cols, dtype=torch.int64, device=device)
        self._cache: dict = {}
        self.local_fn = local_fn or (lambda x, v, i: _local_minmax_cuda(op, x, v, i, self._cache))
        self.combine_fn = combine_fn or (lambda av, ai, off, ov, oi: _minmax_combine_cuda(op, av, ai, off, ov, oi))

    def __call__(self, local: torch.Tensor):
        self.local_fn(local, self.values, self.indices)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self._flat_values, self.values, group=self.group)
            dist.all_gather_into_tensor(self._flat_indices, self.indices, group=self.group)
        else:
            self.all_values.copy_(self.values.reshape(1, -1))
            self.all_indices.copy_(self.indices.reshape(1, -1))
        self.combine_fn(self.all_values, self.all_indices, self.offsets, self.out_values, self.out_indices)
        return self.out_values, self.out_indices


def sharded_index_select(table: torch.Tensor, indices: torch.Tensor, total: int, rank: int, world: int,
                         select: Optional[Callable] = None) -> torch.Tensor:
    """index_select(table, 0, indices) with the output rows sharded: the table is replicated and
    each rank gathers the rows for its own contiguous slice of `indices` (indices[start:stop] of
    the row_shard of `total` = len(indices)). No communication; the output stays sharded."""
    from .ops import index_select

    sh = row_shard(total, rank, world)
    return (select or index_select)(table, 0, indices[sh.start:sh.stop])


class PeerStep:
    """The one-pass step of this rank with the whole-job sum exchanged inside the same launch
    (ctb_chain_rows_allsum): Y = op2(op1(X, r), r) for this rank's rows, the per-row argmin, and
    sum(Y) over all ranks, the same on every rank. The last CTA of each rank's launch stores the
    rank's float64 partial into every rank's workspace over NVLink (CUDA IPC mappings set up here
    once), waits for the others' and adds them in rank order, so a step is one kernel launch with
    no collective call. Every rank must construct it (it exchanges the IPC handles through
    `group`) and call it the same number of times, on one stream; the ranks must be on different
    GPUs. The sum equals ShardedSum's (same per-rank partial, same rank order) bit for bit.

    A rank that does not arrive within `timeout_ns` (0: one second) makes the others' waits run
    out: their sum of that call is NaN and the call is recorded in the workspace. The calls do not
    synchronise the host; `check()` does, and raises CommTimeoutError if any call so far failed."""

    def __init__(self, device: torch.device, rank: int, world: int, group=None, out_dtype=torch.float32,
                 timeout_ns: int = 0):
        import ctypes

        from . import _capi as C

        self.C, self.rank, self.world, self.device = C, rank, world, device
        self.timeout_ns = timeout_ns
        with torch.cuda.device(device):
            ws = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(64)
            self._check(C.lib.ctb_peer_alloc(ctypes.byref(ws), handle))
            self.ws = ws.value
            handles = [bytes(handle.raw)]
            if world > 1:
                import torch.distributed as dist

                handles = [None] * world
                dist.all_gather_object(handles, bytes(handle.raw), group=group)
            self._opened = []
            ptrs = []
            for r in range(world):
                if r == rank:
                    ptrs.append(self.ws)
                    continue
                p = ctypes.c_void_p()
                self._check(C.lib.ctb_peer_open(handles[r], ctypes.byref(p)))
                self._opened.append(p.value)
                ptrs.append(p.value)
            self.peer_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.out = torch.zeros((), dtype=out_dtype, device=device)
        self.parts = torch.zeros(world, dtype=torch.float64, device=device)
        self.epoch = 0

    def _check(self, rc):
        if rc != self.C.OK:
            raise RuntimeError(self.C.last_error())

    def __call__(self, x_local: torch.Tensor, r: torch.Tensor, y: Optional[torch.Tensor] = None,
                 k: Optional[torch.Tensor] = None, op1: str = "sub", op2: str = "mul", row_op: str = "min"):
        C = self.C
        codes = {"add": C.ADD, "sub": C.SUB, "mul": C.MUL, "div": C.DIV}
        if y is None:
            y = torch.empty_like(x_local)
        if k is None:
            k = torch.empty(x_local.shape[0], dtype=torch.int64, device=x_local.device)
        self.epoch += 1
        self._check(C.lib.ctb_chain_rows_allsum(
            codes[op1], codes[op2], C.view(x_local), C.view(r), C.view(r), C.view(y),
            C.MIN if row_op == "min" else C.MAX, C.view(k), self.peer_ptrs.data_ptr(), self.ws,
            self.rank, self.world, self.epoch, C.view(self.out), self.parts.data_ptr(), self.timeout_ns,
            C.stream_handle(x_local.device)))
        return y, self.out, k

    def status(self):
        """(done_epoch, failed_epoch) of this rank's workspace: the last call whose exchange
        completed and the last whose wait ran out (0: none). Synchronises the device."""
        import ctypes

        done, failed = ctypes.c_uint64(0), ctypes.c_uint64(0)
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            self._check(self.C.lib.ctb_peer_status(self.ws, ctypes.byref(done), ctypes.byref(failed)))
        return done.value, failed.value

    def trace(self, calls: Optional[int] = None):
        """Per-call timestamps of this rank's last `calls` calls (at most 64; default all made,
        capped at 64), oldest first, in ns of this GPU's %globaltimer: rows of (CTA 0 started,
        first CTA done, last CTA done, exchange completed). Synchronises the device."""
        import ctypes

        import numpy as np

        buf = (ctypes.c_uint64 * (64 * 4))()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            self._check(self.C.lib.ctb_peer_trace(self.ws, buf))
        ring = np.frombuffer(buf, dtype=np.uint64).reshape(64, 4).astype(np.int64)
        n = min(64, self.epoch if calls is None else calls, self.epoch)
        epochs = range(self.epoch - n + 1, self.epoch + 1)
        return np.stack([ring[e % 64] for e in epochs]) if n else np.zeros((0, 4), np.int64)

    @staticmethod
    def trace_summary(tr) -> dict:
        """Medians (µs) over calls of a trace(): `rows` (CTA 0 start to the last CTA done),
        `tail` (first to last CTA done: the one-wave grid's ragged end), `exchange` (last CTA
        done to the exchange completed: NVLink latency plus the wait for slower ranks), `gap`
        (previous call's exchange completed to this call's CTA 0 start: launch gap)."""
        import numpy as np

        if len(tr) == 0:
            return {}
        med = lambda a: float(np.median(a)) / 1e3 if len(a) else None  # noqa: E731
        return {"rows_us": med(tr[:, 2] - tr[:, 0]), "tail_us": med(tr[:, 2] - tr[:, 1]),
                "exchange_us": med(tr[:, 3] - tr[:, 2]), "gap_us": med(tr[1:, 0] - tr[:-1, 3]),
                "calls": int(len(tr))}

    def check(self):
        """Raises CommTimeoutError unless every call so far completed its exchange."""
        from .errors import CommTimeoutError

        done, failed = self.status()
        if failed or done != self.epoch:
            raise CommTimeoutError(
                f"rank {self.rank}: cross-GPU sum exchange timed out (last failed call {failed}, "
                f"last completed {done}, calls made {self.epoch})")

    def close(self):
        """Unmaps the peers' workspaces and frees this rank's (after a device synchronize)."""
        if self.ws is None:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for p in self._opened:
                self.C.lib.ctb_peer_close(p)
            self.C.lib.ctb_peer_free(self.ws)
        self._opened, self.ws = [], None
