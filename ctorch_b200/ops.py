"""ctorch's eager op API (include/ctorch/ops/{elementwise,reduction,indexing}.h) over torch CUDA
tensors, computed by the sm_100a kernels behind include/ctb/ctb.h.

Each function performs the checks of the matching ctorch front-door (same argument meaning, same
exception types), allocates the output, and makes one C-ABI call on the current stream. Unlike
ctorch's front-door, mixed-dtype operands are promoted in registers on the device instead of being
copied to the host, cast and copied back (src/ops/binary_ops_cpu.cpp:154-184), and outputs are not
zero-filled first, since every kernel writes every output element. There is no CPU fallback:
CPU tensors raise DeviceError.
"""
from __future__ import annotations

import builtins as _bi
from collections import namedtuple
from typing import Sequence

import torch

from . import _capi as C
from .errors import AliasError, DeviceError, DTypeError, ShapeError

ValuesIndices = namedtuple("ValuesIndices", ["values", "indices"])

_PROMOTION_ORDER = [torch.bool, torch.int32, torch.int64, torch.float32, torch.float64]


def promote_types(a: torch.dtype, b: torch.dtype) -> torch.dtype:
    """ctorch's lattice bool < int32 < int64 < float32 < float64 (src/type_promotion.cpp:45-62)."""
    if a not in _PROMOTION_ORDER or b not in _PROMOTION_ORDER:
        raise DTypeError("ctorch::promote_types: bfloat16 not supported")
    return _bi.max(a, b, key=_PROMOTION_ORDER.index)


def _raise(status: int, name: str):
    msg = f"ctorch::{name}: {C.last_error()}"
    if status == C.ERR_DTYPE:
        raise DTypeError(msg)
    if status in (C.ERR_SHAPE, C.ERR_INDEX):
        raise ShapeError(msg)
    if status == C.ERR_CUDA:
        raise DeviceError(msg)
    if status == C.ERR_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _call(status: int, name: str):
    if status != C.OK:
        _raise(status, name)


def _cuda(name: str, *ts: torch.Tensor):
    dev = ts[0].device
    for t in ts:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"ctorch::{name}: expected a tensor")
        if t.device.type != "cuda":
            raise DeviceError(f"ctorch::{name}: ctorch_b200 computes on CUDA tensors only "
                              f"(got a {t.device.type} tensor)")
        if t.device != dev:
            raise DeviceError(f"ctorch::{name}: operands are on different devices")
    return dev


def broadcast_shape(sa: Sequence[int], sb: Sequence[int]) -> tuple:
    """Right-aligned broadcast (src/ops/broadcast.cpp:35-82); ShapeError when incompatible."""
    r = _bi.max(len(sa), len(sb))
    pa = (1,) * (r - len(sa)) + tuple(sa)
    pb = (1,) * (r - len(sb)) + tuple(sb)
    out = []
    for x, y in zip(pa, pb):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise ShapeError(f"ctorch: cannot broadcast shapes {list(sa)} and {list(sb)}")
    return tuple(out)


# ---------------------------------------------------------------- elementwise


def _check_no_bool(a, b, name):
    # src/ops/binary_ops_cpu.cpp:202-208
    if a.dtype == torch.bool or b.dtype == torch.bool:
        raise DTypeError(f"ctorch::{name}: binary arithmetic on bool is not supported "
                         "(cast operands to int32/float first)")


def _binary(op: int, a: torch.Tensor, b: torch.Tensor, name: str) -> torch.Tensor:
    dev = _cuda(name, a, b)
    _check_no_bool(a, b, name)
    dt = promote_types(a.dtype, b.dtype)
    out = torch.empty(broadcast_shape(a.shape, b.shape), dtype=dt, device=dev)
    with torch.cuda.device(dev):
        _call(C.lib.ctb_binary(op, C.view(a), C.view(b), C.view(out), C.stream_handle(dev)), name)
    return out


def add(a, b):
    return _binary(C.ADD, a, b, "add")


def sub(a, b):
    return _binary(C.SUB, a, b, "sub")


def mul(a, b):
    return _binary(C.MUL, a, b, "mul")


def div(a, b):
    return _binary(C.DIV, a, b, "div")


def _byte_range(t: torch.Tensor):
    es = t.element_size()
    base = t.data_ptr()
    extent = 0
    for s, st in zip(t.shape, t.stride()):
        if s > 1 and st != 0:
            extent += (s - 1) * _bi.abs(st) * es
    return base, base + extent + es


def may_overlap(dst: torch.Tensor, src: torch.Tensor) -> bool:
    """src/ops/tensor_iter.cpp:86-110: same storage and overlapping byte ranges."""
    if dst.untyped_storage().data_ptr() != src.untyped_storage().data_ptr():
        return False
    dl, dh = _byte_range(dst)
    sl, sh = _byte_range(src)
    return dl < sh and sl < dh


def _same_view(a, b):
    return (a.data_ptr() == b.data_ptr() and a.shape == b.shape and a.stride() == b.stride()
            and a.dtype == b.dtype)


def _binary_inplace(op: int, a: torch.Tensor, b: torch.Tensor, name: str) -> torch.Tensor:
    # src/ops/binary_ops_cpu.cpp:222-245
    dev = _cuda(name, a, b)
    _check_no_bool(a, b, name)
    dt = promote_types(a.dtype, b.dtype)
    if a.dtype != dt:
        raise DTypeError(f"ctorch::{name}: in-place output dtype must equal the promoted dtype "
                         "of the operands")
    if broadcast_shape(a.shape, b.shape) != tuple(a.shape):
        raise ShapeError(f"ctorch::{name}: in-place output shape must equal the broadcast result "
                         "shape (no implicit reshape)")
    if may_overlap(a, b) and not _same_view(a, b):
        raise AliasError(f"ctorch::{name}: in-place output aliases a non-trivial view of the "
                         "right-hand operand")
    with torch.cuda.device(dev):
        _call(C.lib.ctb_binary(op, C.view(a), C.view(b), C.view(a), C.stream_handle(dev)), name)
    return a


def add_(a, b):
    return _binary_inplace(C.ADD, a, b, "add_")


def sub_(a, b):
    return _binary_inplace(C.SUB, a, b, "sub_")


def mul_(a, b):
    return _binary_inplace(C.MUL, a, b, "mul_")


def div_(a, b):
    return _binary_inplace(C.DIV, a, b, "div_")


def binary_chain(op1: str, op2: str, a, b, c) -> torch.Tensor:
    """op2(op1(a, b), c) in one pass, bit-identical to the two eager ops (float32/float64)."""
    codes = {"add": C.ADD, "sub": C.SUB, "mul": C.MUL, "div": C.DIV}
    dev = _cuda("binary_chain", a, b, c)
    shape = broadcast_shape(broadcast_shape(a.shape, b.shape), c.shape)
    out = torch.empty(shape, dtype=a.dtype, device=dev)
    with torch.cuda.device(dev):
        _call(C.lib.ctb_binary_chain(codes[op1], codes[op2], C.view(a), C.view(b), C.view(c),
                                     C.CODE_OF_TORCH[a.dtype], C.view(out), C.stream_handle(dev)),
              "binary_chain")
    return out


def binary_unary(op: str, uop: str, a, b) -> torch.Tensor:
    """uop(op(a, b)) in one pass (uop: relu, neg or abs), bit-identical to the two eager ops; a and b
    share one dtype."""
    codes = {"add": C.ADD, "sub": C.SUB, "mul": C.MUL, "div": C.DIV}
    ucodes = {"relu": C.RELU, "neg": C.NEG, "abs": C.ABS}
    dev = _cuda("binary_unary", a, b)
    out = torch.empty(broadcast_shape(a.shape, b.shape), dtype=a.dtype, device=dev)
    with torch.cuda.device(dev):
        _call(C.lib.ctb_binary_unary(codes[op], ucodes[uop], C.view(a), C.view(b), C.view(out),
                                     C.stream_handle(dev)), "binary_unary")
    return out


def chain_rows(op1: str, op2: str, a, b, c, row_op: str = "min", write_y: bool = True,
               want_sum: bool = True, out_sum: torch.Tensor | None = None):
    """One pass over a [rows, cols] matrix: y = op2(op1(a, b), c) with b, c one broadcast row,
    plus the per-row argmin/argmax of y and the float64 sum of y (ctb_chain_rows). Returns
    (y or None, row indices int64 [rows], float64 sum tensor [1] or None). y and the indices are
    bit-identical to the eager ops; the sum matches to float64 rounding."""
    codes = {"add": C.ADD, "sub": C.SUB, "mul": C.MUL, "div": C.DIV}
    dev = _cuda("chain_rows", a, b, c)
    y = torch.empty(a.shape, dtype=a.dtype, device=dev) if write_y else None
    idx = torch.empty(a.shape[0], dtype=torch.int64, device=dev)
    s = None
    if want_sum:
        s = out_sum if out_sum is not None else torch.empty(1, dtype=torch.float64, device=dev)
    rop = C.MIN if row_op == "min" else C.MAX
    with torch.cuda.device(dev):
        va, vb, vc, vy, vi = C.view(a), C.view(b), C.view(c), C.view(y), C.view(idx)
        need = C.lib.ctb_chain_rows_scratch_bytes(codes[op1], codes[op2], va, vb, vc, vy, rop, vi) if want_sum else 0
        scratch = _scratch(need, dev)
        _call(C.lib.ctb_chain_rows(codes[op1], codes[op2], va, vb, vc, vy, rop, vi,
                                   s.data_ptr() if s is not None else None,
                                   scratch.data_ptr() if scratch is not None else None, need,
                                   C.stream_handle(dev)), "chain_rows")
    return y, idx, s


def _unary(op: int, x: torch.Tensor, name: str) -> torch.Tensor:
    dev = _cuda(name, x)
    out = torch.empty(x.shape, dtype=x.dtype, device=dev)
    with torch.cuda.device(dev):
        _call(C.lib.ctb_unary(op, C.view(x), C.view(out), C.stream_handle(dev)), name)
    return out


def cast(x: torch.Tensor, dtype) -> torch.Tensor:
    """x converted to `dtype` (a new contiguous tensor; x itself when the dtype already matches
    and x is contiguous), with ctorch's cast semantics (src/ops/cast_cpu.cpp:21-90) computed on
    the GPU. This is the device-side cast that ctorch's CUDA promotion does through the host
    (src/ops/binary_ops_cpu.cpp:154-184), and it also takes non-contiguous views."""
    dev = _cuda("cast", x)
    if dtype not in C.CODE_OF_TORCH or x.dtype not in C.CODE_OF_TORCH:
        raise DTypeError(f"ctorch: cast from {x.dtype} to {dtype} is not supported")
    if dtype == x.dtype and x.is_contiguous():
        return x
    out = torch.empty(x.shape, dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        _call(C.lib.ctb_cast(C.view(x), C.view(out), C.stream_handle(dev)), "cast")
    return out


def contiguous(x: torch.Tensor) -> torch.Tensor:
    """A contiguous copy of a strided CUDA view, made on the device (ctorch's Tensor::contiguous,
    src/tensor.cpp:239-254, materialises strided tensors on the CPU only); x itself when it is
    already contiguous."""
    return cast(x, x.dtype)


def neg(x):
    return _unary(C.NEG, x, "neg")


def abs(x):  # noqa: A001 - ctorch's name
    return _unary(C.ABS, x, "abs")


def exp(x):
    return _unary(C.EXP, x, "exp")


def log(x):
    return _unary(C.LOG, x, "log")


def sqrt(x):
    return _unary(C.SQRT, x, "sqrt")


def relu(x):
    return _unary(C.RELU, x, "relu")


def sigmoid(x):
    return _unary(C.SIGMOID, x, "sigmoid")


def tanh(x):
    return _unary(C.TANH, x, "tanh")


# ---------------------------------------------------------------- reductions


def _reject_bf16(x, name):
    if x.dtype == torch.bfloat16:
        raise DTypeError(f"ctorch::{name}: bfloat16 is not supported")


def _normalise_axis(dim: int, rank: int) -> int:
    d = dim + rank if dim < 0 else dim
    if d < 0 or d >= rank:
        raise ShapeError(f"ctorch::reduction: axis {dim} out of range for tensor of rank {rank}")
    return d


def _canonicalise(x: torch.Tensor, dims) -> int:
    """src/ops/reduction.cpp:52-88: returns the reduce mask (empty dims = every axis)."""
    rank = x.dim()
    if rank > C.MAX_DIMS:
        raise ShapeError("ctorch: tensor rank exceeds kMaxRank")
    if not dims:
        return (1 << rank) - 1
    mask = 0
    for raw in dims:
        d = _normalise_axis(int(raw), rank)
        if mask >> d & 1:
            raise ShapeError(f"ctorch: duplicate axis {d} in reduction dims")
        mask |= 1 << d
    return mask


def _reduced_shape(x, mask, keepdim):
    return tuple((1 if keepdim else None) if mask >> d & 1 else s
                 for d, s in enumerate(x.shape) if not (mask >> d & 1 and not keepdim))


def _scratch(nbytes: int, dev) -> torch.Tensor | None:
    return torch.empty(nbytes, dtype=torch.uint8, device=dev) if nbytes else None


def _reduce(op: int, x: torch.Tensor, dims, keepdim: bool, name: str, out_dtype) -> torch.Tensor:
    dev = _cuda(name, x)
    _reject_bf16(x, name)
    mask = _canonicalise(x, dims)
    out = torch.empty(_reduced_shape(x, mask, keepdim), dtype=out_dtype, device=dev)
    with torch.cuda.device(dev):
        vx, vo = C.view(x), C.view(out)
        need = C.lib.ctb_reduce_scratch_bytes(op, vx, vo, mask)
        scratch = _scratch(need, dev)
        _call(C.lib.ctb_reduce(op, vx, vo, mask, scratch.data_ptr() if scratch is not None else None,
                               need, C.stream_handle(dev)), name)
    return out


def _sum_dtype(dt):
    # src/ops/reduction.cpp:131-144
    return dt if dt in (torch.float32, torch.float64) else torch.int64


def sum(x, dims=None, keepdim=False):  # noqa: A001 - ctorch's name
    return _reduce(C.SUM, x, dims, keepdim, "sum", _sum_dtype(x.dtype))


def prod(x, dims=None, keepdim=False):
    return _reduce(C.PROD, x, dims, keepdim, "prod", _sum_dtype(x.dtype))


def mean(x, dims=None, keepdim=False):
    if x.dtype not in (torch.float32, torch.float64, torch.bfloat16):
        raise DTypeError("ctorch::mean: requires a floating dtype input (cast int/bool to float first)")
    return _reduce(C.MEAN, x, dims, keepdim, "mean", x.dtype)


def _maxmin_values(op, x, dims, keepdim, name):
    # src/ops/reduction_ops_cpu.cpp:416-428: no identity for an empty slice
    _reject_bf16(x, name)
    mask = _canonicalise(x, dims)
    red = 1
    for d, s in enumerate(x.shape):
        if mask >> d & 1:
            red *= s
    if red == 0:
        raise ShapeError(f"ctorch::{name}: cannot reduce a zero-element slice (operation has no identity)")
    return _reduce(op, x, dims, keepdim, name, x.dtype)


def _single_axis(x, dim, name):
    # src/ops/reduction.cpp:90-97 and reduction_ops_cpu.cpp:433-436
    if x.dim() == 0:
        raise ShapeError("ctorch: cannot reduce a 0-d tensor along a single axis "
                         "(use the whole-tensor form instead)")
    axis = _normalise_axis(int(dim), x.dim())
    if x.shape[axis] == 0:
        raise ShapeError(f"ctorch::{name}: cannot reduce a zero-length axis (operation has no identity)")
    return axis


def _with_index(op, x, dim, keepdim, name, values: bool):
    dev = _cuda(name, x)
    _reject_bf16(x, name)
    axis = _single_axis(x, dim, name)
    shape = _reduced_shape(x, 1 << axis, keepdim)
    vals = torch.empty(shape, dtype=x.dtype, device=dev) if values else None
    idx = torch.empty(shape, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        vx = C.view(x)
        need = C.lib.ctb_reduce_index_scratch_bytes(vx, axis)
        scratch = _scratch(need, dev)
        _call(C.lib.ctb_reduce_index(op, vx, C.view(vals), C.view(idx), axis,
                                     scratch.data_ptr() if scratch is not None else None, need,
                                     C.stream_handle(dev)), name)
    return ValuesIndices(vals, idx) if values else idx


def max(x, dims=None, keepdim=False):  # noqa: A001 - ctorch's name
    """max(x) / max(x, [dims], keepdim) -> values; max(x, dim:int, keepdim) -> (values, indices)."""
    if isinstance(dims, int):
        return _with_index(C.MAX, x, dims, keepdim, "max", True)
    return _maxmin_values(C.MAX, x, dims, keepdim, "max")


def min(x, dims=None, keepdim=False):  # noqa: A001 - ctorch's name
    if isinstance(dims, int):
        return _with_index(C.MIN, x, dims, keepdim, "min", True)
    return _maxmin_values(C.MIN, x, dims, keepdim, "min")


def argmax(x, dim: int, keepdim=False):
    return _with_index(C.MAX, x, dim, keepdim, "argmax", False)


def argmin(x, dim: int, keepdim=False):
    return _with_index(C.MIN, x, dim, keepdim, "argmin", False)


# ---------------------------------------------------------------- indexing


def index_select_async(src: torch.Tensor, dim: int, indices: torch.Tensor):
    """Enqueue the gather and return (out, status): status[0:4] (int32) is nonzero if an index was
    out of range, in which case out was not written. No host synchronisation."""
    # src/ops/indexing_cpu.cpp:163-200
    if indices.dim() != 1:
        raise ShapeError(f"ctorch::index_select: indices must be 1-D (got rank {indices.dim()})")
    if indices.dtype not in (torch.int32, torch.int64):
        raise DTypeError("ctorch::index_select: indices dtype must be int32 or int64")
    if src.device != indices.device:
        raise DeviceError("ctorch::index_select: src and indices must live on the same device")
    dev = _cuda("index_select", src, indices)
    if src.dtype == torch.bfloat16:
        raise DTypeError("ctorch::index_select: bfloat16 is not supported")
    rank = src.dim()
    if rank == 0:
        raise ShapeError("ctorch::index_select: cannot index a 0-d tensor")
    adj = dim + rank if dim < 0 else dim
    if adj < 0 or adj >= rank:
        raise ShapeError(f"ctorch::index_select: dim {dim} out of range for tensor of rank {rank}")
    shape = list(src.shape)
    shape[adj] = indices.shape[0]
    out = torch.empty(shape, dtype=src.dtype, device=dev)
    status = torch.empty(16, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _call(C.lib.ctb_index_select(C.view(src), adj, C.view(indices), C.view(out),
                                     status.data_ptr(), C.stream_handle(dev)), "index_select")
    return out, status


def index_select(src: torch.Tensor, dim: int, indices: torch.Tensor) -> torch.Tensor:
    """Gather along `dim`; raises ShapeError (after synchronising) if any index is out of range."""
    out, status = index_select_async(src, dim, indices)
    st = status.cpu()
    if int(st[:4].view(torch.int32)[0]) != 0:
        bad = int(st[8:16].view(torch.int64)[0])
        size = src.shape[dim + src.dim() if dim < 0 else dim]
        raise ShapeError(f"ctorch::index_select: index {bad} out of range for dim {dim} of size {size}")
    return out


def launch_count() -> int:
    """Kernels this thread has launched through the library (see ctb_launch_count)."""
    return int(C.lib.ctb_launch_count())


def launch_count_reset() -> None:
    C.lib.ctb_launch_count_reset()
