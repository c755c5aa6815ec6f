"""ctorch_b200 — B200 (sm_100a) CUDA backend for ctorch's eager tensor-op hot path.

The kernels live in libctb_cuda.so behind the C ABI of include/ctb/ctb.h. Two hosts sit on top
of that ABI:
  * ctorch_plugin/cuda_backend.cpp — the C++ drop-in for ctorch itself: it defines ctorch's four
    CUDA registration hooks and fills every CUDA dispatch slot;
  * this package — the same ops for torch CUDA tensors (ops.py mirrors ctorch's public API and
    error types), plus the row-sharded multi-GPU workload (sharded.py).
"""
from .errors import AliasError, CommTimeoutError, DeviceError, DTypeError, Error, ShapeError  # noqa: F401
from .ops import (  # noqa: F401
    ValuesIndices,
    abs,
    add,
    add_,
    argmax,
    argmin,
    binary_chain,
    binary_unary,
    broadcast_shape,
    cast,
    chain_rows,
    contiguous,
    div,
    div_,
    exp,
    index_select,
    index_select_async,
    launch_count,
    launch_count_reset,
    log,
    max,
    mean,
    min,
    mul,
    mul_,
    neg,
    prod,
    promote_types,
    relu,
    sigmoid,
    sqrt,
    sub,
    sub_,
    sum,
    tanh,
)

__all__ = [n for n in dir() if not n.startswith("_")]
