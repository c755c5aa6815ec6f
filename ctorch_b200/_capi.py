"""ctypes binding of include/ctb/ctb.h (libctb_cuda.so, built in-tree by ctorch_b200/csrc/Makefile).

Importing this module loads the library and fails loudly if it has not been built: the package
has no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libctb_cuda.so")

MAX_DIMS = 16
ABI_VERSION = 1

# dtype codes (ctorch::dtype enumerator order)
F32, F64, I32, I64, BOOL, BF16 = 0, 1, 2, 3, 4, 5
CODE_OF_TORCH = {
    torch.float32: F32,
    torch.float64: F64,
    torch.int32: I32,
    torch.int64: I64,
    torch.bool: BOOL,
    torch.bfloat16: BF16,
}
TORCH_OF_CODE = {v: k for k, v in CODE_OF_TORCH.items()}

# status codes
OK, ERR_DTYPE, ERR_SHAPE, ERR_INDEX, ERR_CUDA, ERR_ARGUMENT, ERR_SCRATCH = range(7)

ADD, SUB, MUL, DIV = range(4)
NEG, ABS, EXP, LOG, SQRT, RELU, SIGMOID, TANH = range(8)
SUM, MEAN, PROD, MAX, MIN = range(5)


class View(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("strides", ctypes.c_int64 * MAX_DIMS),
    ]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C ctorch_b200/csrc` "
            "(or __graft_entry__.build()); ctorch_b200 has no CPU fallback"
        )
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER(View)
    vp, sz, i32, i64, u32, u64 = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int64,
                                  ctypes.c_uint32, ctypes.c_uint64)
    sigs = {
        "ctb_abi_version": (i32, []),
        "ctb_last_error": (ctypes.c_char_p, []),
        "ctb_launch_count": (u64, []),
        "ctb_launch_count_reset": (None, []),
        "ctb_binary": (i32, [i32, P, P, P, vp]),
        "ctb_binary_chain": (i32, [i32, i32, P, P, P, ctypes.c_int32, P, vp]),
        "ctb_unary": (i32, [i32, P, P, vp]),
        "ctb_cast": (i32, [P, P, vp]),
        "ctb_binary_unary": (i32, [i32, i32, P, P, P, vp]),
        "ctb_reduce_scratch_bytes": (sz, [i32, P, P, u32]),
        "ctb_reduce": (i32, [i32, P, P, u32, vp, sz, vp]),
        "ctb_reduce_noalloc": (i32, [i32, P, P, u32, vp]),
        "ctb_reduce_index_scratch_bytes": (sz, [P, i32]),
        "ctb_reduce_index": (i32, [i32, P, P, P, i32, vp, sz, vp]),
        "ctb_index_select": (i32, [P, i32, P, P, vp, vp]),
        "ctb_chain_rows_scratch_bytes": (sz, [i32, i32, P, P, P, P, i32, P]),
        "ctb_chain_rows": (i32, [i32, i32, P, P, P, P, i32, P, vp, vp, sz, vp]),
        "ctb_sum_partial_scratch_bytes": (sz, [P]),
        "ctb_sum_partial": (i32, [P, vp, vp, sz, vp]),
        "ctb_sum_combine": (i32, [vp, i32, P, vp]),
        "ctb_minmax_combine": (i32, [i32, P, P, vp, P, P, vp]),
        "ctb_peer_workspace_bytes": (sz, []),
        "ctb_peer_alloc": (i32, [ctypes.POINTER(vp), vp]),
        "ctb_peer_open": (i32, [vp, ctypes.POINTER(vp)]),
        "ctb_peer_close": (i32, [vp]),
        "ctb_peer_free": (i32, [vp]),
        "ctb_peer_status": (i32, [vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
        "ctb_peer_trace": (i32, [vp, ctypes.POINTER(ctypes.c_uint64)]),
        "ctb_chain_rows_allsum": (i32, [i32, i32, P, P, P, P, i32, P, vp, vp, i32, i32, u64, P, vp, u64, vp]),
        "ctb_fill_random": (i32, [P, i32, u64, u64, i64, ctypes.c_double, ctypes.c_double, vp]),
        "ctb_debug_plan_elementwise": (i32, [P, ctypes.POINTER(P), i32, i32, ctypes.c_char_p, i32,
                                             ctypes.POINTER(ctypes.c_int),
                                             ctypes.POINTER(ctypes.c_int64)]),
        "ctb_debug_plan_reduction": (i32, [P, P, u32, ctypes.c_char_p, i32,
                                           ctypes.POINTER(ctypes.c_int),
                                           ctypes.POINTER(ctypes.c_int)]),
        "ctb_debug_fastdiv": (u64, [u64, u64]),
        "ctb_debug_strip_geometry": (i32, [i64, i64, i64, i64, ctypes.POINTER(ctypes.c_int64),
                                           ctypes.POINTER(ctypes.c_int64)]),
        "ctb_debug_last_reduction_kernel": (i32, [ctypes.c_char_p, i32]),
        "ctb_debug_noalloc_fits": (i32, [sz]),
        "ctb_wait_timeouts": (i32, [ctypes.POINTER(ctypes.c_uint64)]),
        "ctb_debug_wait_timeout": (i32, [u64, ctypes.POINTER(ctypes.c_int)]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.ctb_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH}: ABI version {lib.ctb_abi_version()} != {ABI_VERSION}")
    return lib


lib = _load()


def last_reduction_kernel():
    """Name of the first kernel the calling thread's last reduction launched."""
    buf = ctypes.create_string_buffer(64)
    lib.ctb_debug_last_reduction_kernel(buf, 64)
    return buf.value.decode()


def last_error() -> str:
    return lib.ctb_last_error().decode(errors="replace")


def view(t: torch.Tensor | None) -> View | None:
    """Describe a tensor for the C ABI (data pointer already includes the storage offset)."""
    if t is None:
        return None
    v = View()
    v.data = t.data_ptr()
    v.dtype = CODE_OF_TORCH[t.dtype]
    v.ndim = t.dim()
    if t.dim() > MAX_DIMS:
        v.ndim = t.dim()  # rejected by the library with CTB_ERR_SHAPE
        return v
    for d, (s, st) in enumerate(zip(t.shape, t.stride())):
        v.shape[d] = s
        v.strides[d] = st
    return v


def stream_handle(device: torch.device | None = None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def wait_timeouts() -> int:
    """Timed-out waits counted on the current device (ctb_wait_timeouts); 0 on a healthy GPU."""
    n = ctypes.c_uint64(0)
    rc = lib.ctb_wait_timeouts(ctypes.byref(n))
    if rc != OK:
        raise RuntimeError(last_error())
    return n.value
