"""Python access to the checkers in oracle/ (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import this
module, and only as the checker or as the timed CPU baseline. The ctorch_b200 product never
imports it.

Two checkers live here:

* ``Oracle`` wraps ``liboracle.so``, the C restatement of ctorch's CPU backend
  (``ctb_oracle.c``; each function cites the ctorch file:line it restates). It works on any
  strided numpy view, so the same bytes can be handed to the CUDA backend and to the oracle.
* ``Ref`` wraps ``_ref/libctorch_ref.so``, ctorch's own CPU backend compiled from its sources,
  driven through ctorch's public front-doors with ctorch's own view ops (permute / slice /
  select). It pins the restatement and is the timed reference arm of bench.py.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libctorch_ref.so")

MAX_DIMS = 16

# dtype codes: enumerator order of ctorch::dtype (include/ctorch/dtype.h:24-31)
F32, F64, I32, I64, BOOL = 0, 1, 2, 3, 4
NP_OF_CODE = {F32: np.float32, F64: np.float64, I32: np.int32, I64: np.int64, BOOL: np.bool_}
CODE_OF_NP = {np.dtype(v): k for k, v in NP_OF_CODE.items()}

BINARY_OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3}
UNARY_OPS = {"neg": 0, "abs": 1, "exp": 2, "log": 3, "sqrt": 4, "relu": 5, "sigmoid": 6, "tanh": 7}
REDUCE_OPS = {"sum": 0, "mean": 1, "prod": 2, "max": 3, "min": 4}

OK, ERR_DTYPE, ERR_SHAPE, ERR_INDEX = 0, 1, 2, 3


class OracleError(Exception):
    def __init__(self, code: int, what: str = ""):
        super().__init__(f"oracle status {code} {what}")
        self.code = code


class OrcView(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("strides", ctypes.c_int64 * MAX_DIMS),
    ]


def code_of(dtype) -> int:
    return CODE_OF_NP[np.dtype(dtype)]


def promote(a, b):
    """ctorch's promotion lattice (src/type_promotion.cpp:45-62) on numpy dtypes."""
    order = [np.dtype(np.bool_), np.dtype(np.int32), np.dtype(np.int64), np.dtype(np.float32),
             np.dtype(np.float64)]
    return max(np.dtype(a), np.dtype(b), key=order.index)


def make_view(arr: np.ndarray) -> OrcView:
    """Describe a (possibly strided / broadcast) numpy array; strides converted to elements."""
    v = OrcView()
    v.data = arr.__array_interface__["data"][0]
    v.dtype = code_of(arr.dtype)
    v.ndim = arr.ndim
    es = arr.dtype.itemsize
    for d in range(arr.ndim):
        v.shape[d] = arr.shape[d]
        assert arr.strides[d] % es == 0
        v.strides[d] = arr.strides[d] // es
    return v


def broadcast_shape(sa, sb):
    r = max(len(sa), len(sb))
    sa = (1,) * (r - len(sa)) + tuple(sa)
    sb = (1,) * (r - len(sb)) + tuple(sb)
    out = []
    for x, y in zip(sa, sb):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise OracleError(ERR_SHAPE, "broadcast")
    return tuple(out)


class Oracle:
    """The C restatement (liboracle.so)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built: run `make -C oracle oracle`")
        lib = ctypes.CDLL(path)
        P = ctypes.POINTER(OrcView)
        lib.orc_binary.argtypes = [ctypes.c_int, P, P, P]
        lib.orc_unary.argtypes = [ctypes.c_int, P, P]
        lib.orc_cast.argtypes = [P, P]
        lib.orc_reduce.argtypes = [ctypes.c_int, P, P, ctypes.c_uint32]
        lib.orc_reduce_idx.argtypes = [ctypes.c_int, P, P, P, ctypes.c_int]
        lib.orc_index_select.argtypes = [P, ctypes.c_int, P, P, ctypes.POINTER(ctypes.c_int64)]
        for f in ("orc_binary", "orc_unary", "orc_cast", "orc_reduce", "orc_reduce_idx", "orc_index_select"):
            getattr(lib, f).restype = ctypes.c_int
        self.lib = lib

    @staticmethod
    def _check(st, what=""):
        if st != OK:
            raise OracleError(st, what)

    def binary(self, op: str, a: np.ndarray, b: np.ndarray, out_dtype=None) -> np.ndarray:
        shape = broadcast_shape(a.shape, b.shape)
        out = np.empty(shape, dtype=out_dtype or promote(a.dtype, b.dtype))
        self._check(self.lib.orc_binary(BINARY_OPS[op], make_view(a), make_view(b),
                                        make_view(out)), op)
        return out

    def unary(self, op: str, x: np.ndarray) -> np.ndarray:
        out = np.empty(x.shape, dtype=x.dtype)
        self._check(self.lib.orc_unary(UNARY_OPS[op], make_view(x), make_view(out)), op)
        return out

    def cast(self, x: np.ndarray, dtype) -> np.ndarray:
        out = np.empty(x.shape, dtype=dtype)
        self._check(self.lib.orc_cast(make_view(x), make_view(out)), "cast")
        return out

    @staticmethod
    def reduce_out_dtype(op: str, dt):
        dt = np.dtype(dt)
        if op in ("sum", "prod"):
            return dt if dt.kind == "f" else np.dtype(np.int64)
        return dt

    @staticmethod
    def reduce_mask(ndim, dims):
        if dims is None:
            return (1 << ndim) - 1 if ndim else 0
        m = 0
        for d in dims:
            m |= 1 << (d % ndim)
        return m

    def reduce(self, op: str, x: np.ndarray, dims=None, keepdim=False) -> np.ndarray:
        mask = self.reduce_mask(x.ndim, dims)
        if keepdim:
            shape = tuple(1 if (mask >> d) & 1 else s for d, s in enumerate(x.shape))
        else:
            shape = tuple(s for d, s in enumerate(x.shape) if not (mask >> d) & 1)
        out = np.empty(shape, dtype=self.reduce_out_dtype(op, x.dtype))
        self._check(self.lib.orc_reduce(REDUCE_OPS[op], make_view(x), make_view(out), mask), op)
        return out

    def reduce_idx(self, op: str, x: np.ndarray, dim: int, keepdim=False, values=True):
        axis = dim % x.ndim
        shape = tuple((1 if keepdim else None) if d == axis else s for d, s in enumerate(x.shape))
        shape = tuple(s for s in shape if s is not None)
        idx = np.empty(shape, dtype=np.int64)
        vals = np.empty(shape, dtype=x.dtype) if values else None
        st = self.lib.orc_reduce_idx(REDUCE_OPS[op], make_view(x),
                                     make_view(vals) if values else None, make_view(idx), axis)
        self._check(st, op)
        return (vals, idx) if values else idx

    def index_select(self, src: np.ndarray, dim: int, idx: np.ndarray) -> np.ndarray:
        dim = dim % src.ndim
        shape = list(src.shape)
        shape[dim] = idx.shape[0]
        out = np.empty(shape, dtype=src.dtype)
        bad = ctypes.c_int64(0)
        st = self.lib.orc_index_select(make_view(src), dim, make_view(idx), make_view(out),
                                       ctypes.byref(bad))
        self._check(st, f"index_select bad index {bad.value}")
        return out


class RefError(Exception):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ctorch error {code}: {msg}")
        self.code = code


class Ref:
    """ctorch's own CPU backend (oracle/_ref/libctorch_ref.so), through its public API."""

    ERR_DTYPE, ERR_SHAPE = 1, 2

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built: run `make -C oracle ref`")
        lib = ctypes.CDLL(path)
        vp, ip, i64p = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64)
        lib.ref_last_error.restype = ctypes.c_char_p
        lib.ref_tensor_from.argtypes = [ctypes.c_int, ctypes.c_int, i64p, vp, ip]
        lib.ref_tensor_from.restype = vp
        lib.ref_free.argtypes = [vp]
        lib.ref_ndim.argtypes = [vp]
        lib.ref_dtype.argtypes = [vp]
        lib.ref_shape.argtypes = [vp, i64p]
        lib.ref_strides.argtypes = [vp, i64p]
        lib.ref_offset.argtypes = [vp]
        lib.ref_offset.restype = ctypes.c_int64
        lib.ref_read.argtypes = [vp, vp]
        lib.ref_permute.argtypes = [vp, ctypes.c_int, i64p, ip]
        lib.ref_permute.restype = vp
        lib.ref_slice.argtypes = [vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int64, ip]
        lib.ref_slice.restype = vp
        lib.ref_select.argtypes = [vp, ctypes.c_int, ctypes.c_int64, ip]
        lib.ref_select.restype = vp
        lib.ref_reshape.argtypes = [vp, ctypes.c_int, i64p, ip]
        lib.ref_reshape.restype = vp
        lib.ref_binary.argtypes = [ctypes.c_int, vp, vp, ip]
        lib.ref_binary.restype = vp
        lib.ref_binary_inplace.argtypes = [ctypes.c_int, vp, vp]
        lib.ref_unary.argtypes = [ctypes.c_int, vp, ip]
        lib.ref_unary.restype = vp
        lib.ref_reduce.argtypes = [ctypes.c_int, vp, ctypes.c_int, i64p, ctypes.c_int, ip]
        lib.ref_reduce.restype = vp
        lib.ref_reduce_idx.argtypes = [ctypes.c_int, vp, ctypes.c_int64, ctypes.c_int,
                                       ctypes.POINTER(vp), ip]
        lib.ref_reduce_idx.restype = vp
        lib.ref_arg.argtypes = [ctypes.c_int, vp, ctypes.c_int64, ctypes.c_int, ip]
        lib.ref_arg.restype = vp
        lib.ref_cast.argtypes = [vp, ctypes.c_int, ip]
        lib.ref_cast.restype = vp
        lib.ref_index_select.argtypes = [vp, ctypes.c_int, vp, ip]
        lib.ref_index_select.restype = vp
        self.lib = lib

    def _wrap(self, h, err):
        if err.value != 0 or not h:
            raise RefError(err.value, self.lib.ref_last_error().decode())
        return RefTensor(self, h)

    def tensor(self, arr: np.ndarray) -> "RefTensor":
        arr = np.ascontiguousarray(arr)
        shape = (ctypes.c_int64 * max(1, arr.ndim))(*arr.shape)
        err = ctypes.c_int(0)
        h = self.lib.ref_tensor_from(code_of(arr.dtype), arr.ndim, shape,
                                     arr.__array_interface__["data"][0], ctypes.byref(err))
        return self._wrap(h, err)

    def cast(self, a, dtype):
        err = ctypes.c_int(0)
        return self._wrap(self.lib.ref_cast(a.h, code_of(np.dtype(dtype)), ctypes.byref(err)), err)

    def binary(self, op, a, b):
        err = ctypes.c_int(0)
        return self._wrap(self.lib.ref_binary(BINARY_OPS[op], a.h, b.h, ctypes.byref(err)), err)

    def binary_inplace(self, op, a, b):
        st = self.lib.ref_binary_inplace(BINARY_OPS[op], a.h, b.h)
        if st:
            raise RefError(st, self.lib.ref_last_error().decode())
        return a

    def unary(self, op, a):
        err = ctypes.c_int(0)
        return self._wrap(self.lib.ref_unary(UNARY_OPS[op], a.h, ctypes.byref(err)), err)

    def reduce(self, op, a, dims=None, keepdim=False):
        err = ctypes.c_int(0)
        if dims is None:
            h = self.lib.ref_reduce(REDUCE_OPS[op], a.h, -1, None, 0, ctypes.byref(err))
        else:
            d = (ctypes.c_int64 * max(1, len(dims)))(*dims)
            h = self.lib.ref_reduce(REDUCE_OPS[op], a.h, len(dims), d, int(keepdim),
                                    ctypes.byref(err))
        return self._wrap(h, err)

    def reduce_idx(self, op, a, dim, keepdim=False):
        err = ctypes.c_int(0)
        ih = ctypes.c_void_p(0)
        vh = self.lib.ref_reduce_idx(REDUCE_OPS[op], a.h, dim, int(keepdim), ctypes.byref(ih),
                                     ctypes.byref(err))
        v = self._wrap(vh, err)
        return v, RefTensor(self, ih.value)

    def arg(self, op, a, dim, keepdim=False):
        err = ctypes.c_int(0)
        code = REDUCE_OPS["max" if op == "argmax" else "min"]
        return self._wrap(self.lib.ref_arg(code, a.h, dim, int(keepdim), ctypes.byref(err)), err)

    def index_select(self, src, dim, idx):
        err = ctypes.c_int(0)
        return self._wrap(self.lib.ref_index_select(src.h, dim, idx.h, ctypes.byref(err)), err)


class RefTensor:
    def __init__(self, ref: Ref, h):
        self.ref, self.h = ref, h

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ref_free(self.h)
            self.h = None

    @property
    def ndim(self):
        return self.ref.lib.ref_ndim(self.h)

    @property
    def shape(self):
        n = self.ndim
        buf = (ctypes.c_int64 * max(1, n))()
        self.ref.lib.ref_shape(self.h, buf)
        return tuple(buf[:n])

    @property
    def strides(self):
        n = self.ndim
        buf = (ctypes.c_int64 * max(1, n))()
        self.ref.lib.ref_strides(self.h, buf)
        return tuple(buf[:n])

    @property
    def dtype(self):
        return np.dtype(NP_OF_CODE[self.ref.lib.ref_dtype(self.h)])

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        st = self.ref.lib.ref_read(self.h, out.__array_interface__["data"][0])
        if st:
            raise RefError(st, self.ref.lib.ref_last_error().decode())
        return out

    def _view(self, fn, *args):
        err = ctypes.c_int(0)
        return self.ref._wrap(fn(self.h, *args, ctypes.byref(err)), err)

    def permute(self, dims):
        d = (ctypes.c_int64 * len(dims))(*dims)
        return self._view(self.ref.lib.ref_permute, len(dims), d)

    def slice(self, dim, start, end, step=1):
        return self._view(self.ref.lib.ref_slice, dim, start, end, step)

    def select(self, dim, index):
        return self._view(self.ref.lib.ref_select, dim, index)

    def reshape(self, shape):
        s = (ctypes.c_int64 * max(1, len(shape)))(*shape)
        return self._view(self.ref.lib.ref_reshape, len(shape), s)


_ORACLE = None
_REF = None


def oracle() -> Oracle:
    global _ORACLE
    if _ORACLE is None:
        _ORACLE = Oracle()
    return _ORACLE


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> Ref:
    global _REF
    if _REF is None:
        _REF = Ref()
    return _REF
