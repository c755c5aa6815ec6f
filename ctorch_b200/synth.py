"""Seeded synthetic inputs (no dataset exists for this path; shapes and value distributions follow
the benchmark configurations).

Element i of (seed, stream) is derived from h = splitmix64(key + i) with
key = splitmix64(splitmix64(seed) ^ stream) (splitmix64: Steele, Lea & Flood, "Fast splittable
pseudorandom number generators", OOPSLA 2014). Uniform floats take the top 24 bits,
u = (h >> 40) * 2^-24, and lo + (hi - lo) * u evaluated in double then rounded once to the dtype;
integer uniforms are lo + h mod (hi - lo + 1); normals use Box-Muller on two 53-bit uniforms.
`device_fill` runs the generator on the GPU (ctb_fill_random); `host_fill` is the numpy twin
(bit-identical for the uniform kinds; normals agree to the last bit of the double almost always,
so the rounded float32 values match). `first` is the global index of element 0, so a row shard
generated alone equals the same rows of the whole tensor.
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0x9E3779B97F4A7C15)
_M2 = np.uint64(0xBF58476D1CE4E5B9)
_M3 = np.uint64(0x94D049BB133111EB)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + _M1
        z = (z ^ (z >> np.uint64(30))) * _M2
        z = (z ^ (z >> np.uint64(27))) * _M3
        return z ^ (z >> np.uint64(31))


def _key(seed: int, stream: int) -> np.uint64:
    s = _splitmix64(np.array([seed], dtype=np.uint64))[0]
    return _splitmix64(np.array([s ^ np.uint64(stream)], dtype=np.uint64))[0]


UNIFORM, NORMAL = 0, 1


def host_fill(shape, dtype, dist: int, seed: int, stream: int, lo: float, hi: float,
              first: int = 0, chunk: int = 1 << 24) -> np.ndarray:
    dtype = np.dtype(dtype)
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=dtype)
    key = _key(seed, stream)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        with np.errstate(over="ignore"):
            h = _splitmix64(key + np.arange(first + s, first + e, dtype=np.uint64))
        if dtype.kind == "f":
            if dist == UNIFORM:
                u = (h >> np.uint64(40)).astype(np.float64) * 2.0**-24
                v = lo + (hi - lo) * u
            else:
                u1 = ((h >> np.uint64(11)) + np.uint64(1)).astype(np.float64) * 2.0**-53
                u2 = (_splitmix64(h) >> np.uint64(11)).astype(np.float64) * 2.0**-53
                z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
                v = lo + hi * z
            out[s:e] = v.astype(dtype)
        else:
            if dist != UNIFORM:
                raise ValueError("normal fill needs a float dtype")
            a, b = int(lo), int(hi)
            rng = np.uint64(b - a + 1)
            r = h % rng
            with np.errstate(over="ignore"):
                out[s:e] = (np.uint64(a % 2**64) + r).astype(np.int64).astype(dtype)
    return out.reshape(shape)


def device_fill(t, dist: int, seed: int, stream: int, lo: float, hi: float, first: int = 0):
    """Fills a contiguous CUDA tensor in place with the same sequence as host_fill."""
    import torch

    from . import _capi as C

    assert t.is_cuda and t.is_contiguous()
    with torch.cuda.device(t.device):
        rc = C.lib.ctb_fill_random(C.view(t), dist, seed, stream, first, float(lo), float(hi),
                                   C.stream_handle(t.device))
    if rc != C.OK:
        raise RuntimeError(f"ctb_fill_random: {C.last_error()}")
    return t
