"""ctypes view of the reference's C++ CPU kernels built by ``oracle/Makefile``.

TEST INFRASTRUCTURE ONLY.  ``load()`` returns ``None`` when ``oracle/_ref`` has
not been built (the reference checkout is needed to build it).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libfluxref_cpu.so"
_F = ctypes.POINTER(ctypes.c_float)


def load():
    if not LIB.exists():
        return None
    lib = ctypes.CDLL(str(LIB))
    lib.fxref_rmsnorm_fp32.argtypes = [_F, _F, _F, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float]
    lib.fxref_residual_rmsnorm_fp32.argtypes = [_F, _F, _F, _F, _F, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float]
    lib.fxref_packed_swiglu_fp32.argtypes = [_F, _F, ctypes.c_size_t, ctypes.c_size_t]
    return lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(_F)


def rmsnorm(lib, x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    assert lib.fxref_rmsnorm_fp32(_p(x), _p(w), _p(out), x.size // x.shape[-1], x.shape[-1], eps) == 0
    return out


def residual_rmsnorm(lib, h, r, w, eps):
    h = np.ascontiguousarray(h, np.float32)
    r = np.ascontiguousarray(r, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    norm, res = np.empty_like(h), np.empty_like(h)
    assert lib.fxref_residual_rmsnorm_fp32(_p(h), _p(r), _p(w), _p(norm), _p(res),
                                           h.size // h.shape[-1], h.shape[-1], eps) == 0
    return norm, res


def packed_swiglu(lib, packed):
    packed = np.ascontiguousarray(packed, np.float32)
    half = packed.shape[-1] // 2
    out = np.empty(packed.shape[:-1] + (half,), np.float32)
    assert lib.fxref_packed_swiglu_fp32(_p(packed), _p(out), packed.size // packed.shape[-1], half) == 0
    return out
