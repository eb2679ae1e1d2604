"""ctypes loader of the oracle's C quantiser (oracle/quant_ref.c) - TEST INFRASTRUCTURE, never the product path."""
from __future__ import annotations

import ctypes

import numpy as np

from .build import build

_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.oq_quantize_rows_f32.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                              ctypes.c_void_p]
        _lib.oq_gemm_i32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int64, ctypes.c_void_p]
    return _lib


def quantize_rows(x: np.ndarray):
    """(q int8, fp32 scale (M,)) of the C restatement of Int8Tensor.quantize."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
    M, K = x.shape
    q = np.empty((M, K), dtype=np.int8)
    s = np.empty(M, dtype=np.float32)
    _load().oq_quantize_rows_f32(x.ctypes.data, M, K, q.ctypes.data, s.ctypes.data)
    return q, s


def gemm_i32(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    M, K = a.shape
    N = w.shape[0]
    acc = np.empty((M, N), dtype=np.int32)
    _load().oq_gemm_i32(a.ctypes.data, w.ctypes.data, M, N, K, acc.ctypes.data)
    return acc
