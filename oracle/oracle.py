"""ctypes binding of the CPU oracle (``liboracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py``. It is the checker the CUDA path is
compared against, never a fallback of the product.

Each wrapper mirrors a reference function of ``crates/unltd-tensor/src/quants.rs``
(cited on the C side in ``quants_ref.c``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

# DType ordinals, reference enum order (lib.rs:19-31)
F32, F16, BF16, I8, U8, Q4K, Q6K, Q8_0 = range(8)
QK_K = 256
BLOCK_BYTES = {Q4K: 144, Q6K: 210, Q8_0: 34}
BLOCK_ELEMS = {Q4K: 256, Q6K: 256, Q8_0: 32}


class Q8KBlock(ctypes.Structure):
    _fields_ = [("d", ctypes.c_float), ("qs", ctypes.c_int8 * 256), ("bsums", ctypes.c_int32 * 16)]


_lib = None


def build() -> str:
    """Compile liboracle.so from the committed C sources (make)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(
            os.path.getmtime(os.path.join(HERE, f)) for f in ("quants_ref.c", "quants_ref.h")
        ):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        S = ctypes.c_size_t
        L.ora_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.ora_f16_to_f32.restype = ctypes.c_float
        L.ora_pairwise_sum_f64.argtypes = [P, S]
        L.ora_pairwise_sum_f64.restype = ctypes.c_double
        L.ora_nearest_int.argtypes = [ctypes.c_float]
        L.ora_nearest_int.restype = ctypes.c_int32
        for name in ("ora_dot_f32", "ora_dot_q4_k", "ora_dot_q6_k", "ora_dot_q8_0"):
            f = getattr(L, name)
            f.argtypes = [P, P, S]
            f.restype = ctypes.c_double
        L.ora_quantize_q8_k.argtypes = [P, S, P]
        L.ora_quantize_q8_k.restype = ctypes.c_int
        for name in ("ora_dot_q4_k_q8_k", "ora_dot_q6_k_q8_k"):
            f = getattr(L, name)
            f.argtypes = [P, P, S]
            f.restype = ctypes.c_float
        for name in ("ora_gemv_quant", "ora_gemv_quant_q8k", "ora_gemv_quant_f64"):
            f = getattr(L, name)
            f.argtypes = [P, P, P, S, S, S, ctypes.c_int, ctypes.c_int]
            f.restype = ctypes.c_int
        for name in ("ora_dequantize_q4_k", "ora_dequantize_q6_k", "ora_dequantize_q8_0"):
            f = getattr(L, name)
            f.argtypes = [P, P, S]
            f.restype = ctypes.c_int
        L.ora_argmax.argtypes = [P, S]
        L.ora_argmax.restype = S
        L.ora_row_bytes.argtypes = [ctypes.c_int, S]
        L.ora_row_bytes.restype = S
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def f16_to_f32(h: int) -> np.float32:
    return np.float32(lib().ora_f16_to_f32(h))


def pairwise_sum_f64(v) -> float:
    a = np.ascontiguousarray(v, dtype=np.float64)
    return lib().ora_pairwise_sum_f64(_p(a), a.size)


def nearest_int(f: float) -> int:
    return lib().ora_nearest_int(float(np.float32(f)))


def _u8(w) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(w), dtype=np.uint8) if isinstance(w, (bytes, bytearray)) else w, dtype=np.uint8)


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def dot_f32(x, w) -> float:
    x, w = _f32(x), _f32(w)
    return lib().ora_dot_f32(_p(x), _p(w), x.size)


def dot_q4_k(x, w) -> float:
    x, w = _f32(x), _u8(w)
    return lib().ora_dot_q4_k(_p(x), _p(w), x.size)


def dot_q6_k(x, w) -> float:
    x, w = _f32(x), _u8(w)
    return lib().ora_dot_q6_k(_p(x), _p(w), x.size)


def dot_q8_0(x, w) -> float:
    x, w = _f32(x), _u8(w)
    return lib().ora_dot_q8_0(_p(x), _p(w), x.size)


def quantize_q8_k(x):
    x = _f32(x)
    nb = x.size // QK_K
    arr = (Q8KBlock * max(nb, 1))()
    rc = lib().ora_quantize_q8_k(_p(x), x.size, ctypes.cast(arr, ctypes.c_void_p))
    if rc != 0:
        raise ValueError("quantize_q8_k: len is not a multiple of 256")
    return arr[:nb]


def _q8k_array(blocks):
    arr = (Q8KBlock * max(len(blocks), 1))(*blocks)
    return arr


def dot_q4_k_q8_k(xq, w) -> np.float32:
    w = _u8(w)
    arr = _q8k_array(xq)
    return np.float32(lib().ora_dot_q4_k_q8_k(ctypes.cast(arr, ctypes.c_void_p), _p(w), len(xq)))


def dot_q6_k_q8_k(xq, w) -> np.float32:
    w = _u8(w)
    arr = _q8k_array(xq)
    return np.float32(lib().ora_dot_q6_k_q8_k(ctypes.cast(arr, ctypes.c_void_p), _p(w), len(xq)))


def _gemv(fname, out_dtype, x, w, dim_in, dim_out, dtype, nthreads):
    x, w = _f32(x), _u8(w)
    out = np.zeros(dim_out, dtype=out_dtype)
    rc = getattr(lib(), fname)(_p(out), _p(x), _p(w), w.size, dim_in, dim_out, dtype, nthreads)
    if rc != 0:
        raise ValueError(f"{fname}: status {rc}")
    return out


def gemv_quant(x, w, dim_in, dim_out, dtype, nthreads=1) -> np.ndarray:
    """quants.rs:422 — exact f64 dots rounded to f32."""
    return _gemv("ora_gemv_quant", np.float32, x, w, dim_in, dim_out, dtype, nthreads)


def gemv_quant_f64(x, w, dim_in, dim_out, dtype, nthreads=1) -> np.ndarray:
    """The f64-accumulated ground truth (gemv_quant before its f32 rounding)."""
    return _gemv("ora_gemv_quant_f64", np.float64, x, w, dim_in, dim_out, dtype, nthreads)


def gemv_quant_q8k(x, w, dim_in, dim_out, dtype, nthreads=1) -> np.ndarray:
    """quants.rs:474 — x quantized to Q8_K, ggml-generic integer dots."""
    return _gemv("ora_gemv_quant_q8k", np.float32, x, w, dim_in, dim_out, dtype, nthreads)


def dequantize(w, n, dtype) -> np.ndarray:
    w = _u8(w)
    out = np.zeros(n, dtype=np.float32)
    fname = {Q4K: "ora_dequantize_q4_k", Q6K: "ora_dequantize_q6_k", Q8_0: "ora_dequantize_q8_0"}[dtype]
    rc = getattr(lib(), fname)(_p(out), _p(w), n)
    if rc != 0:
        raise ValueError(f"{fname}: status {rc}")
    return out


def dequantize_q4_k(w, n) -> np.ndarray:
    return dequantize(w, n, Q4K)


def argmax(v) -> int:
    v = _f32(v)
    if v.size == 0:
        raise ValueError("argmax: empty logits")
    return int(lib().ora_argmax(_p(v), v.size))


def row_bytes(dtype, dim_in) -> int:
    return int(lib().ora_row_bytes(dtype, dim_in))
