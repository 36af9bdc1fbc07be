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
            os.path.getmtime(os.path.join(HERE, f)) for f in ("quants_ref.c", "quants_ref.h", "forward_ref.c", "forward_ref.h")
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


# ---- Qwen3.5-style hybrid decode step (forward_ref.c) -----------------------

class _OraCfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_rot", "conv_kernel", "group_count",
        "d_inner", "full_attn_interval", "vocab", "ctx")] + [("rms_eps", ctypes.c_float), ("theta_scale", ctypes.c_double)]


# Per-layer tensor slots, in the order of the ORA_* enum of forward_ref.h.
LAYER_KINDS = [
    "attn_norm.weight", "post_attention_norm.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight",
    "attn_q.weight", "attn_q_norm.weight", "attn_k.weight", "attn_k_norm.weight", "attn_v.weight",
    "attn_output.weight", "attn_qkv.weight", "attn_gate.weight", "ssm_conv1d.weight", "ssm_dt.bias", "ssm_a",
    "ssm_beta.weight", "ssm_alpha.weight", "ssm_norm.weight", "ssm_out.weight",
]
GLOBAL_KINDS = ["token_embd.weight", "output_norm.weight", "output.weight"]


class Qwen35Oracle:
    """CPU decode step (ora_decode_token) over a model given as name ->
    (dtype, array), with its own copy of the session state."""

    def __init__(self, cfg: dict, tensors: dict, ctx: int, state: dict | None = None, position: int = 0,
                 theta_scale: float | None = None):
        L = lib()
        if not hasattr(L, "_fwd_ready"):
            L.ora_decode_token.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32,
                                                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
            L.ora_decode_token.restype = ctypes.c_int
            L._fwd_ready = True
        if theta_scale is None:
            theta_scale = float(np.float32(np.float32(cfg["freq_base"]) ** (np.float32(-2.0) / np.float32(cfg["n_rot"]))))
        self.cfg = cfg
        self.c = _OraCfg(cfg["n_layer"], cfg["n_embd"], cfg["n_ff"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"],
                         cfg["n_rot"], cfg["conv_kernel"], cfg["group_count"], cfg["d_inner"],
                         cfg["full_attn_interval"], cfg["vocab"], ctx, cfg["rms_eps"], theta_scale)
        nslots = len(GLOBAL_KINDS) + len(LAYER_KINDS) * cfg["n_layer"]
        self._keep = []
        ptrs = (ctypes.c_void_p * nslots)()
        dts = (ctypes.c_int * nslots)()
        names = list(GLOBAL_KINDS) + [f"blk.{il}.{k}" for il in range(cfg["n_layer"]) for k in LAYER_KINDS]
        for i, nm in enumerate(names):
            if nm in tensors:
                dt, arr = tensors[nm]
                arr = np.ascontiguousarray(arr)
                self._keep.append(arr)
                ptrs[i] = arr.ctypes.data
                dts[i] = dt
        self.ptrs, self.dts = ptrs, dts
        hd = cfg["d_inner"] // (2 * cfg["group_count"])
        nv, dconv, kvlen = cfg["d_inner"] // hd, 2 * cfg["d_inner"], cfg["n_head_kv"] * cfg["head_dim"]
        attn = [(il + 1) % cfg["full_attn_interval"] == 0 for il in range(cfg["n_layer"])]
        nr, na = attn.count(False), attn.count(True)
        st = state or {}
        self.conv = [np.array(st["conv"][i], np.float32) if st.get("conv") else
                     np.zeros((cfg["conv_kernel"] - 1, dconv), np.float32) for i in range(nr)]
        self.gdn = [np.array(st["gdn"][i], np.float32) if st.get("gdn") else np.zeros((nv, hd, hd), np.float32)
                    for i in range(nr)]
        self.k = [np.zeros((ctx, kvlen), np.float32) for _ in range(na)]
        self.v = [np.zeros((ctx, kvlen), np.float32) for _ in range(na)]
        for i in range(na):
            if st.get("k"):
                self.k[i][:position] = st["k"][i][:position]
                self.v[i][:position] = st["v"][i][:position]
        self.position = position

        def arr(xs):
            a = (ctypes.c_void_p * max(1, len(xs)))()
            for i, x in enumerate(xs):
                a[i] = x.ctypes.data
            return a

        self._conv_p, self._gdn_p, self._k_p, self._v_p = arr(self.conv), arr(self.gdn), arr(self.k), arr(self.v)

    def step(self, token: int, nthreads: int = 8):
        """One token; returns (logits, hidden) and advances the position."""
        logits = np.empty(self.cfg["vocab"], np.float32)
        hidden = np.empty(self.cfg["n_embd"], np.float32)
        rc = lib().ora_decode_token(ctypes.byref(self.c), self.ptrs, self.dts, self._conv_p, self._gdn_p, self._k_p,
                                    self._v_p, self.position, token, logits.ctypes.data, hidden.ctypes.data, nthreads)
        if rc != 0:
            raise ValueError(f"ora_decode_token failed ({rc})")
        self.position += 1
        return logits, hidden

    @staticmethod
    def exact_gemv(on: bool):
        """Process-wide: every projection through gemv_quant (f64 dots)
        instead of gemv_quant_q8k; measures the reference's own Q8_K error."""
        lib().ora_forward_exact_gemv(1 if on else 0)

    @staticmethod
    def row_split(world: int):
        """Process-wide: the input-split projections (ffn_down, ssm_out,
        attn_output) as `world` tensor-parallel ranks compute them (per-rank
        partial gemv_quant_q8k, summed in rank order); 1 = one device."""
        lib().ora_forward_row_split(int(world))

    def greedy(self, token: int, n_steps: int, nthreads: int = 8):
        """greedy.rs: step, argmax (first index of the max), feed back."""
        out, logits, hidden = [], None, None
        for _ in range(n_steps):
            logits, hidden = self.step(token, nthreads)
            token = argmax(logits)
            out.append(token)
        return out, logits, hidden


# ---- f32 kernels of the decode step (forward_ref.c, kernels.rs) --------------

def _fwd_lib():
    L = lib()
    if not hasattr(L, "_fwd_k_ready"):
        P, I, F, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double
        L.ora_rmsnorm.argtypes = [P, P, P, I, F]
        L.ora_l2_norm_rows.argtypes = [P, I, I, F]
        L.ora_gdn_step.argtypes = [P, P, P, P, P, F, F, F, I]
        L.ora_rope_imrope.argtypes = [P, I, D, I]
        L.ora_softmax.argtypes = [P, P, I, F]
        for nm in ("ora_sigmoid", "ora_silu", "ora_softplus"):
            getattr(L, nm).argtypes = [P, P, I]
        L.ora_swiglu.argtypes = [P, P, P, I]
        L.ora_ssm_conv.argtypes = [P, P, I, P, I, I]
        L.ora_expf.argtypes = [F]
        L.ora_expf.restype = F
        L._fwd_k_ready = True
    return L


def rmsnorm(x, w, eps):
    x, w = _f32(x), _f32(w)
    out = np.zeros_like(x)
    _fwd_lib().ora_rmsnorm(_p(out), _p(x), _p(w), x.size, eps)
    return out


def l2_norm_rows(x, dim, eps):
    x = _f32(x).copy()
    _fwd_lib().ora_l2_norm_rows(_p(x), x.size // dim, dim, eps)
    return x


def gdn_step(state, q, k, v, gate, beta, scale):
    state = _f32(state).copy()
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.zeros(q.size, np.float32)
    _fwd_lib().ora_gdn_step(_p(state), _p(out), _p(q), _p(k), _p(v), gate, beta, scale, q.size)
    return state, out


def rope_imrope(x, n_rot, theta_scale, pos):
    x = _f32(x).copy()
    _fwd_lib().ora_rope_imrope(_p(x), n_rot, theta_scale, pos)
    return x


def softmax(x, scale):
    x = _f32(x)
    out = np.zeros_like(x)
    _fwd_lib().ora_softmax(_p(out), _p(x), x.size, scale)
    return out


def _elementwise(name, x):
    x = _f32(x)
    out = np.zeros_like(x)
    getattr(_fwd_lib(), name)(_p(out), _p(x), x.size)
    return out


def sigmoid(x):
    return _elementwise("ora_sigmoid", x)


def silu(x):
    return _elementwise("ora_silu", x)


def softplus(x):
    return _elementwise("ora_softplus", x)


def swiglu(g, u):
    g, u = _f32(g), _f32(u)
    out = np.zeros_like(g)
    _fwd_lib().ora_swiglu(_p(out), _p(g), _p(u), g.size)
    return out


def ssm_conv(x, kernel, d_conv, channels):
    x, kernel = _f32(x), _f32(kernel)
    ncs = x.size // channels
    out = np.zeros((ncs - (d_conv - 1)) * channels, np.float32)
    _fwd_lib().ora_ssm_conv(_p(out), _p(x), ncs, _p(kernel), d_conv, channels)
    return out
