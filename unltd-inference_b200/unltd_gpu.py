"""ctypes binding of libunltd_gpu (include/unltd_gpu.h).

Mirrors the reference crate's operator names (crates/unltd-tensor/src/
quants.rs): ``gemv_quant``, ``gemv_quant_q8k``, ``dequantize_q4_k`` take host
numpy arrays exactly like the Rust functions take slices; the handle API
(``Context``, ``Weight``) takes device pointers (e.g. ``torch.Tensor.data_ptr()``).

There is no CPU fallback: importing works without a GPU (so the library can
be inspected), but every compute call goes through the CUDA library and
raises ``UnltdError`` when it fails or when no device is present.
"""
from __future__ import annotations

import atexit
import ctypes
import os
import sys
import weakref

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libunltd_gpu.so")

# DType ordinals (crates/unltd-tensor/src/lib.rs:19-31)
F32, F16, BF16, I8, U8, Q4K, Q6K, Q8_0 = range(8)
MODE_F32X, MODE_Q8K = 0, 1
STATUS = {
    0: "OK", 1: "INVALID_ARG", 2: "LENGTH", 3: "DIM", 4: "UNSUPPORTED", 5: "CUDA",
    6: "OUT_OF_MEMORY", 7: "NO_DEVICE", 8: "NCCL", 9: "TIMEOUT",
}

# Every symbol include/unltd_gpu.h declares: (name, restype, argtypes)
_P, _S, _I, _I64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int64
SIGNATURES = [
    ("unltd_last_error", ctypes.c_char_p, []),
    ("unltd_abi_version", _I, []),
    ("unltd_row_bytes", _S, [_I, _S]),
    ("unltd_ctx_create", _I, [_I, ctypes.POINTER(_P)]),
    ("unltd_ctx_destroy", _I, [_P]),
    ("unltd_ctx_stream", _I, [_P, ctypes.POINTER(_P)]),
    ("unltd_ctx_set_stream", _I, [_P, _P]),
    ("unltd_ctx_synchronize", _I, [_P]),
    ("unltd_ctx_launch_count", _I64, [_P]),
    ("unltd_weight_upload", _I, [_P, _P, _S, _I, _S, _S, ctypes.POINTER(_P)]),
    ("unltd_weight_upload_rows", _I, [_P, _P, _S, _I, _S, _S, _S, _S, ctypes.POINTER(_P)]),
    ("unltd_weight_free", _I, [_P]),
    ("unltd_weight_info", _I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_S), ctypes.POINTER(_S), ctypes.POINTER(_S)]),
    ("unltd_gemv", _I, [_P, _P, _P, _P, _I]),
    ("unltd_gemv_argmax", _I, [_P, _P, _P, _P, _P, _I]),
    ("unltd_gemv_argmax_shard", _I, [_P, _P, _P, _P, _P, ctypes.c_uint32, _I]),
    ("unltd_gemv_batch", _I, [_P, _P, _P, _P, _I, _I]),
    ("unltd_gemv_argmax_batch", _I, [_P, _P, _P, _P, _P, _I, _I]),
    ("unltd_dequant", _I, [_P, _P, _P]),
    ("unltd_gemv_noalloc", _I, [_P, _P, _P, _I, _P]),
    ("unltd_gemm", _I, [_P, _P, _P, _P, _S]),
    ("unltd_gemm_f32x", _I, [_P, _P, _P, _P, _S]),
    ("unltd_gemv_quant", _I, [_P, _S, _P, _S, _P, _S, _S, _S, _I]),
    ("unltd_gemv_quant_q8k", _I, [_P, _S, _P, _S, _P, _S, _S, _S, _I]),
    ("unltd_dequantize_q4_k", _I, [_P, _S, _P, _S]),
    ("unltd_set_default_device", _I, [_I]),
    ("unltd_forget_host_weights", _I, []),
    ("unltd_comm_unique_id", _I, [_P, _S]),
    ("unltd_comm_init", _I, [_P, _I, _I, _P, _S]),
    ("unltd_gguf_open", _I, [ctypes.c_char_p, _P]),
    ("unltd_gguf_close", _I, [_P]),
    ("unltd_gguf_tensor_count", ctypes.c_int64, [_P]),
    ("unltd_gguf_tensor_info", _I, [_P, ctypes.c_int64, _P, _P, _P, _P, _P, _P]),
    ("unltd_gguf_find_tensor", _I, [_P, ctypes.c_char_p, _P]),
    ("unltd_gguf_get_int", _I, [_P, ctypes.c_char_p, _P]),
    ("unltd_gguf_get_float", _I, [_P, ctypes.c_char_p, _P]),
    ("unltd_gguf_get_string", _I, [_P, ctypes.c_char_p, _P]),
    ("unltd_qwen35_config_from_gguf", _I, [_P, _P]),
    ("unltd_qwen35_load_gguf", _I, [_P, _P]),
    ("unltd_peer_export", _I, [_P, _P, _S]),
    ("unltd_peer_import", _I, [_P, _P, _S]),
    ("unltd_allreduce_sum_f32", _I, [_P, _P, _S]),
    ("unltd_allreduce_max_u64", _I, [_P, _P, _S]),
    ("unltd_qwen35_create", _I, [_P, _P, ctypes.POINTER(_P)]),
    ("unltd_qwen35_create_tp", _I, [_P, _P, _I, _I, ctypes.POINTER(_P)]),
    ("unltd_qwen35_shard", _I, [_P, _I, _I, ctypes.c_char_p, _P, _I, ctypes.POINTER(_I), ctypes.POINTER(_I64),
                                ctypes.POINTER(_I64)]),
    ("unltd_qwen35_session_shape", _I, [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                                        ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    ("unltd_qwen35_set_tensor", _I, [_P, ctypes.c_char_p, _P, _S, _I]),
    ("unltd_qwen35_finalize", _I, [_P]),
    ("unltd_qwen35_destroy", _I, [_P]),
    ("unltd_qwen35_session_create", _I, [_P, _I, ctypes.POINTER(_P)]),
    ("unltd_qwen35_session_destroy", _I, [_P]),
    ("unltd_qwen35_session_set_state", _I, [_P, _I, _P, _P, _P, _P]),
    ("unltd_qwen35_session_get_state", _I, [_P, _P, _P, _P, _P]),
    ("unltd_qwen35_feed", _I, [_P, _P, _I, _P]),
    ("unltd_qwen35_prefill", _I, [_P, _P, _I, _P]),
    ("unltd_qwen35_decode", _I, [_P, ctypes.c_uint32, _I, _P]),
    ("unltd_qwen35_session_info", _I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_P), ctypes.POINTER(_I64)]),
    ("unltd_qwen35_session_read", _I, [_P, _P, _P]),
    ("unltd_qwen35_session_create_batch", _I, [_P, _I, _I, ctypes.POINTER(_P)]),
    ("unltd_qwen35_batch_set_state", _I, [_P, _I, _I, _P, _P, _P, _P]),
    ("unltd_qwen35_batch_get_state", _I, [_P, _I, _P, _P, _P, _P]),
    ("unltd_qwen35_batch_read", _I, [_P, _I, _P, _P]),
    ("unltd_qwen35_batch_decode", _I, [_P, _P, _I, _P]),
    ("unltd_qwen35_batch_info", _I, [_P, ctypes.POINTER(_I), _P]),
]


class UnltdError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


_lib = None

# Live handles by release order (sessions, models, weights, contexts): closed
# in that order at interpreter exit, before module teardown, so no handle is
# released after the context it lives in.
_live = [weakref.WeakSet() for _ in range(4)]


def _track(obj, rank: int):
    _live[rank].add(obj)


def _owner(obj):
    """The Context a session, model or weight lives in."""
    if hasattr(obj, "model"):
        obj = obj.model
    return getattr(obj, "ctx", None)


def _alive(obj) -> bool:
    """True while obj holds a handle and its context has not been destroyed."""
    c = _owner(obj)
    return bool(getattr(obj, "h", None)) and (c is None or bool(getattr(c, "h", None)))


@atexit.register
def _close_all():
    for group in _live:
        for o in list(group):
            try:
                o.close()
            except Exception:
                pass


def lib():
    """Load the in-tree CUDA library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python unltd-inference_b200/build.py` "
                "(there is no CPU fallback)"
            )
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _check(rc: int):
    if rc != 0:
        raise UnltdError(rc, lib().unltd_last_error().decode(errors="replace"))


def last_error() -> str:
    return lib().unltd_last_error().decode(errors="replace")


def row_bytes(dtype: int, dim_in: int) -> int:
    return int(lib().unltd_row_bytes(dtype, dim_in))


def _ptr(a) -> int:
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


class Context:
    """A CUDA stream + scratch on one device (unltd_ctx_create)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        h = ctypes.c_void_p()
        _check(lib().unltd_ctx_create(device, ctypes.byref(h)))
        self.h = h
        self.device = device
        _track(self, 3)
        if stream is not None:
            self.set_stream(stream)

    def set_stream(self, stream: int | None):
        """Launch on `stream` (a cudaStream_t as int). 0 is the legacy default
        stream (torch's default), passed as cudaStreamLegacy; None restores
        the context's own stream."""
        if stream is None:
            _check(lib().unltd_ctx_set_stream(self.h, None))
        else:
            _check(lib().unltd_ctx_set_stream(self.h, ctypes.c_void_p(stream if stream else 0x1)))

    def stream(self) -> int:
        s = ctypes.c_void_p()
        _check(lib().unltd_ctx_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    def synchronize(self):
        _check(lib().unltd_ctx_synchronize(self.h))

    def launch_count(self) -> int:
        return int(lib().unltd_ctx_launch_count(self.h))

    def upload(self, w: np.ndarray, dtype: int, dim_in: int, dim_out: int, row0: int = 0, rows: int | None = None):
        w = np.ascontiguousarray(w, dtype=np.uint8)
        rows = dim_out - row0 if rows is None else rows
        h = ctypes.c_void_p()
        _check(lib().unltd_weight_upload_rows(self.h, w.ctypes.data, w.nbytes, dtype, dim_in, dim_out, row0, rows,
                                              ctypes.byref(h)))
        return Weight(self, h, dtype, dim_in, rows)

    def gemv(self, w: "Weight", x, y, mode: int = MODE_F32X):
        _check(lib().unltd_gemv(self.h, w.h, _ptr(x), _ptr(y), mode))

    def gemv_argmax(self, w: "Weight", x, token, logits=None, mode: int = MODE_Q8K):
        _check(lib().unltd_gemv_argmax(self.h, w.h, _ptr(x), _ptr(logits) if logits is not None else None,
                                       _ptr(token), mode))

    def gemv_argmax_shard(self, w: "Weight", x, key, row0: int, logits=None, mode: int = MODE_Q8K):
        """Vocab shard [row0, row0 + dim_out) of the LM head: this shard's
        argmax key (orderable(logit) << 32 | 0xFFFFFFFF - global row) into
        `key` (one int64); allreduce_max_u64 over the ranks then gives the
        whole vocabulary's first-index maximum."""
        _check(lib().unltd_gemv_argmax_shard(self.h, w.h, _ptr(x), _ptr(logits) if logits is not None else None,
                                             _ptr(key), row0, mode))

    def gemv_batch(self, w: "Weight", X, Y, n_seq: int, mode: int = MODE_Q8K):
        """Y[s] = W . X[s] for n_seq sequences (Q8K_EXACT): each row of Y the
        bits of gemv(w, X[s], Y[s], MODE_Q8K)."""
        _check(lib().unltd_gemv_batch(self.h, w.h, _ptr(X), _ptr(Y), n_seq, mode))

    def gemv_argmax_batch(self, w: "Weight", X, tokens, n_seq: int, logits=None, mode: int = MODE_Q8K):
        _check(lib().unltd_gemv_argmax_batch(self.h, w.h, _ptr(X), _ptr(logits) if logits is not None else None,
                                             _ptr(tokens), n_seq, mode))

    def gemm(self, w: "Weight", X, Y, m_tokens: int, accurate: bool = False):
        """Y[m][n] = sum_k X[m][k] W[n][k] on the tensor cores, f32 accumulate:
        fp16 operands (unltd_gemm), or hi + lo fp16 pairs within 1e-4 of the
        f64 truth (accurate=True, unltd_gemm_f32x)."""
        fn = lib().unltd_gemm_f32x if accurate else lib().unltd_gemm
        _check(fn(self.h, w.h, _ptr(X), _ptr(Y), m_tokens))

    def dequant(self, w: "Weight", out):
        _check(lib().unltd_dequant(self.h, w.h, _ptr(out)))

    def comm_init(self, rank: int, world: int, uid: bytes):
        """NCCL communicator for tensor parallelism (uid from comm_unique_id on rank 0)."""
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        _check(lib().unltd_comm_init(self.h, rank, world, buf, 128))
        self.rank, self.world = rank, world

    def peer_init(self, group=None):
        """Switch this context's all-reduces to the NVLink peer kernel: exchange
        the CUDA IPC handles of every rank's receive area over the
        torch.distributed group (call on every rank after comm_init)."""
        import torch.distributed as dist

        h = ctypes.create_string_buffer(64)
        _check(lib().unltd_peer_export(self.h, h, 64))
        hs = [None] * self.world
        dist.all_gather_object(hs, h.raw, group=group)
        buf = ctypes.create_string_buffer(b"".join(hs), 64 * self.world)
        _check(lib().unltd_peer_import(self.h, buf, 64 * self.world))

    def allreduce_sum(self, buf, count: int):
        _check(lib().unltd_allreduce_sum_f32(self.h, _ptr(buf), count))

    def allreduce_max_u64(self, buf, count: int):
        _check(lib().unltd_allreduce_max_u64(self.h, _ptr(buf), count))

    def close(self):
        if getattr(self, "h", None):
            # release what lives in this context first (sessions, models,
            # weights), so no handle outlives it
            for group in _live[:3]:
                for o in list(group):
                    if _owner(o) is self:
                        o.close()
            lib().unltd_ctx_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return
        try:
            self.close()
        except Exception:
            pass


class Weight:
    def __init__(self, ctx: Context, h, dtype, dim_in, dim_out):
        self.ctx, self.h, self.dtype, self.dim_in, self.dim_out = ctx, h, dtype, dim_in, dim_out
        _track(self, 2)

    def info(self):
        dt, di, do, nb = _I(), _S(), _S(), _S()
        _check(lib().unltd_weight_info(self.h, ctypes.byref(dt), ctypes.byref(di), ctypes.byref(do), ctypes.byref(nb)))
        return dt.value, di.value, do.value, nb.value

    def free(self):
        if _alive(self):
            lib().unltd_weight_free(self.h)
        self.h = None

    close = free

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return
        try:
            if self.ctx.h:
                self.free()
        except Exception:
            pass


# ---- reference-signature API (host numpy buffers) ------------------------------

def gemv_quant(out: np.ndarray, x: np.ndarray, w: np.ndarray, dim_in: int, dim_out: int, dtype: int):
    """quants.rs:422 ``gemv_quant(out, x, w, dim_in, dim_out, dtype)`` on the GPU."""
    _check(lib().unltd_gemv_quant(out.ctypes.data, out.size, x.ctypes.data, x.size, w.ctypes.data, w.nbytes,
                                  dim_in, dim_out, dtype))


def gemv_quant_q8k(out: np.ndarray, x: np.ndarray, w: np.ndarray, dim_in: int, dim_out: int, dtype: int):
    """quants.rs:474 ``gemv_quant_q8k(out, x, w, dim_in, dim_out, dtype)`` on the GPU."""
    _check(lib().unltd_gemv_quant_q8k(out.ctypes.data, out.size, x.ctypes.data, x.size, w.ctypes.data, w.nbytes,
                                      dim_in, dim_out, dtype))


def dequantize_q4_k(out: np.ndarray, w: np.ndarray):
    """quants.rs:534 ``dequantize_q4_k(out, w)`` on the GPU."""
    _check(lib().unltd_dequantize_q4_k(out.ctypes.data, out.size, w.ctypes.data, w.nbytes))


def forget_host_weights():
    _check(lib().unltd_forget_host_weights())


# ---- Qwen3.5-style hybrid decode (unltd_qwen35_*) ------------------------------

class Qwen35Config(ctypes.Structure):
    """unltd_qwen35_config (qwen35.rs:46-80)."""
    _fields_ = [(n, ctypes.c_int32) for n in (
        "n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "head_dim_v", "n_rot",
        "conv_kernel", "state_size", "group_count", "time_step_rank", "d_inner", "full_attn_interval", "vocab")] + [
        ("freq_base", ctypes.c_float), ("rms_eps", ctypes.c_float)]

    @classmethod
    def from_dict(cls, d: dict) -> "Qwen35Config":
        return cls(**{k: d[k] for k, _ in cls._fields_})


def comm_unique_id() -> bytes:
    """A fresh 128-byte NCCL id (call on one rank and distribute it)."""
    buf = ctypes.create_string_buffer(128)
    _check(lib().unltd_comm_unique_id(buf, 128))
    return buf.raw


def exchange_unique_id(group=None) -> bytes:
    """Rank 0 creates the NCCL id and every rank of the torch.distributed
    group receives it (works over gloo or nccl process groups)."""
    import torch.distributed as dist

    obj = [comm_unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def qwen35_shard(cfg: dict, rank: int, world: int, name: str):
    """Host-only shard plan: ([(row_begin, row_end), ...], (in_begin, in_end))."""
    c = Qwen35Config.from_dict(cfg)
    ranges = (ctypes.c_int64 * 512)()
    n, i0, i1 = _I(), _I64(), _I64()
    _check(lib().unltd_qwen35_shard(ctypes.byref(c), rank, world, name.encode(), ranges, 256, ctypes.byref(n),
                                    ctypes.byref(i0), ctypes.byref(i1)))
    return [(ranges[2 * k], ranges[2 * k + 1]) for k in range(n.value)], (i0.value, i1.value)


class Gguf:
    """An opened GGUF file (unltd_gguf_open): metadata and zero-copy tensor
    views of its read-only mapping (gguf.rs:353-520, weights.rs:32-92)."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _check(lib().unltd_gguf_open(os.fsencode(path), ctypes.byref(h)))
        self.h = h

    def tensors(self) -> list:
        """[(name, dtype, ne (4 dims, ne[0] fastest), ndims, nbytes, address)]"""
        out = []
        for i in range(lib().unltd_gguf_tensor_count(self.h)):
            name, dt, nd, data, nb = ctypes.c_char_p(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_void_p(), _S()
            ne = (ctypes.c_int64 * 4)()
            _check(lib().unltd_gguf_tensor_info(self.h, i, ctypes.byref(name), ctypes.byref(dt), ne, ctypes.byref(nd),
                                                ctypes.byref(data), ctypes.byref(nb)))
            out.append((name.value.decode(errors="replace"), dt.value, tuple(ne), nd.value, nb.value, data.value))
        return out

    def tensor_bytes(self, name: str) -> bytes:
        i = ctypes.c_int64()
        _check(lib().unltd_gguf_find_tensor(self.h, name.encode(), ctypes.byref(i)))
        data, nb = ctypes.c_void_p(), _S()
        _check(lib().unltd_gguf_tensor_info(self.h, i.value, None, None, None, None, ctypes.byref(data),
                                            ctypes.byref(nb)))
        return ctypes.string_at(data.value, nb.value) if data.value else b""

    def get_int(self, key: str) -> int:
        v = ctypes.c_int64()
        _check(lib().unltd_gguf_get_int(self.h, key.encode(), ctypes.byref(v)))
        return v.value

    def get_float(self, key: str) -> float:
        v = ctypes.c_double()
        _check(lib().unltd_gguf_get_float(self.h, key.encode(), ctypes.byref(v)))
        return v.value

    def get_string(self, key: str) -> str:
        v = ctypes.c_char_p()
        _check(lib().unltd_gguf_get_string(self.h, key.encode(), ctypes.byref(v)))
        return v.value.decode()

    def qwen35_config(self) -> dict:
        """Qwen35Config::from_gguf (qwen35.rs:130-200) as a config dict."""
        c = Qwen35Config()
        _check(lib().unltd_qwen35_config_from_gguf(self.h, ctypes.byref(c)))
        return {k: getattr(c, k) for k, _ in Qwen35Config._fields_}

    def close(self):
        if getattr(self, "h", None):
            lib().unltd_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return
        try:
            self.close()
        except Exception:
            pass


class Qwen35Model:
    """Qwen35Forward::open on the device: tensors uploaded by GGUF name. With
    world > 1 this is the tensor-parallel shard of `rank` (the context needs
    comm_init first); set_tensor still takes the full tensors."""

    def __init__(self, ctx: Context, cfg: dict, rank: int = 0, world: int = 1):
        self.ctx, self.cfg, self.rank, self.world = ctx, dict(cfg), rank, world
        self._c = Qwen35Config.from_dict(cfg)
        h = ctypes.c_void_p()
        _check(lib().unltd_qwen35_create_tp(ctx.h, ctypes.byref(self._c), rank, world, ctypes.byref(h)))
        self.h = h
        _track(self, 1)

    def set_tensor(self, name: str, data: np.ndarray, dtype: int):
        data = np.ascontiguousarray(data)
        _check(lib().unltd_qwen35_set_tensor(self.h, name.encode(), data.ctypes.data, data.nbytes, dtype))

    def load(self, tensors: dict):
        """tensors: name -> (dtype, array), as synth.qwen35_model returns."""
        for name, (dt, arr) in tensors.items():
            self.set_tensor(name, arr, dt)
        _check(lib().unltd_qwen35_finalize(self.h))

    def load_gguf(self, g: "Gguf"):
        """Every tensor from an opened GGUF file (zero-copy views), then finalize."""
        _check(lib().unltd_qwen35_load_gguf(self.h, g.h))

    def session(self, ctx_len: int) -> "Qwen35Session":
        h = ctypes.c_void_p()
        _check(lib().unltd_qwen35_session_create(self.h, ctx_len, ctypes.byref(h)))
        return Qwen35Session(self, h, ctx_len)

    def batch_session(self, ctx_len: int, n_seq: int) -> "Qwen35BatchSession":
        """n_seq sequences decoded together (unltd_qwen35_session_create_batch)."""
        h = ctypes.c_void_p()
        _check(lib().unltd_qwen35_session_create_batch(self.h, ctx_len, n_seq, ctypes.byref(h)))
        return Qwen35BatchSession(self, h, ctx_len, n_seq)

    def close(self):
        if _alive(self):
            for o in list(_live[0]):  # its sessions first
                if getattr(o, "model", None) is self:
                    o.close()
            lib().unltd_qwen35_destroy(self.h)
        self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return
        try:
            self.close()
        except Exception:
            pass


def _ptr_array(arrs):
    if arrs is None:
        return None, None
    keep = [None if a is None else np.ascontiguousarray(a, dtype=np.float32) for a in arrs]
    arr = (ctypes.c_void_p * max(1, len(keep)))(*[None if a is None else a.ctypes.data for a in keep])
    return arr, keep


class Qwen35Session:
    def __init__(self, model: Qwen35Model, h, ctx_len: int):
        self.model, self.h, self.ctx_len = model, h, ctx_len
        _track(self, 0)

    def set_state(self, position: int, conv=None, gdn=None, kcache=None, vcache=None):
        ptrs = [_ptr_array(a) for a in (conv, gdn, kcache, vcache)]
        _check(lib().unltd_qwen35_session_set_state(self.h, position, *[p[0] for p in ptrs]))

    def shape(self) -> dict:
        cr, gh, kv, v0, v1 = _I64(), _I64(), _I64(), _I64(), _I64()
        _check(lib().unltd_qwen35_session_shape(self.h, ctypes.byref(cr), ctypes.byref(gh), ctypes.byref(kv),
                                                ctypes.byref(v0), ctypes.byref(v1)))
        return {"conv_row": cr.value, "gdn_heads": gh.value, "kv_row": kv.value, "vocab": (v0.value, v1.value)}

    def get_state(self) -> dict:
        """The state at the current position: conv windows, GDN matrices, K/V
        rows (this rank's slices under tensor parallelism)."""
        cfg = self.model.cfg
        hd = cfg["d_inner"] // (2 * cfg["group_count"])
        sh = self.shape()
        nv, dconv, kvlen = sh["gdn_heads"], sh["conv_row"], sh["kv_row"]
        attn = [(il + 1) % cfg["full_attn_interval"] == 0 for il in range(cfg["n_layer"])]
        pos = self.info()["position"]
        st = {"conv": [np.zeros((cfg["conv_kernel"] - 1, dconv), np.float32) for a in attn if not a],
              "gdn": [np.zeros((nv, hd, hd), np.float32) for a in attn if not a],
              "k": [np.zeros((pos, kvlen), np.float32) for a in attn if a],
              "v": [np.zeros((pos, kvlen), np.float32) for a in attn if a]}
        ptrs = [_ptr_array(st[k]) for k in ("conv", "gdn", "k", "v")]
        # _ptr_array copies non-contiguous inputs; these are contiguous, so it points at st's arrays
        _check(lib().unltd_qwen35_session_get_state(self.h, *[p[0] for p in ptrs]))
        return st

    def feed(self, tokens) -> int:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        nxt = np.zeros(1, np.uint32)
        _check(lib().unltd_qwen35_feed(self.h, t.ctypes.data, t.size, nxt.ctypes.data))
        return int(nxt[0])

    def prefill(self, tokens) -> int:
        """The prompt through unltd_qwen35_prefill (batched; same bits as feed)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        nxt = np.zeros(1, np.uint32)
        _check(lib().unltd_qwen35_prefill(self.h, t.ctypes.data, t.size, nxt.ctypes.data))
        return int(nxt[0])

    def decode(self, token: int, n_steps: int, out: np.ndarray | None = None) -> np.ndarray:
        out = np.zeros(n_steps, np.uint32) if out is None else out
        _check(lib().unltd_qwen35_decode(self.h, token, n_steps, out.ctypes.data))
        return out

    def info(self):
        pos, st, nl = _I(), _P(), _I64()
        _check(lib().unltd_qwen35_session_info(self.h, ctypes.byref(pos), ctypes.byref(st), ctypes.byref(nl)))
        return {"position": pos.value, "stream": st.value or 0, "launches_per_step": nl.value}

    def read(self, logits: bool = True, hidden: bool = True):
        cfg = self.model.cfg
        v0, v1 = self.shape()["vocab"]
        lg = np.empty(v1 - v0, np.float32) if logits else None
        hd = np.empty(cfg["n_embd"], np.float32) if hidden else None
        _check(lib().unltd_qwen35_session_read(self.h, None if lg is None else lg.ctypes.data,
                                               None if hd is None else hd.ctypes.data))
        return lg, hd

    def close(self):
        if _alive(self) and getattr(self.model, "h", None):
            lib().unltd_qwen35_session_destroy(self.h)
        self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return
        try:
            if self.model.h:
                self.close()
        except Exception:
            pass


class Qwen35BatchSession(Qwen35Session):
    """A batch session: every call names its sequence; decode steps all."""

    def __init__(self, model: Qwen35Model, h, ctx_len: int, n_seq: int):
        super().__init__(model, h, ctx_len)
        self.n_seq = n_seq

    def set_state(self, seq: int, position: int, conv=None, gdn=None, kcache=None, vcache=None):
        ptrs = [_ptr_array(a) for a in (conv, gdn, kcache, vcache)]
        _check(lib().unltd_qwen35_batch_set_state(self.h, seq, position, *[p[0] for p in ptrs]))

    def positions(self) -> list:
        n = _I()
        pos = np.zeros(self.n_seq, np.int32)
        _check(lib().unltd_qwen35_batch_info(self.h, ctypes.byref(n), pos.ctypes.data))
        return pos.tolist()

    def get_state(self, seq: int) -> dict:
        cfg = self.model.cfg
        hd = cfg["d_inner"] // (2 * cfg["group_count"])
        sh = self.shape()
        nv, dconv, kvlen = sh["gdn_heads"], sh["conv_row"], sh["kv_row"]
        attn = [(il + 1) % cfg["full_attn_interval"] == 0 for il in range(cfg["n_layer"])]
        pos = self.positions()[seq]
        st = {"conv": [np.zeros((cfg["conv_kernel"] - 1, dconv), np.float32) for a in attn if not a],
              "gdn": [np.zeros((nv, hd, hd), np.float32) for a in attn if not a],
              "k": [np.zeros((pos, kvlen), np.float32) for a in attn if a],
              "v": [np.zeros((pos, kvlen), np.float32) for a in attn if a]}
        ptrs = [_ptr_array(st[k]) for k in ("conv", "gdn", "k", "v")]
        _check(lib().unltd_qwen35_batch_get_state(self.h, seq, *[p[0] for p in ptrs]))
        return st

    def decode(self, tokens, n_steps: int) -> np.ndarray:
        """tokens: the first token of every sequence; returns [n_seq][n_steps]."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        assert t.size == self.n_seq
        out = np.zeros((self.n_seq, n_steps), np.uint32)
        _check(lib().unltd_qwen35_batch_decode(self.h, t.ctypes.data, n_steps, out.ctypes.data))
        return out

    def read(self, seq: int, logits: bool = True, hidden: bool = True):
        cfg = self.model.cfg
        v0, v1 = self.shape()["vocab"]
        lg = np.empty(v1 - v0, np.float32) if logits else None
        hd = np.empty(cfg["n_embd"], np.float32) if hidden else None
        _check(lib().unltd_qwen35_batch_read(self.h, seq, None if lg is None else lg.ctypes.data,
                                             None if hd is None else hd.ctypes.data))
        return lg, hd
