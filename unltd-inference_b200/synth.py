"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the reference measures on no public dataset; these
stand in for the real GGUF tensors, which are not available here).

* Q4_K: d, dmin ~ U[1e-3, 1e-2] (f16); the 12 packed scale bytes and the 128
  quant bytes uniform — the scale_min_k4 packing is a bijection between 96
  bits and sixteen 6-bit values, so uniform bytes are uniform scales/mins.
* Q6_K: ql/qh uniform bits, int8 scales ~ U{-32..31}, d ~ U[1e-3, 1e-2].
* Q8_0: d ~ U[1e-3, 1e-2] (f16), q ~ U{-127..127}.
* x ~ N(0, 1) f32.
"""
from __future__ import annotations

import numpy as np

F32, Q4K, Q6K, Q8_0 = 0, 5, 6, 7
BLOCK_BYTES = {Q4K: 144, Q6K: 210, Q8_0: 34}
BLOCK_ELEMS = {Q4K: 256, Q6K: 256, Q8_0: 32}


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(-1, 2)


def quant_weights(dtype: int, dim_in: int, dim_out: int, seed: int) -> np.ndarray:
    """Packed GGUF bytes of a dim_out x dim_in tensor, flat uint8."""
    rng = np.random.default_rng(seed)
    if dtype == F32:
        return rng.standard_normal(dim_in * dim_out, dtype=np.float32).view(np.uint8)
    be, bb = BLOCK_ELEMS[dtype], BLOCK_BYTES[dtype]
    assert dim_in % be == 0
    nblk = dim_out * (dim_in // be)
    w = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
    d = _f16_bytes(rng.uniform(1e-3, 1e-2, size=nblk).astype(np.float32))
    if dtype == Q4K:
        w[:, 0:2] = d
        w[:, 2:4] = _f16_bytes(rng.uniform(1e-3, 1e-2, size=nblk).astype(np.float32))
    elif dtype == Q6K:
        w[:, 192:208] = rng.integers(-32, 32, size=(nblk, 16), dtype=np.int8).view(np.uint8)
        w[:, 208:210] = d
    else:
        w[:, 0:2] = d
        w[:, 2:34] = rng.integers(-127, 128, size=(nblk, 32), dtype=np.int8).view(np.uint8)
    return w.reshape(-1)


def _pack_scale_min_k4(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """The 12 packed bytes of eight 6-bit scales and mins per block (the
    inverse of scale_min_k4, quants.rs:92-102): bytes 0-3 hold sc[0..3] with
    the top two bits of sc[4..7], bytes 4-7 m[0..3] with the top two bits of
    m[4..7], bytes 8-11 the low nibbles of sc[4..7] | m[4..7] << 4."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    out = np.empty(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = (m[..., 0:4] & 63) | ((m[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 0xF) | ((m[..., 4:8] & 0xF) << 4)
    return out


def centered_q4k_weights(dim_in: int, dim_out: int, seed: int) -> np.ndarray:
    """Q4_K blocks whose dequantized values have mean ~0: uniform quants and
    6-bit scales, each group's min equal to its scale and dmin = f16(7.5 d),
    so w = d*sc*q - dmin*sc ~ d*sc*(q - 7.5). Uniform scale/min bytes (the
    benchmark kernels' distribution) give every weight a mean of about
    +240 d, which adds the same large common-mode vector to the residual at
    every layer of a model; with it the greedy stream settles on the vocab
    row with the largest sum. The model generator uses these blocks."""
    rng = np.random.default_rng(seed)
    nblk = dim_out * (dim_in // 256)
    w = np.empty((nblk, 144), np.uint8)
    d = rng.uniform(1e-3, 1e-2, size=nblk).astype(np.float32)
    dh = d.astype(np.float16)
    w[:, 0:2] = dh.view(np.uint8).reshape(-1, 2)
    w[:, 2:4] = (dh.astype(np.float32) * np.float32(7.5)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    sc = rng.integers(0, 64, size=(nblk, 8), dtype=np.uint8)
    w[:, 4:16] = _pack_scale_min_k4(sc, sc)
    w[:, 16:144] = rng.integers(0, 256, size=(nblk, 128), dtype=np.uint8)
    return w.reshape(-1)


def activations(n: int, seed: int, rows: int | None = None) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if rows is None:
        return rng.standard_normal(n, dtype=np.float32)
    return rng.standard_normal((rows, n), dtype=np.float32)


def row_bytes(dtype: int, dim_in: int) -> int:
    if dtype == F32:
        return 4 * dim_in
    return dim_in // BLOCK_ELEMS[dtype] * BLOCK_BYTES[dtype]


# ---- synthetic Qwen3.5-style hybrid model ------------------------------------
# Shapes follow crates/unltd-generation/src/qwen35_forward.rs:139-221; the
# dtypes follow the Q4_K_M mix (Q4_K for most projections and the embedding,
# Q6_K for attn_v, ffn_down and the LM head). Q6_K tensors use the block
# distribution above; Q4_K tensors use centered_q4k_weights (zero-mean
# weights: with uniform scale/min bytes every Q4_K projection adds a large
# common-mode vector to the residual stream and the greedy stream settles on
# one vocab row). f32 tensors (the reference loads them from the GGUF):
#   attn_norm / post_attention_norm / output_norm / ssm_norm ~ U[2e-4, 6e-4]
#     (keeps the 32-layer residual stream at an rms of ~20),
#   attn_q_norm / attn_k_norm ~ U[0.5, 1.5], ssm_conv1d ~ U[-0.5, 0.5],
#   ssm_dt.bias ~ U[-1, 1], ssm_a ~ -U[0.1, 1].
# The session state stands in for a prefilled context: K and V cache rows
# ~ N(0, 1), conv windows ~ N(0, 1), GDN matrices ~ N(0, 0.05^2).

import struct
import zlib

QWEN35_9B = dict(
    n_layer=32, n_embd=4096, n_ff=12288, n_head=16, n_head_kv=4, head_dim=256, head_dim_v=256, n_rot=64,
    conv_kernel=4, state_size=128, group_count=16, time_step_rank=32, d_inner=4096, full_attn_interval=4,
    vocab=151936, freq_base=1e7, rms_eps=1e-6,
)

# Small configuration with the same structure (3 recurrent + 1 attention layer).
QWEN35_TINY = dict(
    n_layer=4, n_embd=512, n_ff=1024, n_head=2, n_head_kv=1, head_dim=256, head_dim_v=256, n_rot=64,
    conv_kernel=4, state_size=128, group_count=2, time_step_rank=4, d_inner=512, full_attn_interval=4,
    vocab=1000, freq_base=1e7, rms_eps=1e-6,
)


def qwen35_dims(cfg: dict) -> dict:
    """Derived dimensions (qwen35.rs:255-291)."""
    hd = cfg["d_inner"] // (2 * cfg["group_count"])
    theta = np.float32(cfg["freq_base"]) ** (np.float32(-2.0) / np.float32(cfg["n_rot"]))
    return dict(
        hd=hd, nv=cfg["d_inner"] // hd, nqk=cfg["group_count"], dconv=2 * cfg["d_inner"],
        kvlen=cfg["n_head_kv"] * cfg["head_dim"],
        attn=[(il + 1) % cfg["full_attn_interval"] == 0 for il in range(cfg["n_layer"])],
        theta_scale=float(np.float32(theta)),
    )


def qwen35_tensor_list(cfg: dict) -> list:
    """(name, dtype, dim_in, dim_out) of every tensor, Q4_K_M mix; F32 tensors
    have dim_out = 1."""
    d = qwen35_dims(cfg)
    n, nff = cfg["n_embd"], cfg["n_ff"]
    t = [("token_embd.weight", Q4K, n, cfg["vocab"]), ("output_norm.weight", F32, n, 1),
         ("output.weight", Q6K, n, cfg["vocab"])]
    for il in range(cfg["n_layer"]):
        p = f"blk.{il}."
        t += [(p + "attn_norm.weight", F32, n, 1), (p + "post_attention_norm.weight", F32, n, 1),
              (p + "ffn_gate.weight", Q4K, n, nff), (p + "ffn_up.weight", Q4K, n, nff),
              (p + "ffn_down.weight", Q6K, nff, n)]
        if d["attn"][il]:
            t += [(p + "attn_q.weight", Q4K, n, 2 * n), (p + "attn_q_norm.weight", F32, cfg["head_dim"], 1),
                  (p + "attn_k.weight", Q4K, n, d["kvlen"]), (p + "attn_k_norm.weight", F32, cfg["head_dim"], 1),
                  (p + "attn_v.weight", Q6K, n, d["kvlen"]), (p + "attn_output.weight", Q4K, n, n)]
        else:
            t += [(p + "attn_qkv.weight", Q4K, n, d["dconv"]), (p + "attn_gate.weight", Q4K, n, n),
                  (p + "ssm_conv1d.weight", F32, cfg["conv_kernel"] * d["dconv"], 1),
                  (p + "ssm_dt.bias", F32, d["nv"], 1), (p + "ssm_a", F32, d["nv"], 1),
                  (p + "ssm_beta.weight", Q4K, n, d["nv"]), (p + "ssm_alpha.weight", Q4K, n, d["nv"]),
                  (p + "ssm_norm.weight", F32, d["hd"], 1), (p + "ssm_out.weight", Q4K, n, n)]
    return t


NORM_RANGE = (2e-4, 6e-4)


def _tensor_seed(seed: int, name: str) -> int:
    return (seed * 1000003 + zlib.crc32(name.encode())) & 0xFFFFFFFF


def _f32_tensor(name: str, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(_tensor_seed(seed, name))
    if name.endswith(("attn_norm.weight", "post_attention_norm.weight", "ssm_norm.weight")) or name == "output_norm.weight":
        lo, hi = NORM_RANGE
    elif name.endswith(("attn_q_norm.weight", "attn_k_norm.weight")):
        lo, hi = 0.5, 1.5
    elif name.endswith("ssm_conv1d.weight"):
        lo, hi = -0.5, 0.5
    elif name.endswith("ssm_dt.bias"):
        lo, hi = -1.0, 1.0
    elif name.endswith("ssm_a"):
        return -rng.uniform(0.1, 1.0, n).astype(np.float32)
    else:
        raise KeyError(name)
    return rng.uniform(lo, hi, n).astype(np.float32)


def qwen35_tensor(cfg: dict, name: str, seed: int):
    """(dtype, array) of one tensor: packed bytes (uint8) or f32 values."""
    for nm, dt, di, do in qwen35_tensor_list(cfg):
        if nm == name:
            if dt == F32:
                return dt, _f32_tensor(nm, di, seed)
            if dt == Q4K:
                return dt, centered_q4k_weights(di, do, _tensor_seed(seed, nm))
            return dt, quant_weights(dt, di, do, _tensor_seed(seed, nm))
    raise KeyError(name)


def qwen35_model(cfg: dict, seed: int) -> dict:
    """name -> (dtype, array) for the whole model."""
    return {nm: qwen35_tensor(cfg, nm, seed) for nm, _, _, _ in qwen35_tensor_list(cfg)}


def qwen35_state(cfg: dict, position: int, seed: int) -> dict:
    """Seeded session state at `position`: per recurrent layer the conv window
    ((K-1) x d_conv, oldest row first) and GDN matrices (n_v x hd x hd); per
    attention layer `position` rows of K and V."""
    d = qwen35_dims(cfg)
    rng = np.random.default_rng(seed)
    st = {"conv": [], "gdn": [], "k": [], "v": []}
    for il in range(cfg["n_layer"]):
        if d["attn"][il]:
            st["k"].append(rng.standard_normal((position, d["kvlen"]), dtype=np.float32))
            st["v"].append(rng.standard_normal((position, d["kvlen"]), dtype=np.float32))
        else:
            st["conv"].append(rng.standard_normal((cfg["conv_kernel"] - 1, d["dconv"]), dtype=np.float32))
            st["gdn"].append((0.05 * rng.standard_normal((d["nv"], d["hd"], d["hd"]), dtype=np.float32)).astype(np.float32))
    return st


# ---- synthetic GGUF files (the reference's loader reads gguf.rs:353-520) ----

_GGML_TYPE = {F32: 0, Q8_0: 8, Q4K: 12, Q6K: 14}
_GGUF_U32, _GGUF_I32, _GGUF_F32, _GGUF_STRING, _GGUF_ARRAY = 4, 5, 6, 8, 9


def _gguf_str(b: bytearray, s: str):
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


def write_gguf(path: str, kvs: list, tensors: list, alignment: int = 32):
    """GGUF v3: kvs = [(key, kind, value)] with kind in 'u32', 'i32', 'f32',
    'str', 'i32[]'; tensors = [(name, ggml_type, ne (ne[0] fastest), bytes)]."""
    b = bytearray(b"GGUF")
    b += struct.pack("<IQQ", 3, len(tensors), len(kvs) + 1)
    _gguf_str(b, "general.alignment")
    b += struct.pack("<II", _GGUF_U32, alignment)
    for key, kind, val in kvs:
        _gguf_str(b, key)
        if kind == "u32":
            b += struct.pack("<II", _GGUF_U32, val)
        elif kind == "i32":
            b += struct.pack("<Ii", _GGUF_I32, val)
        elif kind == "f32":
            b += struct.pack("<If", _GGUF_F32, val)
        elif kind == "str":
            b += struct.pack("<I", _GGUF_STRING)
            _gguf_str(b, val)
        elif kind == "i32[]":
            b += struct.pack("<IIQ", _GGUF_ARRAY, _GGUF_I32, len(val)) + struct.pack(f"<{len(val)}i", *val)
        else:
            raise ValueError(kind)
    off = 0
    offsets = []
    for name, gt, ne, data in tensors:
        _gguf_str(b, name)
        b += struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
        b += struct.pack("<IQ", gt, off)
        offsets.append(off)
        off += (len(data) + alignment - 1) // alignment * alignment
    b += bytes((-len(b)) % alignment)
    with open(path, "wb") as fh:
        fh.write(b)
        for (name, gt, ne, data), o in zip(tensors, offsets):
            fh.write(data)
            fh.write(bytes((-len(data)) % alignment))


def write_qwen35_gguf(path: str, cfg: dict, tensors: dict, context_length: int = 262144):
    """The model as a qwen35 GGUF file: the metadata keys Qwen35Config::from_gguf
    requires (qwen35.rs:23-42) and every tensor in GGUF shape (a weight ne =
    [dim_in, dim_out]; ssm_conv1d.weight ne = [conv_kernel, channels])."""
    a = "qwen35."
    kvs = [("general.architecture", "str", "qwen35"),
           (a + "block_count", "u32", cfg["n_layer"]), (a + "context_length", "u32", context_length),
           (a + "embedding_length", "u32", cfg["n_embd"]), (a + "feed_forward_length", "u32", cfg["n_ff"]),
           (a + "attention.head_count", "u32", cfg["n_head"]),
           (a + "attention.head_count_kv", "u32", cfg["n_head_kv"]),
           (a + "attention.key_length", "u32", cfg["head_dim"]),
           (a + "attention.value_length", "u32", cfg["head_dim_v"]),
           (a + "attention.layer_norm_rms_epsilon", "f32", cfg["rms_eps"]),
           (a + "rope.dimension_count", "u32", cfg["n_rot"]),
           (a + "rope.dimension_sections", "i32[]", [11, 11, 10, 0]),
           (a + "rope.freq_base", "f32", cfg["freq_base"]),
           (a + "ssm.conv_kernel", "u32", cfg["conv_kernel"]), (a + "ssm.state_size", "u32", cfg["state_size"]),
           (a + "ssm.group_count", "u32", cfg["group_count"]),
           (a + "ssm.time_step_rank", "u32", cfg["time_step_rank"]),
           (a + "ssm.inner_size", "u32", cfg["d_inner"]),
           (a + "full_attention_interval", "u32", cfg["full_attn_interval"])]
    out = []
    for name, dt, dim_in, dim_out in qwen35_tensor_list(cfg):
        _, arr = tensors[name]
        data = np.ascontiguousarray(arr).tobytes()
        if dt == F32:
            ne = [cfg["conv_kernel"], dim_in // cfg["conv_kernel"]] if name.endswith("ssm_conv1d.weight") else [dim_in]
        else:
            ne = [dim_in, dim_out]
        out.append((name, _GGML_TYPE[dt], ne, data))
    write_gguf(path, kvs, out)
