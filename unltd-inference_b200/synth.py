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


def activations(n: int, seed: int, rows: int | None = None) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if rows is None:
        return rng.standard_normal(n, dtype=np.float32)
    return rng.standard_normal((rows, n), dtype=np.float32)


def row_bytes(dtype: int, dim_in: int) -> int:
    if dtype == F32:
        return 4 * dim_in
    return dim_in // BLOCK_ELEMS[dtype] * BLOCK_BYTES[dtype]
