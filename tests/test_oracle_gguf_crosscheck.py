"""Cross-check the oracle's dequantization with gguf-py, an independent
implementation of the same GGUF block formats (the reference used it the
same way: benchmarks/reference/ornith-decode-crosscheck.py:22-69).

Q8_0 parity is otherwise unpinned (the reference has no Q8_0 kernel), so this
is the only independent pin of that format.
"""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as QT  # noqa: E402


def _rand_blocks(rng, dtype, nblocks, ora):
    nbytes = ora.BLOCK_BYTES[dtype]
    w = rng.integers(0, 256, size=(nblocks, nbytes), dtype=np.uint8)
    # finite f16 scales so NaN/inf do not hide mapping errors
    d = rng.uniform(-0.02, 0.02, size=nblocks).astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    if dtype == ora.Q4K:
        w[:, 0:2] = d
        w[:, 2:4] = rng.uniform(0, 0.01, size=nblocks).astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    elif dtype == ora.Q6K:
        w[:, 208:210] = d
    else:
        w[:, 0:2] = d
    return w.reshape(-1)


@pytest.mark.parametrize("name", ["Q4K", "Q6K", "Q8_0"])
def test_dequant_matches_gguf_py(ora, name):
    dtype = getattr(ora, name)
    qt = {"Q4K": QT.Q4_K, "Q6K": QT.Q6_K, "Q8_0": QT.Q8_0}[name]
    rng = np.random.default_rng(11)
    nblocks = 64
    w = _rand_blocks(rng, dtype, nblocks, ora)
    n = nblocks * ora.BLOCK_ELEMS[dtype]
    mine = ora.dequantize(w, n, dtype)
    theirs = np.asarray(gguf.quants.dequantize(w.reshape(1, -1), qt), dtype=np.float32).reshape(-1)
    assert theirs.shape == mine.shape
    # gguf-py evaluates in numpy f32 with its own operation order; all three
    # formats give exact products, so the only possible difference is the
    # single rounding of Q4_K's subtraction, which both perform once.
    assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32))
