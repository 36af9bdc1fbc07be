"""CPU check of the GEMV kernels' lane/permutation arithmetic (kernel_model.py)
against the oracle: integer lane sums must be identical, F32X within the
stated tolerance. No GPU needed."""
import numpy as np
import pytest

import kernel_model as km


def _rand_q8(rng):
    return rng.integers(-127, 128, size=256).astype(np.int64)


def test_permutations_are_bijections():
    assert sorted(km.q4_xpos(np.arange(256)).tolist()) == list(range(256))
    assert sorted(km.q6_xpos(np.arange(256)).tolist()) == list(range(256))
    assert sorted(km.q6_pic(np.arange(16)).tolist()) == list(range(16))


def test_q4k_lane_classes_are_pure():
    # every 4-byte word a lane loads holds 4 elements of one scale group and one class e%8
    e = np.arange(256)
    pos = km.q4_xpos(e)
    for w in range(64):
        members = e[(pos >> 2) == w]
        assert len(set((members % 8).tolist())) == 1
        assert len(set((members // 32).tolist())) == 1


def test_q6k_word_pairs_are_pure():
    e = np.arange(256)
    pos = km.q6_xpos(e)
    for w in range(64):
        members = e[(pos >> 2) == w]
        assert len(set((members // 16).tolist())) == 1  # one scale group per word
        by_pos = {int(pp & 3): int(m) for pp, m in zip(pos[(pos >> 2) == w], members)}
        assert by_pos[0] % 8 == by_pos[1] % 8 and by_pos[2] % 8 == by_pos[3] % 8


@pytest.mark.parametrize("seed", range(6))
def test_q4k_q8k_lane_sums_match_reference(ora, seed):
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=144, dtype=np.uint8)
    q8 = _rand_q8(rng)
    s_model, m_model = km.q4k_block_sumi_model(blk, q8)
    s_ref, m_ref = km.q4k_block_sumi_reference(blk, q8)
    assert np.array_equal(s_model, s_ref) and m_model == m_ref


@pytest.mark.parametrize("seed", range(6))
def test_q6k_q8k_lane_sums_match_reference(ora, seed):
    rng = np.random.default_rng(100 + seed)
    blk = rng.integers(0, 256, size=210, dtype=np.uint8)
    q8 = _rand_q8(rng)
    assert np.array_equal(km.q6k_block_sumi_model(blk, q8), km.q6k_block_sumi_reference(blk, q8))


@pytest.mark.parametrize("seed", range(4))
def test_q4k_f32x_model_within_tolerance(ora, seed):
    rng = np.random.default_rng(200 + seed)
    blk = rng.integers(0, 256, size=144, dtype=np.uint8)
    blk[0:2] = np.frombuffer(np.float16(0.004).tobytes(), np.uint8)
    blk[2:4] = np.frombuffer(np.float16(0.002).tobytes(), np.uint8)
    x = rng.standard_normal(256).astype(np.float32)
    exact = ora.dot_q4_k(x, blk)
    got = km.q4k_block_f32x_model(blk, x)
    deq = ora.dequantize_q4_k(blk, 256).astype(np.float64)
    scale = float(np.abs(deq * x).sum())
    assert abs(got - exact) <= 1e-6 * scale
