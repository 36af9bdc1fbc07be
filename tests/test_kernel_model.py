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


def test_warp_span_writer_positions():
    # q8k_span_write_warp: lane l writes element 8l + k at base(l) + 16k with
    # base = 128 (g >> 2) + 4 (g & 3) + (l & 3), g = l >> 2; the same bytes as
    # the per-element class-major position q4k_q8k_xpos, and group g's sum is
    # the sum of lanes 4g .. 4g+3
    lane = np.arange(32)[:, None]
    k = np.arange(8)[None, :]
    g = lane >> 2
    warp_pos = 128 * (g >> 2) + 4 * (g & 3) + (lane & 3) + 16 * k
    assert np.array_equal(warp_pos, km.q4k_q8k_xpos(8 * lane + k))
    assert np.array_equal((8 * lane + k) >> 5, np.broadcast_to(g, (32, 8)))


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


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q6k_mma_fragments_match_reference(seed):
    # the tensor-core Q6_K item's fragment mapping gives the reference's
    # per-class integer sums for 16 rows of random blocks
    import synth
    rng = np.random.default_rng(seed)
    wb = synth.quant_weights(6, 256, 16, seed=100 + seed)
    blks = [wb[r * 210:(r + 1) * 210] for r in range(16)]
    q8 = rng.integers(-127, 128, size=256).astype(np.int64)
    got = km.q6k_rows_mma_model(blks, q8)
    for r in range(16):
        assert np.array_equal(got[r], km.q6k_block_sumi_reference(blks[r], q8))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q4k_minsum_mma_fragments_match_reference(seed):
    # the Q4_K item's min-term MMA (6-bit mins x group sums split into two
    # byte columns) gives the reference's minsum for 16 rows, extreme q8 too
    import synth
    rng = np.random.default_rng(seed)
    wb = synth.quant_weights(synth.Q4K, 256, 16, seed=200 + seed)
    blks = [wb[r * 144:(r + 1) * 144] for r in range(16)]
    for q8 in (rng.integers(-127, 128, size=256), np.full(256, 127), np.full(256, -127),
               np.where(np.arange(256) % 3 == 0, 127, -127)):
        q8 = q8.astype(np.int64)
        got = km.q4k_minsum_mma_model([km.repack_q4k_block(b)[0] for b in blks], q8)
        for r in range(16):
            assert got[r] == km.q4k_block_sumi_reference(blks[r], q8)[1]


def test_q4k_scale_split_batched_sums_equal_reference():
    # design model of a batched (several sequences) Q4_K Q8_K dot: the
    # per-class integer sums of every (row, sequence) pair equal the
    # reference's sumi (quants.rs:328-351), including all-63 scales and the
    # extreme q8 values
    rng = np.random.default_rng(41)
    blks = [rng.integers(0, 256, size=144).astype(np.uint8) for _ in range(12)]
    blks[0][4:16] = 0xFF  # every 6-bit scale and min = 63
    blks[0][16:] = 0xFF  # every quant = 15
    q8s = rng.integers(-127, 128, size=(5, 256)).astype(np.int64)
    q8s[0] = 127
    q8s[1] = -127
    got = km.q4k_sumi_scale_split_batched(blks, q8s)
    for r, blk in enumerate(blks):
        for b in range(q8s.shape[0]):
            ref, _ = km.q4k_block_sumi_reference(blk, q8s[b])
            assert np.array_equal(got[r, b], ref), (r, b)


def test_q4k_batched_gemv_model_bit_identical_to_oracle():
    # the whole batched Q4_K Q8_K GEMV of the design model: for every
    # sequence, the same bits as the reference's gemv_quant_q8k
    import oracle
    import synth

    dim_in, dim_out, B = 1024, 24, 6
    wb = synth.quant_weights(synth.Q4K, dim_in, dim_out, seed=43)
    xs = [synth.activations(dim_in, seed=44 + b) for b in range(B)]
    xs[1][:256] = 0.0  # an all-zero block: d = 0, qs = 0
    q8 = [oracle.quantize_q8_k(x) for x in xs]
    q8_d = np.array([[blk.d for blk in q] for q in q8], np.float32)
    q8_qs = np.array([[list(blk.qs) for blk in q] for q in q8], np.int64)
    got = km.q4k_gemv_q8k_batched_model(wb, dim_in, dim_out, q8_d, q8_qs)
    for b in range(B):
        ref = oracle.gemv_quant_q8k(xs[b], wb, dim_in, dim_out, synth.Q4K)
        assert np.array_equal(got[b].view(np.uint32), ref.view(np.uint32)), b


def test_q6k_batched_gemv_model_bit_identical_to_oracle():
    # Q6_K with full-range int8 scales (-128 and 127 included): the two-operand
    # split of sc * (raw6 - 32) stays exact and the batch gives the
    # reference's bits for every sequence
    import oracle
    import synth

    dim_in, dim_out, B = 768, 20, 5
    wb = synth.quant_weights(synth.Q6K, dim_in, dim_out, seed=45).copy()
    blocks = wb.reshape(-1, 210)
    blocks[0, 192:208] = np.array([-128, 127] * 8, np.int8).view(np.uint8)
    blocks[0, :192] = 0xFF  # raw6 = 63 everywhere in that block
    blocks[1, :192] = 0x00  # raw6 = 0 everywhere: a = -32
    blocks[1, 192:208] = np.array([-128] * 16, np.int8).view(np.uint8)
    xs = [synth.activations(dim_in, seed=46 + b) for b in range(B)]
    q8 = [oracle.quantize_q8_k(x) for x in xs]
    q8_d = np.array([[blk.d for blk in q] for q in q8], np.float32)
    q8_qs = np.array([[list(blk.qs) for blk in q] for q in q8], np.int64)
    got = km.q6k_gemv_q8k_batched_model(wb, dim_in, dim_out, q8_d, q8_qs)
    for b in range(B):
        ref = oracle.gemv_quant_q8k(xs[b], wb, dim_in, dim_out, synth.Q6K)
        assert np.array_equal(got[b].view(np.uint32), ref.view(np.uint32)), b
