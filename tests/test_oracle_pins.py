"""Pin the CPU oracle against the reference's own known-answer tests.

Every case here restates a test of crates/unltd-tensor/src/quants.rs
(lines cited per test), crates/unltd-tensor/src/kernels.rs:435-447 and
crates/unltd-generation/src/greedy.rs, plus the real-model golden blocks
(tests/golden/ornith_pins.json, extracted from quants.rs:1094-1198).
"""
import json
import os
import struct

import numpy as np
import pytest

F16_ONE = 0x3C00
F16_TWO = 0x4000
HERE = os.path.dirname(os.path.abspath(__file__))


def q4_block(d, dmin, scales, qs):
    b = struct.pack("<HH", d, dmin) + bytes(scales) + bytes(qs)
    assert len(b) == 144
    return b


def q6_block(d, ql, qh, scales):
    b = bytes(ql) + bytes(qh) + bytes((s & 0xFF) for s in scales) + struct.pack("<H", d)
    assert len(b) == 210
    return b


def f32bits(v):
    return struct.unpack("<I", struct.pack("<f", float(v)))[0]


def test_f16_to_f32_known_patterns(ora):  # quants.rs:582-596
    f = ora.f16_to_f32
    assert f(0x3C00) == 1.0 and f(0x4000) == 2.0 and f(0xC000) == -2.0
    assert f(0x0000) == 0.0 and f32bits(f(0x8000)) == 0x80000000
    assert np.isinf(f(0x7C00)) and f(0x7C00) > 0
    assert np.isinf(f(0xFC00)) and f(0xFC00) < 0
    assert np.isnan(f(0x7E00))
    assert f32bits(f(0x7E01)) == 0x7FC00000  # quiet NaN, payload 0 (quants.rs:66)
    assert f(0x0001) == np.float32(2.0**-24)
    assert f(0x03FF) == np.float32(2.0**-14 - 2.0**-24)
    assert f(0x7BFF) == 65504.0
    assert f(0x3555) == np.float32(0.333251953125)


def test_f16_to_f32_all_patterns_match_numpy(ora):
    # canonical conversion == IEEE half widening for every non-NaN pattern
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([ora.f16_to_f32(int(v)) for v in range(0, 65536, 7)], dtype=np.float32)
    sel = ref[::7]
    nan = np.isnan(sel)
    assert np.array_equal(got[~nan].view(np.uint32), sel[~nan].view(np.uint32))
    assert np.all(np.isnan(got[nan]))


def test_dot_f32_small_exact(ora):  # quants.rs:598-604
    assert ora.dot_f32([1, 2, 3, 4], [5, 6, 7, 8]) == 70.0
    assert ora.dot_f32([1, 2, 3], [4, 5, 6]) == 32.0


def test_pairwise_partition_is_the_documented_tree(ora):  # kernels.rs:435-447
    assert ora.pairwise_sum_f64([1, 2, 3, 4, 5]) == 15.0
    assert ora.pairwise_sum_f64([1e16, 1.0, -1e16, 1.0]) == 0.0
    assert ora.pairwise_sum_f64([1, 2, 3]) == 6.0
    assert ora.pairwise_sum_f64([]) == 0.0


def test_dequantize_q4_k_hand_values_and_multi_block(ora):  # quants.rs:607-648
    scales = [0] * 12
    scales[0], scales[4], scales[1], scales[5] = 1, 3, 2, 1
    qs = [0] * 128
    qs[0] = 0x12
    a = q4_block(F16_ONE, F16_TWO, scales, qs)
    b = q4_block(0, 0, [0] * 12, [0xAB] * 128)
    out = ora.dequantize_q4_k(a + b, 512)
    assert out[0] == -4.0 and out[1] == -6.0 and out[31] == -6.0
    assert out[32] == 0.0 and out[33] == -2.0
    assert np.all(out[64:512] == 0.0)
    x = np.full(256, 0.5, np.float32)
    exact = ora.dot_q4_k(x, a)
    via = ora.dot_f32(x, out[:256])
    assert abs(via - exact) < 1e-4


def test_dequantize_q4_k_matches_reference_formula_bitwise(ora):  # quants.rs:651-684
    scales = [0x1F, 0x2E, 0x3D, 0x4C, 0x5B, 0x6A, 0x79, 0x03, 0x92, 0x81, 0x70, 0x6F]
    qs = [(i * 7 + 3) & 0xFF for i in range(128)]
    d_bits, dmin_bits = 0x3B21, 0x2C10
    blk = q4_block(d_bits, dmin_bits, scales, qs)
    out = ora.dequantize_q4_k(blk, 256)
    d = np.float32(ora.f16_to_f32(d_bits))
    mn = np.float32(ora.f16_to_f32(dmin_bits))

    def smk(g):
        if g < 4:
            return scales[g] & 63, scales[g + 4] & 63
        return (scales[g + 4] & 0xF) | ((scales[g - 4] >> 6) << 4), (scales[g + 4] >> 4) | ((scales[g] >> 6) << 4)

    e = 0
    for is_ in range(0, 8, 2):
        pair = qs[32 * (is_ // 2): 32 * (is_ // 2) + 32]
        for g, shift in ((is_, 0), (is_ + 1, 4)):
            sc, m = smk(g)
            dg = np.float32(d * np.float32(sc))
            mg = np.float32(mn * np.float32(m))
            for l in range(32):
                expected = np.float32(np.float32(dg * np.float32((pair[l] >> shift) & 0xF)) - mg)
                assert f32bits(out[e]) == f32bits(expected), e
                e += 1


def test_q4_k_zero_block_and_hand_values(ora):  # quants.rs:708-743
    blk = q4_block(F16_ONE, 0, [0] * 12, [0xFF] * 128)
    assert ora.dot_q4_k(np.full(256, 0.5, np.float32), blk) == 0.0
    scales = [0] * 12
    scales[0], scales[4] = 1, 3
    qs = [0] * 128
    qs[0] = 0x01
    blk = q4_block(F16_ONE, F16_TWO, scales, qs)
    x = np.zeros(256, np.float32)
    x[0] = 1
    assert ora.dot_q4_k(x, blk) == -5.0
    x[0], x[1] = 0, 1
    assert ora.dot_q4_k(x, blk) == -6.0
    scales = [0] * 12
    scales[0], scales[4], scales[8] = 0xC0, 0x43, 0x31
    qs = [0] * 128
    qs[64] = 0x01
    blk = q4_block(F16_ONE, F16_ONE, scales, qs)
    x = np.zeros(256, np.float32)
    x[128] = 1
    assert ora.dot_q4_k(x, blk) == 30.0


def test_q4_k_pairwise_tree_is_the_contract(ora):  # quants.rs:746-766
    scales = [0] * 12
    scales[0] = 1
    qs = [0] * 128
    qs[0:4] = [0x0A, 0x01, 0x0A, 0x01]
    blk = q4_block(F16_ONE, 0, scales, qs)
    x = np.zeros(256, np.float32)
    x[0:4] = [1e19, 1.0, -1e19, 1.0]
    assert ora.dot_q4_k(x, blk) == 0.0


def test_q4_k_full_block_matches_layout_reference(ora):  # quants.rs:769-788
    qs = [i & 0xFF for i in range(128)]
    blk = q4_block(F16_ONE, 0, [1] * 12, qs)
    x = np.arange(1, 257, dtype=np.float32)
    exp = 0.0
    for e in range(256):
        g = e // 32
        byte = qs[32 * (g // 2) + e % 32]
        nib = byte & 0xF if g % 2 == 0 else byte >> 4
        exp += (e + 1) * nib
    assert ora.dot_q4_k(x, blk) == exp


def test_q4_k_multiblock_stride(ora):  # quants.rs:791-802
    qs = [0] * 128
    qs[0] = 1
    w = q4_block(F16_ONE, 0, [1] * 12, qs) + q4_block(F16_TWO, 0, [1] * 12, qs)
    assert ora.dot_q4_k(np.ones(512, np.float32), w) == 3.0


def test_q6_k_zero_block_and_hand_values(ora):  # quants.rs:805-872
    blk = q6_block(F16_TWO, [0xFF] * 128, [0xFF] * 64, [0] * 16)
    assert ora.dot_q6_k(np.full(256, 0.5, np.float32), blk) == 0.0
    cases = [
        # (ql edits, qh edits, scales, element, expected)
        ({0: 0x01}, {}, [1] * 16, 0, -62.0),
        ({32: 0x03}, {0: 0x04}, {2: -1}, 32, 26.0),
        ({0: 0x50}, {0: 0x10}, {4: 3}, 64, -66.0),
        ({32: 0x70}, {0: 0x40}, [1] * 16, 96, -18.0),
        ({64: 0x02}, {32: 0x02}, {8: 5}, 128, 20.0),
    ]
    for qle, qhe, sce, elem, expected in cases:
        ql, qh = [0] * 128, [0] * 64
        for k, v in qle.items():
            ql[k] = v
        for k, v in qhe.items():
            qh[k] = v
        if isinstance(sce, dict):
            sc = [0] * 16
            for k, v in sce.items():
                sc[k] = v
        else:
            sc = list(sce)
        blk = q6_block(F16_TWO, ql, qh, sc)
        x = np.zeros(256, np.float32)
        x[elem] = 1
        assert ora.dot_q6_k(x, blk) == expected, elem


def test_q6_k_pairwise_tree_is_the_contract(ora):  # quants.rs:875-901
    ql = [0] * 128
    ql[0:4] = [0x0A, 0x01, 0x0A, 0x01]
    qh = [0] * 64
    qh[0:4] = [2, 2, 2, 2]
    sc = [0] * 16
    sc[0] = 1
    blk = q6_block(F16_ONE, ql, qh, sc)
    x = np.zeros(256, np.float32)
    x[0:4] = [1e19, 1.0, -1e19, 1.0]
    assert ora.dot_q6_k(x, blk) == 0.0


def test_q6_k_full_block_matches_layout_reference(ora):  # quants.rs:904-934
    ql = [i & 0xFF for i in range(128)]
    qh = [i & 0xFF for i in range(64)]
    sc = [i - 8 for i in range(16)]
    blk = q6_block(F16_ONE, ql, qh, sc)
    x = np.arange(1, 257, dtype=np.float32)
    exp = 0.0
    for e in range(256):
        byte = ql[64 * (e // 128) + e % 64]
        nib = byte & 0xF if (e // 64) % 2 == 0 else byte >> 4
        hi2 = (qh[(e % 32) + 32 * (e // 128)] >> (2 * ((e % 128) // 32))) & 3
        q = nib | (hi2 << 4)
        exp += (e + 1) * sc[e // 16] * (q - 32)
    assert ora.dot_q6_k(x, blk) == exp


def test_q6_k_multiblock_stride(ora):  # quants.rs:937-952
    ql = [0] * 128
    ql[0] = 1
    sc = [0] * 16
    sc[0] = 1
    w = q6_block(F16_ONE, ql, [0] * 64, sc) + q6_block(F16_TWO, ql, [0] * 64, sc)
    assert ora.dot_q6_k(np.ones(512, np.float32), w) == -511.0 + -1022.0


def test_nearest_int_replicates_ggml_magic(ora):  # quants.rs:955-965
    ni = ora.nearest_int
    assert [ni(v) for v in (0.0, 2.5, 3.5, -3.5, 126.7, -126.7, 0.5, 1.5)] == [0, 2, 4, -4, 127, -127, 0, 2]


def test_quantize_q8_k_hand_block_and_zero_block(ora):  # quants.rs:968-1000
    x = np.zeros(256, np.float32)
    x[0] = 1
    q = ora.quantize_q8_k(x)
    assert len(q) == 1 and q[0].qs[0] == -127 and all(v == 0 for v in q[0].qs[1:])
    assert q[0].bsums[0] == -127 and all(v == 0 for v in q[0].bsums[1:])
    assert np.float32(q[0].d) == np.float32(1.0) / np.float32(-127.0)
    x[0] = -1
    q = ora.quantize_q8_k(x)
    assert q[0].qs[0] == -127 and np.float32(q[0].d) == np.float32(1.0) / np.float32(127.0)
    q = ora.quantize_q8_k(np.zeros(256, np.float32))
    assert q[0].d == 0.0 and all(v == 0 for v in q[0].qs)
    two = np.zeros(512, np.float32)
    two[256] = 2
    q = ora.quantize_q8_k(two)
    assert len(q) == 2 and q[0].d == 0.0 and q[1].qs[0] == -127


def test_dot_q4_k_q8_k_hand_values(ora):  # quants.rs:1003-1021
    scales = [0] * 12
    scales[0], scales[4] = 1, 3
    qs = [0] * 128
    qs[0] = 1
    blk = q4_block(F16_ONE, F16_TWO, scales, qs)
    x = np.zeros(256, np.float32)
    x[0] = 127
    assert ora.dot_q4_k_q8_k(ora.quantize_q8_k(x), blk) == -635.0


def test_dot_q6_k_q8_k_hand_values(ora):  # quants.rs:1024-1057
    ql = [0] * 128
    ql[0] = 1
    sc = [0] * 16
    sc[0] = 1
    blk = q6_block(F16_ONE, ql, [0] * 64, sc)
    x = np.zeros(256, np.float32)
    x[0] = 127
    assert ora.dot_q6_k_q8_k(ora.quantize_q8_k(x), blk) == -3937.0
    ql = [0] * 128
    ql[32] = 1
    sc = [0] * 16
    sc[2] = -1
    blk = q6_block(F16_ONE, ql, [0] * 64, sc)
    x = np.zeros(256, np.float32)
    x[32] = 127
    assert ora.dot_q6_k_q8_k(ora.quantize_q8_k(x), blk) == 3937.0


def _pins():
    with open(os.path.join(HERE, "golden", "ornith_pins.json")) as f:
        return json.load(f)


def _pin_xs():
    i = np.arange(256)
    xp = (((i * 7919) % 1009).astype(np.float32) / np.float32(1009.0) - np.float32(0.5)).astype(np.float32)
    xa = (((i * 31 + 17) % 257).astype(np.float32) / np.float32(257.0) - np.float32(0.5)).astype(np.float32)
    return xp, xa


def test_q8k_dots_close_to_exact_dots(ora):  # quants.rs:1060-1083
    pins = _pins()
    xp, _ = _pin_xs()
    q = ora.quantize_q8_k(xp)
    for name in ("Q4K_B0", "Q4K_B15"):
        raw = bytes.fromhex(pins["blocks_hex"][name])
        assert abs(ora.dot_q4_k(xp, raw) - float(ora.dot_q4_k_q8_k(q, raw))) < 0.5
    for name in ("Q6K_B0", "Q6K_B15"):
        raw = bytes.fromhex(pins["blocks_hex"][name])
        assert abs(ora.dot_q6_k(xp, raw) - float(ora.dot_q6_k_q8_k(q, raw))) < 0.5


def test_ornith_decode_pin(ora):  # quants.rs:1155-1222 (gguf-py values)
    pins = _pins()
    xp, xa = _pin_xs()
    hot7 = np.zeros(256, np.float32)
    hot7[7] = 1
    hot200 = np.zeros(256, np.float32)
    hot200[200] = 1
    tol = pins["tolerance"]
    for c in pins["cases"]:
        raw = bytes.fromhex(pins["blocks_hex"][c["block"]])
        dot = ora.dot_q6_k if len(raw) == 210 else ora.dot_q4_k
        assert abs(dot(xp, raw) - c["dot_x_pattern"]) < tol
        assert abs(dot(xa, raw) - c["dot_x_alt"]) < tol
        assert abs(dot(hot7, raw) - c["w7"]) < tol
        assert abs(dot(hot200, raw) - c["w200"]) < tol


def test_argmax_first_index_on_ties(ora):  # greedy.rs:18-27
    assert ora.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert ora.argmax([5.0]) == 0
    assert ora.argmax([-1.0, -1.0]) == 0
    with pytest.raises(ValueError):
        ora.argmax([])


def test_row_bytes_sizes_are_exact(ora):  # min_forward.rs:283-293
    assert ora.row_bytes(ora.F32, 4096) == 16384
    assert ora.row_bytes(ora.Q4K, 4096) == 16 * 144
    assert ora.row_bytes(ora.Q6K, 4096) == 16 * 210
    assert ora.row_bytes(ora.Q8_0, 64) == 2 * 34
    assert ora.row_bytes(ora.Q4K, 4097) == 0
    assert ora.row_bytes(ora.Q8_0, 33) == 0


def test_gemv_refusals_mirror_reference_asserts(ora):  # quants.rs:430-452, 482-505
    w = bytes(144)
    with pytest.raises(ValueError):  # dim_in not a multiple of 256
        ora.gemv_quant(np.zeros(300, np.float32), w, 300, 1, ora.Q4K)
    with pytest.raises(ValueError):  # len(w) != rows * row_bytes
        ora.gemv_quant(np.zeros(256, np.float32), w, 256, 2, ora.Q4K)
    with pytest.raises(ValueError):  # Q8_0 has no q8_K path in the reference
        ora.gemv_quant_q8k(np.zeros(32, np.float32), bytes(34), 32, 1, ora.Q8_0)


def test_gemv_rows_equal_row_dots_and_threads_agree(ora):
    rng = np.random.default_rng(5)
    for dt, nbytes in ((ora.Q4K, 144), (ora.Q6K, 210)):
        w = rng.integers(0, 256, size=3 * 2 * nbytes, dtype=np.uint8)
        # keep the f16 scales finite and small
        for r in range(6):
            off = r * nbytes + (0 if dt == ora.Q4K else 208)
            w[off:off + 2] = np.frombuffer(np.float16(0.01 * (r + 1)).tobytes(), np.uint8)
            if dt == ora.Q4K:
                w[off + 2:off + 4] = np.frombuffer(np.float16(0.002).tobytes(), np.uint8)
        x = rng.standard_normal(512).astype(np.float32)
        y1 = ora.gemv_quant(x, w, 512, 3, dt, 1)
        y4 = ora.gemv_quant(x, w, 512, 3, dt, 4)
        dot = ora.dot_q4_k if dt == ora.Q4K else ora.dot_q6_k
        rb = 2 * nbytes
        for j in range(3):
            assert y1[j] == np.float32(dot(x, w[j * rb:(j + 1) * rb]))
        assert np.array_equal(y1, y4)
        q1 = ora.gemv_quant_q8k(x, w, 512, 3, dt, 1)
        q4 = ora.gemv_quant_q8k(x, w, 512, 3, dt, 3)
        assert np.array_equal(q1.view(np.uint32), q4.view(np.uint32))
