"""Known-answer tests of the decode-step oracle (oracle/forward_ref.c).

Each case restates an assertion of the reference's own unit tests of the f32
kernels (crates/unltd-tensor/src/kernels.rs, tests module 410-922), so the
oracle that checks the GPU decode step is pinned to the reference. Where the
reference computes its expectation through f64 (sigmoid/silu/softplus at 1),
the same expectation is computed here with numpy f64.
"""
import math
from fractions import Fraction

import numpy as np

import oracle

f32 = np.float32


def fma(a, b, c):
    """Fused multiply-add with one rounding (exact rational arithmetic)."""
    return float(Fraction(a) * Fraction(b) + Fraction(c))


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_rmsnorm_exact_cases():  # kernels.rs:450-487
    assert list(oracle.rmsnorm([1.0] * 4, [1.0] * 4, 0.0)) == [1.0] * 4
    out = oracle.rmsnorm([3.0, 4.0], [1.0, 1.0], 0.0)
    mean = f32((9.0 + 16.0) / 2.0)
    scale = f32(1.0) / np.sqrt(mean + f32(0.0))
    assert bits(out).tolist() == bits([f32(3.0) * scale, f32(4.0) * scale]).tolist()
    assert list(oracle.rmsnorm([0.0, 0.0], [2.0, 3.0], 1e-6)) == [0.0, 0.0]
    sq = f32(1e8) * f32(1e8)
    assert float(sq) != 1e16
    out = oracle.rmsnorm([1e8] * 4, [1.0] * 4, 0.0)
    scale = f32(1.0) / np.sqrt(sq + f32(0.0))
    assert (bits(out) == bits(f32(1e8) * scale)).all()


def test_softmax_max_subtraction_and_partition():  # kernels.rs:563-592
    o1 = oracle.softmax([1000.0, 1001.0, 1002.0], 1.0)
    o2 = oracle.softmax([-2.0, -1.0, 0.0], 1.0)
    assert (bits(o1) == bits(o2)).all()
    e = [float(oracle._fwd_lib().ora_expf(v)) for v in (-2.0, -1.0, 0.0)]
    s = (e[0] + e[1]) + e[2]
    assert bits(o1).tolist() == bits([f32(v / s) for v in e]).tolist()
    assert abs((float(o1[0]) + float(o1[1])) + float(o1[2]) - 1.0) < 1e-7
    assert (bits(oracle.softmax([-2.0, -1.0, 0.0], 2.0)) == bits(oracle.softmax([-4.0, -2.0, 0.0], 1.0))).all()


def test_swiglu_hand_values():  # kernels.rs:595-608
    assert list(oracle.swiglu([0.0, 3.0], [7.0, 0.0])) == [0.0, 0.0]
    out = oracle.swiglu([1.0], [2.0])
    t = 1.0
    e = f32(t * (1.0 / (1.0 + math.exp(-t))) * 2.0)
    assert bits(out)[0] == bits(e)
    assert abs(float(out[0]) - 1.4621172) < 1e-6


def test_sigmoid_silu_softplus_formulas():  # kernels.rs:626-660
    assert list(oracle.sigmoid([0.0] * 3)) == [0.5] * 3
    assert list(oracle.silu([0.0] * 3)) == [0.0] * 3
    assert oracle.softplus([0.0])[0] == f32(math.log(2.0))
    sig = 1.0 / (1.0 + math.exp(-1.0))
    assert bits(oracle.sigmoid([1.0]))[0] == bits(f32(sig))
    assert bits(oracle.silu([1.0]))[0] == bits(f32(1.0 * sig))
    sp = oracle.softplus([1.0])[0]
    assert bits(sp) == bits(f32(math.log(1.0 + math.exp(1.0))))
    assert abs(float(sp) - 1.3132617) < 1e-6
    s = oracle.sigmoid([-1.0, 1.0])
    assert bits(s).tolist() == bits([f32(1.0 / (1.0 + math.exp(1.0))), f32(1.0 / (1.0 + math.exp(-1.0)))]).tolist()
    # softplus passes large inputs through (kernels.rs:217-226)
    assert oracle.softplus([25.0])[0] == f32(25.0)


def test_l2_norm_rows_reference_formula():  # kernels.rs:663-691
    assert list(oracle.l2_norm_rows([3.0, 4.0], 2, 1e-6)) == [f32(0.6), f32(0.8)]
    assert list(oracle.l2_norm_rows([0.0, 0.0], 2, 0.1)) == [0.0, 0.0]
    x = np.array([1.0, 2.0, 3.0], np.float32)
    out = oracle.l2_norm_rows(x, 3, 1e-6)
    scale = f32(1.0) / max(np.sqrt(f32(1.0 + 4.0 + 9.0)), f32(1e-6))
    assert (bits(out) == bits(x * scale)).all()
    assert list(oracle.l2_norm_rows([3.0, 4.0, 6.0, 8.0], 2, 1e-6)) == [f32(0.6), f32(0.8)] * 2


def test_ssm_conv_hand_values_and_f32_order():  # kernels.rs:694-728
    assert list(oracle.ssm_conv([1.0, 10.0, 2.0, 20.0, 3.0, 30.0], [1.0, 2.0, 3.0, 4.0], 2, 2)) == [7.0, 100.0, 11.0, 160.0]
    assert list(oracle.ssm_conv([1e16, 1.0, -1e16, 1.0], [1.0] * 4, 4, 1)) == [1.0]
    k = np.array([0.1, 0.2, 0.3, 0.4], np.float32)
    x = np.array([1.5, 2.5, 3.5, 4.5, 5.5, 6.5], np.float32)
    out = oracle.ssm_conv(x, k, 2, 2)
    for t in range(2):
        for c in range(2):
            s = f32(0.0)
            for tau in range(2):
                s = f32(s + f32(x[(t + tau) * 2 + c] * k[tau * 2 + c]))
            assert bits(out[t * 2 + c]) == bits(s)


def test_rope_imrope_interleaved_pairs():  # kernels.rs:731-778
    x = oracle.rope_imrope([1.0, 99.0, 0.0, 99.0, 7.0, 8.0], 4, 0.01, 1)
    s, c = math.sin(1.0), math.cos(1.0)
    assert bits(x[0]) == bits(f32(fma(c, 1.0, -(s * 0.0))))
    assert bits(x[2]) == bits(f32(fma(s, 1.0, c * 0.0)))
    assert (x[1], x[3], x[4], x[5]) == (99.0, 99.0, 7.0, 8.0)
    orig = np.array([1.5, -2.25, 3.0, 4.0], np.float32)
    assert (oracle.rope_imrope(orig, 4, 0.01, 0) == orig).all()
    orig = np.arange(12, dtype=np.float32)
    x = oracle.rope_imrope(orig, 12, 0.01, 1)

    def rot(x0, x1, a):
        s, c = math.sin(a), math.cos(a)
        return f32(fma(c, float(x0), -(s * float(x1)))), f32(fma(s, float(x0), c * float(x1)))

    r0, r6 = rot(orig[0], orig[6], 1.0)
    r3, r9 = rot(orig[3], orig[9], 0.01 ** 3)
    want = orig.copy()
    want[[0, 3, 6, 9]] = [r0, r3, r6, r9]
    assert (bits(x) == bits(want)).all()


def test_gdn_fused_step_hand_values():  # kernels.rs:799-844, 846-862
    st, out = oracle.gdn_step([1.0, 0.0, 0.0, 1.0], [1.0, 0.0], [1.0, 1.0], [3.0, 4.0], 0.0, 1.0, 1.0)
    assert list(st) == [3.0, 3.0, 2.0, 4.0] and list(out) == [3.0, 3.0]
    st, out = oracle.gdn_step([3.0, 3.0, 2.0, 4.0], [1.0, 1.0], [1.0, 1.0], [3.0, 4.0], 0.0, 1.0, 2.0)
    assert list(st) == [1.0, 0.0, 0.0, 1.0] and list(out) == [2.0, 2.0]


def test_gdn_fused_step_replicates_documented_f32_chain():  # kernels.rs:865-898
    q = np.array([0.25, -0.5, 0.75], np.float32)
    k = np.array([-0.125, 0.5, 0.375], np.float32)
    v = np.array([1.0, -2.0, 0.5], np.float32)
    beta, scale = f32(0.8), f32(0.0625)
    st0 = np.eye(3, dtype=np.float32).reshape(-1)
    st, out = oracle.gdn_step(st0, q, k, v, 0.0, beta, scale)
    rep = st0.copy()
    for j in range(3):
        acc = 0.0
        for i in range(3):
            acc += float(f32(rep[i * 3 + j] * k[i]))
        d = f32(f32(v[j] - f32(acc)) * beta)
        for i in range(3):
            rep[i * 3 + j] = f32(rep[i * 3 + j] + f32(k[i] * d))
    rep_out = np.zeros(3, np.float32)
    for j in range(3):
        acc = 0.0
        for i in range(3):
            acc += float(f32(rep[i * 3 + j] * q[i]))
        rep_out[j] = f32(f32(acc) * scale)
    assert (bits(st) == bits(rep)).all() and (bits(out) == bits(rep_out)).all()


def test_decode_step_is_deterministic_and_stateful():
    """The oracle's decode step: same inputs give the same bits for any
    thread count; the state carries over (the same token again differs)."""
    import synth

    cfg = synth.QWEN35_TINY
    t = synth.qwen35_model(cfg, 3)
    st = synth.qwen35_state(cfg, 10, 4)
    a = oracle.Qwen35Oracle(cfg, t, 32, st, 10)
    b = oracle.Qwen35Oracle(cfg, t, 32, st, 10)
    la, ha = a.step(7, nthreads=2)
    lb, hb = b.step(7, nthreads=1)
    assert (bits(la) == bits(lb)).all() and (bits(ha) == bits(hb)).all()
    la2, _ = a.step(7)
    assert not np.array_equal(la2, la)
    assert a.position == 12


def test_row_split_restates_rank_order_sums():
    """Qwen35Oracle.row_split(world): the input-split projections as
    per-rank partial gemv_quant_q8k over equal column slices, summed in rank
    order. One projection restated in numpy from the one-device
    gemv_quant_q8k of each slice gives the same bits as a decode step built
    on it predicts: world 1 is the one-device step again, world 2 moves the
    hidden state by rounding only (same greedy token, close values)."""
    import synth

    # one GEMV: rank partials summed in rank order (f32)
    for dtype, din in ((synth.Q4K, 1024), (synth.Q6K, 2048)):
        dout = 37
        wb = synth.quant_weights(dtype, din, dout, seed=din)
        x = synth.activations(din, seed=din + 1)
        rbf = oracle.row_bytes(dtype, din)
        W = np.frombuffer(bytes(wb), np.uint8).reshape(dout, rbf)
        for world in (2, 4):
            cols = din // world
            rbs = oracle.row_bytes(dtype, cols)
            y = None
            for r in range(world):
                ws = np.ascontiguousarray(W[:, r * rbs:(r + 1) * rbs])
                p = oracle.gemv_quant_q8k(x[r * cols:(r + 1) * cols], ws, cols, dout, dtype)
                y = p if y is None else (y + p).astype(np.float32)
            full = oracle.gemv_quant_q8k(x, wb, din, dout, dtype)
            assert np.max(np.abs(y - full)) <= 1e-4 * np.max(np.abs(full))
    # the forward
    cfg = synth.QWEN35_TINY
    t = synth.qwen35_model(cfg, 3)
    st = synth.qwen35_state(cfg, 10, 4)
    l1, h1 = oracle.Qwen35Oracle(cfg, t, 32, st, 10).step(7)
    oracle.Qwen35Oracle.row_split(2)
    try:
        l2, h2 = oracle.Qwen35Oracle(cfg, t, 32, st, 10).step(7)
    finally:
        oracle.Qwen35Oracle.row_split(1)
    l3, h3 = oracle.Qwen35Oracle(cfg, t, 32, st, 10).step(7)
    assert (bits(l3) == bits(l1)).all() and (bits(h3) == bits(h1)).all()
    assert not np.array_equal(bits(h2), bits(h1))
    assert oracle.argmax(l2) == oracle.argmax(l1)
    assert np.max(np.abs(h2 - h1)) <= 1e-3 * np.max(np.abs(h1))
