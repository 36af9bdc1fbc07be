"""The exact resolution of sequential f64 sums used by the decode kernels
(forward.cu: attn_combine_quant_kernel, gdn_dot, resolve_sum), checked in
numpy: whenever the error bound decides a result, that result must be the f32
rounding of the reference's left-to-right f64 sum (np.cumsum is that sum).
Adversarial inputs included: heavy cancellation, tiny results, wide ranges."""
import numpy as np
import pytest

f32 = np.float32


def chunked_resolve(t, chunk):
    """Mirror of the kernels: in-order chunk sums with running |partial| sums,
    combined in order; B = 2^-51 (2 T1 + T2 + T3)."""
    O = 0.0
    T1 = T2 = T3 = 0.0
    for w0 in range(0, len(t), chunk):
        c = t[w0:w0 + chunk]
        run = np.cumsum(c)
        Sw = float(run[-1])
        Qw = float(np.cumsum(np.abs(run))[-1])
        T1 += Qw
        T2 += len(c) * abs(O)
        O = O + Sw
        T3 += abs(O)
    B = 2.0 ** -51 * (2.0 * T1 + T2 + T3)
    lo, hi = f32(O - B), f32(O + B)
    return (lo == hi), lo


def positive_resolve(t):
    """resolve_sum for nonnegative terms (rmsnorm, l2 norm): B = (n+8) 2^-51 S."""
    S = float(np.sum(t))  # any order
    B = (len(t) + 8) * 2.0 ** -51 * S
    n = len(t)
    lo, hi = f32((S - B) / n), f32((S + B) / n)
    return lo == hi, lo


def _terms(rng, n, kind):
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    if kind == "cancel":  # large alternating terms, small sum
        b = (np.abs(b) * np.where(np.arange(n) % 2, 1, -1) * 1e3).astype(np.float32)
    elif kind == "wide":
        a = (a * np.exp(rng.uniform(-30, 30, n))).astype(np.float32)
    elif kind == "softmax":  # attention: weights in (0, 1], values N(0,1)
        a = rng.random(n).astype(np.float32) ** 8
    return a.astype(np.float64) * b.astype(np.float64)  # exact products, as the kernels form them


@pytest.mark.parametrize("kind", ["normal", "cancel", "wide", "softmax"])
@pytest.mark.parametrize("chunk", [32, 64])
def test_chunked_bound_never_misresolves(kind, chunk):
    rng = np.random.default_rng(hash((kind, chunk)) & 0xFFFF)
    resolved = 0
    for trial in range(300):
        n = int(rng.integers(1, 2200 if chunk == 64 else 129))
        t = _terms(rng, n, kind)
        ok, v = chunked_resolve(t, chunk)
        ref = f32(np.cumsum(t)[-1])
        if ok:
            resolved += 1
            assert v == ref or (np.isnan(v) and np.isnan(ref)), (kind, n, trial)
    assert resolved > 250  # the fallback stays rare


def test_chunked_bound_detects_a_boundary_case():
    # a sum built to sit on an f32 rounding boundary is not claimed
    half_ulp = 2.0 ** -24
    t = np.array([1.0, half_ulp, 1e-300], np.float64)
    ok, _ = chunked_resolve(t, 2)
    assert not ok


def test_positive_bound_never_misresolves():
    rng = np.random.default_rng(5)
    for trial in range(300):
        n = int(rng.integers(1, 5000))
        x = (rng.standard_normal(n) * np.exp(rng.uniform(-5, 5))).astype(np.float32)
        t = (x * x).astype(np.float32).astype(np.float64)  # f32 squares, summed in f64
        ok, v = positive_resolve(t)
        if ok:
            assert v == f32(np.cumsum(t)[-1] / n)
