"""GPU parity of the tensor-core prefill GEMM (unltd_gemm, unltd_gemm_f32x) against the oracle.

Ground truth: f64 products of X and the oracle's exact dequantized weights
(every Q4_K weight is exact in f32), i.e. gemv_quant (quants.rs:422) per
token before its final rounding. The kernel feeds the tensor cores fp16
operands (unit roundoff u = 2^-11): X rounded once; W = q * fp16(d*sc) -
fp16(dmin*m) in one fp16 FMA; f32 accumulation. Per element that gives
|Y - T| <= 2^-9 * sum_k |X_k| (|W_k| + |d sc q|_k + |dmin m|_k), which the
test asserts (a rigorous bound with margin), and it reports the normwise error.

The accurate mode (unltd_gemm_f32x) carries X and W as hi + lo fp16 pairs
(22 significant bits each; the dropped Xl Wl term is below 2^-22 relative):
it must meet gemv_quant's bar, max |Y - T| / max |T| <= 1e-4, and per element
|Y - T| <= 2^-14 * sum_k |X_k| |W_k| (the f32 accumulation over K included).
"""
import numpy as np
import pytest

import oracle
import synth
import unltd_gpu as ug

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
BOUND = 2.0 ** -9


def q4k_magnitudes(wb, K, N):
    """|d*sc*q| + |dmin*m| per weight (the unreduced terms), row-major [N][K]."""
    blk = np.asarray(wb, np.uint8).reshape(-1, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float64)[:, 0]
    dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float64)[:, 0]
    s = blk[:, 4:16].astype(np.int64)
    sc = np.zeros((len(blk), 8), np.int64)
    m = np.zeros((len(blk), 8), np.int64)
    sc[:, :4], m[:, :4] = s[:, 0:4] & 63, s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
    m[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    qs = blk[:, 16:].astype(np.int64).reshape(-1, 4, 32)
    q = np.stack([qs & 0xF, qs >> 4], axis=2).reshape(-1, 256)  # element order 64p + 32h + l
    g = np.arange(256) // 32
    mag = np.abs(d[:, None] * sc[:, g] * q) + np.abs(dmin[:, None] * m[:, g])
    return mag.reshape(N, K)


def _check(Y, X, W, wb, K, N):
    X64 = X.astype(np.float64)
    T = X64 @ W.T
    mag = np.abs(X64) @ (np.abs(W) + q4k_magnitudes(wb, K, N)).T
    err = np.abs(Y - T)
    assert np.all(np.isfinite(Y))
    assert np.all(err <= BOUND * mag + 1e-30), float(np.max(err / (mag + 1e-30)))
    return float(np.max(err) / np.max(np.abs(T)))


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from __graft_entry__ import build

    build()
    torch.cuda.set_device(0)
    torch.cuda.set_stream(torch.cuda.Stream())
    c = ug.Context(0, stream=torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def _gemm(ctx, wb, K, N, X, accurate=False):
    M = X.shape[0]
    w = ctx.upload(wb, ug.Q4K, K, N)
    Xd = torch.from_numpy(np.ascontiguousarray(X)).cuda()
    Y = torch.full((M, N), float("nan"), device="cuda")
    ctx.gemm(w, Xd, Y, M, accurate=accurate)
    ctx.synchronize()
    out = Y.cpu().numpy()
    w.free()
    return out


@pytest.mark.parametrize("M,N,K", [(1, 192, 256), (37, 200, 512), (300, 500, 1024), (256, 384, 4096)])
def test_gemm_small_within_bf16_bound(ctx, M, N, K):
    wb = synth.quant_weights(ug.Q4K, K, N, seed=M + N + K)
    X = synth.activations(K, seed=K + 1, rows=M)
    Y = _gemm(ctx, wb, K, N, X).astype(np.float64)
    W = oracle.dequantize(wb, K * N, ug.Q4K).reshape(N, K).astype(np.float64)
    assert _check(Y, X, W, wb, K, N) < 2e-3


def test_gemm_config2_full_size(ctx):
    """X 512 x 4096, W Q4_K 12288 x 4096."""
    M, N, K = 512, 12288, 4096
    wb = synth.quant_weights(ug.Q4K, K, N, seed=2024)
    X = synth.activations(K, seed=2025, rows=M)
    Y = _gemm(ctx, wb, K, N, X).astype(np.float64)
    W = oracle.dequantize(wb, K * N, ug.Q4K).reshape(N, K).astype(np.float64)
    normwise = _check(Y, X, W, wb, K, N)
    # the reference's own prefill is gemv_quant_q8k per token: its error on
    # the same data, for comparison (a sample of tokens)
    ref_err = 0.0
    for t in range(0, M, 64):
        yq = oracle.gemv_quant_q8k(X[t], wb, K, N, ug.Q4K, nthreads=8).astype(np.float64)
        tt = W @ X[t].astype(np.float64)
        ref_err = max(ref_err, float(np.max(np.abs(yq - tt)) / np.max(np.abs(tt))))
    print(f"config2 normwise max-rel error vs f64 truth: {normwise:.3e} (reference q8_K path: {ref_err:.3e})")
    assert normwise <= ref_err


ACC_MAXREL = 1e-4
ACC_ELEM = 2.0 ** -14


def _check_accurate(Y, X, W):
    X64 = X.astype(np.float64)
    T = X64 @ W.T
    err = np.abs(Y - T)
    assert np.all(np.isfinite(Y))
    mag = np.abs(X64) @ np.abs(W).T
    assert np.all(err <= ACC_ELEM * mag + 1e-30), float(np.max(err / (mag + 1e-30)))
    maxrel = float(np.max(err) / np.max(np.abs(T)))
    assert maxrel <= ACC_MAXREL, maxrel
    return maxrel


@pytest.mark.parametrize("M,N,K", [(1, 192, 256), (37, 200, 512), (129, 500, 1024), (256, 384, 4096)])
def test_gemm_accurate_small(ctx, M, N, K):
    wb = synth.quant_weights(ug.Q4K, K, N, seed=M + N + K)
    X = synth.activations(K, seed=K + 1, rows=M)
    X[0, :5] = [1e-3, -300.0, 0.0, 7.0, -1e-6]  # a wide dynamic range in one row
    if M > 2:
        X[2] = 0.0                               # an all-zero token row
    Y = _gemm(ctx, wb, K, N, X, accurate=True).astype(np.float64)
    W = oracle.dequantize(wb, K * N, ug.Q4K).reshape(N, K).astype(np.float64)
    _check_accurate(Y, X, W)


def test_gemm_accurate_config2_full_size(ctx):
    """BASELINE config 2 in the accurate mode: within 1e-4 max-rel of the f64 truth."""
    M, N, K = 512, 12288, 4096
    wb = synth.quant_weights(ug.Q4K, K, N, seed=2024)
    X = synth.activations(K, seed=2025, rows=M)
    Y = _gemm(ctx, wb, K, N, X, accurate=True).astype(np.float64)
    W = oracle.dequantize(wb, K * N, ug.Q4K).reshape(N, K).astype(np.float64)
    maxrel = _check_accurate(Y, X, W)
    print(f"config2 accurate mode max-rel error vs f64 truth: {maxrel:.3e}")
