"""GPU parity of the tensor-core prefill GEMM (unltd_gemm) against the oracle.

Ground truth: f64 products of X and the oracle's exact dequantized weights
(every Q4_K weight is exact in f32), i.e. gemv_quant (quants.rs:422) per
token before its final rounding. The kernel rounds X and W once to bf16
(unit roundoff 2^-8) and accumulates in f32, so per element
|Y - T| <= 2^-7 * sum_k |X_k W_k| (+ f32 accumulation, far below); the test
asserts that bound and reports the normwise error.
"""
import numpy as np
import pytest

import oracle
import synth
import unltd_gpu as ug

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
BOUND = 2.0 ** -7


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


def _gemm(ctx, wb, K, N, X):
    M = X.shape[0]
    w = ctx.upload(wb, ug.Q4K, K, N)
    Xd = torch.from_numpy(np.ascontiguousarray(X)).cuda()
    Y = torch.full((M, N), float("nan"), device="cuda")
    ctx.gemm(w, Xd, Y, M)
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
    T = X.astype(np.float64) @ W.T
    mag = np.abs(X.astype(np.float64)) @ np.abs(W).T
    err = np.abs(Y - T)
    assert np.all(np.isfinite(Y))
    assert np.all(err <= BOUND * mag + 1e-30), float(np.max(err / (mag + 1e-30)))
    # rows are tokens: each row equals the GEMV of that token within the same bound
    assert np.max(err) / np.max(np.abs(T)) < 1e-2


def test_gemm_config2_full_size(ctx):
    """X 512 x 4096, W Q4_K 12288 x 4096."""
    M, N, K = 512, 12288, 4096
    wb = synth.quant_weights(ug.Q4K, K, N, seed=2024)
    X = synth.activations(K, seed=2025, rows=M)
    Y = _gemm(ctx, wb, K, N, X).astype(np.float64)
    W = oracle.dequantize(wb, K * N, ug.Q4K).reshape(N, K).astype(np.float64)
    X64 = X.astype(np.float64)
    T = X64 @ W.T
    mag = np.abs(X64) @ np.abs(W).T
    err = np.abs(Y - T)
    assert np.all(err <= BOUND * mag + 1e-30), float(np.max(err / (mag + 1e-30)))
    normwise = float(np.max(err) / np.max(np.abs(T)))
    print(f"config2 normwise max-rel error vs f64 truth: {normwise:.3e}")
    assert normwise < 1e-2
