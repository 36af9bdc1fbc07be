"""GPU parity of the batched decode GEMV (unltd_gemv_batch, unltd_gemv_argmax_batch).

Bar: for every sequence s of the batch, y_s is bit-identical to
gemv_quant_q8k (quants.rs:474-515) of x_s alone (the oracle), and to the
single-sequence unltd_gemv in Q8K_EXACT mode; the batched argmax gives each
sequence the first index of its maximum (greedy.rs:18-27).
"""
import numpy as np
import pytest

import oracle
import synth
import unltd_gpu as ug

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


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


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _xs(dim_in, n, seed):
    X = np.stack([synth.activations(dim_in, seed=seed + s) for s in range(n)]).astype(np.float32)
    if n > 2:
        X[1] *= 1e-3          # a small-magnitude sequence
        X[2, : dim_in // 2] = 0.0  # zero spans
    return X


# Q4_K rows of 512 and 4096 inputs; Q6_K rows of 512 (padded 432-byte
# stride), 4096 and 12288 (16-block chunks); row counts that leave partial
# tiles and CTAs with different row counts
SHAPES = [(ug.Q4K, 512, 300), (ug.Q4K, 4096, 1000), (ug.Q4K, 4096, 4096), (ug.Q6K, 512, 77),
          (ug.Q6K, 4096, 1000), (ug.Q6K, 12288, 700), (ug.Q6K, 8192, 129)]


@pytest.mark.parametrize("n_seq", [1, 3, 8, 13, 32])
@pytest.mark.parametrize("dtype,dim_in,dim_out", SHAPES)
def test_batch_bit_identical(ctx, dtype, dim_in, dim_out, n_seq):
    wb = synth.quant_weights(dtype, dim_in, dim_out, seed=dim_in + 3 * dim_out + dtype)
    X = _xs(dim_in, n_seq, seed=100 + dim_out)
    w = ctx.upload(wb, dtype, dim_in, dim_out)
    Y = torch.full((n_seq, dim_out), float("nan"), device="cuda")
    ctx.gemv_batch(w, _dev(X), Y, n_seq)
    # the single-sequence path on the same device, one sequence at a time
    y1 = torch.full((dim_out,), float("nan"), device="cuda")
    got = None
    singles = []
    for s in range(n_seq):
        ctx.gemv(w, _dev(X[s]), y1, ug.MODE_Q8K)
        ctx.synchronize()
        singles.append(y1.cpu().numpy().copy())
    got = Y.cpu().numpy()
    w.free()
    for s in range(n_seq):
        assert np.array_equal(_bits(got[s]), _bits(singles[s])), (s, np.flatnonzero(_bits(got[s]) != _bits(singles[s]))[:8])
    # the oracle, for the first and the last sequence
    for s in {0, n_seq - 1}:
        ref = oracle.gemv_quant_q8k(X[s], wb, dim_in, dim_out, dtype, nthreads=8)
        assert np.array_equal(_bits(got[s]), _bits(ref)), (s, np.flatnonzero(_bits(got[s]) != _bits(ref))[:8])


@pytest.mark.parametrize("dtype,dim_in,dim_out", [(ug.Q6K, 4096, 151936), (ug.Q4K, 512, 1000), (ug.Q6K, 512, 1000)])
def test_batch_argmax(ctx, dtype, dim_in, dim_out):
    n_seq = 32 if dim_out > 100000 else 7
    wb = synth.quant_weights(dtype, dim_in, dim_out, seed=dim_out + dtype)
    X = _xs(dim_in, n_seq, seed=5)
    w = ctx.upload(wb, dtype, dim_in, dim_out)
    L = torch.full((n_seq, dim_out), float("nan"), device="cuda")
    tok = torch.zeros(n_seq, dtype=torch.int32, device="cuda")
    for rep in range(2):  # the argmax state is reset by each call
        ctx.gemv_argmax_batch(w, _dev(X), tok, n_seq, logits=L)
        ctx.synchronize()
        toks = tok.cpu().numpy().view(np.uint32)
        logits = L.cpu().numpy()
        for s in range(n_seq):
            assert int(toks[s]) == int(np.argmax(logits[s])), (rep, s)
    # without logits, the same tokens
    tok2 = torch.zeros(n_seq, dtype=torch.int32, device="cuda")
    ctx.gemv_argmax_batch(w, _dev(X), tok2, n_seq)
    ctx.synchronize()
    assert np.array_equal(tok2.cpu().numpy(), tok.cpu().numpy())
    for s in (0, n_seq - 1):
        ref = oracle.gemv_quant_q8k(X[s], wb, dim_in, dim_out, dtype, nthreads=8)
        assert np.array_equal(_bits(logits[s]), _bits(ref))
        assert int(toks[s]) == oracle.argmax(ref)
    w.free()


def test_batch_rejects(ctx):
    wb = synth.quant_weights(ug.Q4K, 512, 64, seed=1)
    w = ctx.upload(wb, ug.Q4K, 512, 64)
    X = _dev(np.zeros((33, 512), np.float32))
    Y = torch.zeros((33, 64), device="cuda")
    for n in (0, 33):
        with pytest.raises(ug.UnltdError):
            ctx.gemv_batch(w, X, Y, n)
    with pytest.raises(ug.UnltdError):
        ctx.gemv_batch(w, X, Y, 4, mode=ug.MODE_F32X)
    w.free()
