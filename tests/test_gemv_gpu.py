"""GPU parity of the decode GEMV path against the CPU oracle, through the C ABI.

Bars (tolerances written here):
* dequantization: bit-exact (NaN compares equal to NaN);
* MODE_Q8K_EXACT: bit-identical to gemv_quant_q8k (quants.rs:474-515);
* MODE_F32X: max_j |y_j - t_j| / max_j |t_j| <= 1e-4 against the
  f64-accumulated gemv_quant (quants.rs:422-466), and per element
  |y_j - t_j| <= 1e-5 * sum_i |w_ji x_i|;
* fused argmax: the same index as greedy.rs:18-27 on the oracle's logits.
"""
import numpy as np
import pytest

import oracle
import synth
import unltd_gpu as ug

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

F32X_NORMWISE = 1e-4
F32X_ELEMWISE = 1e-5


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


def _same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return np.array_equal(a.view(np.uint32)[~nan], b.view(np.uint32)[~nan]) and np.array_equal(np.isnan(a), np.isnan(b))


def _run(ctx, wb, dtype, dim_in, dim_out, x, mode):
    w = ctx.upload(wb, dtype, dim_in, dim_out)
    xd = _dev(x)
    y = torch.full((dim_out,), float("nan"), device="cuda")
    ctx.gemv(w, xd, y, mode)
    ctx.synchronize()
    out = y.cpu().numpy()
    w.free()
    return out


def _abs_mag(wb, dtype, dim_in, dim_out, x):
    deq = oracle.dequantize(wb, dim_in * dim_out, dtype).reshape(dim_out, dim_in).astype(np.float64)
    return np.abs(deq) @ np.abs(x.astype(np.float64))


# (6144, 77): K-chunks of 8 blocks; (8192, 300) and (12288, 64): chunks of 16
SHAPES_K = [(256, 1), (512, 3), (1024, 37), (4096, 256), (4096, 4096), (6144, 77), (8192, 300), (12288, 64),
            (768, 9000)]


@pytest.mark.parametrize("dtype", [ug.Q4K, ug.Q6K])
@pytest.mark.parametrize("dim_in,dim_out", SHAPES_K)
def test_q8k_exact_bit_identical(ctx, dtype, dim_in, dim_out):
    wb = synth.quant_weights(dtype, dim_in, dim_out, seed=dim_in + dim_out)
    x = synth.activations(dim_in, seed=7 + dim_out)
    got = _run(ctx, wb, dtype, dim_in, dim_out, x, ug.MODE_Q8K)
    ref = oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, dtype, nthreads=8)
    assert _same_bits(got, ref), np.flatnonzero(got.view(np.uint32) != ref.view(np.uint32))[:10]


@pytest.mark.parametrize("dtype", [ug.Q4K, ug.Q6K, ug.Q8_0])
@pytest.mark.parametrize("dim_in,dim_out", SHAPES_K + [(96, 5), (4096 + 32, 17)])
def test_f32x_within_tolerance(ctx, dtype, dim_in, dim_out):
    if dtype != ug.Q8_0 and dim_in % 256:
        pytest.skip("K-quants need dim_in % 256 == 0")
    wb = synth.quant_weights(dtype, dim_in, dim_out, seed=3 * dim_in + dim_out)
    x = synth.activations(dim_in, seed=11 + dim_out)
    got = _run(ctx, wb, dtype, dim_in, dim_out, x, ug.MODE_F32X).astype(np.float64)
    truth = oracle.gemv_quant_f64(x, wb, dim_in, dim_out, dtype, nthreads=8)
    assert np.max(np.abs(got - truth)) <= F32X_NORMWISE * np.max(np.abs(truth))
    mag = _abs_mag(wb, dtype, dim_in, dim_out, x)
    assert np.all(np.abs(got - truth) <= F32X_ELEMWISE * mag + 1e-30)


@pytest.mark.parametrize("dtype", [ug.Q4K, ug.Q6K, ug.Q8_0])
@pytest.mark.parametrize("dim_in,dim_out", [(256, 1), (512, 7), (4096, 33)])
def test_dequant_bit_exact(ctx, dtype, dim_in, dim_out):
    rng = np.random.default_rng(dim_in * 7 + dim_out)
    wb = rng.integers(0, 256, size=dim_out * synth.row_bytes(dtype, dim_in), dtype=np.uint8)
    # keep most scales finite but include subnormal, zero and negative f16 scales
    nb = wb.size // synth.BLOCK_BYTES[dtype]
    blocks = wb.reshape(nb, synth.BLOCK_BYTES[dtype])
    off = 208 if dtype == ug.Q6K else 0
    vals = np.array([0.003, -0.007, 6.0e-8, 0.0, 1.5e-5, 2.0], np.float16)
    blocks[:, off:off + 2] = vals[rng.integers(0, len(vals), nb)].view(np.uint8).reshape(nb, 2)
    w = ctx.upload(wb, dtype, dim_in, dim_out)
    out = torch.empty(dim_out * dim_in, device="cuda")
    ctx.dequant(w, out)
    ctx.synchronize()
    ref = oracle.dequantize(wb, dim_in * dim_out, dtype)
    assert _same_bits(out.cpu().numpy(), ref)
    w.free()


def test_q8k_edge_inputs(ctx):
    """Zero spans (amax = 0), ties in |x| (first index wins), a negative max."""
    dim_in, dim_out = 1024, 40
    for dtype in (ug.Q4K, ug.Q6K):
        wb = synth.quant_weights(dtype, dim_in, dim_out, seed=5)
        x = synth.activations(dim_in, seed=6)
        x[0:256] = 0.0
        x[256:512] = np.where(np.arange(256) % 2 == 0, 3.0, -3.0).astype(np.float32)
        x[600] = -50.0
        x[800] = 7.5
        x[801] = -7.5
        got = _run(ctx, wb, dtype, dim_in, dim_out, x, ug.MODE_Q8K)
        ref = oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, dtype)
        assert _same_bits(got, ref)


def test_reference_hand_blocks_through_gpu(ctx):
    """quants.rs:1003-1057 hand values, run through the GPU Q8_K path."""
    scales = [1, 0, 0, 0, 3, 0, 0, 0, 0, 0, 0, 0]
    qs = [1] + [0] * 127
    blk = np.frombuffer(np.array([0x3C00, 0x4000], np.uint16).tobytes() + bytes(scales) + bytes(qs), np.uint8)
    x = np.zeros(256, np.float32)
    x[0] = 127
    assert _run(ctx, blk, ug.Q4K, 256, 1, x, ug.MODE_Q8K)[0] == -635.0
    ql = [1] + [0] * 127
    sc = [1] + [0] * 15
    blk6 = np.frombuffer(bytes(ql) + bytes(64) + bytes(s & 0xFF for s in sc) + np.uint16(0x3C00).tobytes(), np.uint8)
    assert _run(ctx, blk6, ug.Q6K, 256, 1, x, ug.MODE_Q8K)[0] == -3937.0
    ql = [0] * 128
    ql[32] = 1
    sc = [0] * 16
    sc[2] = -1
    blk6 = np.frombuffer(bytes(ql) + bytes(64) + bytes(s & 0xFF for s in sc) + np.uint16(0x3C00).tobytes(), np.uint8)
    x = np.zeros(256, np.float32)
    x[32] = 127
    assert _run(ctx, blk6, ug.Q6K, 256, 1, x, ug.MODE_Q8K)[0] == 3937.0


def test_reference_golden_blocks_through_gpu(ctx):
    """The reference's real-model blocks (two Q6_K, two Q4_K of a Q4_K_M GGUF,
    quants.rs:1094-1152, fixture tests/golden/ornith_pins.json) through the
    GPU: the dequantized weights bit-exact with the oracle and equal to the
    gguf-py single weights w[7], w[200] the reference pins (quants.rs:1169-1198);
    F32X dots within the reference's 1e-4 of the gguf-py values for both
    deterministic x (quants.rs:1157-1166); Q8K_EXACT dots bit-identical to the
    oracle's gemv_quant_q8k."""
    import json
    import os

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ornith_pins.json")) as f:
        pins = json.load(f)
    i = np.arange(256)
    xp = (((i * 7919) % 1009).astype(np.float32) / np.float32(1009.0) - np.float32(0.5)).astype(np.float32)
    xa = (((i * 31 + 17) % 257).astype(np.float32) / np.float32(257.0) - np.float32(0.5)).astype(np.float32)
    tol = pins["tolerance"]
    for case in pins["cases"]:
        raw = np.frombuffer(bytes.fromhex(pins["blocks_hex"][case["block"]]), np.uint8)
        dtype = ug.Q4K if case["block"].startswith("Q4K") else ug.Q6K
        w = ctx.upload(raw, dtype, 256, 1)
        deq = torch.empty(256, device="cuda")
        ctx.dequant(w, deq)
        ctx.synchronize()
        got = deq.cpu().numpy()
        assert _same_bits(got, oracle.dequantize(raw, 256, dtype)), case["block"]
        assert abs(float(got[7]) - case["w7"]) <= tol and abs(float(got[200]) - case["w200"]) <= tol, case
        for x, want in ((xp, case["dot_x_pattern"]), (xa, case["dot_x_alt"])):
            y = torch.full((1,), float("nan"), device="cuda")
            ctx.gemv(w, _dev(x), y, ug.MODE_F32X)
            ctx.synchronize()
            assert abs(float(y.item()) - want) <= tol, (case["block"], float(y.item()), want)
            ctx.gemv(w, _dev(x), y, ug.MODE_Q8K)
            ctx.synchronize()
            ref = oracle.gemv_quant_q8k(x, raw, 256, 1, dtype)
            assert _same_bits(y.cpu().numpy(), ref), case["block"]
        w.free()


@pytest.mark.parametrize("mode", [ug.MODE_Q8K, ug.MODE_F32X])
def test_fused_argmax_matches_greedy(ctx, mode):
    dim_in, dim_out = 4096, 20000
    wb = synth.quant_weights(ug.Q6K, dim_in, dim_out, seed=21)
    rb = synth.row_bytes(ug.Q6K, dim_in)
    # duplicate the future maximum row later in the tensor: ties keep the first index
    x = synth.activations(dim_in, seed=22)
    ref_logits = oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, ug.Q6K, nthreads=8)
    top = int(np.argmax(ref_logits))
    wb = wb.copy()
    wb[(dim_out - 3) * rb:(dim_out - 2) * rb] = wb[top * rb:(top + 1) * rb]
    w = ctx.upload(wb, ug.Q6K, dim_in, dim_out)
    xd = _dev(x)
    tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    logits = torch.empty(dim_out, device="cuda")
    for _ in range(3):  # the reduction state must reset between calls
        ctx.gemv_argmax(w, xd, tok, logits=logits, mode=mode)
        ctx.synchronize()
        lg = logits.cpu().numpy()
        assert int(tok.item()) == oracle.argmax(lg)
    if mode == ug.MODE_Q8K:
        assert int(tok.item()) == top
    w.free()


def test_argmax_shard_key(ctx):
    """unltd_gemv_argmax_shard on one GPU: the key of rows [row0, row0 + n)
    of a head is orderable(max logit) << 32 | 0xFFFFFFFF - (row0 + first
    local argmax), over three calls in a row."""
    dim_in, vocab, row0, n = 4096, 9000, 3000, 4000
    wb = synth.quant_weights(ug.Q6K, dim_in, vocab, seed=81)
    x = synth.activations(dim_in, seed=82)
    ref = oracle.gemv_quant_q8k(x, wb, dim_in, vocab, ug.Q6K, nthreads=8)[row0:row0 + n]
    w = ctx.upload(wb, ug.Q6K, dim_in, vocab, row0=row0, rows=n)
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    lg = torch.empty(n, device="cuda")
    i = oracle.argmax(ref)
    b = int(ref[i:i + 1].view(np.uint32)[0])
    ordv = (~b & 0xFFFFFFFF) if b >= 0x80000000 else (b | 0x80000000)
    want = (ordv << 32) | (0xFFFFFFFF - (row0 + i))
    for _ in range(3):
        ctx.gemv_argmax_shard(w, _dev(x), key, row0, logits=lg, mode=ug.MODE_Q8K)
        ctx.synchronize()
        assert _same_bits(lg.cpu().numpy(), ref)
        assert int(key.item()) & 0xFFFFFFFFFFFFFFFF == want
    w.free()


def test_argmax_nan_rules(ctx):
    """A NaN logit never wins, except at index 0 (greedy.rs strict '>')."""
    dim_in, dim_out = 256, 50
    wb = synth.quant_weights(ug.Q6K, dim_in, dim_out, seed=31).copy()
    rb = synth.row_bytes(ug.Q6K, dim_in)
    x = synth.activations(dim_in, seed=32)
    nan16 = np.array([0x7E00], np.uint16).view(np.uint8)
    w2 = wb.copy()
    w2[7 * rb + 208: 7 * rb + 210] = nan16  # row 7 -> NaN
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    w = ctx.upload(w2, ug.Q6K, dim_in, dim_out)
    logits = torch.empty(dim_out, device="cuda")
    ctx.gemv_argmax(w, _dev(x), tok, logits=logits, mode=ug.MODE_Q8K)
    ctx.synchronize()
    assert int(tok.item()) == oracle.argmax(logits.cpu().numpy())
    w.free()
    w3 = wb.copy()
    w3[208:210] = nan16  # row 0 -> NaN: the scan never moves off index 0
    w = ctx.upload(w3, ug.Q6K, dim_in, dim_out)
    ctx.gemv_argmax(w, _dev(x), tok, logits=logits, mode=ug.MODE_Q8K)
    ctx.synchronize()
    assert int(tok.item()) == 0 == oracle.argmax(logits.cpu().numpy())
    w.free()


def test_reference_signature_host_api(ctx):
    dim_in, dim_out = 4096, 300
    for dtype in (ug.Q4K, ug.Q6K):
        wb = synth.quant_weights(dtype, dim_in, dim_out, seed=41)
        x = synth.activations(dim_in, seed=42)
        out = np.zeros(dim_out, np.float32)
        ug.gemv_quant_q8k(out, x, wb, dim_in, dim_out, dtype)
        assert _same_bits(out, oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, dtype))
        ug.gemv_quant(out, x, wb, dim_in, dim_out, dtype)
        truth = oracle.gemv_quant_f64(x, wb, dim_in, dim_out, dtype)
        assert np.max(np.abs(out - truth)) <= F32X_NORMWISE * np.max(np.abs(truth))
    # out in pinned (device-mapped) host memory: the GEMV writes it directly
    pinned = torch.full((dim_out,), float("nan")).pin_memory().numpy()
    for dtype in (ug.Q4K, ug.Q6K):
        wb = synth.quant_weights(dtype, dim_in, dim_out, seed=44)
        x = synth.activations(dim_in, seed=45)
        ug.gemv_quant_q8k(pinned, x, wb, dim_in, dim_out, dtype)
        assert _same_bits(pinned, oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, dtype))
    # one buffer rewritten in place with other weights: the cache, keyed by
    # the pointer, notices (sampled fingerprint) and uploads again
    buf = synth.quant_weights(ug.Q4K, dim_in, dim_out, seed=47).copy()
    for seed in (47, 48):
        buf[:] = synth.quant_weights(ug.Q4K, dim_in, dim_out, seed=seed)
        ug.gemv_quant_q8k(pinned, x, buf, dim_in, dim_out, ug.Q4K)
        assert _same_bits(pinned, oracle.gemv_quant_q8k(x, buf, dim_in, dim_out, ug.Q4K))
    wq = synth.quant_weights(ug.Q8_0, dim_in, dim_out, seed=46)
    ug.gemv_quant(pinned, x, wq, dim_in, dim_out, ug.Q8_0)
    truth = oracle.gemv_quant_f64(x, wq, dim_in, dim_out, ug.Q8_0)
    assert np.max(np.abs(pinned - truth)) <= F32X_NORMWISE * np.max(np.abs(truth))
    wb = synth.quant_weights(ug.Q4K, 4096, 1, seed=43)
    out = np.zeros(4096, np.float32)
    ug.dequantize_q4_k(out, wb)
    assert _same_bits(out, oracle.dequantize_q4_k(wb, 4096))
    ug.forget_host_weights()


def test_row_range_upload_equals_slice(ctx):
    dim_in, dim_out = 4096, 100
    wb = synth.quant_weights(ug.Q4K, dim_in, dim_out, seed=51)
    x = synth.activations(dim_in, seed=52)
    full = _run(ctx, wb, ug.Q4K, dim_in, dim_out, x, ug.MODE_Q8K)
    w = ctx.upload(wb, ug.Q4K, dim_in, dim_out, row0=30, rows=40)
    y = torch.empty(40, device="cuda")
    ctx.gemv(w, _dev(x), y, ug.MODE_Q8K)
    ctx.synchronize()
    assert _same_bits(y.cpu().numpy(), full[30:70])
    w.free()


def test_full_size_lm_head_q8k_and_argmax(ctx):
    """Config 1d at full size: Q6_K 4096 -> 151936, bit-exact logits and token."""
    dim_in, dim_out = 4096, 151936
    wb = synth.quant_weights(ug.Q6K, dim_in, dim_out, seed=61)
    x = synth.activations(dim_in, seed=62)
    w = ctx.upload(wb, ug.Q6K, dim_in, dim_out)
    logits = torch.empty(dim_out, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.gemv_argmax(w, _dev(x), tok, logits=logits, mode=ug.MODE_Q8K)
    ctx.synchronize()
    ref = oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, ug.Q6K, nthreads=8)
    assert _same_bits(logits.cpu().numpy(), ref)
    assert int(tok.item()) == oracle.argmax(ref)
    w.free()


# BASELINE configs 1a-1c at full size, on the benchmark's own seeded inputs
# (bench.py SEEDS: weights 1000 + i, x 1001 + i)
FULL_CONFIG1 = [("1a_q4k_gate_up", ug.Q4K, 4096, 12288, 1000), ("1b_q6k_down", ug.Q6K, 12288, 4096, 1001),
                ("1c_q8_0", ug.Q8_0, 4096, 4096, 1002)]


@pytest.mark.parametrize("name,dtype,dim_in,dim_out,seed", FULL_CONFIG1, ids=[c[0] for c in FULL_CONFIG1])
def test_full_size_config1_gemvs(ctx, name, dtype, dim_in, dim_out, seed):
    """Q8K_EXACT bit-identical to gemv_quant_q8k (the K-quants; the reference
    has no Q8_0 dot), F32X within the stated bounds of the f64 truth."""
    wb = synth.quant_weights(dtype, dim_in, dim_out, seed)
    x = synth.activations(dim_in, seed + 1)
    if dtype != ug.Q8_0:
        got = _run(ctx, wb, dtype, dim_in, dim_out, x, ug.MODE_Q8K)
        assert _same_bits(got, oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, dtype, nthreads=8))
    got = _run(ctx, wb, dtype, dim_in, dim_out, x, ug.MODE_F32X).astype(np.float64)
    truth = oracle.gemv_quant_f64(x, wb, dim_in, dim_out, dtype, nthreads=8)
    assert np.max(np.abs(got - truth)) <= F32X_NORMWISE * np.max(np.abs(truth))
    assert np.all(np.abs(got - truth) <= F32X_ELEMWISE * _abs_mag(wb, dtype, dim_in, dim_out, x) + 1e-30)


def test_launches_are_counted(ctx):
    n0 = ctx.launch_count()
    _run(ctx, synth.quant_weights(ug.Q4K, 256, 4, seed=1), ug.Q4K, 256, 4, synth.activations(256, seed=2), ug.MODE_F32X)
    assert ctx.launch_count() >= n0 + 2  # repack + gemv (x quantized in the GEMV's prologue)


def _misaligned(x):
    """x on the device at an address 4 bytes past a 16-byte boundary: the
    GEMV cannot load it as float4 and falls back to the prep kernel."""
    buf = torch.zeros(x.size + 4, device="cuda")
    v = buf[1:1 + x.size]
    v.copy_(torch.from_numpy(x))
    assert v.data_ptr() % 16 == 4
    return v


@pytest.mark.parametrize("dtype,mode", [(ug.Q4K, ug.MODE_F32X), (ug.Q6K, ug.MODE_F32X), (ug.Q8_0, ug.MODE_F32X),
                                        (ug.Q4K, ug.MODE_Q8K), (ug.Q6K, ug.MODE_Q8K)])
@pytest.mark.parametrize("dim_in,dim_out", [(256, 3), (4096, 300), (12288, 40), (4096 + 96, 33)])
def test_prologue_quantization_equals_prep(ctx, dtype, mode, dim_in, dim_out):
    """x quantized in the GEMV's own prologue (aligned x) gives the same bits
    as the image of the separate prep kernel (misaligned x), with and without
    the fused argmax, zero spans and outliers included."""
    if dtype != ug.Q8_0 and dim_in % 256:
        pytest.skip("K-quants need dim_in % 256 == 0")
    wb = synth.quant_weights(dtype, dim_in, dim_out, seed=dim_in + 5 * dim_out)
    w = ctx.upload(wb, dtype, dim_in, dim_out)
    xs = [synth.activations(dim_in, seed=dim_out + 9)]
    x2 = xs[0].copy()
    x2[:256] = 0.0           # a zero span
    # F32X: a non-finite last span (NaN outputs either way); Q8K: a large outlier
    x2[-1] = np.float32(np.inf) if mode == ug.MODE_F32X else np.float32(-1e30)
    xs.append(x2)
    for x in xs:
        outs = []
        for xd in (_dev(x), _misaligned(x)):
            y = torch.full((dim_out,), 1.0, device="cuda")
            ctx.gemv(w, xd, y, mode)
            tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
            lg = torch.full((dim_out,), 2.0, device="cuda")
            ctx.gemv_argmax(w, xd, tok, logits=lg, mode=mode)
            ctx.synchronize()
            outs.append((y.cpu().numpy(), lg.cpu().numpy(), int(tok.item())))
        assert _same_bits(outs[0][0], outs[1][0])
        assert _same_bits(outs[0][1], outs[1][1]) and _same_bits(outs[0][0], outs[0][1])
        assert outs[0][2] == outs[1][2] == oracle.argmax(outs[0][1])
    w.free()
