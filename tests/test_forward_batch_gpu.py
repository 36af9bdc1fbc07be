"""Batch decode (unltd_qwen35_session_create_batch / unltd_qwen35_batch_decode):
n_seq sequences with their own states and positions decoded together, every
weight matrix read once per step for all of them (unltd_gemv_batch).

The reference decodes one sequence per step (qwen35_forward.rs:289), so the
bar is per sequence: its greedy tokens, logits, hidden state and session
state are bit-identical to a one-sequence session started from the same
state (itself bit-identical to the oracle), and to the oracle directly for
some sequences.
"""
import os

import numpy as np
import pytest

import oracle
import synth
import unltd_gpu as ug

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from __graft_entry__ import build

    build()
    c = ug.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def tiny(ctx):
    cfg = synth.QWEN35_TINY
    tensors = synth.qwen35_model(cfg, 11)
    m = ug.Qwen35Model(ctx, cfg)
    m.load(tensors)
    yield cfg, tensors, m
    m.close()


def _single(m, ctx_len, pos, st, token, n):
    s = m.session(ctx_len)
    if st is None:
        s.set_state(pos)
    else:
        s.set_state(pos, st["conv"], st["gdn"], st["k"], st["v"])
    toks = s.decode(token, n)
    lg, hd = s.read()
    gs = s.get_state()
    s.close()
    return toks, lg, hd, gs


@pytest.mark.parametrize("n_seq", [2, 5, 32])
def test_tiny_batch_matches_single_sequences(tiny, n_seq):
    cfg, tensors, m = tiny
    ctx_len, n = 96, 10
    rng = np.random.default_rng(n_seq)
    pos = [int(p) for p in rng.integers(0, 70, n_seq)]
    pos[0] = 40
    if n_seq > 2:
        pos[1] = 0  # an empty context
    states = [None if p == 0 else synth.qwen35_state(cfg, p, 100 + z) for z, p in enumerate(pos)]
    first = [int(t) for t in rng.integers(0, cfg["vocab"], n_seq)]
    b = m.batch_session(ctx_len, n_seq)
    for z in range(n_seq):
        st = states[z]
        if st is None:
            b.set_state(z, pos[z])
        else:
            b.set_state(z, pos[z], st["conv"], st["gdn"], st["k"], st["v"])
    toks = b.decode(first, n)
    assert b.positions() == [p + n for p in pos]
    check = range(n_seq) if n_seq <= 5 else [0, 1, 7, n_seq - 1]
    for z in check:
        stoks, slg, shd, sgs = _single(m, ctx_len, pos[z], states[z], first[z], n)
        assert toks[z].tolist() == stoks.tolist(), z
        lg, hd = b.read(z)
        assert (bits(lg) == bits(slg)).all(), z
        assert (bits(hd) == bits(shd)).all(), z
        gs = b.get_state(z)
        for key in ("conv", "gdn", "k", "v"):
            for a, c in zip(gs[key], sgs[key]):
                assert (bits(a) == bits(c)).all(), (z, key)
    # the oracle, directly, for sequence 0
    o = oracle.Qwen35Oracle(cfg, tensors, ctx_len, states[0], pos[0])
    otoks, ologits, ohidden = o.greedy(first[0], n)
    assert toks[0].tolist() == otoks
    lg, hd = b.read(0)
    assert (bits(lg) == bits(ologits)).all()
    assert (bits(hd) == bits(ohidden)).all()
    # a second call continues every sequence
    more = b.decode(toks[:, -1], 3)
    assert more.shape == (n_seq, 3)
    b.close()


def test_batch_session_errors(ctx, tiny):
    cfg, tensors, m = tiny
    for bad in (0, 33):
        with pytest.raises(ug.UnltdError):
            m.batch_session(64, bad)
    b = m.batch_session(32, 3)
    with pytest.raises(ug.UnltdError):
        b.set_state(3, 0)
    with pytest.raises(ug.UnltdError):
        b.decode([1, 2, cfg["vocab"]], 1)  # a token outside the vocab
    b.set_state(0, 30)
    with pytest.raises(ug.UnltdError):
        b.decode([1, 2, 3], 3)  # sequence 0 would pass the context
    # the one-sequence calls refuse a batch session
    with pytest.raises(ug.UnltdError):
        ug.Qwen35Session.decode(b, 1, 1)
    b.close()


def test_9b_batch32_from_2048_context(ctx):
    """BASELINE config 4, batch 32 on one GPU: 32 sequences from 2048-token
    contexts (four distinct seeded states, each sequence its own first token);
    sequences 0-3 and 31 bit-identical to one-sequence sessions, sequence 0 to
    the oracle."""
    cfg = synth.QWEN35_9B
    tensors = synth.qwen35_model(cfg, 2026)
    m = ug.Qwen35Model(ctx, cfg)
    m.load(tensors)
    n_seq, n, pos = 32, 4, 2048
    states = [synth.qwen35_state(cfg, pos, 2027 + i) for i in range(4)]
    first = [1000 + 37 * z for z in range(n_seq)]
    ctx_len = pos + n + 4
    b = m.batch_session(ctx_len, n_seq)
    for z in range(n_seq):
        st = states[z % 4]
        b.set_state(z, pos, st["conv"], st["gdn"], st["k"], st["v"])
    toks = b.decode(first, n)
    reads = {z: b.read(z) for z in (0, 1, 2, 3, 31)}
    b.close()
    for z in (0, 1, 2, 3, 31):
        stoks, slg, shd, _ = _single(m, ctx_len, pos, states[z % 4], first[z], n)
        assert toks[z].tolist() == stoks.tolist(), z
        assert (bits(reads[z][0]) == bits(slg)).all(), z
        assert (bits(reads[z][1]) == bits(shd)).all(), z
    m.close()
    o = oracle.Qwen35Oracle(cfg, tensors, ctx_len, states[0], pos)
    otoks, ologits, ohidden = o.greedy(first[0], n, nthreads=os.cpu_count() or 8)
    assert toks[0].tolist() == otoks
    assert (bits(reads[0][0]) == bits(ologits)).all()
    print("9B batch-32 streams (first 4):", toks[:4].tolist())
