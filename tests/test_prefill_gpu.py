"""Batched prefill (unltd_qwen35_prefill) against the token-by-token prompt
(unltd_qwen35_feed, itself bit-identical to the oracle) and the oracle.

The reference prefills one token per step (qwen35_forward.rs:8-12,
greedy.rs:55-65); the prefill runs a chunk's projections as batched GEMVs
with the same per-token arithmetic, so the bar is bit-identity: the next
token, the last token's logits and hidden state, and the whole session state
(conv windows, GDN matrices, K/V rows).
"""
import os
import time

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


def _same_state(a, b):
    for key in ("conv", "gdn", "k", "v"):
        assert len(a[key]) == len(b[key])
        for x, y in zip(a[key], b[key]):
            assert (bits(x) == bits(y)).all(), key


def _pair(m, ctx_len, pos, st, prompt):
    """(prefill session, feed session) after the same prompt from the same state."""
    out = []
    for how in ("prefill", "feed"):
        s = m.session(ctx_len)
        if st is None:
            s.set_state(pos)
        else:
            s.set_state(pos, st["conv"], st["gdn"], st["k"], st["v"])
        nxt = s.prefill(prompt) if how == "prefill" else s.feed(prompt)
        out.append((s, nxt))
    return out


@pytest.mark.parametrize("n", [1, 6, 32, 70])
def test_tiny_prefill_matches_feed_and_oracle(tiny, n):
    cfg, tensors, m = tiny
    prompt = [int(t) for t in np.random.default_rng(n).integers(0, cfg["vocab"], n)]
    (sp, np_), (sf, nf) = _pair(m, 96, 0, None, prompt)
    assert np_ == nf
    lp, hp = sp.read()
    lf, hf = sf.read()
    assert (bits(lp) == bits(lf)).all() and (bits(hp) == bits(hf)).all()
    assert sp.info()["position"] == n
    _same_state(sp.get_state(), sf.get_state())
    # the oracle's prompt loop
    o = oracle.Qwen35Oracle(cfg, tensors, 96)
    for t in prompt:
        ologits, ohidden = o.step(t)
    assert np_ == oracle.argmax(ologits)
    assert (bits(lp) == bits(ologits)).all() and (bits(hp) == bits(ohidden)).all()
    # decoding continues identically
    assert sp.decode(np_, 4).tolist() == sf.decode(nf, 4).tolist()
    sp.close()
    sf.close()


def test_tiny_prefill_from_a_state(tiny):
    """A prompt appended to a 40-position context (recurrent windows and K/V
    rows already there); two prefill calls in a row."""
    cfg, tensors, m = tiny
    st = synth.qwen35_state(cfg, 40, 3)
    prompt = [int(t) for t in np.random.default_rng(4).integers(0, cfg["vocab"], 45)]
    (sp, _), (sf, nf) = _pair(m, 128, 40, st, prompt[:20])
    np2 = sp.prefill(prompt[20:])
    nf2 = sf.feed(prompt[20:])
    assert np2 == nf2
    assert (bits(sp.read()[0]) == bits(sf.read()[0])).all()
    _same_state(sp.get_state(), sf.get_state())
    sp.close()
    sf.close()


def test_prefill_errors(tiny):
    cfg, tensors, m = tiny
    s = m.session(16)
    with pytest.raises(ug.UnltdError):
        s.prefill([cfg["vocab"]])
    with pytest.raises(ug.UnltdError):
        s.prefill(list(range(17)))
    assert s.prefill([]) == 0
    s.close()
    b = m.batch_session(16, 2)
    with pytest.raises(ug.UnltdError):
        ug.Qwen35Session.prefill(b, [1, 2])
    b.close()


def test_9b_prefill_matches_feed(ctx):
    """The synthetic 9B model: a 96-token prompt after a 2048-position
    context, prefill against feed, bit for bit, with both timed."""
    cfg = synth.QWEN35_9B
    tensors = synth.qwen35_model(cfg, 2026)
    st = synth.qwen35_state(cfg, 2048, 2027)
    m = ug.Qwen35Model(ctx, cfg)
    m.load(tensors)
    prompt = [int(t) for t in np.random.default_rng(9).integers(0, cfg["vocab"], 96)]
    res = {}
    for how in ("prefill", "feed"):
        s = m.session(2048 + 96 + 8)
        s.set_state(2048, st["conv"], st["gdn"], st["k"], st["v"])
        fn = s.prefill if how == "prefill" else s.feed
        fn(prompt[:8])  # warm-up (workspace, graph)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        nxt = fn(prompt[8:])
        dt = time.perf_counter() - t0
        res[how] = (nxt, s.read(), s.get_state(), dt)
        s.close()
    m.close()
    print(f"9B prompt of 88 tokens: prefill {88 / res['prefill'][3]:.0f} tok/s, feed {88 / res['feed'][3]:.0f} tok/s")
    assert res["prefill"][0] == res["feed"][0]
    assert (bits(res["prefill"][1][0]) == bits(res["feed"][1][0])).all()
    assert (bits(res["prefill"][1][1]) == bits(res["feed"][1][1])).all()
    _same_state(res["prefill"][2], res["feed"][2])
