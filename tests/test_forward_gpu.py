"""GPU decode step of the Qwen3.5-style hybrid model (unltd_qwen35_*) against
the CPU oracle (oracle/forward_ref.c, a restatement of qwen35_forward.rs).

Both sides run every projection as gemv_quant_q8k and keep the reference's
f32/f64 operation order, so the greedy token streams must be identical and
the logits and hidden states equal bit for bit.
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


def test_tiny_greedy_stream_bit_exact(tiny):
    cfg, tensors, m = tiny
    st = synth.qwen35_state(cfg, 40, 12)
    s = m.session(64)
    s.set_state(40, st["conv"], st["gdn"], st["k"], st["v"])
    toks = s.decode(5, 12)
    o = oracle.Qwen35Oracle(cfg, tensors, 64, st, 40)
    otoks, ologits, ohidden = o.greedy(5, 12)
    assert toks.tolist() == otoks
    lg, hd = s.read()
    assert (bits(hd) == bits(ohidden)).all()
    assert (bits(lg) == bits(ologits)).all()
    assert s.info()["position"] == 52
    # the session state (conv windows, GDN matrices, K/V rows) equals the oracle's
    gs = s.get_state()
    for i in range(len(o.conv)):
        assert (bits(gs["conv"][i]) == bits(o.conv[i])).all()
        assert (bits(gs["gdn"][i]) == bits(o.gdn[i])).all()
    for i in range(len(o.k)):
        assert (bits(gs["k"][i]) == bits(o.k[i][:52])).all()
        assert (bits(gs["v"][i]) == bits(o.v[i][:52])).all()
    s.close()


def test_tiny_loaded_from_gguf_matches_oracle(ctx, tiny, tmp_path):
    """The model written as a GGUF file and loaded from its mapping
    (unltd_qwen35_config_from_gguf + unltd_qwen35_load_gguf) decodes the same
    greedy stream and logits as the oracle."""
    cfg, tensors, _ = tiny
    path = str(tmp_path / "tiny.gguf")
    synth.write_qwen35_gguf(path, cfg, tensors)
    with ug.Gguf(path) as g:
        gcfg = g.qwen35_config()
        m = ug.Qwen35Model(ctx, gcfg)
        m.load_gguf(g)
    st = synth.qwen35_state(cfg, 40, 12)
    s = m.session(64)
    s.set_state(40, st["conv"], st["gdn"], st["k"], st["v"])
    toks = s.decode(5, 12)
    o = oracle.Qwen35Oracle(cfg, tensors, 64, st, 40)
    otoks, ologits, _ = o.greedy(5, 12)
    assert toks.tolist() == otoks
    lg, _ = s.read()
    assert (bits(lg) == bits(ologits)).all()
    s.close()
    m.close()


def test_tiny_prompt_from_position_zero(tiny):
    """feed() teacher-forces a prompt from an empty state (n_ctx = 1 at the
    first step), then decode() continues greedily."""
    cfg, tensors, m = tiny
    prompt = [3, 141, 59, 265, 358, 979]
    s = m.session(32)
    nxt = s.feed(prompt)
    o = oracle.Qwen35Oracle(cfg, tensors, 32)
    for t in prompt:
        ologits, ohidden = o.step(t)
    assert nxt == oracle.argmax(ologits)
    lg, hd = s.read()
    assert (bits(lg) == bits(ologits)).all() and (bits(hd) == bits(ohidden)).all()
    toks = s.decode(nxt, 5)
    otoks, _, _ = o.greedy(nxt, 5)
    assert toks.tolist() == otoks
    s.close()


def test_tiny_state_round_trip(tiny):
    """get_state returns what set_state loaded (the checkpoint/resume pair)."""
    cfg, tensors, m = tiny
    st = synth.qwen35_state(cfg, 17, 9)
    s = m.session(24)
    s.set_state(17, st["conv"], st["gdn"], st["k"], st["v"])
    gs = s.get_state()
    for key in ("conv", "gdn", "k", "v"):
        for a, b in zip(gs[key], st[key]):
            assert (bits(a) == bits(b)).all(), key
    # resuming a copy of a state continues exactly like the original session
    a = s.decode(11, 3)
    s2 = m.session(24)
    s2.set_state(17, st["conv"], st["gdn"], st["k"], st["v"])
    b = s2.decode(11, 3)
    assert a.tolist() == b.tolist()
    assert (bits(s.read()[0]) == bits(s2.read()[0])).all()
    s.close()
    s2.close()


def test_tiny_graph_matches_uncaptured(tiny):
    cfg, tensors, m = tiny
    st = synth.qwen35_state(cfg, 20, 5)
    out = []
    for no_graph in ("0", "1"):
        os.environ["UNLTD_NO_GRAPH"] = no_graph
        try:
            s = m.session(40)
            s.set_state(20, st["conv"], st["gdn"], st["k"], st["v"])
            out.append((s.decode(9, 6).tolist(), s.read()))
            s.close()
        finally:
            os.environ.pop("UNLTD_NO_GRAPH", None)
    assert out[0][0] == out[1][0]
    assert (bits(out[0][1][0]) == bits(out[1][1][0])).all()


def test_model_and_session_errors(ctx, tiny):
    cfg, tensors, m = tiny
    bad = dict(cfg, n_head=3)
    with pytest.raises(ug.UnltdError) as e:
        ug.Qwen35Model(ctx, bad)
    assert e.value.status == 1
    m2 = ug.Qwen35Model(ctx, cfg)
    with pytest.raises(ug.UnltdError) as e:
        m2.set_tensor("blk.0.ffn_gate.weight", tensors["blk.0.ffn_gate.weight"][1], ug.Q6K)
    assert e.value.status == 4
    with pytest.raises(ug.UnltdError) as e:
        m2.set_tensor("blk.0.ffn_gate.weight", tensors["blk.0.ffn_gate.weight"][1][:-1], ug.Q4K)
    assert e.value.status == 2
    with pytest.raises(ug.UnltdError) as e:
        m2.set_tensor("blk.9.ffn_gate.weight", tensors["blk.0.ffn_gate.weight"][1], ug.Q4K)
    assert e.value.status == 1
    with pytest.raises(ug.UnltdError) as e:
        m2.load({})
    assert "missing tensor" in str(e.value)
    m2.close()
    s = m.session(8)
    with pytest.raises(ug.UnltdError) as e:
        s.decode(cfg["vocab"], 1)
    assert e.value.status == 1
    s.decode(1, 8)
    with pytest.raises(ug.UnltdError) as e:
        s.decode(1, 1)
    assert e.value.status == 2 and "context full" in str(e.value)
    s.close()


def test_9b_greedy_stream_from_2048_context(ctx):
    """the synthetic 9B-class model, KV cache prefilled to
    2048 positions; 16 greedy tokens (at least 8 distinct: the stream does not
    settle on one vocab row), the final hidden state and logits bit-identical
    to the oracle."""
    cfg = synth.QWEN35_9B
    tensors = synth.qwen35_model(cfg, 2026)
    st = synth.qwen35_state(cfg, 2048, 2027)
    m = ug.Qwen35Model(ctx, cfg)
    m.load(tensors)
    n = 16
    s = m.session(2048 + n + 4)
    s.set_state(2048, st["conv"], st["gdn"], st["k"], st["v"])
    toks = s.decode(1000, n)
    lg, hd = s.read()
    s.close()
    m.close()
    o = oracle.Qwen35Oracle(cfg, tensors, 2048 + n + 4, st, 2048)
    otoks, ologits, ohidden = o.greedy(1000, n, nthreads=os.cpu_count() or 8)
    print("9B greedy stream:", toks.tolist(), "oracle:", otoks)
    assert toks.tolist() == otoks
    assert len(set(otoks)) >= 8, otoks
    assert (bits(hd) == bits(ohidden)).all()
    assert (bits(lg) == bits(ologits)).all()
