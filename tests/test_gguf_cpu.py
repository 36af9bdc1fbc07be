"""GGUF reader of the library (csrc/gguf.cu), no GPU: the synthetic tiny
model written as a GGUF file comes back tensor for tensor (names, ggml types
mapped to unltd dtypes, GGUF shapes, bytes), the qwen35 config is derived as
Qwen35Config::from_gguf does (qwen35.rs:23-42, 130-200), and malformed files
are refused with an error status, never a crash."""
import os
import struct

import numpy as np
import pytest

import synth
import unltd_gpu as ug

CFG = synth.QWEN35_TINY


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    tensors = synth.qwen35_model(CFG, 11)
    path = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    synth.write_qwen35_gguf(path, CFG, tensors)
    return path, tensors


def test_tensors_round_trip(tiny):
    path, tensors = tiny
    with ug.Gguf(path) as g:
        listed = {t[0]: t for t in g.tensors()}
        assert set(listed) == set(tensors)
        for name, dt, dim_in, dim_out in synth.qwen35_tensor_list(CFG):
            _, gdt, ne, nd, nb, addr = listed[name]
            assert gdt == dt and addr
            arr = np.ascontiguousarray(tensors[name][1])
            assert nb == arr.nbytes
            assert g.tensor_bytes(name) == arr.tobytes()
            if dt != synth.F32:
                assert (nd, ne[0], ne[1]) == (2, dim_in, dim_out)
            assert addr % 32 == 0  # general.alignment


def test_qwen35_config(tiny):
    path, _ = tiny
    with ug.Gguf(path) as g:
        c = g.qwen35_config()
        assert g.get_string("general.architecture") == "qwen35"
        assert g.get_int("qwen35.block_count") == CFG["n_layer"]
    for k, v in CFG.items():
        assert c[k] == pytest.approx(v), k


def _kvs(skip=None, sections=(11, 11, 10, 0)):
    a = "qwen35."
    kv = [("general.architecture", "str", "qwen35")] + [
        (a + k, "u32", 4) for k in ("block_count", "context_length", "embedding_length", "feed_forward_length",
                                    "attention.head_count", "attention.head_count_kv", "attention.key_length",
                                    "attention.value_length", "rope.dimension_count", "ssm.conv_kernel",
                                    "ssm.state_size", "ssm.group_count", "ssm.time_step_rank", "ssm.inner_size",
                                    "full_attention_interval")] + [
        (a + "attention.layer_norm_rms_epsilon", "f32", 1e-6), (a + "rope.freq_base", "f32", 1e7),
        (a + "rope.dimension_sections", "i32[]", list(sections))]
    return [x for x in kv if x[0] != skip]


def _emb():
    return [("token_embd.weight", 0, [4, 3], np.arange(12, dtype=np.float32).tobytes())]


def test_config_refuses_missing_or_mistyped_keys(tmp_path):
    p = str(tmp_path / "m.gguf")
    synth.write_gguf(p, _kvs(), _emb())
    with ug.Gguf(p) as g:
        assert g.qwen35_config()["vocab"] == 3
    for bad in (_kvs(skip="qwen35.ssm.inner_size"), _kvs(sections=(11, 11, 10))):
        synth.write_gguf(p, bad, _emb())
        with ug.Gguf(p) as g, pytest.raises(ug.UnltdError):
            g.qwen35_config()
    wrong = [(k, "i32", v) if k == "qwen35.block_count" else (k, t, v) for k, t, v in _kvs()]
    synth.write_gguf(p, wrong, _emb())
    with ug.Gguf(p) as g, pytest.raises(ug.UnltdError):
        g.qwen35_config()


def test_malformed_files_are_refused(tmp_path, tiny):
    path, _ = tiny
    good = open(path, "rb").read()
    p = str(tmp_path / "bad.gguf")
    cases = [b"GGUX" + good[4:],                      # magic
             good[:4] + struct.pack("<I", 7) + good[8:],  # version
             good[:200],                                 # metadata cut short
             good[:len(good) - 1000]]                    # last tensor past the end
    for data in cases:
        open(p, "wb").write(data)
        with pytest.raises(ug.UnltdError):
            ug.Gguf(p)
    with pytest.raises(ug.UnltdError):
        ug.Gguf(str(tmp_path / "does-not-exist.gguf"))


def test_mutations_never_crash(tmp_path):
    # random byte flips in the header region and random truncations: the
    # reader either parses or returns an error status
    p = str(tmp_path / "m.gguf")
    synth.write_gguf(p, _kvs(), _emb())
    good = bytearray(open(p, "rb").read())
    rng = np.random.default_rng(5)
    parsed = 0
    for _ in range(300):
        b = bytearray(good)
        for _ in range(int(rng.integers(1, 4))):
            b[int(rng.integers(0, len(b)))] = int(rng.integers(0, 256))
        if rng.random() < 0.3:
            b = b[:int(rng.integers(0, len(b)))]
        open(p, "wb").write(bytes(b))
        try:
            with ug.Gguf(p) as g:
                g.tensors()
                parsed += 1
        except ug.UnltdError:
            pass
    assert parsed > 0


def test_centered_q4k_model_blocks(ora):
    """The model generator's Q4_K blocks: every group's min equals its scale
    (scale_min_k4 of the packed bytes, quants.rs:92-102), dmin = f16(7.5 d),
    and the dequantized weights have mean ~0 (uniform blocks: ~+1.2)."""
    import numpy as np

    import synth

    w = synth.centered_q4k_weights(4096, 16, seed=5)
    blocks = w.reshape(-1, 144)
    for blk in blocks[:8]:
        s = blk[4:16]
        for g in range(8):
            if g < 4:
                sc, m = s[g] & 63, s[g + 4] & 63
            else:
                sc = (s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4)
                m = (s[g + 4] >> 4) | ((s[g] >> 6) << 4)
            assert sc == m
        d = np.frombuffer(blk[0:2].tobytes(), np.float16)[0]
        dmin = np.frombuffer(blk[2:4].tobytes(), np.float16)[0]
        assert dmin == np.float16(np.float32(d) * np.float32(7.5))
    deq = ora.dequantize_q4_k(w, 4096 * 16)
    assert abs(float(deq.mean())) < 0.02 and 0.5 < float(deq.std()) < 2.0
    plain = ora.dequantize_q4_k(synth.quant_weights(synth.Q4K, 4096, 16, seed=5), 4096 * 16)
    assert float(plain.mean()) > 0.5
