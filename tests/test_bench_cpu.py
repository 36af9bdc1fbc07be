"""bench.py on the CPU: the reference arm's JSON line, its silence on ranks
other than 0, the algorithmic byte counts the GB/s figures divide by, and the
host-side sharding of the config-1 weights used at N > 1 GPUs."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [REPO]

import bench  # noqa: E402
import synth  # noqa: E402


def _run_ref(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_reference_arm_prints_one_contract_line():
    lines = [l for l in _run_ref({}).splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 1
    assert d["config"]["workload"] == "config1_mixed_gemv_decode"
    assert d["config"]["step_bytes"] == bench.STEP_BYTES
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_silently():
    assert _run_ref({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}).strip() == ""


def test_algorithmic_bytes_match_the_stated_weight_sizes():
    # weight bytes of configs 1a-1d: 0.5625 / 0.8203125 / 1.0625 B per element
    weights = {"a_q4k_gate_up": 28_311_552, "b_q6k_down": 41_287_680, "c_q8_0": 17_825_792,
               "d_q6k_lm_head": 510_504_960}
    total = 0
    for n, dt, di, do, _ in bench.MIX:
        b = bench.algorithmic_bytes(dt, di, do, n.startswith("d_"))
        assert b == weights[n] + 4 * di + 4 * do + (4 if n.startswith("d_") else 0)
        total += b
    assert total == bench.STEP_BYTES == 598_717_956


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("item", range(len(bench.MIX)))
def test_config1_shards_partition_the_weights(world, item):
    n, dt, di, do, split = bench.MIX[item]
    if dt == synth.Q6K and n.startswith("d_"):
        di, do = 512, 1001  # the LM head's split at a size the test builds quickly
    wb = synth.quant_weights(dt, di, do, 5)
    rb = synth.row_bytes(dt, di)
    parts = [bench.shard_weights(wb, dt, di, do, split, r, world) for r in range(world)]
    if split == "rows":
        assert np.array_equal(np.concatenate([p[0] for p in parts]), wb)
        assert [p[3] for p in parts] == list(np.cumsum([0] + [p[2] for p in parts[:-1]]))
        assert all(p[1] == di and p[0].size == p[2] * rb for p in parts)
    else:
        be, bb = synth.BLOCK_ELEMS[dt], synth.BLOCK_BYTES[dt]
        cols = [p[0].reshape(do, -1) for p in parts]
        assert np.array_equal(np.concatenate(cols, axis=1).reshape(-1), wb)
        for p in parts:
            assert p[1] % be == 0 and p[3] % be == 0 and p[2] == do
            assert p[0].size == do * (p[1] // be) * bb
        assert sum(p[1] for p in parts) == di


def test_decode_bytes_per_token_components():
    # the 9B-class model at a 2048-position context: packed projection and
    # LM-head weights with the one embedding row 4,826,052,864 B, K/V rows
    # 134,217,728 B, GDN matrices read and written 2 x 50,331,648 B, plus the
    # f32 tensors and the conv windows
    cfg = synth.QWEN35_9B
    d = synth.qwen35_dims(cfg)
    packed = f32_bytes = embd = 0
    for nm, dt, di, do in synth.qwen35_tensor_list(cfg):
        if nm == "token_embd.weight":
            embd = synth.row_bytes(dt, di)
        elif dt == synth.F32:
            f32_bytes += 4 * di * do
        else:
            packed += synth.row_bytes(dt, di) * do
    assert packed + embd == 4_826_052_864
    n_recr = cfg["n_layer"] - sum(d["attn"])
    conv = n_recr * 4 * cfg["conv_kernel"] * d["dconv"]
    expect = packed + f32_bytes + embd + 134_217_728 + 2 * 50_331_648 + conv
    assert bench.decode_bytes_per_token(cfg, 2047) == expect
