"""Tensor-parallel decode (tests/tp_decode_check.py under torchrun) against
the CPU oracle, and the sharded GEMV forms through the C ABI
(tests/tp_shard_check.py). On 2 GPUs with the small model: identical greedy
stream, logits and hidden state within 1e-3 max-rel (the row-split
projections sum partial outputs across GPUs, so the f32 rounding differs from
the single-device reference), through both all-reduce paths, the NVLink peer
kernel and NCCL. On 4 and 8 GPUs (skipped on smaller boxes) with the 9B-class
model: see test_tp_9b_decode_matches_oracle."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
HERE = os.path.dirname(os.path.abspath(__file__))
TOL = 1e-3


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("allreduce", ["peer", "nccl"])
def test_tp2_tiny_decode_matches_oracle(allreduce):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from __graft_entry__ import build

    build()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "tp_decode_check.py"), "--model", "tiny", "--steps", "8", "--allreduce", allreduce]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    out = json.loads(line)
    print(out)
    assert out["same_stream_on_all_ranks"] and out["argmax_matches_gathered_logits"]
    assert out["stream_matches_oracle"], out
    assert out["logits_maxrel"] <= TOL and out["hidden_maxrel"] <= TOL, out


@pytest.mark.parametrize("allreduce", ["peer", "nccl"])
def test_tp2_vocab_split_argmax_and_column_split_gemv(allreduce):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from __graft_entry__ import build

    build()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "tp_shard_check.py"), "--allreduce", allreduce]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    out = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    print(out)
    assert out["same_token_on_all_ranks"] and out["token_matches_oracle"] and out["logits_bit_identical"], out
    assert out["colsplit_maxrel"] <= 1e-4, out
    if allreduce == "peer":  # rank-order sums: the same bits everywhere
        assert out["colsplit_same_on_all_ranks"], out


def _run_torchrun(world, script, *args):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, script), *args]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    out = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    print(out)
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_9b_decode_matches_oracle(world):
    """The 9B-class model at 4 and 8 GPUs: at 8 every rank holds one KV head
    shared by its pair of query heads and 4 of the 32 recurrent v heads; the
    row-split sums run through the NVLink peer kernel fused into the GEMVs.

    Over 32 layers the f32 rounding of the split sums moves a few Q8_K
    activation quants by one step, so the final hidden state drifts from the
    single-device oracle (8.8e-4 max-rel at 8 GPUs), and the LM head, whose
    dot products cancel, amplifies that drift in its logits (5.1e-3 max-rel
    at 8 GPUs). The logits are therefore checked bit for bit against the
    oracle's output norm and LM head applied to this run's own hidden state,
    the hidden state within 1e-3, and the greedy stream exactly."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from __graft_entry__ import build

    build()
    out = _run_torchrun(world, "tp_decode_check.py", "--model", "9b", "--steps", "4", "--allreduce", "peer")
    assert out["same_stream_on_all_ranks"] and out["argmax_matches_gathered_logits"]
    assert out["stream_matches_oracle"], out
    assert out["logits_bit_identical_given_hidden"], out
    assert out["hidden_maxrel"] <= TOL, out


@pytest.mark.parametrize("world", [4, 8])
def test_tp_shard_forms_at_world(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from __graft_entry__ import build

    build()
    out = _run_torchrun(world, "tp_shard_check.py", "--allreduce", "peer")
    assert out["same_token_on_all_ranks"] and out["token_matches_oracle"] and out["logits_bit_identical"], out
    assert out["colsplit_maxrel"] <= 1e-4, out
    assert out["colsplit_same_on_all_ranks"], out
