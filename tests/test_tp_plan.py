"""Host-side checks of the tensor-parallel decode (no GPU): the shard plan
that unltd_qwen35_create_tp applies to every GGUF tensor, and the NCCL id
exchange over a world-size-2 gloo process group."""
import os
import socket

import numpy as np
import pytest

import synth
import unltd_gpu as ug

WORLDS = (1, 2, 4, 8)


def _coverage(cfg, name, world):
    rows, ins = [], []
    for r in range(world):
        rr, ii = ug.qwen35_shard(cfg, r, world, name)
        rows.append(rr)
        ins.append(ii)
    return rows, ins


def _count(ranges, n):
    c = np.zeros(n, np.int64)
    for a, b in ranges:
        assert 0 <= a < b <= n
        c[a:b] += 1
    return c


@pytest.mark.parametrize("cfg", [synth.QWEN35_9B, synth.QWEN35_TINY], ids=["9b", "tiny"])
@pytest.mark.parametrize("world", WORLDS)
def test_shard_plan_partitions(cfg, world):
    if cfg is synth.QWEN35_TINY and world > 2:
        pytest.skip("the tiny model has 2 q heads")
    d = synth.qwen35_dims(cfg)
    nvl, nhl = d["nv"] // world, cfg["n_head"] // world
    for name, dt, di, do in synth.qwen35_tensor_list(cfg):
        kind = name.split(".", 2)[-1] if name.startswith("blk.") else name
        n = di if dt == synth.F32 else do
        rows, ins = _coverage(cfg, name, world)
        counts = _count([x for rr in rows for x in rr], n)
        if kind in ("ffn_gate.weight", "ffn_up.weight", "output.weight", "attn_q.weight", "attn_gate.weight",
                    "ssm_beta.weight", "ssm_alpha.weight", "ssm_dt.bias", "ssm_a"):
            assert (counts == 1).all(), name  # output rows partitioned
        elif kind in ("ffn_down.weight", "attn_output.weight", "ssm_out.weight"):
            assert (counts == world).all(), name  # every rank all rows ...
            cin = _count(ins, di)
            assert (cin == 1).all(), name  # ... of a partition of the input columns
            assert all((b - a) % 256 == 0 for a, b in ins)
        elif kind in ("attn_k.weight", "attn_v.weight"):
            # kv heads partitioned, or shared by the ranks of one kv group
            g = cfg["n_head"] // cfg["n_head_kv"]
            assert (counts == max(1, g // nhl)).all(), name
        elif kind in ("attn_qkv.weight", "ssm_conv1d.weight"):
            hd, nqk = d["hd"], d["nqk"]
            unit = hd * (cfg["conv_kernel"] if kind == "ssm_conv1d.weight" else 1)
            qk = counts[: 2 * nqk * unit]
            v = counts[2 * nqk * unit:]
            assert (v == 1).all(), name  # v channels partitioned
            assert qk.min() >= 1 and (qk == qk[0]).all(), name  # every q/k head on the same number of ranks
        else:
            assert (counts == world).all(), name  # replicated
        if kind not in ("ffn_down.weight", "attn_output.weight", "ssm_out.weight"):
            assert all(ii == (0, di if dt != synth.F32 else 1) for ii in ins), name


def test_shard_plan_rejects_uneven_split():
    cfg = dict(synth.QWEN35_9B, n_head=12, n_embd=3072, d_inner=3072)
    with pytest.raises(ug.UnltdError):
        ug.qwen35_shard(cfg, 0, 8, "blk.3.attn_q.weight")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = ug.exchange_unique_id()
    except ug.UnltdError as e:  # no usable network interface for NCCL's bootstrap
        uid = b"unavailable: " + str(e).encode()
    with open(os.path.join(out_dir, f"uid{rank}"), "wb") as f:
        f.write(uid)
    dist.barrier()
    dist.destroy_process_group()


def test_unique_id_exchange_gloo(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_exchange_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    a, b = (open(tmp_path / f"uid{r}", "rb").read() for r in range(2))
    if a.startswith(b"unavailable"):
        pytest.skip(a.decode(errors="replace"))
    assert a == b and len(a) == 128
