"""The two sharded GEMV forms of tensor parallelism through the C ABI, on N
GPUs (one process each, under torchrun), e.g.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \
        --master-addr 127.0.0.1 --master-port 29513 tests/tp_shard_check.py

* vocab split: every rank holds rows [row0, row0 + n) of a Q6_K LM head and
  runs unltd_gemv_argmax_shard; unltd_allreduce_max_u64 of the keys must give
  the first-index maximum of the whole head's logits (greedy.rs:18-27), and
  the token must equal the oracle's on the full Q8_K logits (a row's logit
  does not depend on the split, so the logits are bit-identical);
* column split: every rank holds input blocks [b0, b1) of a Q6_K matrix and
  runs unltd_gemv (Q8K_EXACT) on its slice of x; unltd_allreduce_sum_f32 of
  the partial outputs must match the oracle's single-device gemv_quant_q8k
  within 1e-4 of max |y| (only the f32 rounding of the per-rank sums differs).

Rank 0 prints one JSON line.
"""
import argparse
import datetime
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [os.path.join(REPO, "unltd-inference_b200"), os.path.join(REPO, "oracle"), REPO]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
import synth  # noqa: E402
import unltd_gpu as ug  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--allreduce", default="peer", choices=["peer", "nccl"])
    ap.add_argument("--vocab", type=int, default=20011)
    args = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_stream(torch.cuda.Stream())
    ctx = ug.Context(local, stream=torch.cuda.current_stream().cuda_stream)
    ctx.comm_init(rank, world, ug.exchange_unique_id())
    if args.allreduce == "peer":
        ctx.peer_init()
    out = {"world": world, "allreduce": args.allreduce}

    # ---- vocab-split LM head ----
    dim_in, vocab = 4096, args.vocab
    rb = synth.row_bytes(ug.Q6K, dim_in)
    wb = synth.quant_weights(ug.Q6K, dim_in, vocab, seed=71).copy()
    x = synth.activations(dim_in, seed=72)
    full = oracle.gemv_quant_q8k(x, wb, dim_in, vocab, ug.Q6K, nthreads=8) if rank == 0 else None
    if rank == 0:
        # a tie across the shard boundary: the copy in the later shard must lose
        top = int(np.argmax(full))
        if top < vocab - 2:
            wb[(vocab - 2) * rb:(vocab - 1) * rb] = wb[top * rb:(top + 1) * rb]
            full = oracle.gemv_quant_q8k(x, wb, dim_in, vocab, ug.Q6K, nthreads=8)
    t = torch.from_numpy(wb)
    dist.broadcast(t, 0)
    wb = t.numpy()
    per = -(-vocab // world)
    r0, r1 = rank * per, min(vocab, (rank + 1) * per)
    w = ctx.upload(wb, ug.Q6K, dim_in, vocab, row0=r0, rows=r1 - r0)
    xd = torch.from_numpy(x).cuda()
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    logits = torch.empty(r1 - r0, device="cuda")
    toks = []
    for _ in range(3):  # the argmax state resets between calls
        ctx.gemv_argmax_shard(w, xd, key, r0, logits=logits, mode=ug.MODE_Q8K)
        ctx.allreduce_max_u64(key, 1)
        ctx.synchronize()
        toks.append(0xFFFFFFFF - (int(key.item()) & 0xFFFFFFFF))
    lp = torch.full((per,), float("nan"), device="cuda")
    lp[:r1 - r0] = logits
    gl = [torch.empty(per) for _ in range(world)]
    dist.all_gather(gl, lp.cpu())
    all_toks = [None] * world
    dist.all_gather_object(all_toks, toks)
    w.free()

    # ---- column-split Q6_K GEMV (ffn_down shape) ----
    din, dout = 12288, 4096
    wd = synth.quant_weights(ug.Q6K, din, dout, seed=73)
    xx = synth.activations(din, seed=74)
    nblk = din // 256
    bper = -(-nblk // world)
    b0, b1 = rank * bper, min(nblk, (rank + 1) * bper)
    rbd = synth.row_bytes(ug.Q6K, din)
    rows = wd.reshape(dout, rbd)[:, b0 * 210:b1 * 210]
    ws = ctx.upload(np.ascontiguousarray(rows).reshape(-1), ug.Q6K, (b1 - b0) * 256, dout)
    y = torch.empty(dout, device="cuda")
    ctx.gemv(ws, torch.from_numpy(xx[b0 * 256:b1 * 256].copy()).cuda(), y, ug.MODE_Q8K)
    ctx.allreduce_sum(y, dout)
    ctx.synchronize()
    ys = [None] * world
    dist.all_gather_object(ys, y.cpu().numpy())
    ws.free()

    if rank == 0:
        lg = np.concatenate([g.numpy() for g in gl])
        lg = np.concatenate([lg[i * per:i * per + min(per, vocab - i * per)] for i in range(world)])
        out["same_token_on_all_ranks"] = all(t == all_toks[0] for t in all_toks)
        out["token"] = all_toks[0][0]
        out["token_matches_oracle"] = all_toks[0][0] == oracle.argmax(full) == top
        out["logits_bit_identical"] = bool(np.array_equal(lg.view(np.uint32), full.view(np.uint32)))
        # against the single-device Q8_K product: the split changes only the
        # f32 rounding of the per-rank sums
        ref = oracle.gemv_quant_q8k(xx, wd, din, dout, ug.Q6K, nthreads=8).astype(np.float64)
        out["colsplit_maxrel"] = float(np.max(np.abs(ys[0] - ref)) / np.max(np.abs(ref)))
        out["colsplit_same_on_all_ranks"] = all(np.array_equal(v, ys[0]) for v in ys)
        print(json.dumps(out), flush=True)
    dist.barrier()
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
