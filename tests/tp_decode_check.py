"""Tensor-parallel greedy decode on N GPUs against the single-process CPU
oracle; run with torchrun (one process per GPU), e.g.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \
        --master-addr 127.0.0.1 --master-port 29512 tests/tp_decode_check.py --model tiny

Every rank holds its shard (unltd_qwen35_create_tp); rank 0 compares the
greedy stream, the full logits (gathered from the vocab shards) and the
hidden state with the oracle and prints one JSON line: bit for bit against
the oracle of the sharded arithmetic (Qwen35Oracle.row_split(world): the
input-split projections as per-rank partial gemv_quant_q8k summed in rank
order), and as a drift against the one-device oracle (the rank-order sums
round differently from the reference's single chain).
"""
import argparse
import datetime
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [os.path.join(REPO, "unltd-inference_b200"), os.path.join(REPO, "oracle"), REPO]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import synth  # noqa: E402
import unltd_gpu as ug  # noqa: E402


def load_model(cfg, seed, rank, model_name):
    """The synthetic model, generated once per machine: rank 0 writes every
    tensor to a cache directory (one .npy each, a marker file last); the
    other ranks, and later runs, map the files read-only."""
    cache = os.path.join(os.environ.get("UNLTD_MODEL_CACHE", "/tmp/unltd_model_cache"), f"{model_name}_{seed}")
    marker = os.path.join(cache, "complete")
    if rank == 0 and not os.path.exists(marker):
        tensors = synth.qwen35_model(cfg, seed)
        os.makedirs(cache, exist_ok=True)
        for name, (dt, arr) in tensors.items():
            np.save(os.path.join(cache, name + ".npy"), arr)
        with open(marker, "w") as f:
            f.write("ok")
    dist.barrier()
    out = {}
    for name, dt, _, _ in synth.qwen35_tensor_list(cfg):
        out[name] = (dt, np.load(os.path.join(cache, name + ".npy"), mmap_mode="r"))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", choices=["tiny", "9b"])
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--position", type=int, default=40)
    ap.add_argument("--first-token", type=int, default=None, help="first token (default: 5 tiny, 7 for the 9B model)")
    ap.add_argument("--no-oracle", action="store_true")
    ap.add_argument("--batch", type=int, default=1,
                    help="sequences of a batch session (first tokens first-token + 37 z); sequences 0 and B-1 checked")
    ap.add_argument("--allreduce", default="peer", choices=["peer", "nccl"],
                    help="peer: one kernel over NVLink peer memory; nccl: ncclAllReduce")
    args = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    cfg = synth.QWEN35_TINY if args.model == "tiny" else synth.QWEN35_9B
    seed = 11 if args.model == "tiny" else 2026
    pos0, n = args.position, args.steps
    tensors = load_model(cfg, seed, rank, args.model)
    st = synth.qwen35_state(cfg, pos0, seed + 1)
    ctx = ug.Context(local)
    ctx.comm_init(rank, world, ug.exchange_unique_id())
    if args.allreduce == "peer":
        ctx.peer_init()
    m = ug.Qwen35Model(ctx, cfg, rank, world)
    m.load(tensors)
    if args.batch > 1:
        return batch_main(args, cfg, tensors, st, ctx, m, rank, world, pos0, n)
    s = m.session(pos0 + n + 10)
    s.set_state(pos0, st["conv"], st["gdn"], st["k"], st["v"])
    start = args.first_token if args.first_token is not None else (5 if args.model == "tiny" else 7)
    warm = s.decode(start, 2)  # captures the step graph
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    toks = s.decode(int(warm[-1]), n)
    dt = time.perf_counter() - t0
    toks = np.concatenate([warm, toks])
    lg, hd = s.read()
    v0, v1 = s.shape()["vocab"]
    parts = [None] * world
    dist.all_gather_object(parts, (v0, v1, lg))
    streams = [None] * world
    dist.all_gather_object(streams, toks.tolist())
    out = {"model": args.model, "world": world, "allreduce": args.allreduce, "steps": n, "position": pos0,
           "tokens": toks.tolist(),
           "same_stream_on_all_ranks": all(x == streams[0] for x in streams),
           "tok_s": round(n / dt, 2), "ms_per_token": round(dt / n * 1e3, 4)}
    if rank == 0:
        logits = np.zeros(cfg["vocab"], np.float32)
        for a, b, l in parts:
            logits[a:b] = l
        out["argmax_matches_gathered_logits"] = bool(int(np.argmax(logits)) == int(toks[-1]))
        if not args.no_oracle:
            import oracle

            o = oracle.Qwen35Oracle(cfg, tensors, pos0 + n + 10, st, pos0)
            # the oracle's greedy loop, keeping every step's top-2 logit margin
            otoks, margins, tok = [], [], start
            for _ in range(n + 2):
                ol, oh = o.step(tok, nthreads=os.cpu_count() or 8)
                tok = oracle.argmax(ol)
                top2 = np.sort(ol)[-2:]
                otoks.append(tok)
                margins.append(float((top2[1] - top2[0]) / abs(top2[1])))
            out["oracle_tokens"] = otoks
            out["oracle_top2_margin_rel"] = [round(m, 6) for m in margins]
            out["distinct_tokens"] = len(set(otoks))
            out["stream_matches_oracle"] = otoks == toks.tolist()
            out["logits_maxrel"] = float(np.max(np.abs(logits - ol)) / np.max(np.abs(ol)))
            out["hidden_maxrel"] = float(np.max(np.abs(hd - oh)) / np.max(np.abs(oh)))
            d64 = lambda a, b: float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(np.asarray(b, np.float64)))
            out["logits_normwise"] = d64(logits, ol)
            out["hidden_normwise"] = d64(hd, oh)
            # the oracle's output norm and LM head (gemv_quant_q8k) applied to this
            # run's own final hidden state: the vocab-split head depends on its
            # input only, so given the same hidden state its logits are the same bits
            xn = oracle.rmsnorm(hd, tensors["output_norm.weight"][1], cfg["rms_eps"])
            own = oracle.gemv_quant_q8k(xn, tensors["output.weight"][1], cfg["n_embd"], cfg["vocab"], ug.Q6K,
                                        nthreads=os.cpu_count() or 8)
            out["logits_bit_identical_given_hidden"] = bool(np.array_equal(own.view(np.uint32),
                                                                           logits.view(np.uint32)))
            # the oracle of the sharded arithmetic: the same steps bit for bit
            oracle.Qwen35Oracle.row_split(world)
            try:
                so = oracle.Qwen35Oracle(cfg, tensors, pos0 + n + 10, st, pos0)
                stoks, sl, sh, tok = [], None, None, start
                for _ in range(n + 2):
                    sl, sh = so.step(tok, nthreads=os.cpu_count() or 8)
                    tok = oracle.argmax(sl)
                    stoks.append(tok)
            finally:
                oracle.Qwen35Oracle.row_split(1)
            out["stream_matches_split_oracle"] = stoks == toks.tolist()
            out["logits_bit_identical_to_split_oracle"] = bool(np.array_equal(sl.view(np.uint32), logits.view(np.uint32)))
            out["hidden_bit_identical_to_split_oracle"] = bool(np.array_equal(sh.view(np.uint32), hd.view(np.uint32)))
        print(json.dumps(out), flush=True)
    s.close()
    m.close()
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()


def batch_main(args, cfg, tensors, st, ctx, m, rank, world, pos0, n):
    """A batch session on every rank: each sequence from the same state with
    its own first token; sequences 0 and B-1 against the oracle of the
    sharded arithmetic, bit for bit."""
    B = args.batch
    start = args.first_token if args.first_token is not None else (5 if args.model == "tiny" else 7)
    first = [(start + 37 * z) % cfg["vocab"] for z in range(B)]
    b = m.batch_session(pos0 + n + 10, B)
    for z in range(B):
        b.set_state(z, pos0, st["conv"], st["gdn"], st["k"], st["v"])
    warm = b.decode(first, 2)
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    toks = b.decode(warm[:, -1], n)
    dt = time.perf_counter() - t0
    toks = np.concatenate([warm, toks], axis=1)
    v0, v1 = b.shape()["vocab"]
    check = sorted({0, B - 1})
    reads = {z: b.read(z) for z in check}
    parts = [None] * world
    dist.all_gather_object(parts, (v0, v1, {z: reads[z][0] for z in check}))
    streams = [None] * world
    dist.all_gather_object(streams, toks.tolist())
    out = {"model": args.model, "world": world, "batch": B, "steps": n, "position": pos0,
           "same_streams_on_all_ranks": all(x == streams[0] for x in streams),
           "tok_s": round(B * n / dt, 1)}
    if rank == 0 and not args.no_oracle:
        import oracle

        ok_tok, ok_lg, ok_hd = True, True, True
        oracle.Qwen35Oracle.row_split(world)
        try:
            for z in check:
                logits = np.zeros(cfg["vocab"], np.float32)
                for a, c, lgs in parts:
                    logits[a:c] = lgs[z]
                so = oracle.Qwen35Oracle(cfg, tensors, pos0 + n + 10, st, pos0)
                tok, stoks = first[z], []
                for _ in range(n + 2):
                    sl, sh = so.step(tok, nthreads=os.cpu_count() or 8)
                    tok = oracle.argmax(sl)
                    stoks.append(tok)
                ok_tok &= stoks == toks[z].tolist()
                ok_lg &= bool(np.array_equal(sl.view(np.uint32), logits.view(np.uint32)))
                ok_hd &= bool(np.array_equal(sh.view(np.uint32), reads[z][1].view(np.uint32)))
        finally:
            oracle.Qwen35Oracle.row_split(1)
        out["checked_sequences"] = check
        out["streams_match_split_oracle"] = ok_tok
        out["logits_bit_identical_to_split_oracle"] = ok_lg
        out["hidden_bit_identical_to_split_oracle"] = ok_hd
    if rank == 0:
        print(json.dumps(out), flush=True)
    b.close()
    m.close()
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
