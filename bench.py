"""Benchmark of the quantized decode-GEMV path (driver contract: one JSON line).

Workload (the mixed-format GEMVs at Q4_K_M decode shapes):
  (a) Q4_K 4096 -> 12288, (b) Q6_K 12288 -> 4096, (c) Q8_0 4096 -> 4096,
  (d) Q6_K LM head 4096 -> 151936 + greedy argmax.
One step = one pass of (a)-(d) on seeded synthetic weights and x ~ N(0,1).
The weights of one step (598 MB) exceed the 126 MB L2, so every step streams
them from HBM; no separate flush is needed.

`gemv_back_to_back` (one GPU): BASELINE config 0 (Q4_K 4096 x 4096) and each
config-1 shape alone, as device throughput of GEMVs issued back to back: a
CUDA graph of launches cycling through distinct uploads of the weights whose
total exceeds the L2, CUDA-event timed (the decode step issues its GEMVs this
way).

Arithmetic: the K-quant GEMVs run MODE_Q8K_EXACT (bit-identical to the
reference's gemv_quant_q8k, its production path); Q8_0 has no Q8_K path in the
reference and runs MODE_F32X. The F32X rate of the whole mix is reported too.

N > 1 GPUs (torchrun): the projections are sharded as in a tensor-parallel
decode: (a) and (c) column-split (rows), (b) row-split on its inputs followed
by an all-reduce of y, (d) vocab-split with a cross-GPU argmax (all-reduce MAX
of a packed 64-bit key); both all-reduces are the library's NVLink peer kernel
(NCCL through torch.distributed if the peer mapping is unavailable). Total work
is fixed: strong scaling. `e2e` at N > 1 adds, every step, each rank's x copy
from pinned host memory and its y shard and the token back into pinned host
memory, device-timed and taken as the max over ranks.

--impl reference times the reference's CPU implementation of the same step
(the oracle restatement of quants.rs: gemv_quant_q8k single-threaded per
projection as the reference runs them, the LM head row-parallel over all
host cores as min_forward.rs:245-264 does) on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(REPO, "unltd-inference_b200"), os.path.join(REPO, "oracle")]

import numpy as np  # noqa: E402

import synth  # noqa: E402

METRIC = "Q4_K/Q6_K GEMV GB/s vs B200 HBM peak; 9B-class decode tok/s at 1/2/4/8 GPUs"
UNIT = "GB/s"
Q4K, Q6K, Q8_0 = synth.Q4K, synth.Q6K, synth.Q8_0
# (name, dtype, dim_in, dim_out, split): split = "rows" (column-parallel) | "cols" (row-parallel)
MIX = [
    ("a_q4k_gate_up", Q4K, 4096, 12288, "rows"),
    ("b_q6k_down", Q6K, 12288, 4096, "cols"),
    ("c_q8_0", Q8_0, 4096, 4096, "rows"),
    ("d_q6k_lm_head", Q6K, 4096, 151936, "rows"),
]
SEEDS = {n: 1000 + i for i, (n, *_rest) in enumerate(MIX)}


def algorithmic_bytes(dtype, dim_in, dim_out, argmax=False):
    """Packed weights + x read once + y written (+ the 4-byte token)."""
    return synth.row_bytes(dtype, dim_in) * dim_out + 4 * dim_in + 4 * dim_out + (4 if argmax else 0)


STEP_BYTES = sum(algorithmic_bytes(dt, di, do, n.startswith("d_")) for n, dt, di, do, _ in MIX)


def _peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _bf16_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"


def _traffic():
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, device: int):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        names = {
            0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
            0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown",
        }
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in names.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.0002)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self):
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def _dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def shard_weights(wb, dtype, dim_in, dim_out, split, rank, world):
    """Host-side shard of a packed tensor: rows [r0, r1) or input blocks [b0, b1)."""
    rb = synth.row_bytes(dtype, dim_in)
    if world == 1:
        return wb, dim_in, dim_out, 0
    if split == "rows":
        per = -(-dim_out // world)
        r0, r1 = rank * per, min(dim_out, (rank + 1) * per)
        return wb[r0 * rb:r1 * rb], dim_in, r1 - r0, r0
    be = synth.BLOCK_ELEMS[dtype]
    nblk = dim_in // be
    per = -(-nblk // world)
    b0, b1 = rank * per, min(nblk, (rank + 1) * per)
    bb = synth.BLOCK_BYTES[dtype]
    m = wb.reshape(dim_out, rb)[:, b0 * bb:b1 * bb]
    return np.ascontiguousarray(m).reshape(-1), (b1 - b0) * be, dim_out, b0 * be


L2_BYTES = 126 * 2**20


def back_to_back(ctx, stream, dt, di, do, seed, mode, reps_min=24):
    """Device throughput of one GEMV shape issued back to back: C distinct
    uploads of the weights (C x bytes > L2, so every launch streams its
    weights from HBM), R launches cycling through them captured in one CUDA
    graph (no host launch gaps; consecutive GEMVs chain with programmatic
    dependent launch as in the decode step), timed with CUDA events on the
    launch stream. Returns (us per GEMV, GB/s of algorithmic bytes)."""
    import torch

    base = synth.quant_weights(dt, di, do, seed)
    wbytes = synth.row_bytes(dt, di) * do
    C = max(1, -(-int(1.2 * L2_BYTES) // wbytes))
    ws = []
    for c in range(C):
        wb = base.copy()
        wb[:16] ^= np.uint8(c)  # a distinct tensor per copy
        ws.append(ctx.upload(wb, dt, di, do))
    x = torch.from_numpy(synth.activations(di, seed + 1)).cuda()
    y = torch.empty(do, device="cuda")
    R = max(reps_min, C)
    R = -(-R // C) * C
    for w in ws:
        ctx.gemv(w, x, y, mode)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        for r in range(R):
            ctx.gemv(ws[r % C], x, y, mode)
    ctx.set_stream(stream.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(3):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (3 * R)
    del g
    for w in ws:
        w.free()
    return us, algorithmic_bytes(dt, di, do) / (us * 1e-6) / 1e9


def cpu_baseline(steps=3):
    """The oracle (reference restatement) on one full config-1 step, median of `steps`."""
    import oracle

    ncores = os.cpu_count() or 1
    data = []
    for n, dt, di, do, _ in MIX:
        data.append((n, dt, di, do, synth.quant_weights(dt, di, do, SEEDS[n]), synth.activations(di, SEEDS[n] + 1)))
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        for n, dt, di, do, wb, x in data:
            if n.startswith("d_"):
                y = oracle.gemv_quant_q8k(x, wb, di, do, dt, ncores)
                oracle.argmax(y)
            elif dt == Q8_0:
                oracle.gemv_quant(x, wb, di, do, dt, 1)
            else:
                oracle.gemv_quant_q8k(x, wb, di, do, dt, 1)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {
        "value": round(STEP_BYTES / t / 1e9, 4),
        "unit": UNIT,
        "cores": ncores,
        "kind": "port",
        "sample": f"{steps} full config-1 steps (median {t:.3f} s/step): projections single-threaded, "
                  f"LM head row-parallel on {ncores} threads, as the reference runs them",
    }


def decode_bytes_per_token(cfg, position, n_seq=1):
    """Bytes one greedy decode step must move: every projection's packed
    weights, the LM head, the f32 norms and conv kernels (once per step), and
    per sequence one embedding row, the GDN matrices (read and written), the
    conv windows and the K/V rows of the `position + 1` cached positions
    (qwen35_forward.rs step)."""
    d = synth.qwen35_dims(cfg)
    total = 0
    for nm, dt, di, do in synth.qwen35_tensor_list(cfg):
        if nm == "token_embd.weight":
            total += n_seq * synth.row_bytes(dt, di)
        else:
            total += synth.row_bytes(dt, di) * do
    n_attn = sum(d["attn"])
    n_recr = cfg["n_layer"] - n_attn
    total += n_seq * n_recr * (2 * 4 * d["nv"] * d["hd"] * d["hd"] + 4 * cfg["conv_kernel"] * d["dconv"])
    total += n_seq * n_attn * 2 * 4 * (position + 1) * d["kvlen"]
    return total


def decode_batch_bench(m, cfg, st, pos0, n_seq, n_steps, profile_region=False, world=1, dist=None):
    """BASELINE config 4 at batch n_seq: n_seq sequences from the
    2048-position state (each its own first token) decoded together through
    unltd_qwen35_batch_decode, on one GPU or tensor-parallel over `world`
    (every rank holds its shard of the weights and of every sequence's
    state); every weight matrix is read once per step for all sequences.
    Device-timed on each rank's session stream, the max over ranks."""
    import torch

    b = m.batch_session(pos0 + n_steps + 16, n_seq)
    for z in range(n_seq):
        b.set_state(z, pos0, st["conv"], st["gdn"], st["k"], st["v"])
    first = [1000 + 37 * z for z in range(n_seq)]
    warm = b.decode(first, 4)
    ext = torch.cuda.ExternalStream(b.info()["stream"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if profile_region:
        torch.cuda.profiler.start()
    t0 = time.perf_counter()
    e0.record(ext)
    toks = b.decode(warm[:, -1], n_steps)
    e1.record(ext)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if profile_region:
        torch.cuda.profiler.stop()
    ms_step = e0.elapsed_time(e1) / n_steps
    if dist:
        tt = torch.tensor([ms_step, wall], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_step, wall = float(tt[0]), float(tt[1])
    bps = decode_bytes_per_token(cfg, pos0 + 4 + n_steps // 2, n_seq)
    peak, peak_kind = _peaks()
    gbs = bps / (ms_step * 1e-3) / 1e9
    out = {"workload": f"config4_qwen35_9b_synthetic_greedy_decode_ctx2048_batch{n_seq}" +
                       (f"_tp{world}" if world > 1 else ""), "n_seq": n_seq,
           "steps": n_steps, "n_gpus": world, "tok_s": round(n_seq * 1e3 / ms_step, 1),
           "ms_per_step": round(ms_step, 4), "e2e_tok_s": round(n_seq * n_steps / wall, 1), "bytes_per_step": bps,
           "hbm_gbs": round(gbs, 1), "hbm_gbs_per_gpu": round(gbs / world, 1),
           "roofline_frac": round(gbs / world / peak, 4), "peak": peak, "peak_kind": peak_kind,
           "launches_per_step": b.info()["launches_per_step"],
           "arithmetic": "Q8K_EXACT projections (one weight pass for all sequences); every sequence bit-identical "
                         "to a one-sequence session",
           "distinct_tokens_seq0": len(set(int(t) for t in toks[0]))}
    b.close()
    return out


def prefill_bench(m, cfg, st, pos0, n, profile_region=False):
    """A prompt of n seeded tokens after the 2048-position state through
    unltd_qwen35_prefill (32-token chunks, each weight read once per chunk;
    the same bits as the token-by-token unltd_qwen35_feed). Device-timed on
    the session stream."""
    import torch

    s = m.session(pos0 + n + 40)
    s.set_state(pos0, st["conv"], st["gdn"], st["k"], st["v"])
    prompt = [int(t) for t in np.random.default_rng(7).integers(0, cfg["vocab"], n + 32)]
    s.prefill(prompt[:32])  # warm-up: workspace, batched operands
    ext = torch.cuda.ExternalStream(s.info()["stream"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if profile_region:
        torch.cuda.profiler.start()
    t0 = time.perf_counter()
    e0.record(ext)
    s.prefill(prompt[32:])
    e1.record(ext)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if profile_region:
        torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1)
    s.close()
    return {"workload": f"qwen35_9b_synthetic_prefill_{n}_tokens_after_ctx2048", "tokens": n,
            "tok_s": round(n / (ms * 1e-3), 1), "ms": round(ms, 3), "e2e_tok_s": round(n / wall, 1),
            "arithmetic": "Q8K_EXACT projections batched over 32-token chunks; state and next token bit-identical "
                          "to the token-by-token prompt"}


def decode_bench(n_tokens, with_cpu, rank=0, world=1, dist=None, profile_region=False, batch=32, profile_batch=False,
                 prefill=256, layers=0, profile_prefill=False):
    """BASELINE configs 3 and 4: greedy decode of the synthetic 9B-class hybrid
    model from a 2048-position context through unltd_qwen35_decode, on one GPU
    or tensor-parallel over `world` GPUs (one process each). Device-timed on
    each rank's session stream; the max over ranks is reported."""
    import torch

    import unltd_gpu as ug

    cfg = dict(synth.QWEN35_9B)
    if layers:  # profiling: the same attention and recurrent layers, fewer of them, small FFN and vocab
        cfg.update(n_layer=layers, n_ff=1024, vocab=4096)
    pos0 = 2048
    tensors = synth.qwen35_model(cfg, 2026)
    st = synth.qwen35_state(cfg, pos0, 2027)
    ctx = ug.Context(torch.cuda.current_device())
    if world > 1:
        ctx.comm_init(rank, world, ug.exchange_unique_id())
        ctx.peer_init()  # the step's all-reduces as one NVLink peer kernel each
    m = ug.Qwen35Model(ctx, cfg, rank, world)
    m.load(tensors)
    s = m.session(pos0 + n_tokens + 16)
    s.set_state(pos0, st["conv"], st["gdn"], st["k"], st["v"])
    warm = s.decode(1000, 8)
    info = s.info()
    ext = torch.cuda.ExternalStream(info["stream"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if profile_region:
        torch.cuda.profiler.start()
    t0 = time.perf_counter()
    e0.record(ext)
    toks = s.decode(int(warm[-1]), n_tokens)
    e1.record(ext)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if profile_region:
        torch.cuda.profiler.stop()
    ms_tok = e0.elapsed_time(e1) / n_tokens
    if dist:
        tt = torch.tensor([ms_tok, wall], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_tok, wall = float(tt[0]), float(tt[1])
    bpt = decode_bytes_per_token(cfg, pos0 + 8 + n_tokens // 2)
    peak, peak_kind = _peaks()
    gbs = bpt / (ms_tok * 1e-3) / 1e9  # whole job; each GPU moves about 1/world of it
    out = {
        "workload": ("config3_qwen35_9b_synthetic_greedy_decode_ctx2048" if world == 1 else
                     f"config4_qwen35_9b_synthetic_greedy_decode_ctx2048_tp{world}"),
        "n_tokens": n_tokens, "batch": 1, "n_gpus": world,
        "tok_s": round(1e3 / ms_tok, 2), "ms_per_token": round(ms_tok, 4),
        "e2e_tok_s": round(n_tokens / wall, 2),
        "bytes_per_token": bpt, "hbm_gbs": round(gbs, 1), "hbm_gbs_per_gpu": round(gbs / world, 1),
        "roofline_frac": round(gbs / world / peak, 4), "peak": peak, "peak_kind": peak_kind,
        "launches_per_step": info["launches_per_step"], "graph": "one CUDA graph per token",
        "arithmetic": ("Q8K_EXACT projections; f32/f64 ops in the reference's order (hidden states bit-identical to "
                       "the oracle)" if world == 1 else
                       "Q8K_EXACT projections; row-split partial outputs summed in rank order by the NVLink peer "
                       "all-reduce kernel (bit-identical to the oracle of the sharded arithmetic; same greedy stream "
                       "as the one-device oracle)"),
        "tokens_tail": [int(t) for t in toks[-4:]],
        "distinct_tokens": len(set(int(t) for t in toks)),
    }
    s.close()
    if world == 1 and prefill > 0:
        out["prefill"] = prefill_bench(m, cfg, st, pos0, prefill, profile_prefill)
    if batch > 1:
        out["batch"] = 1
        out["batch%d" % batch] = decode_batch_bench(m, cfg, st, pos0, batch, max(4, n_tokens // 4), profile_batch,
                                                    world, dist)
    m.close()
    ctx.close()
    if with_cpu and rank == 0:
        import oracle

        o = oracle.Qwen35Oracle(cfg, tensors, pos0 + 8, st, pos0)
        ncores = os.cpu_count() or 1
        t0 = time.perf_counter()
        o.step(1000, nthreads=ncores)
        cpu_s = time.perf_counter() - t0
        out["cpu_baseline"] = {"tok_s": round(1.0 / cpu_s, 4), "cores": ncores, "kind": "port",
                               "sample": "1 decode step of the same model and state (oracle restatement of "
                                         "qwen35_forward.rs, projections row-parallel on all cores)"}
    del tensors
    return out


def gemm_bench(ctx, stream, reps):
    """BASELINE config 2 (X 512 x 4096, W Q4_K 12288 x 4096) through unltd_gemm
    (fast, fp16 operands) and unltd_gemm_f32x (accurate), CUDA-event timed
    over `reps` back-to-back calls each (X conversion kernel included)."""
    import torch

    GM, GN, GK = 512, 12288, 4096
    gw = ctx.upload(synth.quant_weights(Q4K, GK, GN, 2024), Q4K, GK, GN)
    GX = torch.from_numpy(synth.activations(GK, 2025, rows=GM)).cuda()
    GY = torch.empty((GM, GN), device="cuda")
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_it = max(reps, 10)
    flops = 2.0 * GM * GN * GK
    peak_tf, peak_tf_kind = _bf16_peak()
    timed = {}
    for accurate in (False, True):
        for _ in range(3):
            ctx.gemm(gw, GX, GY, GM, accurate=accurate)
        torch.cuda.synchronize()
        g0.record(stream)
        for _ in range(n_it):
            ctx.gemm(gw, GX, GY, GM, accurate=accurate)
        g1.record(stream)
        torch.cuda.synchronize()
        timed[accurate] = g0.elapsed_time(g1) / n_it
    gms = timed[False]
    out = {
        "workload": "config2_prefill_gemm_q4k_512x4096x12288", "ms": round(gms, 4),
        "tflops": round(flops / (gms * 1e-3) / 1e12, 1), "peak_tflops": peak_tf, "peak_kind": peak_tf_kind,
        "frac": round(flops / (gms * 1e-3) / 1e12 / peak_tf, 4),
        "note": "unltd_gemm: includes the X f32->fp16 conversion kernel; fp16 operands, f32 accumulation",
        "accurate": {"ms": round(timed[True], 4), "tflops": round(flops / (timed[True] * 1e-3) / 1e12, 1),
                     "frac": round(flops / (timed[True] * 1e-3) / 1e12 / peak_tf, 4),
                     "note": "unltd_gemm_f32x: X and W as hi + lo fp16 pairs, three MMAs per K slice "
                             "(within 1e-4 max-rel of the f64 truth); useful flops counted once"},
    }
    gw.free()
    return out


def run_reference(args):
    rank, world, _ = _dist_env()
    if rank != 0:
        return
    import oracle

    ncores = os.cpu_count() or 1
    data = []
    for n, dt, di, do, _ in MIX:
        data.append((n, dt, di, do, synth.quant_weights(dt, di, do, SEEDS[n]), synth.activations(di, SEEDS[n] + 1)))

    def step():
        for n, dt, di, do, wb, x in data:
            if n.startswith("d_"):
                oracle.argmax(oracle.gemv_quant_q8k(x, wb, di, do, dt, ncores))
            elif dt == Q8_0:
                oracle.gemv_quant(x, wb, di, do, dt, 1)
            else:
                oracle.gemv_quant_q8k(x, wb, di, do, dt, 1)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt_s = (time.perf_counter() - t0) / max(args.steps, 1)
    v = STEP_BYTES / dt_s / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt_s * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8xint8->int32,f32",
        "data": "synthetic (seeded, BASELINE config 1 shapes)",
        "config": {"workload": "config1_mixed_gemv_decode", "gemvs": [m[0] for m in MIX],
                   "step_bytes": STEP_BYTES},
        "cpu_baseline": {"value": round(v, 4), "unit": UNIT, "cores": ncores, "kind": "port",
                         "sample": f"full config-1 steps; projections single-threaded, LM head on {ncores} threads"},
        "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--only", default=None, help="comma-separated subset of the mix (profiling)")
    ap.add_argument("--mode", default="q8k", choices=["q8k", "f32x"], help="arithmetic of the K-quant GEMVs")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-3 decode measurement")
    ap.add_argument("--decode-tokens", type=int, default=64)
    ap.add_argument("--decode-batch", type=int, default=32, help="sequences of the batch-decode measurement (1: none)")
    ap.add_argument("--decode-only", action="store_true", help="measure only the decode step (profiling)")
    ap.add_argument("--gemm-only", action="store_true", help="measure only the config-2 GEMM (profiling)")
    ap.add_argument("--profile-region", action="store_true",
                    help="bracket the timed decode with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    ap.add_argument("--profile-batch", action="store_true",
                    help="bracket the timed batch decode instead (ncu --profile-from-start off)")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="bracket the timed prefill instead (ncu --profile-from-start off)")
    ap.add_argument("--decode-layers", type=int, default=0,
                    help="profiling: a model with this many layers of the 9B shapes (small FFN and vocab)")
    ap.add_argument("--batch-gemv", default=None, metavar="DTYPE:DIM_IN:DIM_OUT:N_SEQ",
                    help="profiling: four unltd_gemv_batch calls on seeded weights (e.g. q4k:4096:12288:32)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import torch

    import unltd_gpu as ug

    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    # exactly one JSON line on stdout: everything else (NCCL's banner included)
    # goes to stderr; the line is written to the saved stdout at the end
    out_fd = os.dup(1)
    os.dup2(2, 1)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    torch.cuda.set_stream(torch.cuda.Stream())
    stream = torch.cuda.current_stream()
    ctx = ug.Context(local, stream=stream.cuda_stream)

    if args.batch_gemv:
        dt, di, do, ns = args.batch_gemv.split(":")
        dtype = {"q4k": ug.Q4K, "q6k": ug.Q6K}[dt]
        di, do, ns = int(di), int(do), int(ns)
        w = ctx.upload(synth.quant_weights(dtype, di, do, seed=3), dtype, di, do)
        X = torch.randn(ns, di, device="cuda")
        Y = torch.empty(ns, do, device="cuda")
        for _ in range(4):
            ctx.gemv_batch(w, X, Y, ns)
        torch.cuda.synchronize()
        w.free()
        ctx.close()
        return

    if args.gemm_only:
        if rank == 0:
            os.write(out_fd, (json.dumps({"metric": "config-2 GEMM", "gemm_prefill": gemm_bench(ctx, stream, args.steps)})
                              + "\n").encode())
        ctx.close()
        return

    if args.decode_only:
        d = decode_bench(args.decode_tokens, with_cpu=False, rank=rank, world=world, dist=dist, batch=args.decode_batch,
                         profile_batch=args.profile_batch, layers=args.decode_layers,
                         prefill=0 if args.decode_layers and not args.profile_prefill else 256,
                         profile_region=args.profile_region, profile_prefill=args.profile_prefill)
        if rank == 0:
            os.write(out_fd, (json.dumps({"metric": "decode tok/s", "decode": d}) + "\n").encode())
        ctx.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    # N > 1: the row-split sums and the cross-GPU argmax MAX through the
    # library's own all-reduce (one NVLink peer kernel each; NCCL if the
    # peer mapping is unavailable), the same on every rank
    lib_comm = False
    if world > 1:
        ok = 1
        try:
            ctx.comm_init(rank, world, ug.exchange_unique_id())
            ctx.peer_init()
        except Exception as e:  # noqa: BLE001
            print(f"library all-reduce unavailable ({e}); using torch.distributed", file=sys.stderr)
            ok = 0
        flag = torch.tensor([ok], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        lib_comm = bool(flag.item())

    # ---- workload ----
    items = []
    mix = [m for m in MIX if args.only is None or m[0] in args.only.split(",")]
    head_mode = ug.MODE_Q8K if args.mode == "q8k" else ug.MODE_F32X
    for n, dt, di, do, split in mix:
        wb = synth.quant_weights(dt, di, do, SEEDS[n])
        x = synth.activations(di, SEEDS[n] + 1)
        swb, sdi, sdo, off = shard_weights(wb, dt, di, do, split, rank, world)
        w = ctx.upload(swb, dt, sdi, sdo)
        xs = x[off:off + sdi] if split == "cols" else x
        items.append({
            "name": n, "dtype": dt, "dim_in": di, "dim_out": do, "split": split, "w": w, "off": off,
            "x_host": x, "x": torch.from_numpy(np.ascontiguousarray(xs)).cuda(),
            "y": torch.empty(sdo, device="cuda"), "mode": ug.MODE_F32X if dt == Q8_0 else head_mode,
            "bytes": algorithmic_bytes(dt, di, do, n.startswith("d_")),
            "local_bytes": algorithmic_bytes(dt, sdi, sdo, n.startswith("d_")),
        })
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    del wb

    def run_item(it, mode=None):
        m = it["mode"] if mode is None else (ug.MODE_F32X if it["dtype"] == Q8_0 else mode)
        if it["name"].startswith("d_"):
            if lib_comm:  # vocab shard: this shard's key, then the MAX over ranks
                ctx.gemv_argmax_shard(it["w"], it["x"], key, it["off"], logits=it["y"], mode=m)
                ctx.allreduce_max_u64(key, 1)
                return
            ctx.gemv_argmax(it["w"], it["x"], tok, logits=it["y"], mode=m)
            if world > 1:
                # local index -> global key (orderable(logit) << 32 | ~global_idx), then MAX
                li = tok.to(torch.int64)
                v = it["y"][li.clamp_max(it["y"].numel() - 1)]
                b = v.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
                ordv = torch.where(b >= 0x80000000, (~b) & 0xFFFFFFFF, b | 0x80000000)
                key.copy_((ordv << 32) | (0xFFFFFFFF - (li + it["off"])))
                dist.all_reduce(key, op=dist.ReduceOp.MAX)
        else:
            ctx.gemv(it["w"], it["x"], it["y"], m)
            if world > 1 and it["split"] == "cols":
                if lib_comm:
                    ctx.allreduce_sum(it["y"], it["y"].numel())
                else:
                    dist.all_reduce(it["y"])

    # the roofline's kernel: the LM head, 85% of the step's bytes
    dom = max(range(len(items)), key=lambda i: items[i]["bytes"])

    def step(mode=None, events=None, only=None):
        # events bracket item `only` (or every item when only is None); an
        # event between two kernels ends the programmatic-launch overlap, so
        # the timed steps bracket the roofline's kernel alone
        for i, it in enumerate(items):
            mark = events is not None and (only is None or i == only)
            if mark:
                events[i][0].record(stream)
            run_item(it, mode)
            if mark:
                events[i][1].record(stream)

    # clocks are sampled from the warm-up through the per-GEMV pass after the
    # timed steps (the timed region alone lasts a few milliseconds)
    sampler = ClockSampler(local)
    sampler.__enter__()
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    # ---- timed: device-resident inputs ----
    K = args.steps
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in items]
          for _ in range(K)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = ctx.launch_count()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t_start.record(stream)
    for k in range(K):
        step(events=ev[k], only=dom)
    t_end.record(stream)
    torch.cuda.synchronize()
    launches = ctx.launch_count() - n0
    ms = t_start.elapsed_time(t_end)
    if dist:
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_step = ms / K
    value = STEP_BYTES / (ms_step * 1e-3) / 1e9
    dom_ms = statistics.mean(ev[k][dom][0].elapsed_time(ev[k][dom][1]) for k in range(K))
    # per-GEMV breakdown (diagnostic, untimed): every item between events
    for k in range(K):
        step(events=ev[k])
    torch.cuda.synchronize()
    per_item_ms = [statistics.mean(ev[k][i][0].elapsed_time(ev[k][i][1]) for k in range(K)) for i in range(len(items))]
    sampler.__exit__(None, None, None)

    # ---- per-shape device throughput, back to back (BASELINE config 0 and the
    # config-1 shapes): CUDA graphs over distinct weight copies ----
    b2b = None
    if world == 1 and args.only is None:
        peak_b, _ = _peaks()
        b2b = {}
        shapes = [("config0_q4k_4096x4096", Q4K, 4096, 4096, 1234)] + [(n, dt, di, do, SEEDS[n]) for n, dt, di, do, _
                                                                       in MIX]
        for name, dt, di, do, seed in shapes:
            m = ug.MODE_F32X if dt == Q8_0 else head_mode
            us, gbs = back_to_back(ctx, stream, dt, di, do, seed, m)
            b2b[name] = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak_b, 4),
                         "mode": "F32X" if m == ug.MODE_F32X else "Q8K_EXACT"}

    # ---- F32X rate of the same mix ----
    for _ in range(2):
        step(mode=ug.MODE_F32X)
    torch.cuda.synchronize()
    t_start.record(stream)
    for _ in range(K):
        step(mode=ug.MODE_F32X)
    t_end.record(stream)
    torch.cuda.synchronize()
    ms_f32x = t_start.elapsed_time(t_end) / K
    if dist:
        tt = torch.tensor([ms_f32x], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_f32x = float(tt.item())

    # ---- e2e through the reference-signature C ABI, host buffers ----
    e2e = None
    if world == 1 and not args.no_e2e and args.only is None:
        host = []
        for n, dt, di, do, _s in MIX:
            wb = synth.quant_weights(dt, di, do, SEEDS[n])
            xp = torch.from_numpy(synth.activations(di, SEEDS[n] + 1)).pin_memory()
            yp = torch.empty(do, dtype=torch.float32).pin_memory()
            host.append((n, dt, di, do, wb, xp.numpy(), yp.numpy()))

        def e2e_step():
            for n, dt, di, do, wb, xh, yh in host:
                if dt == Q8_0:
                    ug.gemv_quant(yh, xh, wb, di, do, dt)
                else:
                    ug.gemv_quant_q8k(yh, xh, wb, di, do, dt)
                if n.startswith("d_"):
                    int(np.argmax(yh))  # greedy.rs argmax on the host, as the reference does

        for _ in range(2):
            e2e_step()
        t0 = time.perf_counter()
        for _ in range(K):
            e2e_step()
        e2e_s = (time.perf_counter() - t0) / K
        e2e = {
            "value": round(STEP_BYTES / e2e_s / 1e9, 2), "unit": UNIT,
            "h2d_bytes_per_step": int(sum(4 * di for _, _, di, _, _ in MIX)),
            "d2h_bytes_per_step": int(sum(4 * do for _, _, _, do, _ in MIX)),
            "ms_per_step": round(e2e_s * 1e3, 4),
            "path": "unltd_gemv_quant_q8k / unltd_gemv_quant (host buffers, pinned; weights cached after first call)",
        }
        ug.forget_host_weights()
    elif world > 1 and not args.no_e2e and args.only is None:
        # every rank: its x slice from pinned host memory, the sharded mix with
        # its all-reduces, its y shard and the greedy token back into pinned
        # host memory, one stream synchronisation per step (the host reads the
        # token); device-timed on the launch stream, max over ranks
        xin = [it["x"].cpu().pin_memory() for it in items]
        yout = [torch.empty(it["y"].numel(), dtype=torch.float32).pin_memory() for it in items]
        kout = torch.empty(1, dtype=torch.int64).pin_memory()

        def e2e_step_tp():
            for i, it in enumerate(items):
                it["x"].copy_(xin[i], non_blocking=True)
                run_item(it)
                yout[i].copy_(it["y"], non_blocking=True)
                if it["name"].startswith("d_"):
                    kout.copy_(key, non_blocking=True)
            stream.synchronize()
            return 0xFFFFFFFF - (int(kout.item()) & 0xFFFFFFFF)

        for _ in range(2):
            e2e_step_tp()
        dist.barrier()
        torch.cuda.synchronize()
        t_start.record(stream)
        for _ in range(K):
            e2e_step_tp()
        t_end.record(stream)
        torch.cuda.synchronize()
        io = torch.tensor([t_start.elapsed_time(t_end) / K, sum(4 * x.numel() for x in xin),
                           sum(4 * y.numel() for y in yout) + 8], device="cuda", dtype=torch.float64)
        ms_e2e = io[:1].clone()
        dist.all_reduce(ms_e2e, op=dist.ReduceOp.MAX)
        dist.all_reduce(io, op=dist.ReduceOp.SUM)
        e2e = {
            "value": round(STEP_BYTES / (float(ms_e2e.item()) * 1e-3) / 1e9, 2), "unit": UNIT,
            "h2d_bytes_per_step": int(io[1].item()), "d2h_bytes_per_step": int(io[2].item()),
            "ms_per_step": round(float(ms_e2e.item()), 4),
            "path": "Context.gemv / gemv_argmax_shard + library all-reduce on every rank; x from and y, token "
                    "to pinned host buffers each step (bytes summed over ranks); device-timed, max over ranks",
        }

    # ---- batched prefill GEMM on the tensor cores ----
    gemm = None
    if world == 1 and args.only is None and not args.no_gemm:
        gemm = gemm_bench(ctx, stream, K)

    decode = None
    if args.only is None and not args.no_decode:
        try:
            decode = decode_bench(args.decode_tokens, with_cpu=not args.no_cpu_baseline and world == 1, rank=rank,
                                  world=world, dist=dist, batch=args.decode_batch)
        except Exception as e:  # report it in the line; the GEMV measurement above stands
            decode = {"error": f"{type(e).__name__}: {e}"[:400]}

    peak, peak_kind = _peaks()
    step_bytes = sum(it["bytes"] for it in items)
    value = step_bytes / (ms_step * 1e-3) / 1e9
    dom_bytes = items[dom]["local_bytes"]
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic = _traffic().get("gemv_q6k_q8k_lm_head_per_launch")
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8xint8->int32,f32 (Q8K_EXACT); Q8_0: F32X",
        "data": "synthetic (seeded weights and x ~ N(0,1), BASELINE config 1 shapes)",
        "config": {
            "workload": "config1_mixed_gemv_decode", "gemvs": [it["name"] for it in items], "step_bytes": step_bytes,
            "parallelism": f"tp{world}" if world > 1 else "single",
            "collectives": ("library all-reduce (NVLink peer kernel)" if lib_comm else
                            "torch.distributed NCCL") if world > 1 else None, "l2": "inputs larger than L2 (598 MB/step)",
            "mode": "Q8K_EXACT (Q8_0 in F32X)",
        },
        "per_gemv": {it["name"]: {"ms": round(per_item_ms[i], 4),
                                  "gbs": round(it["local_bytes"] / (per_item_ms[i] * 1e-3) / 1e9, 1)}
                     for i, it in enumerate(items)},
        "gemv_back_to_back": b2b,
        "f32x_mode": {"value": round(step_bytes / (ms_f32x * 1e-3) / 1e9, 2), "unit": UNIT,
                      "ms_per_step": round(ms_f32x, 4)},
        "roofline": {"bound": "hbm", "kernel": "gemv_lean_kernel Q6_K Q8K_EXACT on the int8 tensor cores + fused argmax (LM head, x quantized in its prologue)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic},
        "gpu_launches": int(launches),
        "clocks": sampler.summary(),
        "e2e": e2e,
        "gemm_prefill": gemm,
        "decode": decode,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.only is None:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        sys.stdout.flush()
        os.write(out_fd, (json.dumps(line) + "\n").encode())
    for it in items:
        it["w"].free()
    if dist:
        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps its peer area while another still sums
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
