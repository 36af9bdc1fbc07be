"""Generate ``reference_drift_9b.json``: how far the reference's own Q8_K
activation quantization moves the hidden state and the logits of the
synthetic 9B-class model, the yardstick of the tensor-parallel decode test.

The reference's forward runs every projection through gemv_quant_q8k
(crates/unltd-tensor/src/quants.rs:474; qwen35_forward.rs). This script runs
the CPU oracle of that forward twice over the same token stream (the Q8_K
run's greedy tokens, teacher-forced into the second run): once as the
reference does, once with every projection through gemv_quant (quants.rs:422,
f64 dots rounded once to f32). Per step it records the max-relative and
normwise (L2) differences of the final hidden state and of the logits. A
sharded run, whose rank-order partial sums move the Q8_K quants now and then,
is held to stay within these differences (tests/test_forward_tp_gpu.py).

Usage: python tests/golden/make_reference_drift.py   (about 10 minutes on 8 cores)
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(REPO, "unltd-inference_b200"), os.path.join(REPO, "oracle")]

import numpy as np  # noqa: E402

import oracle  # noqa: E402
import synth  # noqa: E402

# the configuration of tests/tp_decode_check.py --model 9b
SEED, POSITION, START, STEPS = 2026, 40, 7, 6


def _diff(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b))), float(np.linalg.norm(a - b) / np.linalg.norm(b))


def main() -> None:
    nthreads = os.cpu_count() or 8
    cfg = synth.QWEN35_9B
    tensors = synth.qwen35_model(cfg, SEED)
    st = synth.qwen35_state(cfg, POSITION, SEED + 1)
    oracle.Qwen35Oracle.exact_gemv(False)
    o = oracle.Qwen35Oracle(cfg, tensors, POSITION + STEPS + 4, st, POSITION)
    tok, fed, q8k = START, [], []
    for _ in range(STEPS):
        fed.append(tok)
        lg, hd = o.step(tok, nthreads)
        q8k.append((lg, hd))
        tok = oracle.argmax(lg)
    oracle.Qwen35Oracle.exact_gemv(True)
    try:
        e = oracle.Qwen35Oracle(cfg, tensors, POSITION + STEPS + 4, st, POSITION)
        steps = []
        for i, t in enumerate(fed):
            lg, hd = e.step(t, nthreads)
            hm, hn = _diff(q8k[i][1], hd)
            lm, ln = _diff(q8k[i][0], lg)
            steps.append({"token_in": int(t), "hidden_maxrel": hm, "hidden_normwise": hn,
                          "logits_maxrel": lm, "logits_normwise": ln})
    finally:
        oracle.Qwen35Oracle.exact_gemv(False)
    out = {
        "what": "reference Q8_K forward vs the same forward with gemv_quant projections, teacher-forced",
        "model": "synth.QWEN35_9B", "seed": SEED, "position": POSITION, "start": START, "steps": steps,
    }
    with open(os.path.join(HERE, "reference_drift_9b.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
