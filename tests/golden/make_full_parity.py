"""Generates tests/golden/full_2b.json: the CPU oracle's outputs on the
full-size 2B decider (BASELINE configs 2 and 4) for the GPU parity tests.

The oracle (oracle/, a C++ restatement of the reference's CPU path) runs
here once; a 512-token forward takes minutes and the config-4 request (a
3584-token state and 8 questions) much longer, too slow for a test run. The
weights and ids come from tests/model_util.py (seeded numpy streams), so a
test rebuilds the same model and compares against the stored logits and
probabilities. Usage:

    python tests/golden/make_full_parity.py [--threads N]
"""
import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

from model_util import (FULL_POINTER_DIM, FULL_SEED, cfg2_request, cfg4_request, full_model_tensors,  # noqa: E402
                        probabilities, tensor_checksums)
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "full_2b.json")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    args = ap.parse_args()
    O.build()
    O.set_threads(args.threads)
    t0 = time.time()
    c, tensors = full_model_tensors()
    sums = tensor_checksums(tensors)
    m = O.OracleModel(c, tensors, "int8-compute", 32, 2.0)
    del tensors
    print(f"model ready in {time.time() - t0:.0f} s", flush=True)
    out = {"what": "CPU oracle outputs on the 2B decider (24 layers, vocab 248320, LoRA r32, int8-compute)",
           "weights": {"seed": FULL_SEED, "pointer_dim": FULL_POINTER_DIM, "checksums": sums}}
    t0 = time.time()
    ids, opt = cfg2_request(c["vocab_size"])
    hidden = m.forward(ids)
    logits = m.head_logits(hidden, opt)
    out["cfg2"] = {"n": len(ids), "options": opt, "kind": "noul", "logits": [float(x) for x in logits],
                   "probabilities": [float(x) for x in probabilities(logits, "noul")],
                   "answer_row_norm": float(np.linalg.norm(hidden[-1].astype(np.float64)))}
    print(f"cfg2 in {time.time() - t0:.0f} s: {out['cfg2']['probabilities']}", flush=True)
    t0 = time.time()
    state, qs = cfg4_request(c["vocab_size"])
    prefix = m.prefill(state)
    print(f"cfg4 state in {time.time() - t0:.0f} s", flush=True)
    qout = []
    for q, opt, kind in qs:
        rows = m.forward_after(prefix, q)
        lg = m.head_logits(rows, opt)
        qout.append({"kind": kind, "options": opt, "logits": [float(x) for x in lg],
                     "probabilities": [float(x) for x in probabilities(lg, kind)]})
        print(f"  {kind}: {qout[-1]['probabilities']}", flush=True)
    out["cfg4"] = {"state_tokens": len(state), "questions": qout}
    print(f"cfg4 in {time.time() - t0:.0f} s", flush=True)
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
