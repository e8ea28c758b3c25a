"""Generates tests/golden/full_2b.json: the CPU oracle's outputs on the
full-size 2B decider (BASELINE configs 2 and 4) for the GPU parity tests.

The oracle (oracle/, a C++ restatement of the reference's CPU path) runs
here once: a 512-token forward takes tens of seconds on a CPU and the
config-4 request (a 3584-token state and 8 questions) minutes, too slow for a
test run. The weights and ids come from tests/model_util.py (seeded numpy
streams), so a test rebuilds the same model and compares against the stored
probabilities. The file holds:

- int8-compute: config 2 and config 4 probabilities, and the oracle's own
  movement when the embedded input rows are scaled by (1 + 1e-7 N(0, 1))
  (`noise`: a few seeded perturbations). The int8-compute forward re-quantises
  every projection input, so a perturbation far below FP32 rounding flips
  int8 codes that compound over 24 layers: this band is how far the
  reference's own output moves under any reordering of its FP32 work;
- checkpoint precision (no quantisation, FP32 throughout): the same two
  requests, where the 1e-3 probability bar is checked without int8 flips.

Usage:

    python tests/golden/make_full_parity.py [--threads N] [--noise-cfg2 6] [--noise-cfg4 2]
    python tests/golden/make_full_parity.py --add-noise cfg4 --count 4   # more samples
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

from model_util import (FULL_POINTER_DIM, FULL_SEED, NOISE_REL, cfg2_request, cfg4_request,  # noqa: E402
                        full_model_tensors, perturbed_embedding, probabilities, tensor_checksums)
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "full_2b.json")


def run_cfg2(m, c):
    ids, opt = cfg2_request(c["vocab_size"])
    hidden = m.forward(ids)
    logits = m.head_logits(hidden, opt)
    return {"n": len(ids), "options": opt, "kind": "noul", "logits": [float(x) for x in logits],
            "probabilities": [float(x) for x in probabilities(logits, "noul")]}


def run_cfg4(m, c):
    state, qs = cfg4_request(c["vocab_size"])
    prefix = m.prefill(state)
    out = []
    for q, opt, kind in qs:
        lg = m.head_logits(m.forward_after(prefix, q), opt)
        out.append({"kind": kind, "options": opt, "logits": [float(x) for x in lg],
                    "probabilities": [float(x) for x in probabilities(lg, kind)]})
    return {"state_tokens": len(state), "questions": out}


def ids_of(which, c):
    if which == "cfg2":
        return cfg2_request(c["vocab_size"])[0]
    state, qs = cfg4_request(c["vocab_size"])
    return np.concatenate([state] + [q for q, _, _ in qs])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    ap.add_argument("--noise-cfg2", type=int, default=6)
    ap.add_argument("--noise-cfg4", type=int, default=2)
    ap.add_argument("--add-noise", choices=["cfg2", "cfg4"], default=None,
                    help="append --count more perturbed int8-compute samples of one config to the existing file")
    ap.add_argument("--count", type=int, default=4)
    args = ap.parse_args()
    O.build()
    O.set_threads(args.threads)
    c, tensors = full_model_tensors()
    if args.add_noise:
        with open(OUT) as f:
            out = json.load(f)
        which = args.add_noise
        fn = run_cfg2 if which == "cfg2" else run_cfg4
        samples = out["int8-compute"][which]["noise"]
        for k in range(len(samples), len(samples) + args.count):
            t0 = time.time()
            t2 = dict(tensors)
            t2["embed_tokens.weight"] = perturbed_embedding(tensors, ids_of(which, c), seed=100 + k)
            m = O.OracleModel(c, t2, "int8-compute", 32, 2.0)
            r = fn(m, c)
            del m, t2
            samples.append([q["probabilities"] for q in r["questions"]] if which == "cfg4" else [r["probabilities"]])
            print(f"noise {which} {k} in {time.time() - t0:.0f} s", flush=True)
            with open(OUT, "w") as f:
                json.dump(out, f, indent=1)
                f.write("\n")
        return
    out = {"what": "CPU oracle outputs on the 2B decider (24 layers, vocab 248320, LoRA r32)",
           "weights": {"seed": FULL_SEED, "pointer_dim": FULL_POINTER_DIM, "checksums": tensor_checksums(tensors)},
           "noise_rel": NOISE_REL}

    def model(precision, tensors_):
        t0 = time.time()
        m = O.OracleModel(c, tensors_, precision, 32, 2.0)
        print(f"  {precision} model in {time.time() - t0:.0f} s", flush=True)
        return m

    for precision in ("int8-compute", "checkpoint"):
        key = "int8-compute" if precision == "int8-compute" else "checkpoint"
        m = model(precision, tensors)
        res = {}
        for which, fn in (("cfg2", run_cfg2), ("cfg4", run_cfg4)):
            t0 = time.time()
            res[which] = fn(m, c)
            print(f"{precision} {which} in {time.time() - t0:.0f} s", flush=True)
        del m
        out[key] = res
    # The int8-compute oracle's own movement under 1e-7 input noise.
    for which, fn, count in (("cfg2", run_cfg2, args.noise_cfg2), ("cfg4", run_cfg4, args.noise_cfg4)):
        samples = []
        for k in range(count):
            t0 = time.time()
            t2 = dict(tensors)
            t2["embed_tokens.weight"] = perturbed_embedding(tensors, ids_of(which, c), seed=100 + k)
            m = model("int8-compute", t2)
            r = fn(m, c)
            del m, t2
            samples.append([q["probabilities"] for q in r["questions"]] if which == "cfg4" else [r["probabilities"]])
            print(f"noise {which} {k} in {time.time() - t0:.0f} s", flush=True)
        out["int8-compute"][which]["noise"] = samples
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
