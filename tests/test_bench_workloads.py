"""Host-side checks of the benchmark's request generators (BASELINE configs
4 and 5): every request is a valid input for dg_logits_batch and the sampled
sizes follow the configs."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402
from decider_gpu.sharding import RequestShape, request_cost, shard_requests  # noqa: E402


def _valid(req, vocab):
    state = req.get("state", [])
    assert len(req["questions"]) >= 1
    for ids, pos in req["questions"]:
        ids = np.asarray(ids)
        assert ids.min() >= 0 and ids.max() < vocab
        assert 2 <= len(pos) <= 5 and max(pos) + 1 < len(ids)  # the answer row is the last token
        assert len(state) + len(ids) <= 4096  # the reference's window


def test_config4_requests():
    state, qs = bench._cfg4_requests(248320, 1000)
    assert len(state) == 3584 and len(qs) == 8
    assert all(len(ids) == 64 and min(pos) >= 48 for ids, pos in qs)  # options in the last 16 tokens
    assert sorted({len(pos) for _, pos in qs}) == [2, 4, 5]  # noul, choice(4), score(5)
    _valid({"state": state, "questions": qs}, 248320)


def test_config5_sample_and_its_sharding():
    reqs, toks, lengths = bench._cfg5_sample(248320, 48)
    assert len(reqs) == 48 and all(128 <= L <= 4096 for L in lengths)
    for r, L, t in zip(reqs, lengths, toks):
        _valid(r, 248320)
        q = len(r["questions"])
        assert 1 <= q <= 4
        assert t == (L if q == 1 else L - 64 + 64 * q)
    # The draw is seeded: the same sample every run.
    again, _, _ = bench._cfg5_sample(248320, 48)
    assert all(np.array_equal(a["questions"][0][0], b["questions"][0][0]) for a, b in zip(reqs, again))
    shapes = [RequestShape(len(r.get("state", ())), tuple(len(q[0]) for q in r["questions"])) for r in reqs]
    plan = shard_requests([request_cost(s) for s in shapes], 8)
    assert sorted(i for p in plan for i in p) == list(range(48))
    per_rank = [sum(toks[i] for i in p) for p in plan]
    assert max(per_rank) < 1.5 * (sum(toks) / 8)
