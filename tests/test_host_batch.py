"""NativeEngine.evaluate_batch (many requests in one dg_logits_batch call)
against NativeEngine.evaluate_encoded request by request (src/lib.rs:477-559),
on a deterministic stand-in for the device model, so the host logic runs on
the CPU: question order, the shared state and the questions that do not
continue it, the token limit, per-request errors, and the readout."""
import json
import os

import numpy as np
import pytest

from conftest import TINY


class FakeModel:
    """Logits that depend only on the full token sequence and the absolute
    position, as the real model's do, so a question scored after a shared
    prefix and the same question scored alone agree."""

    def __init__(self):
        self.lanes = 1
        self.batches = 0

    @staticmethod
    def _score(full, positions):
        for p in positions:
            if p + 1 >= len(full):
                from decider_gpu import DecideError, ErrorKind
                raise DecideError(ErrorKind.ENGINE, "invalid encoding positions or window")
        return np.array([(sum(full[:p + 1]) % 97) / 10.0 + 0.01 * p for p in positions], np.float32)

    def prefill(self, ids):
        return list(ids)

    def logits(self, ids, positions, prefix=None):
        pre = list(prefix) if prefix is not None else []
        return self._score(pre + list(ids), [p + len(pre) for p in positions])

    def logits_batch(self, reqs):
        from decider_gpu import DecideError
        self.batches += 1
        out, status, err = [], np.zeros(len(reqs), np.int32), None
        for i, r in enumerate(reqs):
            state = list(r.get("state", []))
            try:
                out.append([self.logits(ids, pos, state) for ids, pos in r["questions"]])
            except DecideError as e:
                status[i] = 1
                err = err or str(e)
                out.append([np.zeros(len(pos), np.float32) for _, pos in r["questions"]])
        return out, status, np.ones(len(reqs), np.float32), err

    def set_lanes(self, k):
        self.lanes = k


@pytest.fixture()
def engine():
    from decider_gpu import NativeEngine, Precision
    cfg = json.load(open(os.path.join(TINY, "strands_decider_config.json")))
    return NativeEngine(FakeModel(), cfg, Precision.INT8_COMPUTE)


def _q(kind, state, tail, n_opt):
    from decider_gpu import Encoding
    ids = list(state) + list(tail)
    pos = list(range(len(ids) - 1 - n_opt, len(ids) - 1))
    labels = {"noul": ["false", "true"], "choice": ["a", "b", "c", "d"][:n_opt],
              "score": [str(i) for i in range(n_opt)]}[kind]
    legend = {str(i): f"level {i}" for i in range(n_opt)} if kind == "score" else None
    return (kind, labels, Encoding(ids, pos, len(ids) - 1)) + ((legend,) if legend else ())


def _requests():
    rng = np.random.default_rng(3)
    ids = lambda n: [int(x) for x in rng.integers(0, 1000, n)]
    state = ids(50)
    other = ids(50)
    reqs = [
        ({"b_choice": _q("choice", state, ids(12), 4), "a_noul": _q("noul", state, ids(9), 2),
          "c_score": _q("score", state, ids(15), 5)}, 50),
        ({"only": _q("noul", [], ids(30), 2)}, 0),
        # the second question does not continue the first one's state: its own forward
        ({"x": _q("noul", state, ids(8), 2), "y": _q("choice", other, ids(8), 3)}, 50),
        ({"big": _q("noul", [], ids(9000), 2)}, 0),  # over the token limit
    ]
    from decider_gpu import Encoding
    bad = ("noul", ["false", "true"], Encoding(ids(10), [8, 9], 9))  # option at the answer position
    reqs.append(({"bad": bad}, 0))
    return reqs


def test_batch_matches_one_request_at_a_time(engine):
    from decider_gpu import DecideError, ErrorKind
    reqs = _requests()
    engine.set_lanes(2)
    assert engine.model.lanes == 2
    got = engine.evaluate_batch(reqs)
    assert engine.model.batches == 1
    for (questions, state_tokens), g in zip(reqs, got):
        try:
            exp = engine.evaluate_encoded(questions, state_tokens)
        except DecideError as e:
            assert isinstance(g, DecideError) and g.kind == e.kind, (g, e)
            continue
        assert g == exp
    assert isinstance(got[3], DecideError) and got[3].kind == ErrorKind.RESOURCE_LIMIT
    assert isinstance(got[4], DecideError) and got[4].kind == ErrorKind.ENGINE
    assert "invalid encoding positions" in str(got[4])
    assert list(got[0]["answers"]) == ["a_noul", "b_choice", "c_score"]  # name order


def test_batch_of_nothing_and_of_only_refused_requests(engine):
    assert engine.evaluate_batch([]) == []
    from decider_gpu import DecideError
    big = _requests()[3]
    got = engine.evaluate_batch([big])
    assert isinstance(got[0], DecideError) and engine.model.batches == 0
