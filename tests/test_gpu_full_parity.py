"""End-to-end parity of the full-size 2B decider against the CPU oracle, on
the readout of NativeEngine::evaluate (src/lib.rs:525-548): noul / choice /
score probabilities after temperature and softmax.

The model is BASELINE config 2's shape (24 layers = 6 x [3 Gated DeltaNet +
1 gated GQA attention], hidden 2048, vocab 248320, rank-32 LoRA, pointer head
of 256) with seeded weights (tests/model_util.py: full_model_tensors). The
oracle's outputs on it are committed in tests/golden/full_2b.json
(tests/golden/make_full_parity.py): a 512-token CPU forward takes tens of
seconds and the config-4 request minutes, so they are not recomputed here.

- config 2: one 512-token prompt, one noul question (dg_logits);
- config 4: one request with a 3584-token state and 8 questions of 64 tokens
  (noul, 4-way choice, 5-level score in turn) continuing from the state
  (dg_logits_batch, the throughput form of NativeEngine::evaluate).

Two bars:
- checkpoint precision (FP32 throughout, no quantisation): every probability
  within 1e-3 absolute, the north_star's final bar;
- int8-compute: the forward re-quantises every projection input, so one FP32
  rounding difference anywhere (the reference's glibc expf / log1pf are not
  correctly rounded and cannot be reproduced on a GPU) can flip an int8 code,
  and over 24 layers of random weights flips compound. The oracle itself moves
  its probabilities by up to 1.1e-2 (config 2) and 2.5e-2 (config 4) when its
  input rows are scaled by (1 + 1e-7 N(0, 1)) (the fixture's `noise`
  samples: 6 per config). The bar is 1e-3 or twice the largest such movement
  over the request's questions, whichever is larger, in both arithmetic
  modes: the sensitivity belongs to the request's forward (the questions
  share its state and layers), and a handful of embedding perturbations
  samples it too thinly to bound each question on its own (the GPU's
  differences sit elsewhere: in transcendental functions, sums and int8
  flips inside the layers). Each test prints the per-question error and band.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from model_util import (FULL_POINTER_DIM, cfg2_request, cfg4_request, full_model_tensors, probabilities,
                        tensor_checksums)

pytestmark = pytest.mark.gpu

PROB_TOL = 1e-3  # north_star: final noul / choice / score probabilities within 1e-3 absolute


@pytest.fixture(scope="module")
def full():
    from decider_gpu import GpuModel
    with open(os.path.join(GOLDEN, "full_2b.json")) as f:
        golden = json.load(f)
    c, t = full_model_tensors()
    sums = tensor_checksums(t)
    for name, v in golden["weights"]["checksums"].items():
        # The same seeded stream on both machines; a mismatch is not a parity failure.
        assert abs(sums[name] - v) <= 1e-6 * max(1.0, abs(v)), ("weight stream differs", name, sums[name], v)
    models = {p: GpuModel(c, p, 32, 2.0, FULL_POINTER_DIM, 0, 4096) for p in ("int8-compute", "checkpoint")}
    for name in list(t):
        code, shape, arr = t.pop(name)
        for m in models.values():
            m.set_tensor(name, code, shape, arr)
        del arr
    for m in models.values():
        m.finalize()
    assert models["int8-compute"].fast_path
    return models, golden


def _run(m, which):
    if which == "cfg2":
        ids, opt = cfg2_request()
        return [(probabilities(m.logits(ids, opt), "noul"), "noul")]
    state, qs = cfg4_request()
    got, status, _, err = m.logits_batch([{"state": state, "questions": [(q, opt) for q, opt, _ in qs]}])
    assert not status.any(), err
    return [(probabilities(got[0][i], kind), kind) for i, (_, _, kind) in enumerate(qs)]


def _reference(golden, key, which):
    g = golden[key][which]
    qs = [g] if which == "cfg2" else g["questions"]
    return [np.array(q["probabilities"]) for q in qs]


def _noise_band(golden, which):
    """Largest movement of each question's probabilities in the oracle's own
    perturbed runs."""
    ref = _reference(golden, "int8-compute", which)
    band = np.zeros(len(ref))
    for sample in golden["int8-compute"][which]["noise"]:
        for i, p in enumerate(sample):
            band[i] = max(band[i], float(np.abs(np.array(p) - ref[i]).max()))
    return band


@pytest.mark.parametrize("exact", [True, False], ids=["reference-order", "fma"])
@pytest.mark.parametrize("which", ["cfg2", "cfg4"])
def test_checkpoint_precision_probabilities_within_1e3(full, which, exact):
    """FMA mode puts the FP32-weight projections on the tensor cores (3 x TF32)."""
    models, golden = full
    m = models["checkpoint"]
    m.set_exact(exact)
    got = _run(m, which)
    ref = _reference(golden, "checkpoint", which)
    errs = [float(np.abs(p - r).max()) for (p, _), r in zip(got, ref)]
    print(f"checkpoint {which} ({'reference order' if exact else 'fma'}): max probability error per question "
          f"{['%.2e' % e for e in errs]}")
    assert max(errs) <= PROB_TOL, errs


@pytest.mark.parametrize("exact", [True, False], ids=["reference-order", "fma"])
@pytest.mark.parametrize("which", ["cfg2", "cfg4"])
def test_int8_compute_probabilities_within_the_oracles_own_band(full, which, exact):
    models, golden = full
    m = models["int8-compute"]
    m.set_exact(exact)
    got = _run(m, which)
    ref = _reference(golden, "int8-compute", which)
    band = _noise_band(golden, which)
    errs = np.array([float(np.abs(p - r).max()) for (p, _), r in zip(got, ref)])
    tol = np.full(len(errs), max(PROB_TOL, 2 * float(band.max())))
    print(f"int8-compute {which} ({'reference order' if exact else 'fma'}): probability error per question "
          f"{np.array2string(errs, precision=2)}; the oracle's own 1e-7 band {np.array2string(band, precision=2)}; "
          f"within 1e-3: {int((errs <= PROB_TOL).sum())} of {len(errs)}")
    assert (errs <= tol).all(), (errs, band)
    for (p, kind), r in zip(got, ref):
        if kind == "choice":
            top2 = np.sort(r)[-2:]
            if top2[1] - top2[0] > 2 * float(tol.max()):
                assert int(np.argmax(p)) == int(np.argmax(r)), (p, r)
