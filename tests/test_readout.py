"""Host readout (temperature, softmax, typed answers, confidences) against the
reference's tiny-fixture response (src/lib.rs:734-752, src/schema.rs:145-177)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, TINY


def test_answers_match_upstream_response():
    from decider_gpu import answer, softmax
    ref = json.load(open(os.path.join(TINY, "reference.json")))
    cfg = json.load(open(os.path.join(TINY, "strands_decider_config.json")))
    request = json.load(open(os.path.join(GOLDEN, "request.json")))
    for name, q in request["questions"].items():
        kind = q["type"]
        logits = np.array(ref["probes"][name]["logits"], np.float32)
        t = np.float32(cfg["temperature_by_kind"].get(kind, cfg["temperature"]))
        p = softmax((logits / t).astype(np.float32))
        crit = q["criteria"]
        labels = list(crit.keys()) if kind == "choice" else (
            ["false", "true"] if kind == "noul" else [str(i) for i in range(len(crit))])
        legend = {str(i): v for i, v in enumerate(crit)} if kind == "score" else None
        got = answer(kind, labels, p, cfg["ordinal_smoothing"], legend)
        exp = ref["response"]["answers"][name]
        assert got["type"] == exp["type"]
        for key, val in exp.items():
            if isinstance(val, float):
                assert abs(got[key] - val) < 1e-5, (name, key)
            elif isinstance(val, dict) and key == "probabilities":
                for lab, pv in val.items():
                    assert abs(got[key][lab] - pv) < 1e-5, (name, lab)
            elif key not in ("legend",):
                assert got[key] == val, (name, key)


def test_confidence_measures_distinguish_ordinal_precision_and_choice_certainty():
    # src/lib.rs:867-875
    from decider_gpu import choice_confidence, score_confidence
    assert choice_confidence([0.5, 0.5]) == 0.0
    assert choice_confidence([0.0, 1.0]) == 1.0
    assert score_confidence([0.0, 0.5, 0.5, 0.0], 0.0) > score_confidence([0.5, 0.0, 0.0, 0.5], 0.0)


def test_config_readers_validate_like_the_reference(tmp_path):
    from decider_gpu.host import read_decider_config, read_lora_config, read_text_config
    assert read_decider_config(TINY)["pointer_dim"] == 4
    assert read_lora_config(TINY) == (2, 2.0)
    assert read_text_config(TINY)["hidden_size"] == 8
    bad = dict(json.load(open(os.path.join(TINY, "strands_decider_config.json"))), max_length=5000)
    (tmp_path / "strands_decider_config.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="decision window"):
        read_decider_config(str(tmp_path))
