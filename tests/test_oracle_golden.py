"""Pins the CPU oracle to the reference's golden vectors and known answers.

Golden vectors: tests/golden/tiny (the reference's tests/fixtures/tiny,
PyTorch/Transformers FP32 outputs) checked at the reference's own tolerances
(src/lib.rs:705-752). Known answers and properties: src/int8.rs:176-276,
src/tensor.rs:606-803, src/lib.rs:754-832.
"""
import json
import os

import numpy as np
import pytest

from conftest import TINY


@pytest.fixture(scope="module")
def O(oracle_mod):
    return oracle_mod


# --------------------------------------------------------------- src/int8.rs
def test_dot_matches_integer_reference_for_all_block_lengths(O):
    # src/int8.rs:176-193
    for n in range(0, 65):
        a = np.array([(i * 71 + 128) & 0xFF for i in range(n + 1)], np.uint8).view(np.int8)
        b = np.array([(i * 37 + 128) & 0xFF for i in range(n + 1)], np.uint8)
        expected = int(np.sum(a[1:].astype(np.int64) * b[1:].view(np.int8).astype(np.int64)))
        assert O.scalar_dot(a[1:], b[1:]) == expected
    assert O.scalar_dot([-128] * 64, [128] * 64) == 1_048_576
    assert O.scalar_dot([-128] * 64, [127] * 64) == -1_040_384


def test_oversized_blocks_are_rejected(O):
    # src/int8.rs:266-276
    with pytest.raises(O.OracleError):
        O.scalar_dot([1] * 65, [1] * 65)
    with pytest.raises(O.OracleError):
        O.scalar_dot([1] * 16, [1] * 15)


def test_scaled_dot_extreme_known_answer(O):
    # src/int8.rs:238-263: 64*16384*1 + 64*16384*0.25
    s = np.array([1.0, 0.5], np.float32)
    got = O.scaled_dot([-128] * 128, s, [128] * 128, s)
    assert got == np.float32(64.0 * 16384.0 * 1.0 + 64.0 * 16384.0 * 0.25)


# --------------------------------------------------------------- src/tensor.rs
def test_integer_projection_matches_independent_float_reference(O):
    # src/tensor.rs:606-662
    for inp in [1, 15, 16, 17, 63, 64, 65, 131]:
        for rows in [1, 19]:
            output, groups = 31, (inp + 63) // 64
            i = np.arange(rows * inp)
            x = np.where(i < inp, 0.0, ((i * 43 % 255) - 127.0) / 8.0).astype(np.float32)
            x = x.reshape(rows, inp)
            values = ((np.arange(output * inp) * 71 + 128) & 0xFF).astype(np.uint8).reshape(output, inp)
            scales = (((np.arange(output * groups) % 7) + 1) / 32.0).astype(np.float32).reshape(output, groups)
            bias = (np.arange(output) / 16.0).astype(np.float32)
            actual = O.linear_int8_prequant(x, values, scales) + bias  # bias added as the reference does
            q, qs = O.quantize_inputs(x)
            wf = values.view(np.int8).astype(np.float64) * np.repeat(scales, 64, axis=1)[:, :inp]
            xf = q.astype(np.float64) * np.repeat(qs, 64, axis=1)[:, :inp]
            expected = bias.astype(np.float64) + xf @ wf.T
            assert np.all(np.abs(actual - expected) < 1e-3 + np.abs(expected) * 1e-6)


def test_dynamic_quantization_bounds_error_and_rejects_nonfinite(O):
    # src/tensor.rs:769-803
    width = 131
    x = ((np.arange(width * 3) % 79) - 39.0).astype(np.float32) / 11.0
    x[:64] = 0.0
    x[64:128] = np.frombuffer(np.uint32(1).tobytes(), np.float32)[0]
    q, s = O.quantize_inputs(x.reshape(3, width))
    assert s.shape == (3, 3)
    assert np.all(np.isfinite(s)) and np.all(s > 0)
    restored = q.astype(np.float32) * np.repeat(s, 64, axis=1)[:, :width]
    assert np.all(np.abs(restored - x.reshape(3, width)) <= np.repeat(s, 64, axis=1)[:, :width] / 2 + 1e-6)
    for bad in [np.nan, np.inf, -np.inf]:
        assert O.quantize_inputs(np.array([[bad]], np.float32)) is None
        out = O.linear(np.array([[bad]], np.float32), np.array([[1.0]], np.float32), "int8-compute")
        assert not np.isfinite(out[0, 0])


def test_weight_quantization_error_bound(O):
    # src/weights.rs:841-866 (bound: half a step)
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (17, 200)).astype(np.float32)
    w[3, :64] = 0.0
    v, s = O.quantize_weights(w, 8)
    assert s[3, 0] == 1.0
    step = np.repeat(s, 64, axis=1)[:, :200]
    assert np.all(np.abs(v.view(np.int8) * step - w) <= step / 2 + 1e-9)


# --------------------------------------------------------------- tiny golden fixture
@pytest.fixture(scope="module")
def tiny(O):
    return O.OracleModel.from_dir(TINY, "checkpoint")


def test_torso_and_pointer_match_pytorch_fixture(tiny):
    # src/lib.rs:705-732: logits within 1e-5, hidden states within 2e-5
    with open(os.path.join(TINY, "raw-reference.json")) as f:
        cases = json.load(f)
    for case in cases:
        enc = case["encoding"]
        hidden = tiny.forward(enc["input_ids"])
        np.testing.assert_array_less(np.abs(hidden - np.array(case["hidden"], np.float32)), 2e-5)
        logits = tiny.head_logits(hidden, enc["option_positions"])
        np.testing.assert_array_less(np.abs(logits - np.array(case["logits"])), 1e-5)


def test_request_probes_match_upstream_logits(tiny):
    # src/lib.rs:734-752 (the logits part; encodings come from the fixture)
    with open(os.path.join(TINY, "reference.json")) as f:
        ref = json.load(f)
    for name, probe in ref["probes"].items():
        enc = probe["encoding"]
        hidden = tiny.forward(enc["input_ids"])
        logits = tiny.head_logits(hidden, enc["option_positions"])
        np.testing.assert_array_less(np.abs(logits - np.array(probe["logits"])), 1e-5, err_msg=name)


def test_future_tokens_cannot_change_past_hidden_states(tiny):
    # src/lib.rs:754-759
    a = tiny.forward([1, 2, 5, 3, 7, 11])
    b = tiny.forward([1, 2, 5, 3, 9, 10])
    assert np.array_equal(a[:4], b[:4])


@pytest.mark.parametrize("precision", ["checkpoint", "int8", "int8-compute", "int4"])
def test_prefix_cache_reproduces_full_forward_rows_exactly(O, precision):
    # src/lib.rs:796-832
    m = O.OracleModel.from_dir(TINY, precision)
    ids = [(i * 7 + i // 5) % 32 for i in range(140)]
    for total, split in [(2, 1), (7, 2), (6, 5), (40, 3), (75, 70), (75, 10), (140, 64)]:
        full = m.forward(ids[:total])
        prefix = m.prefill(ids[:split])
        assert len(prefix) == split
        rest = m.forward_after(prefix, ids[split:total])
        assert np.array_equal(rest, full[split:]), (precision, split, total)
        assert np.array_equal(m.forward_after(prefix, ids[split:total]), rest)


def test_rejects_out_of_vocabulary_and_overlong_sequences(O, tiny):
    # src/qwen.rs:436-446, src/lib.rs:849
    with pytest.raises(O.OracleError, match="outside vocabulary"):
        tiny.forward([100])
    with pytest.raises(O.OracleError, match="4096 tokens"):
        tiny.forward([])


@pytest.mark.parametrize("precision", ["checkpoint", "int8-compute"])
def test_layer_trace_and_single_layer_restate_the_forward(O, precision):
    """The per-layer residual trace that the GPU per-layer parity test feeds
    in (teacher forcing) is the forward itself: every layer re-run alone on
    its traced input reproduces the next traced rows bit for bit
    (src/qwen.rs:470-494), and the trace starts at the embedded ids."""
    m = O.OracleModel.from_dir(TINY, precision)
    ids = [(i * 11 + 3) % 32 for i in range(23)]
    trace = m.layer_trace(ids)
    assert trace.shape[0] == m.config["num_hidden_layers"] + 1
    for i in range(trace.shape[0] - 1):
        assert np.array_equal(m.layer(i, trace[i]), trace[i + 1]), i
    # Rows with the same id enter the first layer identically.
    assert np.array_equal(trace[0][0], trace[0][ids.index(ids[0], 1)]) if ids.count(ids[0]) > 1 else True
    assert np.isfinite(trace).all()


def test_layer_probe_records_the_projection_inputs(O):
    """The per-layer flipped-code check reads the FP32 inputs of a layer's four
    projection groups from the oracle: the probe's output equals the plain
    layer's, and each recorded input is what its projection consumed (the
    normalised input rows equal rms(x) with the layer's centred weight, and the
    SwiGLU rows are finite and [n][intermediate])."""
    from model_util import random_tensors, small_config
    for lt in ("linear_attention", "full_attention"):
        c = small_config(layer_types=(lt,))
        t = random_tensors(c, rank=32, pointer_dim=0, seed=5)
        m = O.OracleModel(c, t, "int8-compute", 32, 2.0)
        x = np.random.default_rng(1).standard_normal((37, c["hidden_size"])).astype(np.float32)
        out, ins = m.layer_probe(0, x)
        assert np.array_equal(out, m.layer(0, x))
        mixw = c["num_attention_heads"] * c["head_dim"] if lt == "full_attention" else \
            c["linear_num_value_heads"] * c["linear_value_head_dim"]
        assert [a.shape for a in ins] == [(37, c["hidden_size"]), (37, mixw), (37, c["hidden_size"]),
                                          (37, c["intermediate_size"])]
        w = t["layers.0.input_layernorm.weight"][2].astype(np.float64)
        xd = x.astype(np.float64)
        ref = xd / np.sqrt((xd * xd).mean(axis=1, keepdims=True) + 1e-6) * (1 + w)
        assert np.abs(ins[0] - ref).max() < 1e-5 * np.abs(ref).max()
        assert all(np.isfinite(a).all() and np.abs(a).max() > 0 for a in ins)
        assert all(O.quantize_inputs(a) is not None for a in ins)
