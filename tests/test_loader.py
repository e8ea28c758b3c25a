"""The library's own checkpoint loader (dg_engine_load / dg_read_checkpoint_config)
against the Python host readers and the reference's validation messages.
The config tests need no device; the tensor-loading tests are marked gpu."""
import json
import os
import shutil

import numpy as np
import pytest

from decider_gpu.engine import read_checkpoint_config_native
from decider_gpu._lib import GpuError
from decider_gpu.host import read_decider_config, read_lora_config, read_text_config

TINY = os.path.join(os.path.dirname(__file__), "golden", "tiny")


def _copy(tmp_path):
    d = tmp_path / "ckpt"
    shutil.copytree(TINY, d)
    return str(d)


def _edit(path, **changes):
    with open(path) as f:
        c = json.load(f)
    for k, v in changes.items():
        if v is None:
            c.pop(k, None)
        else:
            c[k] = v
    with open(path, "w") as f:
        json.dump(c, f)


def test_native_config_matches_the_host_readers():
    got = read_checkpoint_config_native(TINY)
    t = read_text_config(TINY)
    rank, scale = read_lora_config(TINY)
    assert got["hidden_size"] == t["hidden_size"] and got["vocab_size"] == t["vocab_size"]
    assert got["num_hidden_layers"] == t["num_hidden_layers"]
    assert got["layer_types"] == [1 if x == "full_attention" else 0 for x in t["layer_types"]]
    assert got["head_dim"] == t["head_dim"] and got["linear_conv_kernel_dim"] == t["linear_conv_kernel_dim"]
    assert got["rope_theta"] == np.float32(t["rope_parameters"]["rope_theta"])
    assert got["partial_rotary_factor"] == np.float32(t["rope_parameters"]["partial_rotary_factor"])
    assert got["rms_norm_eps"] == np.float32(t["rms_norm_eps"])
    assert got["lora_rank"] == rank and got["lora_scale"] == np.float32(scale)
    assert got["pointer_dim"] == read_decider_config(TINY)["pointer_dim"]


@pytest.mark.parametrize("file,changes,message", [
    ("strands_decider_config.json", {"head_type": "classifier"}, "pointer head"),
    ("strands_decider_config.json", {"force_bos": True}, "default BOS"),
    ("strands_decider_config.json", {"pointer_dim": 0}, "pointer dimension"),
    ("strands_decider_config.json", {"temperature": None}, "calibration"),
    ("strands_decider_config.json", {"ordinal_smoothing": 1.5}, "calibration"),
    ("lora/adapter_config.json", {"r": 0}, "invalid LoRA rank"),
    ("lora/adapter_config.json", {"lora_alpha": -1}, "invalid LoRA alpha"),
    ("lora/adapter_config.json", {"use_dora": True}, "unsupported LoRA adapter"),
    ("base/config.json", {"model_type": "llama"}, "qwen3_5"),
])
def test_native_config_rejects_what_the_reference_rejects(tmp_path, file, changes, message):
    d = _copy(tmp_path)
    _edit(os.path.join(d, file), **changes)
    with pytest.raises(GpuError, match=message):
        read_checkpoint_config_native(d)


def test_native_config_rejects_an_unsupported_activation(tmp_path):
    d = _copy(tmp_path)
    p = os.path.join(d, "base", "config.json")
    with open(p) as f:
        c = json.load(f)
    c["text_config"]["hidden_act"] = "gelu"
    with open(p, "w") as f:
        json.dump(c, f)
    with pytest.raises(GpuError, match="unsupported Qwen"):
        read_checkpoint_config_native(d)


def test_native_config_reports_a_missing_directory(tmp_path):
    with pytest.raises(GpuError, match="cannot read"):
        read_checkpoint_config_native(str(tmp_path / "nowhere"))


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["checkpoint", "int8", "int8-compute", "int4"])
def test_native_loader_matches_the_host_loader(precision):
    from decider_gpu import GpuModel
    ids = [3, 7, 1, 30, 12, 5, 9, 22]
    a = GpuModel.from_dir(TINY, precision, max_tokens=64)
    b = GpuModel.load_native(TINY, precision, max_tokens=64)
    assert np.array_equal(a.forward(ids), b.forward(ids))
    assert np.array_equal(a.logits(ids, [5, 6]), b.logits(ids, [5, 6]))


@pytest.mark.gpu
def test_native_loader_rejects_a_truncated_safetensors_file(tmp_path):
    from decider_gpu import GpuModel
    d = _copy(tmp_path)
    p = os.path.join(d, "head.safetensors")
    with open(p, "rb") as f:
        raw = f.read()
    with open(p, "wb") as f:
        f.write(raw[:-4])
    with pytest.raises(GpuError, match="do not match|length does not match"):
        GpuModel.load_native(d, "checkpoint", max_tokens=64)
