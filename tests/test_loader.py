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


# Budgets of the tiny checkpoint (vocab 32, hidden 8, max_length 256), charged
# as WeightBudget::charge does (src/loading.rs:61-80): the embedding [32, 8] is
# 32*8*4 bytes plus 32*ceil(8/64)*4 bytes of possible group scales = 1152; the
# aggregate check counts it twice (2304); the forward workspace for 256 tokens
# is (256*16*16 + 256*2*2 + 2*2*2) floats = 266272 bytes (widest projection
# 16, rotary dim 2, recurrent state 2 x 2 x 2).
@pytest.mark.parametrize("limits,message", [
    ({"max_tensor_bytes": 1151}, "embedding: allocation of 1152 bytes exceeds budget 1151"),
    ({"max_weight_bytes": 2303}, "checkpoint weights and conversion scratch: allocation of 2304 bytes exceeds budget 2303"),
    ({"max_workspace_bytes": 266271}, "forward workspace: allocation of 266272 bytes exceeds budget 266271"),
])
def test_load_limits_refuse_before_any_device_memory(limits, message):
    """NativeEngine::load_with_limits (src/lib.rs:287-367) at the C ABI: the
    reference's budgets and messages, checked before the engine exists (so the
    refusal needs no GPU)."""
    from decider_gpu import GpuModel
    with pytest.raises(GpuError) as e:
        GpuModel.load_native(TINY, "int8-compute", max_tokens=64, limits=limits)
    assert message in str(e.value), str(e.value)


def test_default_load_limits_are_the_references():
    import ctypes as C
    from decider_gpu._lib import LoadLimits, load
    lim = LoadLimits()
    load().dg_load_limits_default(C.byref(lim))
    assert (lim.max_tensor_bytes, lim.max_weight_bytes, lim.max_workspace_bytes) == (2 << 30, 12 << 30, 2 << 30)


def test_load_limits_count_every_checkpoint_tensor(tmp_path):
    """The files' tensors are charged from their headers before any payload is
    read (read_tensors, src/weights.rs:316-325), unsupported extra tensors
    included: an adapter file with one extra [300, 300] tensor passes the
    architecture check but is refused by that tensor's own charge
    (300*300*4 + 300*5*4 = 366000 bytes)."""
    import struct
    from decider_gpu import GpuModel
    d = _copy(tmp_path)
    p = os.path.join(d, "lora", "adapter_model.safetensors")
    with open(p, "rb") as f:
        raw = f.read()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    payload = raw[8 + n:]
    end = max(v["data_offsets"][1] for k, v in header.items() if k != "__metadata__")
    header["extra.weight"] = {"dtype": "F32", "shape": [300, 300], "data_offsets": [end, end + 300 * 300 * 4]}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb + payload[:end] + bytes(300 * 300 * 4))
    with pytest.raises(GpuError) as e:
        GpuModel.load_native(d, "int8-compute", max_tokens=64, limits={"max_tensor_bytes": 100000})
    assert "extra.weight: allocation of 366000 bytes exceeds budget 100000" in str(e.value), str(e.value)
