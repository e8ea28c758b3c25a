"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of the CPU oracle (liboracle.so).

The oracle is a C++ restatement of decider-engine's CPU prefill path
(src/int8.rs, src/tensor.rs, src/weights.rs, src/qwen.rs, src/lib.rs). Only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may use it, as
the checker and the timed CPU baseline; the product never imports it.

Parity pin: tests/test_oracle_golden.py checks it against the reference's own
golden vectors (tiny fixture, copied by tests/golden/make_golden.py) and the
known-answer tests of src/int8.rs and src/tensor.rs.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

_c = ctypes
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")

PRECISIONS = {"checkpoint": 0, "int8": 1, "int8-compute": 2, "int4": 3}
EPILOGUES = {"write": 0, "add": 1, "swiglu": 2}


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.or_last_error.restype = _c.c_char_p
        L.or_set_threads.argtypes = [_c.c_int]
        L.or_scalar_dot.restype = _c.c_int32
        L.or_scalar_dot.argtypes = [_i8p, _u8p, _c.c_size_t]
        L.or_scaled_dot.restype = _c.c_float
        L.or_scaled_dot.argtypes = [_i8p, _f32p, _u8p, _f32p, _c.c_size_t]
        L.or_dot_scores.restype = _c.c_float
        L.or_dot_scores.argtypes = [_f32p, _f32p, _c.c_size_t]
        L.or_softmax.argtypes = [_f32p, _c.c_size_t]
        L.or_quantize_inputs.restype = _c.c_int
        L.or_quantize_inputs.argtypes = [_f32p, _c.c_size_t, _c.c_size_t, _i8p, _f32p]
        L.or_quantize_weights.argtypes = [_f32p, _c.c_size_t, _c.c_size_t, _c.c_int, _u8p, _f32p]
        L.or_linear.restype = _c.c_int
        L.or_linear.argtypes = [_f32p, _c.c_size_t, _c.c_size_t, _f32p, _c.c_size_t, _c.c_int,
                                _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t, _c.c_float,
                                _c.c_int, _f32p]
        L.or_linear_int8_prequant.argtypes = [_f32p, _c.c_size_t, _c.c_size_t, _u8p, _f32p,
                                              _c.c_size_t, _f32p]
        L.or_model_new.restype = _c.c_void_p
        L.or_model_new.argtypes = [_c.c_void_p, _c.c_void_p, _c.c_void_p]
        L.or_model_set.argtypes = [_c.c_void_p, _c.c_char_p, _c.c_int, _c.c_void_p, _c.c_int,
                                   _c.c_void_p]
        L.or_model_build.restype = _c.c_int
        L.or_model_build.argtypes = [_c.c_void_p, _c.c_int, _c.c_size_t, _c.c_float]
        L.or_model_free.argtypes = [_c.c_void_p]
        L.or_prefix_free.argtypes = [_c.c_void_p]
        L.or_prefix_len.restype = _c.c_size_t
        L.or_prefix_len.argtypes = [_c.c_void_p]
        L.or_forward.restype = _c.c_int
        L.or_forward.argtypes = [_c.c_void_p, _u32p, _c.c_size_t, _c.c_void_p, _c.c_int,
                                 _c.c_void_p, _c.POINTER(_c.c_void_p)]
        L.or_head_logits.restype = _c.c_int
        L.or_forward_trace.argtypes = [_c.c_void_p, _u32p, _c.c_size_t, _c.c_void_p]
        L.or_layer.argtypes = [_c.c_void_p, _c.c_int, _f32p, _c.c_size_t, _f32p]
        L.or_head_logits.argtypes = [_c.c_void_p, _f32p, _c.c_size_t, _c.c_void_p, _c.c_size_t,
                                     _f32p]
        L.or_layer_probe.restype = _c.c_int
        L.or_layer_probe.argtypes = [_c.c_void_p, _c.c_int, _f32p, _c.c_size_t, _f32p, _f32p, _f32p,
                                     _f32p, _f32p]
        L.or_gated_delta_rule.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _c.c_size_t,
                                          _c.c_size_t, _c.c_size_t, _f32p, _f32p]
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


def _err():
    return OracleError(lib().or_last_error().decode("utf-8", "replace"))


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def scalar_dot(a, b) -> int:
    a = np.ascontiguousarray(a, np.int8)
    b = np.ascontiguousarray(np.asarray(b).astype(np.int64) & 0xFF, np.uint8)
    if len(a) != len(b) or len(a) > 64:
        raise OracleError("dot needs equal lengths of at most 64")
    return int(lib().or_scalar_dot(a, b, len(a)))


def scaled_dot(x, xs, w, ws) -> np.float32:
    x = np.ascontiguousarray(x, np.int8)
    w = np.ascontiguousarray(np.asarray(w).astype(np.int64) & 0xFF, np.uint8)
    return np.float32(lib().or_scaled_dot(x, np.ascontiguousarray(xs, np.float32), w,
                                          np.ascontiguousarray(ws, np.float32), len(x)))


def dot_scores(a, b) -> np.float32:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return np.float32(lib().or_dot_scores(a, b, len(a)))


def softmax(v) -> np.ndarray:
    v = np.array(v, np.float32)
    lib().or_softmax(v, len(v))
    return v


def quantize_inputs(x: np.ndarray):
    """QuantizedInputs::new on [rows, width]; None if any input is non-finite."""
    x = np.ascontiguousarray(x, np.float32)
    rows, width = x.shape
    groups = (width + 63) // 64
    q = np.zeros((rows, width), np.int8)
    s = np.zeros((rows, groups), np.float32)
    if not lib().or_quantize_inputs(x, rows, width, q, s):
        return None
    return q, s


def quantize_weights(w: np.ndarray, bits: int = 8):
    """Data::quantize of an F32 [rows, width] tensor (values as u8, scales)."""
    w = np.ascontiguousarray(w, np.float32)
    rows, width = w.shape
    groups = (width + 63) // 64
    n = rows * width if bits == 8 else (rows * width + 1) // 2
    v = np.zeros(n, np.uint8)
    s = np.zeros((rows, groups), np.float32)
    lib().or_quantize_weights(w, rows, width, bits, v, s)
    return (v.reshape(rows, width) if bits == 8 else v), s


def _ptr(a):
    return None if a is None else a.ctypes.data


def linear(x, w, precision="int8-compute", bias=None, lora_a=None, lora_b=None, scale=0.0,
           epilogue="write", out=None) -> np.ndarray:
    """Linear::apply_into on one projection (weights F32 [output, input])."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    rows, inp = x.shape
    output = w.shape[0]
    bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
    la = None if lora_a is None else np.ascontiguousarray(lora_a, np.float32)
    lb = None if lora_b is None else np.ascontiguousarray(lora_b, np.float32)
    rank = 0 if la is None else la.shape[0]
    res = np.zeros((rows, output), np.float32) if out is None else np.array(out, np.float32)
    if lib().or_linear(x, rows, inp, w, output, PRECISIONS[precision], _ptr(bias), _ptr(la),
                       _ptr(lb), rank, float(scale), EPILOGUES[epilogue], res):
        raise _err()
    return res


def linear_int8_prequant(x, wq, ws) -> np.ndarray:
    """linear_int8 column sums over pre-quantized weights (no bias, no LoRA)."""
    x = np.ascontiguousarray(x, np.float32)
    wq = np.ascontiguousarray(np.asarray(wq).view(np.uint8) if np.asarray(wq).dtype == np.int8
                              else wq, np.uint8)
    rows, inp = x.shape
    out = np.zeros((rows, wq.shape[0]), np.float32)
    lib().or_linear_int8_prequant(x, rows, inp, wq, np.ascontiguousarray(ws, np.float32),
                                  wq.shape[0], out)
    return out


def gated_delta_rule(q, k, v, g, beta, state=None):
    """Gated delta rule recurrence for one (sequence, head): returns (o, state)."""
    n, dk = q.shape
    dv = v.shape[1]
    st = np.zeros((dk, dv), np.float32) if state is None else np.array(state, np.float32)
    o = np.zeros((n, dv), np.float32)
    lib().or_gated_delta_rule(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
                              np.ascontiguousarray(v, np.float32), np.ascontiguousarray(g, np.float32),
                              np.ascontiguousarray(beta, np.float32), n, dk, dv, st, o)
    return o, st


# ----------------------------------------------------------------- safetensors
_DT = {"F32": (np.float32, 0), "BF16": (np.uint16, 1), "F16": (np.uint16, 2)}


def read_safetensors(path):
    """Minimal safetensors reader: {name: (dtype_code, shape, ndarray)}."""
    with open(path, "rb") as f:
        raw = f.read()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    out = {}
    base = 8 + n
    for name, info in header.items():
        if name == "__metadata__":
            continue
        np_dt, code = _DT[info["dtype"]]
        lo, hi = info["data_offsets"]
        arr = np.frombuffer(raw[base + lo:base + hi], dtype=np_dt).copy()
        out[name] = (code, list(info["shape"]), arr)
    return out


class OracleModel:
    """Model::load + Head::load from a directory in the reference's layout
    (src/lib.rs:287-367), or from in-memory tensors."""

    def __init__(self, config: dict, tensors: dict, precision="int8-compute", rank=None,
                 scale=None):
        L = lib()
        c = config
        dims = np.array([c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"],
                         c["vocab_size"], c["num_attention_heads"], c["num_key_value_heads"],
                         c["head_dim"], c["linear_conv_kernel_dim"], c["linear_key_head_dim"],
                         c["linear_value_head_dim"], c["linear_num_key_heads"],
                         c["linear_num_value_heads"]], np.int64)
        rp = c["rope_parameters"]
        fl = np.array([c["rms_norm_eps"], rp["rope_theta"], rp["partial_rotary_factor"]], np.float32)
        lt = np.array([1 if t == "full_attention" else 0 for t in c["layer_types"]], np.int32)
        self.config = c
        self.h = L.or_model_new(dims.ctypes.data, fl.ctypes.data, lt.ctypes.data)
        for name, (code, shape, arr) in tensors.items():
            arr = np.ascontiguousarray(arr)
            shp = np.array(shape, np.int64)
            L.or_model_set(self.h, name.encode(), code, shp.ctypes.data, len(shape), arr.ctypes.data)
        if L.or_model_build(self.h, PRECISIONS[precision], int(rank), float(scale)):
            raise _err()

    @classmethod
    def from_dir(cls, d, precision="checkpoint"):
        with open(os.path.join(d, "base", "config.json")) as f:
            cfg = json.load(f)["text_config"]
        with open(os.path.join(d, "lora", "adapter_config.json")) as f:
            ad = json.load(f)
        rank = int(ad["r"])
        scale = np.float32(np.float32(ad["lora_alpha"]) / np.float32(rank))
        tensors = {}
        prefix = "model.language_model."
        for k, v in read_safetensors(os.path.join(d, "base", "model.safetensors")).items():
            if k.startswith(prefix):
                tensors[k[len(prefix):]] = v
        tensors.update(read_safetensors(os.path.join(d, "lora", "adapter_model.safetensors")))
        for k, v in read_safetensors(os.path.join(d, "head.safetensors")).items():
            tensors["head." + k] = v
        return cls(cfg, tensors, precision, rank, scale)

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_model_free(self.h)
            self.h = None

    def _run(self, ids, past=None, capture=False, want_hidden=True):
        ids = np.ascontiguousarray(ids, np.uint32)
        n = len(ids)
        hidden = np.zeros((n, self.config["hidden_size"]), np.float32) if want_hidden else None
        pref = ctypes.c_void_p()
        rc = lib().or_forward(self.h, ids, n, None if past is None else past.h, int(capture),
                              None if hidden is None else hidden.ctypes.data, ctypes.byref(pref))
        if rc:
            raise _err()
        return hidden, (OraclePrefix(pref.value) if capture else None)

    def forward(self, ids):
        return self._run(ids)[0]

    def prefill(self, ids):
        return self._run(ids, capture=True, want_hidden=False)[1]

    def forward_after(self, prefix, ids):
        return self._run(ids, past=prefix)[0]

    def layer_trace(self, ids):
        """Residual rows through the layer loop of Model::run: [layers + 1][n][hidden],
        the embedded input and then each layer's output (before the final norm)."""
        ids = np.ascontiguousarray(ids, np.uint32)
        c = self.config
        out = np.zeros((c["num_hidden_layers"] + 1, len(ids), c["hidden_size"]), np.float32)
        if lib().or_forward_trace(self.h, ids, len(ids), out.ctypes.data):
            raise _err()
        return out

    def layer(self, index, x):
        """One layer teacher-forced on residual rows x [n][hidden] (positions 0..n-1)."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        if lib().or_layer(self.h, int(index), x, x.shape[0], out):
            raise _err()
        return out

    def layer_probe(self, index, x):
        """`layer`, also returning the FP32 inputs of the layer's four projection
        groups: (out, [input norm, mixer output, post norm, SwiGLU rows])."""
        x = np.ascontiguousarray(x, np.float32)
        c = self.config
        n = x.shape[0]
        full = c["layer_types"][index] == "full_attention"
        mixw = (c["num_attention_heads"] * c["head_dim"] if full
                else c["linear_num_value_heads"] * c["linear_value_head_dim"])
        out = np.zeros_like(x)
        ins = [np.zeros((n, w), np.float32) for w in (c["hidden_size"], mixw, c["hidden_size"],
                                                      c["intermediate_size"])]
        if lib().or_layer_probe(self.h, int(index), x, n, out, *ins):
            raise _err()
        return out, ins

    def head_logits(self, hidden, positions):
        hidden = np.ascontiguousarray(hidden, np.float32)
        pos = np.ascontiguousarray(positions, np.uint64)
        out = np.zeros(len(pos), np.float32)
        if lib().or_head_logits(self.h, hidden, hidden.shape[0], pos.ctypes.data, len(pos), out):
            raise _err()
        return out


class OraclePrefix:
    def __init__(self, h):
        self.h = h

    def __len__(self):
        return int(lib().or_prefix_len(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_prefix_free(self.h)
            self.h = None
