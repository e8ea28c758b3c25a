"""Python host mirror of the reference's model seam over the C ABI.

`GpuModel` stands where qwen::Model + Head stand in the reference
(src/qwen.rs:291-424, src/lib.rs:87-131): `forward`, `prefill`,
`forward_after` and `logits` run on the B200 through libdecider_gpu.so.
`Linear` is the isolated INT8 projection and
`gated_delta_rule` the isolated recurrence (config 3).
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct

import numpy as np

from ._lib import GpuError, ModelConfig, check, load

PRECISIONS = {"checkpoint": 0, "int8": 1, "int8-compute": 2, "int4": 3}
_DT = {"F32": (np.float32, 0), "BF16": (np.uint16, 1), "F16": (np.uint16, 2)}


def _u32(a):
    a = np.ascontiguousarray(a, np.uint32)
    return a, a.ctypes.data


def read_safetensors(path: str) -> dict:
    """Safetensors reader (header bound and length check as read_tensors,
    src/weights.rs:305-318): {name: (dtype_code, shape, ndarray)}."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        raw = f.read()
    n = struct.unpack("<Q", raw[:8])[0]
    if n > 16 * 1024 * 1024 or n + 8 > size:
        raise GpuError("invalid or oversized safetensors header")
    header = json.loads(raw[8:8 + n])
    out, base, data_len = {}, 8 + n, 0
    for name, info in header.items():
        if name == "__metadata__":
            continue
        if info["dtype"] not in _DT:
            raise GpuError(f"{name}: unsupported weight dtype {info['dtype']}")
        np_dt, code = _DT[info["dtype"]]
        lo, hi = info["data_offsets"]
        data_len = max(data_len, hi)
        out[name] = (code, list(info["shape"]), np.frombuffer(raw[base + lo:base + hi], dtype=np_dt))
    if base + data_len != size:
        raise GpuError("safetensors file length does not match metadata")
    return out


def text_config_to_struct(cfg: dict, rank: int, scale: float, pointer_dim: int):
    lt = (C.c_int32 * len(cfg["layer_types"]))(
        *[1 if t == "full_attention" else 0 for t in cfg["layer_types"]])
    rp = cfg["rope_parameters"]
    s = ModelConfig(
        cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["vocab_size"],
        cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"],
        cfg["linear_conv_kernel_dim"], cfg["linear_key_head_dim"], cfg["linear_value_head_dim"],
        cfg["linear_num_key_heads"], cfg["linear_num_value_heads"], cfg["rms_norm_eps"],
        rp["rope_theta"], rp["partial_rotary_factor"], C.cast(lt, C.POINTER(C.c_int32)),
        rank, scale, pointer_dim)
    return s, lt


def read_checkpoint_config_native(d: str) -> dict:
    """The library's own reading of a checkpoint's configs (dg_read_checkpoint_config,
    no device needed), as a dict of the dg_model_config fields."""
    s = ModelConfig()
    lt = (C.c_int32 * 4096)()
    check(load().dg_read_checkpoint_config(d.encode(), C.byref(s), lt, 4096))
    out = {name: getattr(s, name) for name, _ in ModelConfig._fields_ if name != "layer_types"}
    out["layer_types"] = [int(lt[i]) for i in range(s.num_hidden_layers)]
    return out


class _Question(C.Structure):
    _fields_ = [("ids", C.c_void_p), ("n", C.c_size_t), ("opt_pos", C.c_void_p), ("n_opt", C.c_size_t)]


class _Request(C.Structure):
    _fields_ = [("past", C.c_void_p), ("state_ids", C.c_void_p), ("n_state", C.c_size_t),
                ("questions", C.c_void_p), ("n_questions", C.c_size_t)]


class GpuPrefix:
    """Device-resident, immutable prefix cache (Prefix, src/qwen.rs:509-526)."""

    def __init__(self, model: "GpuModel", handle: int):
        self._model = model
        self.h = handle

    def __len__(self):
        return int(load().dg_prefix_len(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            load().dg_prefix_free(self.h)
            self.h = None


class GpuModel:
    """Qwen3.5 torso + pointer head resident on one B200."""

    def __init__(self, text_config: dict, precision: str = "int8-compute", rank: int = 32,
                 lora_scale: float = 2.0, pointer_dim: int = 0, device: int = 0, max_tokens: int = 4096):
        L = load()
        self.config = dict(text_config)
        self.precision = precision
        self.pointer_dim = pointer_dim
        s, self._lt = text_config_to_struct(text_config, rank, lora_scale, pointer_dim)
        h = C.c_void_p()
        check(L.dg_engine_create(C.byref(s), PRECISIONS[precision], device, max_tokens, C.byref(h)))
        self.h = h.value
        self.hidden = text_config["hidden_size"]

    def set_tensor(self, name: str, dtype: int, shape, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        shp = (C.c_int64 * len(shape))(*shape)
        check(load().dg_engine_set_tensor(self.h, name.encode(), dtype, shp, len(shape), data.ctypes.data))

    def set_tensors(self, tensors: dict) -> None:
        for name, (code, shape, arr) in tensors.items():
            self.set_tensor(name, code, shape, arr)

    def fill_synthetic(self, seed: int = 0, stddev: float = 0.02) -> None:
        check(load().dg_engine_fill_synthetic(self.h, seed, stddev))

    def finalize(self) -> "GpuModel":
        check(load().dg_engine_finalize(self.h))
        return self

    def sibling(self) -> "GpuModel":
        """A second engine on this one's device that reads this one's weights
        (dg_engine_create_sibling): its own stream and buffers, so the two
        can serve requests concurrently from different host threads."""
        h = C.c_void_p()
        check(load().dg_engine_create_sibling(self.h, C.byref(h)))
        m = GpuModel.__new__(GpuModel)
        m.config, m.precision, m.pointer_dim, m._lt = self.config, self.precision, self.pointer_dim, self._lt
        m.hidden = self.hidden
        m.h = h.value
        return m

    def set_lanes(self, lanes: int) -> None:
        """Concurrent lanes of logits_batch (dg_engine_set_lanes): the batch's
        requests are dealt to `lanes` engines sharing these weights, each run
        from its own host thread."""
        check(load().dg_engine_set_lanes(self.h, int(lanes)))

    @property
    def lanes(self) -> int:
        return int(load().dg_engine_lanes(self.h))

    def last_batch_ms(self) -> float:
        """Device time of the last logits_batch call, first kernel to the end of its last lane."""
        return float(load().dg_engine_last_batch_ms(self.h))

    @property
    def fast_path(self) -> bool:
        return bool(load().dg_engine_fast_path(self.h))

    def set_exact(self, exact: bool) -> None:
        check(load().dg_engine_set_exact(self.h, int(exact)))

    def gemm_timing(self, enable: bool) -> None:
        """Bracket every tcgen05 projection launch with CUDA events (resets the totals)."""
        check(load().dg_engine_gemm_timing(self.h, int(enable)))

    def gemm_timing_layers(self, first_layer: int, layers: int) -> None:
        """Events around the projections of layers [first_layer, first_layer + layers) only."""
        check(load().dg_engine_gemm_timing_layers(self.h, int(first_layer), int(layers)))

    def gemm_time_all(self):
        """(summed 2*M*N*K ops, launches) of every projection of the timed forwards."""
        ops, n = C.c_double(), C.c_uint64()
        check(load().dg_engine_gemm_time_all(self.h, C.byref(ops), C.byref(n)))
        return ops.value, n.value

    def gemm_time(self):
        """(summed launch ms, summed 2*M*N*K ops, launches) since gemm_timing()."""
        ms, ops, n = C.c_double(), C.c_double(), C.c_uint64()
        check(load().dg_engine_gemm_time(self.h, C.byref(ms), C.byref(ops), C.byref(n)))
        return ms.value, ops.value, n.value

    def __del__(self):
        if getattr(self, "h", None):
            load().dg_engine_free(self.h)
            self.h = None

    # ---- Model::forward / prefill / forward_after
    def forward(self, ids, prefix: GpuPrefix | None = None) -> np.ndarray:
        ids, p = _u32(ids)
        out = np.zeros((len(ids), self.hidden), np.float32)
        check(load().dg_forward_hidden(self.h, None if prefix is None else prefix.h, p, len(ids),
                                       out.ctypes.data))
        return out

    def forward_segments(self, seqs, prefix: GpuPrefix | None = None) -> np.ndarray:
        """Several equal-length sequences continuing `prefix`, as one forward
        (dg_forward_segments_hidden): returns [len(seqs)][seg_len][hidden]."""
        seqs = [np.asarray(q) for q in seqs]
        n = len(seqs[0])
        assert all(len(q) == n for q in seqs), "sequences must have one length"
        ids, p = _u32(np.concatenate(seqs))
        out = np.zeros((len(seqs) * n, self.hidden), np.float32)
        check(load().dg_forward_segments_hidden(self.h, None if prefix is None else prefix.h, p, n, len(seqs),
                                                out.ctypes.data))
        return out.reshape(len(seqs), n, self.hidden)

    def prefill(self, ids) -> GpuPrefix:
        ids, p = _u32(ids)
        h = C.c_void_p()
        check(load().dg_prefill(self.h, p, len(ids), C.byref(h)))
        return GpuPrefix(self, h.value)

    def forward_after(self, prefix: GpuPrefix, ids) -> np.ndarray:
        return self.forward(ids, prefix)

    # ---- NativeEngine::logits (src/lib.rs:400-419)
    def logits(self, ids, positions, prefix: GpuPrefix | None = None) -> np.ndarray:
        ids, p = _u32(ids)
        pos = np.ascontiguousarray(positions, np.uint64)
        out = np.zeros(len(pos), np.float32)
        check(load().dg_logits(self.h, None if prefix is None else prefix.h, p, len(ids), pos.ctypes.data,
                               len(pos), out.ctypes.data))
        return out

    def layer(self, index: int, x: np.ndarray) -> np.ndarray:
        """One decoder layer teacher-forced on residual rows x [n][hidden]
        (positions 0..n-1, no prefix): dg_debug_layer."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        check(load().dg_debug_layer(self.h, int(index), x.ctypes.data, x.shape[0], out.ctypes.data))
        return out

    def layer_codes(self, index: int, x: np.ndarray):
        """`layer`, also returning the int8 codes of the layer's four quantised
        projection inputs: (out, [input norm, mixer output, post norm, SwiGLU
        rows]) (dg_debug_layer_codes)."""
        x = np.ascontiguousarray(x, np.float32)
        c = self.config
        n = x.shape[0]
        full = c["layer_types"][index] == "full_attention"
        mixw = (c["num_attention_heads"] * c["head_dim"] if full
                else c["linear_num_value_heads"] * c["linear_value_head_dim"])
        widths = (c["hidden_size"], mixw, c["hidden_size"], c["intermediate_size"])
        out = np.zeros_like(x)
        codes = np.zeros(n * sum(widths), np.int8)
        check(load().dg_debug_layer_codes(self.h, int(index), x.ctypes.data, n, out.ctypes.data,
                                          codes.ctypes.data))
        blocks, off = [], 0
        for w in widths:
            blocks.append(codes[off:off + n * w].reshape(n, w))
            off += n * w
        return out, blocks

    # ---- batched requests (dg_logits_batch): the throughput form of
    # NativeEngine::evaluate (src/lib.rs:477-559)
    def logits_batch(self, requests):
        """requests: dicts with `questions` [(ids, option_positions), ...] and
        optionally `state` (ids prefilled once and shared by the questions) or
        `past` (a GpuPrefix). Returns (logits per request: a list of arrays per
        question, status per request (0 ok), device ms per request, first error
        message or None)."""
        keep = []
        reqs = (_Request * max(1, len(requests)))()
        sizes = []
        for r, q in enumerate(requests):
            qs = (_Question * len(q["questions"]))()
            sz = []
            for i, (ids, pos) in enumerate(q["questions"]):
                ids, p = _u32(ids)
                pos = np.ascontiguousarray(pos, np.uint64)
                keep += [ids, pos]
                qs[i].ids, qs[i].n, qs[i].opt_pos, qs[i].n_opt = p, len(ids), pos.ctypes.data, len(pos)
                sz.append(len(pos))
            keep.append(qs)
            sizes.append(sz)
            reqs[r].questions, reqs[r].n_questions = C.cast(qs, C.c_void_p), len(qs)
            past = q.get("past")
            reqs[r].past = None if past is None else past.h
            state = q.get("state")
            if state is not None and len(state):
                st, sp = _u32(state)
                keep.append(st)
                reqs[r].state_ids, reqs[r].n_state = sp, len(st)
        total = sum(sum(sz) for sz in sizes)
        out = np.zeros(max(1, total), np.float32)
        status = np.zeros(max(1, len(requests)), np.int32)
        ms = np.zeros(max(1, len(requests)), np.float32)
        rc = load().dg_logits_batch(self.h, C.cast(reqs, C.c_void_p), len(requests), out.ctypes.data, status.ctypes.data, ms.ctypes.data)
        err = load().dg_last_error().decode() if rc else None
        res, o = [], 0
        for sz in sizes:
            per = []
            for k in sz:
                per.append(out[o:o + k].copy())
                o += k
            res.append(per)
        return res, status[:len(requests)].copy(), ms[:len(requests)].copy(), err

    @classmethod
    def load_native(cls, d: str, precision: str = "checkpoint", device: int = 0, max_tokens: int = 4096,
                    limits: dict | None = None):
        """`from_dir` through the library's own checkpoint loader
        (dg_engine_load_with_limits): the C ABI reads the configs and the
        safetensors files itself. `limits` (NativeEngine::load_with_limits,
        src/lib.rs:287-367) maps max_tensor_bytes / max_weight_bytes /
        max_workspace_bytes to byte budgets; missing keys keep the defaults."""
        from ._lib import LoadLimits
        from .host import read_decider_config, read_text_config
        m = cls.__new__(cls)
        m.config = dict(read_text_config(d))
        m.precision = precision
        m.pointer_dim = read_decider_config(d)["pointer_dim"]
        m.hidden = m.config["hidden_size"]
        lim = LoadLimits()
        load().dg_load_limits_default(C.byref(lim))
        for k, v in (limits or {}).items():
            setattr(lim, k, int(v))
        h = C.c_void_p()
        m.h = None
        check(load().dg_engine_load_with_limits(d.encode(), PRECISIONS[precision], C.byref(lim), device, max_tokens,
                                                C.byref(h)))
        m.h = h.value
        return m

    @classmethod
    def from_dir(cls, d: str, precision: str = "checkpoint", device: int = 0, max_tokens: int = 4096):
        """Model::load + Head::load from a checkpoint directory in the
        reference's layout (src/lib.rs:287-367): base/config.json,
        base/model.safetensors, lora/adapter_config.json,
        lora/adapter_model.safetensors, head.safetensors and
        strands_decider_config.json."""
        from .host import read_decider_config, read_lora_config, read_text_config
        dc = read_decider_config(d)
        cfg = read_text_config(d)
        rank, scale = read_lora_config(d)
        m = cls(cfg, precision, rank, scale, dc["pointer_dim"], device, max_tokens)
        prefix = "model.language_model."
        base = read_safetensors(os.path.join(d, "base", "model.safetensors"))
        m.set_tensors({k[len(prefix):]: v for k, v in base.items() if k.startswith(prefix)})
        adapter = read_safetensors(os.path.join(d, "lora", "adapter_model.safetensors"))
        if not adapter:
            raise GpuError("empty LoRA adapter")
        m.set_tensors(adapter)
        m.set_tensors({"head." + k: v for k, v in read_safetensors(os.path.join(d, "head.safetensors")).items()})
        return m.finalize()


class Linear:
    """Isolated group-64 INT8 projection with optional rank-32 LoRA (config 1)."""

    def __init__(self, w: np.ndarray, lora_a=None, lora_b=None, lora_scale: float = 0.0, device: int = 0):
        w = np.ascontiguousarray(w, np.float32)
        self.n, self.k = w.shape
        la = None if lora_a is None else np.ascontiguousarray(lora_a, np.float32)
        lb = None if lora_b is None else np.ascontiguousarray(lora_b, np.float32)
        rank = 0 if la is None else la.shape[0]
        h = C.c_void_p()
        check(load().dg_linear_create(w.ctypes.data, self.n, self.k, None if la is None else la.ctypes.data,
                                      None if lb is None else lb.ctypes.data, rank, lora_scale, device,
                                      C.byref(h)))
        self.h = h.value

    def set_exact(self, exact: bool) -> None:
        check(load().dg_linear_set_exact(self.h, int(exact)))

    def __call__(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros((x.shape[0], self.n), np.float32)
        check(load().dg_linear_forward(self.h, x.ctypes.data, x.shape[0], y.ctypes.data))
        return y

    def forward_device(self, x_ptr: int, m: int, y_ptr: int, dots_ptr: int | None = None) -> None:
        check(load().dg_linear_forward_device(self.h, x_ptr, m, y_ptr, dots_ptr))

    def forward_device_noalloc(self, x_ptr: int, m: int, y_ptr: int) -> None:
        """`forward_device` without any device allocation: the per-call scratch
        is a fixed 8 MiB static area per device (rows beyond it are rejected).
        Calls on one device must not overlap in time; the first call on a
        device should come before any stream capture begins."""
        check(load().dg_linear_forward_device_noalloc(self.h, x_ptr, m, y_ptr))

    def last_times(self):
        """(total_ms, gemm_ms) of the last forward: device time from the
        activation quantiser to the end of the projection, and of the
        projection kernel alone (CUDA events on the handle's stream)."""
        t, g = C.c_float(), C.c_float()
        check(load().dg_linear_last_times(self.h, C.byref(t), C.byref(g)))
        return t.value, g.value

    def stream(self) -> int:
        return int(load().dg_linear_stream(self.h) or 0)

    def last_quantized(self, m: int):
        xq = np.zeros((m, self.k), np.int8)
        xs = np.zeros((self.k // 64, m), np.float32)
        check(load().dg_linear_last_quantized(self.h, m, xq.ctypes.data, xs.ctypes.data))
        return xq, xs

    def __del__(self):
        if getattr(self, "h", None):
            load().dg_linear_free(self.h)
            self.h = None


def gated_delta_rule(q_ptr, k_ptr, v_ptr, g_ptr, beta_ptr, batch, t, heads, state_ptr, o_ptr, stream=0):
    """Isolated gated delta rule on device buffers (config 3); see
    dg_gated_delta_rule_device in include/decider_gpu.h."""
    check(load().dg_gated_delta_rule_device(q_ptr, k_ptr, v_ptr, g_ptr, beta_ptr, batch, t, heads, state_ptr,
                                            o_ptr, stream))


def gated_delta_chunk_workspace_bytes(batch, t, heads) -> int:
    return int(load().dg_gated_delta_chunk_workspace_bytes(batch, t, heads))


def gated_delta_rule_chunked(q_ptr, k_ptr, v_ptr, g_ptr, beta_ptr, batch, t, heads, state_ptr, o_ptr, ws_ptr,
                             ws_bytes, stream=0):
    """Chunked form of `gated_delta_rule` with a caller-owned device workspace."""
    check(load().dg_gated_delta_rule_chunked_device(q_ptr, k_ptr, v_ptr, g_ptr, beta_ptr, batch, t, heads,
                                                    state_ptr, o_ptr, ws_ptr, ws_bytes, stream))


def measure_i8_peak(device: int = 0, iters: int = 1 << 16):
    """(TOP/s, ms) of the dense tcgen05 kind::i8 probe on `device`
    (dg_measure_i8_peak): one CTA per SM issuing back-to-back 128 x 256 x 32
    MMAs. The INT8 tensor-core ceiling next to twice the measured bf16 rate."""
    tops, ms = C.c_double(), C.c_float()
    check(load().dg_measure_i8_peak(int(device), int(iters), C.byref(tops), C.byref(ms)))
    return tops.value, ms.value
