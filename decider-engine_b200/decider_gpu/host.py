"""Host logic around the device model, mirroring decider-engine's API surface
for the prefill path: config reading (src/lib.rs:188-222,287-358),
`NativeEngine.raw_logits` / shared-prefix `logits` (src/lib.rs:383-419), the
temperature/softmax readout (src/lib.rs:525-548, src/tensor.rs:534-546) and the
typed answers (src/prompt.rs:228-257, src/schema.rs:145-177).

Prompt rendering and tokenisation stay with the caller: the boundary takes
token IDs and option positions (`Encoding`, src/lib.rs:160-165).
"""
from __future__ import annotations

import enum
import json
import math
import os
from dataclasses import dataclass, field

import numpy as np

ENGINE_ID = "strands-decider-2b-native"


class Precision(enum.Enum):
    CHECKPOINT = "checkpoint"
    INT8 = "int8"
    INT8_COMPUTE = "int8-compute"
    INT4 = "int4"

    def engine_id(self) -> str:  # src/lib.rs:57-65
        return {"checkpoint": ENGINE_ID, "int8": ENGINE_ID + "-int8",
                "int8-compute": ENGINE_ID + "-int8-compute", "int4": ENGINE_ID + "-int4"}[self.value]


class ErrorKind(enum.Enum):  # src/error.rs:7-21
    INVALID_REQUEST = "invalid_request"
    CONTEXT_WINDOW = "context_window"
    RESOURCE_LIMIT = "resource_limit"
    MODEL_MISMATCH = "model_mismatch"
    ENGINE = "engine"


class DecideError(Exception):
    def __init__(self, kind: ErrorKind, message: str):
        super().__init__(message)
        self.kind = kind
        self.message = message


@dataclass
class Encoding:  # src/lib.rs:160-165
    input_ids: list
    option_positions: list
    answer_position: int


def _json(path: str) -> dict:
    with open(path, "rb") as f:
        raw = f.read(1024 * 1024 + 1)
    if len(raw) > 1024 * 1024:
        raise DecideError(ErrorKind.ENGINE, f"{path}: metadata exceeds 1048576 bytes")
    return json.loads(raw)


def read_decider_config(d: str) -> dict:
    """read_config, src/lib.rs:188-222."""
    p = os.path.join(d, "strands_decider_config.json")
    if not os.path.exists(p):
        p = os.path.join(d, "hobson_config.json")
    c = _json(p)
    if (c.get("base_model") != "Qwen/Qwen3.5-2B-Base" or c.get("head_type") != "pointer"
            or not c.get("use_lora") or c.get("force_bos", False)):
        raise ValueError("native engine requires Qwen3.5-2B-Base, pointer head, LoRA, and default BOS behavior")
    t = c.get("temperature", 0)
    tk = c.get("temperature_by_kind", {}) or {}
    sm = c.get("ordinal_smoothing", 0.0)
    if (not 0 < c["max_length"] <= 4096 or not 0 < c["pointer_dim"] <= 4096 or not math.isfinite(t) or t <= 0
            or any(not math.isfinite(v) or v <= 0 for v in tk.values()) or not math.isfinite(sm)
            or not 0.0 <= sm <= 1.0):
        raise ValueError("invalid decision window, pointer dimension, or calibration")
    c.setdefault("temperature_by_kind", {})
    c.setdefault("ordinal_smoothing", 0.0)
    return c


def read_text_config(d: str) -> dict:
    base = _json(os.path.join(d, "base", "config.json"))
    if base.get("model_type") != "qwen3_5":
        raise ValueError("base model must be qwen3_5")
    c = base["text_config"]
    # Config::validate, src/qwen.rs:133-188
    rp = c["rope_parameters"]
    r = int(c["head_dim"] * np.float32(rp["partial_rotary_factor"]))
    if (c.get("attention_bias") or not c.get("attn_output_gate") or c.get("hidden_act") != "silu"
            or rp.get("rope_type") != "default" or r == 0 or r > c["head_dim"] or r % 2):
        raise ValueError("unsupported Qwen normalization, activation, attention, or RoPE config")
    return c


def read_lora_config(d: str):
    """Rank and alpha/r scale, src/lib.rs:300-358."""
    a = _json(os.path.join(d, "lora", "adapter_config.json"))
    rank = a.get("r")
    if not isinstance(rank, int) or not 0 < rank <= 4096:
        raise ValueError("invalid LoRA rank")
    alpha = a.get("lora_alpha")
    if not isinstance(alpha, (int, float)) or not math.isfinite(alpha) or alpha <= 0:
        raise ValueError("invalid LoRA alpha")
    if (a.get("peft_type") != "LORA" or a.get("bias") != "none" or a.get("use_dora") or a.get("use_rslora")
            or a.get("fan_in_fan_out") or a.get("rank_pattern") or a.get("alpha_pattern")
            or a.get("modules_to_save")):
        raise ValueError("unsupported LoRA adapter configuration")
    scale = np.float32(np.float32(alpha) / np.float32(rank))
    return rank, float(scale)


# ---------------------------------------------------------------- readout
def softmax(v) -> np.ndarray:
    """softmax, src/tensor.rs:534-546 (max, exp, sequential sum, divide)."""
    v = np.asarray(v, np.float32).copy()
    mx = np.float32(-np.inf)
    for x in v:
        mx = max(mx, x)
    total = np.float32(0.0)
    for i in range(len(v)):
        v[i] = np.float32(np.exp(np.float32(v[i] - mx)))
        total = np.float32(total + v[i])
    if total > 0:
        v = (v / total).astype(np.float32)
    return v


def choice_confidence(p) -> float:  # src/schema.rs:145-151
    if len(p) <= 1:
        return 1.0
    n = np.float32(len(p))
    return float(np.clip((n * np.float32(max(p)) - 1) / (n - 1), 0.0, 1.0))


def score_confidence(p, smoothing: float) -> float:  # src/schema.rs:152-177
    if len(p) <= 1:
        return 1.0
    p = np.asarray(p, np.float32)
    total = np.float32(sum(p))
    if total <= 0:
        return 0.0
    mean = np.float32(sum(np.float32(i) * v / total for i, v in enumerate(p)))
    sigma = np.float32(math.sqrt(sum(v / total * (np.float32(i) - mean) ** 2 for i, v in enumerate(p))))
    mx = np.float32((len(p) - 1) / 2.0)
    floor = np.float32(math.sqrt(max(smoothing, 0.0)))
    if mx <= floor:
        return 1.0 if sigma <= floor else 0.0
    return float(np.clip((mx - sigma) / (mx - floor), 0.0, 1.0))


def answer(kind: str, labels: list, p, smoothing: float, legend=None) -> dict:
    """Rendered::answer, src/prompt.rs:228-257."""
    p = [float(x) for x in p]
    probs = dict(zip(labels, p))
    if kind == "noul":
        return {"type": "noul", "noul": p[1]}
    if kind == "choice":
        best = 0
        for i in range(1, len(p)):
            if p[i] > p[best]:
                best = i
        return {"type": "choice", "choice": labels[best], "probabilities": probs,
                "confidence": choice_confidence(p)}
    return {"type": "score", "score": float(sum(np.float32(i) * np.float32(v) for i, v in enumerate(p))),
            "probabilities": probs, "legend": legend or {}, "confidence": score_confidence(p, smoothing)}


@dataclass
class InferenceLimits:  # src/limits.rs:10-43 (token budget used by the forward path)
    max_total_tokens: int = 8192


@dataclass
class NativeEngine:
    """The reference's NativeEngine over the device model, for pre-encoded
    questions (src/lib.rs:267-559)."""
    model: object
    config: dict
    precision: Precision
    forward_calls: int = field(default=0)

    @classmethod
    def load_with_precision(cls, d: str, precision: Precision = Precision.CHECKPOINT, device: int = 0):
        from .engine import GpuModel
        cfg = read_decider_config(d)
        return cls(GpuModel.from_dir(d, precision.value, device, cfg["max_length"]), cfg, precision)

    def max_length(self) -> int:
        return self.config["max_length"]

    def model_id(self) -> str:
        return self.precision.engine_id()

    def raw_logits(self, enc: Encoding) -> np.ndarray:
        """src/lib.rs:383-396"""
        ids = enc.input_ids
        if (not ids or len(ids) > self.max_length() or enc.answer_position != len(ids) - 1
                or not enc.option_positions or any(p >= enc.answer_position for p in enc.option_positions)):
            raise DecideError(ErrorKind.ENGINE, "invalid encoding positions or window")
        return self.logits(enc, None)

    def logits(self, enc: Encoding, shared) -> np.ndarray:
        """NativeEngine::logits, src/lib.rs:400-419; `shared` = (state ids, prefix)."""
        self.forward_calls += 1
        if shared is not None:
            sids, prefix = shared
            n = len(sids)
            if (len(enc.input_ids) > n and list(enc.input_ids[:n]) == list(sids)
                    and all(p >= n for p in enc.option_positions)):
                return self.model.logits(enc.input_ids[n:], [p - n for p in enc.option_positions], prefix)
        return self.model.logits(enc.input_ids, enc.option_positions)

    def set_lanes(self, lanes: int) -> None:
        """Requests of evaluate_batch served `lanes` at a time on this GPU
        (dg_engine_set_lanes)."""
        self.model.set_lanes(lanes)

    def _readout(self, items, logits) -> dict:
        """Temperature, softmax and typed answers of one request
        (src/lib.rs:525-548)."""
        answers, used = {}, 0
        for (name, q), lg in zip(items, logits):
            kind, labels, enc = q[0], q[1], q[2]
            legend = q[3] if len(q) > 3 else None
            t = np.float32(self.config["temperature_by_kind"].get(kind, self.config["temperature"]))
            p = softmax((np.asarray(lg, np.float32) / t).astype(np.float32))
            if not np.all(np.isfinite(p)):
                raise DecideError(ErrorKind.ENGINE, "non-finite decision probabilities")
            answers[name] = answer(kind, labels, p, self.config["ordinal_smoothing"], legend)
            used += len(enc.input_ids)
        return {"model": self.model_id(), "answers": answers, "usage": {"input_tokens": used, "output_tokens": 0}}

    def evaluate_batch(self, requests, limits: InferenceLimits | None = None) -> list:
        """`evaluate_encoded` for many requests in one device call
        (dg_logits_batch): requests is a list of (questions, state_tokens).
        Each request keeps evaluate's semantics: its questions in name order,
        one shared state when it has two or more questions (a question that
        does not continue the state runs as its own forward, as
        NativeEngine::logits does), the token limit checked first. Returns,
        per request, the response dict or the DecideError it raised; one bad
        request does not stop the others."""
        limits = limits or InferenceLimits()
        out = [None] * len(requests)
        dev, where = [], []  # device requests; (request index, [question slots]) for each
        plans = []
        for r, (questions, state_tokens) in enumerate(requests):
            total = sum(len(q[2].input_ids) for q in questions.values())
            if total > limits.max_total_tokens:
                out[r] = DecideError(ErrorKind.RESOURCE_LIMIT,
                                     f"request binds {total} total tokens; limit is {limits.max_total_tokens}")
                continue
            items = sorted(questions.items())
            plans.append((r, items))
            shared, alone = [], []
            sids = list(items[0][1][2].input_ids[:state_tokens]) if len(items) >= 2 else None
            for k, (_, q) in enumerate(items):
                enc, n = q[2], len(sids) if sids is not None else 0
                if (sids is not None and len(enc.input_ids) > n and list(enc.input_ids[:n]) == sids
                        and all(p >= n for p in enc.option_positions)):
                    shared.append((k, (list(enc.input_ids[n:]), [p - n for p in enc.option_positions])))
                else:
                    alone.append((k, (list(enc.input_ids), list(enc.option_positions))))
            if shared:
                dev.append({"state": sids, "questions": [x for _, x in shared]})
                where.append((r, [k for k, _ in shared]))
            for k, x in alone:
                dev.append({"questions": [x]})
                where.append((r, [k]))
        logits, status, _, err = self.model.logits_batch(dev) if dev else ([], [], [], None)
        per = {r: [None] * len(items) for r, items in plans}
        failed = {}
        for d, (r, slots) in enumerate(where):
            if status[d]:
                failed.setdefault(r, err or "device request failed")
                continue
            for k, lg in zip(slots, logits[d]):
                per[r][k] = lg
        for r, items in plans:
            if r in failed:
                out[r] = DecideError(ErrorKind.ENGINE, failed[r])
                continue
            try:
                out[r] = self._readout(items, per[r])
            except DecideError as e:
                out[r] = e
        return out

    def evaluate_encoded(self, questions: dict, state_tokens: int, limits: InferenceLimits | None = None):
        """`evaluate` after prompt binding (src/lib.rs:494-559): questions maps
        name -> (kind, labels, Encoding[, legend]); BTreeMap order; one shared
        prefill when there are two or more questions."""
        limits = limits or InferenceLimits()
        total = sum(len(q[2].input_ids) for q in questions.values())
        if total > limits.max_total_tokens:
            raise DecideError(ErrorKind.RESOURCE_LIMIT,
                              f"request binds {total} total tokens; limit is {limits.max_total_tokens}")
        items = sorted(questions.items())
        shared = None
        if len(items) >= 2:
            sids = list(items[0][1][2].input_ids[:state_tokens])
            self.forward_calls += 1
            shared = (sids, self.model.prefill(sids))
        answers, used = {}, 0
        for name, q in items:
            kind, labels, enc = q[0], q[1], q[2]
            legend = q[3] if len(q) > 3 else None
            lg = self.logits(enc, shared)
            t = np.float32(self.config["temperature_by_kind"].get(kind, self.config["temperature"]))
            p = softmax((lg / t).astype(np.float32))
            if not np.all(np.isfinite(p)):
                raise DecideError(ErrorKind.ENGINE, "non-finite decision probabilities")
            answers[name] = answer(kind, labels, p, self.config["ordinal_smoothing"], legend)
            used += len(enc.input_ids)
        return {"model": self.model_id(), "answers": answers, "usage": {"input_tokens": used, "output_tokens": 0}}
