"""Seeded synthetic Qwen3.5 decider checkpoints for parity tests (shared by
the oracle and the GPU engine)."""
import numpy as np


def small_config(hidden=256, intermediate=512, layer_types=("linear_attention",) * 3 + ("full_attention",),
                 heads=2, kv_heads=1, head_dim=256, key_heads=2, value_heads=2, dk=128, vocab=1000):
    return {
        "hidden_size": hidden, "intermediate_size": intermediate, "num_hidden_layers": len(layer_types),
        "vocab_size": vocab, "layer_types": list(layer_types), "num_attention_heads": heads,
        "num_key_value_heads": kv_heads, "head_dim": head_dim, "rms_norm_eps": 1e-6,
        "linear_conv_kernel_dim": 4, "linear_key_head_dim": dk, "linear_value_head_dim": dk,
        "linear_num_key_heads": key_heads, "linear_num_value_heads": value_heads,
        "rope_parameters": {"rope_theta": 1e7, "partial_rotary_factor": 0.25, "rope_type": "default"},
        "attention_bias": False, "attn_output_gate": True, "hidden_act": "silu",
    }


def cfg2_config(layers=24, vocab=248320):
    """the 2B decider shape (hidden 2048, 6 x [3 Gated
    DeltaNet + 1 gated GQA attention] layers, 8 Q / 2 KV heads of 256, DeltaNet
    16 x 128, SwiGLU 6144)."""
    lt = (["linear_attention"] * 3 + ["full_attention"]) * (layers // 4)
    return {
        "hidden_size": 2048, "intermediate_size": 6144, "num_hidden_layers": layers, "vocab_size": vocab,
        "layer_types": lt, "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 256,
        "rms_norm_eps": 1e-6, "linear_conv_kernel_dim": 4, "linear_key_head_dim": 128,
        "linear_value_head_dim": 128, "linear_num_key_heads": 16, "linear_num_value_heads": 16,
        "rope_parameters": {"rope_theta": 1e7, "partial_rotary_factor": 0.25, "rope_type": "default"},
        "attention_bias": False, "attn_output_gate": True, "hidden_act": "silu",
    }


def expected_shapes(c, rank, pointer_dim):
    H, I = c["hidden_size"], c["intermediate_size"]
    qw, kw = c["num_attention_heads"] * c["head_dim"], c["num_key_value_heads"] * c["head_dim"]
    kd = c["linear_num_key_heads"] * c["linear_key_head_dim"]
    vd = c["linear_num_value_heads"] * c["linear_value_head_dim"]
    W, VH = 2 * kd + vd, c["linear_num_value_heads"]
    shapes, projections = {}, []

    def proj(key, i, o):
        shapes[key + ".weight"] = [o, i]
        projections.append(key)
        shapes["base_model.model." + key + ".lora_A.weight"] = [rank, i]
        shapes["base_model.model." + key + ".lora_B.weight"] = [o, rank]

    for li, t in enumerate(c["layer_types"]):
        p = f"layers.{li}."
        if t == "full_attention":
            proj(p + "self_attn.q_proj", H, 2 * qw)
            proj(p + "self_attn.k_proj", H, kw)
            proj(p + "self_attn.v_proj", H, kw)
            proj(p + "self_attn.o_proj", qw, H)
            shapes[p + "self_attn.q_norm.weight"] = [c["head_dim"]]
            shapes[p + "self_attn.k_norm.weight"] = [c["head_dim"]]
        else:
            proj(p + "linear_attn.in_proj_qkv", H, W)
            proj(p + "linear_attn.in_proj_z", H, vd)
            proj(p + "linear_attn.in_proj_a", H, VH)
            proj(p + "linear_attn.in_proj_b", H, VH)
            proj(p + "linear_attn.out_proj", vd, H)
            shapes[p + "linear_attn.conv1d.weight"] = [W, 1, c["linear_conv_kernel_dim"]]
            shapes[p + "linear_attn.dt_bias"] = [VH]
            shapes[p + "linear_attn.A_log"] = [VH]
            shapes[p + "linear_attn.norm.weight"] = [c["linear_value_head_dim"]]
        proj(p + "mlp.gate_proj", H, I)
        proj(p + "mlp.up_proj", H, I)
        proj(p + "mlp.down_proj", I, H)
        shapes[p + "input_layernorm.weight"] = [H]
        shapes[p + "post_attention_layernorm.weight"] = [H]
    shapes["embed_tokens.weight"] = [c["vocab_size"], H]
    shapes["norm.weight"] = [H]
    if pointer_dim:
        shapes.update({"head.norm.weight": [H], "head.norm.bias": [H], "head.q.weight": [pointer_dim, H],
                       "head.q.bias": [pointer_dim], "head.k.weight": [pointer_dim, H],
                       "head.k.bias": [pointer_dim]})
    return shapes


def random_tensors(c, rank=32, pointer_dim=64, seed=0, std=0.02, norm_jitter=0.1, bias_std=0.1, f32=False):
    """{name: (0 (F32), shape, array)}: N(0, std^2) weights, norms 1 + jitter,
    biases N(0, bias_std^2). f32=True draws the normals directly in float32
    (numpy's float32 ziggurat: a different, faster stream, for the 2B-sized
    parity models)."""
    rng = np.random.default_rng(seed)
    if f32:
        normal = lambda shape: rng.standard_normal(shape, dtype=np.float32)
    else:
        normal = lambda shape: rng.standard_normal(shape)
    out = {}
    for name, shape in expected_shapes(c, rank, pointer_dim).items():
        if "norm" in name and name.endswith(".weight"):
            arr = (1.0 + norm_jitter * normal(shape)).astype(np.float32)
        elif name.endswith(".bias"):
            arr = (bias_std * normal(shape)).astype(np.float32)
        elif name.endswith("embed_tokens.weight"):
            arr = normal(shape).astype(np.float32)
        else:
            s = std
            if "lora_B" in name or "lora_A" in name:
                s = 0.05
            arr = normal(shape)
            arr *= np.float32(s) if f32 else s
            arr = arr.astype(np.float32, copy=False)
        out[name] = (0, list(shape), arr)
    return out


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ---------------------------------------------------------------- full-size parity inputs
# The 2B decider of BASELINE config 2 (24 layers, vocab 248320, rank-32 LoRA
# with alpha/r = 2, pointer head of 256), seeded weights N(0, 0.02^2) with
# norms 1 and zero biases, shared by tests/golden/make_full_parity.py (which
# runs the CPU oracle once and commits its outputs) and the GPU tests.
FULL_SEED = 20261202
FULL_POINTER_DIM = 256
# Relative size of the input perturbation that measures the oracle's own
# sensitivity (far below FP32 rounding of the layers' arithmetic).
NOISE_REL = 1e-7
# temperature_by_kind of the reference's tiny fixture config (noul 0.8,
# choice 0.7, score 1.2).
TEMPERATURES = {"noul": 0.8, "choice": 0.7, "score": 1.2}
KIND_OPTIONS = {"noul": 2, "choice": 4, "score": 5}


def full_model_tensors():
    c = cfg2_config(24)
    t = random_tensors(c, rank=32, pointer_dim=FULL_POINTER_DIM, seed=FULL_SEED, std=0.02, norm_jitter=0.0,
                       bias_std=0.0, f32=True)
    return c, t


def tensor_checksums(tensors, names=("layers.0.linear_attn.in_proj_qkv.weight", "layers.23.mlp.down_proj.weight",
                                     "embed_tokens.weight", "head.q.weight")):
    """float64 sums of a few tensors: the fixture records them so a test can
    tell a different random stream from a parity failure."""
    return {n: float(np.asarray(tensors[n][2], np.float64).sum()) for n in names}


def cfg2_request(vocab=248320):
    """512 ids uniform over the vocabulary (seed 0), one
    noul question with options at [509, 510], answer at 511."""
    ids = np.random.default_rng(0).integers(0, vocab, 512).astype(np.uint32)
    return ids, [509, 510]


def cfg4_request(vocab=248320, seed=4):
    """a 3584-token state, then 8 questions of 64 tokens,
    kinds noul / choice (4) / score (5) in turn, options in each question's
    last 16 tokens."""
    rng = np.random.default_rng(seed)
    state = rng.integers(0, vocab, 3584).astype(np.uint32)
    kinds = [("noul", "choice", "score")[i % 3] for i in range(8)]
    qs = [(rng.integers(0, vocab, 64).astype(np.uint32), [48 + 2 * j for j in range(KIND_OPTIONS[k])], k)
          for k in kinds]
    return state, qs


def probabilities(logits, kind):
    """The reference's readout (src/lib.rs:525-548): logits / T_kind, then
    softmax (max, exp, sequential sum, divide; src/tensor.rs:534-546)."""
    v = (np.asarray(logits, np.float32) / np.float32(TEMPERATURES[kind])).astype(np.float32)
    mx = np.float32(v.max())
    e = np.exp((v - mx).astype(np.float32)).astype(np.float32)
    total = np.float32(0.0)
    for x in e:
        total = np.float32(total + x)
    return (e / total).astype(np.float32)


def perturbed_embedding(tensors, ids, seed, rel=None):
    """The embedding tensor with the rows of `ids` scaled by (1 + rel N(0, 1))
    (seeded): the oracle's sensitivity probe."""
    code, shp, arr = tensors["embed_tokens.weight"]
    rows = np.unique(np.asarray(ids, np.int64))
    out = arr.copy()
    rng = np.random.default_rng(seed)
    out[rows] = (arr[rows] * (1 + (NOISE_REL if rel is None else rel) * rng.standard_normal(arr[rows].shape))
                 ).astype(np.float32)
    return code, shp, out

