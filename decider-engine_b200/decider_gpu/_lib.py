"""ctypes binding of libdecider_gpu.so (the C ABI in include/decider_gpu.h).

The library is built in-tree (decider-engine_b200/build.py). There is no CPU
fallback: if the shared library is missing, loading raises.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_ROOT, "libdecider_gpu.so")

# Every entry point declared in include/decider_gpu.h.
SYMBOLS = [
    "dg_last_error", "dg_launch_count",
    "dg_engine_create", "dg_engine_create_sibling", "dg_engine_set_lanes", "dg_engine_lanes",
    "dg_engine_last_batch_ms", "dg_engine_set_tensor", "dg_engine_fill_synthetic", "dg_engine_finalize",
    "dg_engine_load", "dg_engine_load_with_limits", "dg_load_limits_default", "dg_read_checkpoint_config",
    "dg_engine_fast_path", "dg_engine_set_exact", "dg_engine_free", "dg_engine_stream",
    "dg_engine_last_forward_ms", "dg_engine_last_launches", "dg_engine_gemm_timing", "dg_engine_gemm_time",
    "dg_engine_gemm_timing_layers", "dg_engine_gemm_time_all", "dg_measure_i8_peak",
    "dg_forward_hidden", "dg_prefill", "dg_prefix_len", "dg_prefix_free", "dg_logits",
    "dg_logits_batch", "dg_debug_layer", "dg_debug_layer_codes", "dg_forward_segments_hidden",
    "dg_linear_create", "dg_linear_forward", "dg_linear_forward_device", "dg_linear_forward_device_noalloc",
    "dg_linear_last_quantized",
    "dg_linear_set_exact", "dg_linear_test_wait_fault", "dg_linear_stream", "dg_linear_last_times", "dg_linear_free",
    "dg_gated_delta_rule_device", "dg_gated_delta_chunk_workspace_bytes", "dg_gated_delta_rule_chunked_device",
    "dg_attention_workspace_bytes", "dg_attention_device", "dg_quantize_weights_device",
]


class ModelConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int32), ("intermediate_size", C.c_int32), ("num_hidden_layers", C.c_int32),
        ("vocab_size", C.c_int32), ("num_attention_heads", C.c_int32), ("num_key_value_heads", C.c_int32),
        ("head_dim", C.c_int32), ("linear_conv_kernel_dim", C.c_int32), ("linear_key_head_dim", C.c_int32),
        ("linear_value_head_dim", C.c_int32), ("linear_num_key_heads", C.c_int32),
        ("linear_num_value_heads", C.c_int32), ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float),
        ("partial_rotary_factor", C.c_float), ("layer_types", C.POINTER(C.c_int32)),
        ("lora_rank", C.c_int32), ("lora_scale", C.c_float), ("pointer_dim", C.c_int32),
    ]


_lib = None


class LoadLimits(C.Structure):
    """dg_load_limits: LoadLimits (src/loading.rs:8-24), bytes."""
    _fields_ = [("max_tensor_bytes", C.c_uint64), ("max_weight_bytes", C.c_uint64),
                ("max_workspace_bytes", C.c_uint64)]


def load() -> C.CDLL:
    """Load libdecider_gpu.so; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libdecider_gpu.so is not built ({LIB_PATH}); run decider-engine_b200/build.py")
    L = C.CDLL(LIB_PATH)
    vp, i32, sz, f32p, u32p = C.c_void_p, C.c_int, C.c_size_t, C.c_void_p, C.c_void_p
    L.dg_last_error.restype = C.c_char_p
    L.dg_launch_count.restype = C.c_uint64
    L.dg_engine_create.argtypes = [C.POINTER(ModelConfig), i32, i32, i32, C.POINTER(vp)]
    L.dg_engine_create_sibling.argtypes = [vp, C.POINTER(vp)]
    L.dg_engine_set_lanes.argtypes = [vp, i32]
    L.dg_engine_lanes.argtypes = [vp]
    L.dg_engine_last_batch_ms.argtypes = [vp]
    L.dg_engine_last_batch_ms.restype = C.c_float
    L.dg_engine_load.argtypes = [C.c_char_p, i32, i32, i32, C.POINTER(vp)]
    L.dg_engine_load_with_limits.argtypes = [C.c_char_p, i32, C.POINTER(LoadLimits), i32, i32, C.POINTER(vp)]
    L.dg_load_limits_default.argtypes = [C.POINTER(LoadLimits)]
    L.dg_load_limits_default.restype = None
    L.dg_read_checkpoint_config.argtypes = [C.c_char_p, C.POINTER(ModelConfig), C.POINTER(C.c_int32), i32]
    L.dg_engine_set_tensor.argtypes = [vp, C.c_char_p, i32, vp, i32, vp]
    L.dg_engine_fill_synthetic.argtypes = [vp, C.c_uint64, C.c_float]
    L.dg_engine_finalize.argtypes = [vp]
    L.dg_engine_fast_path.argtypes = [vp]
    L.dg_engine_set_exact.argtypes = [vp, i32]
    L.dg_engine_free.argtypes = [vp]
    L.dg_engine_free.restype = None
    L.dg_engine_stream.argtypes = [vp]
    L.dg_engine_stream.restype = vp
    L.dg_engine_last_forward_ms.argtypes = [vp]
    L.dg_engine_last_forward_ms.restype = C.c_float
    L.dg_engine_last_launches.argtypes = [vp]
    L.dg_engine_gemm_timing.argtypes = [vp, i32]
    L.dg_engine_gemm_timing_layers.argtypes = [vp, i32, i32]
    L.dg_engine_gemm_time_all.argtypes = [vp, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]
    L.dg_engine_gemm_time.argtypes = [vp, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_uint64)]
    L.dg_linear_stream.argtypes = [vp]
    L.dg_linear_stream.restype = vp
    L.dg_linear_last_times.argtypes = [vp, C.POINTER(C.c_float), C.POINTER(C.c_float)]
    L.dg_forward_hidden.argtypes = [vp, vp, u32p, sz, f32p]
    L.dg_prefill.argtypes = [vp, u32p, sz, C.POINTER(vp)]
    L.dg_prefix_len.argtypes = [vp]
    L.dg_prefix_len.restype = sz
    L.dg_prefix_free.argtypes = [vp]
    L.dg_prefix_free.restype = None
    L.dg_logits.argtypes = [vp, vp, u32p, sz, vp, sz, f32p]
    L.dg_logits_batch.argtypes = [vp, vp, sz, f32p, vp, vp]
    L.dg_forward_segments_hidden.argtypes = [vp, vp, u32p, sz, sz, f32p]
    L.dg_attention_workspace_bytes.argtypes = [i32, i32, i32, i32]
    L.dg_attention_workspace_bytes.restype = sz
    L.dg_attention_device.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, i32, vp, sz, vp]
    L.dg_debug_layer.argtypes = [vp, i32, f32p, sz, f32p]
    L.dg_quantize_weights_device.argtypes = [vp, sz, sz, i32, vp, vp, vp]
    L.dg_measure_i8_peak.argtypes = [i32, i32, C.POINTER(C.c_double), C.POINTER(C.c_float)]
    L.dg_debug_layer_codes.argtypes = [vp, i32, f32p, sz, f32p, vp]
    L.dg_linear_create.argtypes = [f32p, i32, i32, f32p, f32p, i32, C.c_float, i32, C.POINTER(vp)]
    L.dg_linear_forward.argtypes = [vp, f32p, i32, f32p]
    L.dg_linear_forward_device.argtypes = [vp, vp, i32, vp, vp]
    L.dg_linear_forward_device_noalloc.argtypes = [vp, vp, i32, vp]
    L.dg_linear_test_wait_fault.argtypes = [vp, i32, C.c_uint64]
    L.dg_linear_last_quantized.argtypes = [vp, i32, vp, vp]
    L.dg_linear_set_exact.argtypes = [vp, i32]
    L.dg_linear_free.argtypes = [vp]
    L.dg_linear_free.restype = None
    L.dg_gated_delta_rule_device.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp]
    L.dg_gated_delta_chunk_workspace_bytes.argtypes = [i32, i32, i32]
    L.dg_gated_delta_chunk_workspace_bytes.restype = sz
    L.dg_gated_delta_rule_chunked_device.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp, sz, vp]
    _lib = L
    return L


class GpuError(RuntimeError):
    pass


def check(rc: int) -> None:
    if rc:
        raise GpuError(load().dg_last_error().decode("utf-8", "replace"))


def launch_count() -> int:
    return int(load().dg_launch_count())
