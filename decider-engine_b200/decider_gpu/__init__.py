"""decider_gpu: B200 (sm_100a) prefill engine for the Strands Decider 2B.

Device code lives in libdecider_gpu.so (csrc/, C ABI in include/decider_gpu.h);
this package is the host-side mirror of the reference's model seam and API.
"""
from ._lib import LIB_PATH, SYMBOLS, GpuError, launch_count, load
from .engine import (GpuModel, GpuPrefix, Linear, gated_delta_chunk_workspace_bytes, gated_delta_rule,
                     gated_delta_rule_chunked, measure_i8_peak, read_safetensors)
from .host import (DecideError, Encoding, ErrorKind, InferenceLimits, NativeEngine, Precision, answer,
                   choice_confidence, score_confidence, softmax)

__all__ = ["LIB_PATH", "SYMBOLS", "GpuError", "launch_count", "load", "GpuModel", "GpuPrefix", "Linear",
           "gated_delta_rule", "gated_delta_rule_chunked", "gated_delta_chunk_workspace_bytes", "measure_i8_peak", "read_safetensors", "DecideError", "Encoding", "ErrorKind", "InferenceLimits",
           "NativeEngine", "Precision", "answer", "choice_confidence", "score_confidence", "softmax"]
