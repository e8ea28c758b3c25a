"""The C-ABI library loads on a CPU-only host and exports every entry point
declared in include/*.h (no device calls)."""
import ctypes
import glob
import os
import re

from conftest import ROOT


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(dg_[a-z0-9_]+)\s*\(", text))
    return names


def test_header_declares_the_python_symbol_list():
    import decider_gpu
    assert declared_symbols() == set(decider_gpu.SYMBOLS)


def test_library_exports_every_declared_symbol():
    import decider_gpu
    assert os.path.exists(decider_gpu.LIB_PATH), "build libdecider_gpu.so first (__graft_entry__.build)"
    lib = ctypes.CDLL(decider_gpu.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_no_device_call_needed_for_errors():
    import decider_gpu
    L = decider_gpu.load()
    assert L.dg_last_error() == b""
    # A null config is rejected on the host before any CUDA call.
    h = ctypes.c_void_p()
    assert L.dg_engine_create(None, 2, 0, 16, ctypes.byref(h)) != 0
    assert b"null" in L.dg_last_error()


def test_quantize_rejects_bad_arguments_before_any_device_call():
    import decider_gpu
    L = decider_gpu.load()
    fake = 0x1000  # never dereferenced: the checks run first
    for rows, width, bits, msg in [(1, 64, 5, b"bits must be 8 or 4"), (1, 0, 8, b"bad width")]:
        assert L.dg_quantize_weights_device(fake, rows, width, bits, fake, fake, None) != 0
        assert msg in L.dg_last_error()
    assert L.dg_quantize_weights_device(None, 1, 64, 8, fake, fake, None) != 0
    assert b"null" in L.dg_last_error()
