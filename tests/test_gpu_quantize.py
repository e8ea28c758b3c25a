"""Weight quantisation on the device (dg_quantize_weights_device) against the
oracle's Data::quantize (src/weights.rs:98-146): every scale and every code
byte equal, for 8 and 4 bits, at the 2B model's projection shapes and at the
edges the reference's arithmetic has: an all-zero group (scale 1), groups
whose max / bound falls below FLT_MIN (the FLT_MIN floor, subnormal
weights), exact halfway values (round half away from zero), clamping at the
bound, a partial last group, and 4-bit packing across row ends (odd width).
The engine quantises every projection with this kernel while it builds."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    return torch


def _device_quantize(torch, w, bits):
    from decider_gpu._lib import check, load
    L = load()
    rows, width = w.shape
    groups = (width + 63) // 64
    nbytes = rows * width if bits == 8 else (rows * width + 1) // 2
    wd = torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda()
    q = torch.full((max(nbytes, 1),), 0xA5, dtype=torch.uint8, device="cuda")
    s = torch.full((max(rows * groups, 1),), float("nan"), dtype=torch.float32, device="cuda")
    check(L.dg_quantize_weights_device(wd.data_ptr(), rows, width, bits, q.data_ptr(), s.data_ptr(),
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return q.cpu().numpy()[:nbytes], s.cpu().numpy()[:rows * groups].reshape(rows, groups)


def _compare(torch, w, bits):
    from oracle import oracle as O
    rv, rs = O.quantize_weights(w, bits)
    gv, gs = _device_quantize(torch, w, bits)
    assert np.array_equal(gs.view(np.uint32), rs.view(np.uint32)), "scales differ"
    assert np.array_equal(gv, rv.reshape(-1)), "codes differ"


def _edge_rows(width):
    """Rows that exercise the quantiser's special cases, `width` wide."""
    rng = np.random.default_rng(7)
    rows = []
    rows.append(np.zeros(width, np.float32))                                   # every group all zero
    rows.append(np.full(width, 1e-38, np.float32) * rng.choice([-1, 1], width))  # max / bound < FLT_MIN
    rows.append((rng.integers(1, 100, width) * np.float32(1e-45)).astype(np.float32))  # subnormal weights
    ties = (rng.integers(-126, 126, width) + 0.5).astype(np.float32)           # exact halves, scale 1
    ties[::64] = 127.0
    rows.append(ties)
    clamp = rng.normal(0, 1, width).astype(np.float32)
    clamp[::64] = -1e30                                     # one huge value per group, the rest round to 0
    rows.append(clamp)
    small = (rng.integers(-6, 6, width) + 0.5).astype(np.float32)              # 4-bit halves, scale 1
    small[::64] = 7.0
    rows.append(small)
    return np.stack(rows)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,width", [(6144, 2048), (2048, 6144), (16, 2048), (2048, 4096)])
def test_device_quantisation_matches_data_quantize_at_2b_shapes(torch_cuda, bits, rows, width):
    rng = np.random.default_rng(rows * 31 + width + bits)
    w = rng.normal(0.0, 0.02, (rows, width)).astype(np.float32)
    edge = _edge_rows(width)
    w[:len(edge)] = edge
    _compare(torch_cuda, w, bits)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("rows,width", [(3, 65), (5, 1), (7, 127), (1, 64), (4, 200)])
def test_device_quantisation_ragged_widths(torch_cuda, bits, rows, width):
    rng = np.random.default_rng(rows * 1000 + width * 10 + bits)
    w = rng.normal(0.0, 1.0, (rows, width)).astype(np.float32)
    w[0, : min(width, 64)] = 0.0
    _compare(torch_cuda, w, bits)
