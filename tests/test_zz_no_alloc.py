"""The allocation-free projection call against the allocating one.

dg_linear_forward_device_noalloc runs the same kernels as
dg_linear_forward_device with its scratch in a fixed static device area, so
the bar is this suite's projection tolerance at its tightest: bit-identical
outputs (reference order and fused-multiply-add order alike), on two calls in
a row through the C ABI. Its file name sorts last so it also runs after every
other GPU test in one session.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    return torch


def _case(seed, m, n, k, rank=32):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    la = (0.05 * rng.standard_normal((rank, k))).astype(np.float32) if rank else None
    lb = (0.05 * rng.standard_normal((n, rank))).astype(np.float32) if rank else None
    return x, w, la, lb


def _both(torch, lin, x, n):
    """(allocating result, allocation-free result) for the rows of x."""
    m = x.shape[0]
    xd = torch.from_numpy(x).cuda()
    ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    got = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    lin.forward_device(xd.data_ptr(), m, ref.data_ptr())
    lin.forward_device_noalloc(xd.data_ptr(), m, got.data_ptr())
    torch.cuda.synchronize()
    return ref.cpu().numpy(), got.cpu().numpy()


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("n,k,rank", [(6144, 2048, 32), (300, 256, 32), (512, 1024, 0)])
def test_noalloc_matches_allocating_call_twice(torch_cuda, exact, n, k, rank):
    from decider_gpu import Linear
    x, w, la, lb = _case(n + k + rank, 512, n, k, rank)
    lin = Linear(w, la, lb, 2.0)
    lin.set_exact(exact)
    # Two calls in a row on the same scratch area: full rows, then fewer rows
    # of different values (the second must not see the first's leftovers).
    for rows in (x, x[::-1][:200].copy() * 0.5):
        ref, got = _both(torch_cuda, lin, rows, n)
        assert np.isfinite(got).all()
        assert np.array_equal(got, ref), f"max |diff| {np.abs(got - ref).max()}"


def test_noalloc_rejects_rows_beyond_its_area(torch_cuda):
    from decider_gpu import Linear
    from decider_gpu._lib import GpuError
    n, k, m = 256, 2048, 4096  # 4096 rows x 2048 bytes alone fill the 8 MiB area
    _, w, la, lb = _case(3, 1, n, k)
    lin = Linear(w, la, lb, 2.0)
    x = torch_cuda.zeros((m, k), dtype=torch_cuda.float32, device="cuda")
    y = torch_cuda.zeros((m, n), dtype=torch_cuda.float32, device="cuda")
    with pytest.raises(GpuError, match="bytes of scratch"):
        lin.forward_device_noalloc(x.data_ptr(), m, y.data_ptr())
    # The handle still works after the refusal.
    rows = np.ones((8, k), np.float32)
    ref, got = _both(torch_cuda, lin, rows, n)
    assert np.array_equal(got, ref)


def test_noalloc_calls_take_no_device_memory(torch_cuda):
    """The property the entry point exists for: once its first call on the
    device has resolved the static area, further calls take no device memory
    (the device's free bytes do not move over many calls of varying sizes)."""
    from decider_gpu import Linear
    n, k = 6144, 2048
    x, w, la, lb = _case(7, 512, n, k)
    lin = Linear(w, la, lb, 2.0)
    xd = torch_cuda.from_numpy(x).cuda()
    yd = torch_cuda.empty((512, n), dtype=torch_cuda.float32, device="cuda")
    lin.forward_device_noalloc(xd.data_ptr(), 512, yd.data_ptr())  # first call: set-up
    torch_cuda.cuda.synchronize()
    free0, _ = torch_cuda.cuda.mem_get_info()
    for rows in (512, 17, 300, 1, 512):
        lin.forward_device_noalloc(xd.data_ptr(), rows, yd.data_ptr())
    torch_cuda.cuda.synchronize()
    free1, _ = torch_cuda.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
