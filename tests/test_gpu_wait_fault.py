"""The projection kernel's failure path, made to run without a GPU fault.

Every wait of the tcgen05 projection pipeline is bounded: when one runs out,
the kernel records kWaitTimeout and the wait's location in its status word,
sets a CTA-wide abort flag, lets its copies in flight land, frees its tensor
memory and returns, and the host turns the status into an error. Here the
wait is made to run out on purpose through dg_linear_test_wait_fault: the MMA
issuer leaves out the completion signal of one 64-wide K group (so the
promotion warps' wait for it can never end) and every wait is bounded by
1 ms. The call must fail with the timeout and its location, and the same
handle must then compute the normal result again (its tensor memory was
freed and the context is intact)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    return torch


def test_a_wait_that_never_ends_times_out_and_the_handle_recovers(torch_cuda):
    from decider_gpu import Linear
    from decider_gpu._lib import GpuError, check, load
    torch = torch_cuda
    rng = np.random.default_rng(5)
    m, n, k = 256, 512, 1024
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    lin = Linear(w)  # reference-order mode: no split-K, one CTA per output tile
    xd = torch.from_numpy(x).cuda()
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    lin.forward_device(xd.data_ptr(), m, y.data_ptr())
    ref = y.cpu().numpy().copy()
    L = load()
    check(L.dg_linear_test_wait_fault(lin.h, 3, 1_000_000))  # group 3 never completes; 1 ms waits
    y.fill_(float("nan"))
    with pytest.raises(GpuError) as e:
        lin.forward_device(xd.data_ptr(), m, y.data_ptr())
    msg = str(e.value)
    print(msg)
    assert "device pipeline wait timed out" in msg and "device error code 2" in msg, msg
    assert "location" in msg
    check(L.dg_linear_test_wait_fault(lin.h, -1, 0))
    for _ in range(2):
        y.fill_(float("nan"))
        lin.forward_device(xd.data_ptr(), m, y.data_ptr())
        assert np.array_equal(y.cpu().numpy(), ref)
    with pytest.raises(GpuError, match="out of range"):
        check(L.dg_linear_test_wait_fault(lin.h, k // 64, 1_000_000))
