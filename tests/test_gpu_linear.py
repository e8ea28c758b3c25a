"""Parity of the tcgen05 INT8 projection with the CPU oracle.

Bar: quantised activations and per-group int32 accumulators bit-exact; FP32
outputs bit-exact in reference order (exact mode); fused-multiply-add mode
within 1e-5 relative (normwise) of the oracle.
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


@pytest.mark.parametrize("m,n,k", [(1, 256, 128), (200, 300, 256), (130, 512, 2048), (77, 1024, 6144)])
def test_projection_bit_exact_with_oracle_in_reference_order(oracle_mod, m, n, k):
    from decider_gpu import Linear
    x, w, la, lb = _case(m + n + k, m, n, k)
    lin = Linear(w, la, lb, 2.0)
    got = lin(x)
    exp = oracle_mod.linear(x, w, "int8-compute", lora_a=la, lora_b=lb, scale=2.0)
    q, s = oracle_mod.quantize_inputs(x)
    gq, gs = lin.last_quantized(m)
    assert np.array_equal(gq, q)
    assert np.array_equal(gs, s.T)
    assert np.array_equal(got, exp), f"max |diff| {np.abs(got - exp).max()}"


def test_projection_without_lora_matches_oracle(oracle_mod):
    from decider_gpu import Linear
    x, w, _, _ = _case(5, 64, 512, 1024, rank=0)
    got = Linear(w)(x)
    exp = oracle_mod.linear(x, w, "int8-compute")
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("tile_n", ["64", "128"])
def test_fma_mode_within_tolerance(oracle_mod, monkeypatch, tile_n):
    """FMA mode on both tile widths; 128-column tiles run LoRA-B on the tensor
    cores (3 x TF32), whose error (about 2^-21 of |mid| |B|) stays far inside
    the 1e-5 bar."""
    from decider_gpu import Linear
    monkeypatch.setenv("DG_GEMM_TILE_N", tile_n)
    x, w, la, lb = _case(7, 256, 768, 2048)
    lin = Linear(w, la, lb, 2.0)
    lin.set_exact(False)
    got = lin(x)
    exp = oracle_mod.linear(x, w, "int8-compute", lora_a=la, lora_b=lb, scale=2.0)
    rel = np.linalg.norm(got - exp) / np.linalg.norm(exp)
    assert rel < 1e-5, rel


def test_tensor_core_lora_keeps_rows_past_m_out(oracle_mod, monkeypatch):
    """A ragged row count (the last 128-row tile partly empty) through the
    tensor-core LoRA path: LoRA-A rows past M come in as zeros."""
    from decider_gpu import Linear
    monkeypatch.setenv("DG_GEMM_TILE_N", "128")
    x, w, la, lb = _case(9, 200, 512, 1024)
    lin = Linear(w, la, lb, 2.0)
    lin.set_exact(False)
    got = lin(x)
    exp = oracle_mod.linear(x, w, "int8-compute", lora_a=la, lora_b=lb, scale=2.0)
    assert np.isfinite(got).all()
    assert np.linalg.norm(got - exp) / np.linalg.norm(exp) < 1e-5


def test_config1_group_accumulators_bit_exact(oracle_mod, torch_cuda):
    """512 x 6144 x 2048: every int32 group dot the tensor
    cores produced equals an independent int32 product of the same quantised
    operands; FP32 rows checked against the oracle on a row sample."""
    torch = torch_cuda
    from decider_gpu import Linear
    m, n, k = 512, 6144, 2048
    rng = np.random.default_rng(0)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    lin = Linear(w)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((m, n), dtype=torch.float32, device="cuda")
    G = k // 64
    dots = torch.empty((G, m, n), dtype=torch.int32, device="cuda")
    lin.forward_device(xd.data_ptr(), m, yd.data_ptr(), dots.data_ptr())
    torch.cuda.synchronize()
    xq, xs = lin.last_quantized(m)
    wq, ws = oracle_mod.quantize_weights(w, 8)
    a = torch.from_numpy(xq).cuda()
    b = torch.from_numpy(wq.view(np.int8)).cuda()
    for g in range(G):
        ref = torch._int_mm(a[:, g * 64:(g + 1) * 64].contiguous(), b[:, g * 64:(g + 1) * 64].t().contiguous())
        assert torch.equal(ref, dots[g]), f"group {g}"
    rows = np.r_[0:8, 250:258, 504:512]
    exp = oracle_mod.linear_int8_prequant(x[rows], wq, ws)
    assert np.array_equal(yd.cpu().numpy()[rows], exp)


def test_nonfinite_input_is_an_error():
    from decider_gpu import GpuError, Linear
    x, w, _, _ = _case(9, 4, 256, 128, rank=0)
    x[2, 5] = np.nan
    with pytest.raises(GpuError, match="non-finite"):
        Linear(w)(x)
