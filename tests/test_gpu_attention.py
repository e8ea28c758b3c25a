"""Gated causal GQA attention (causal_attention and the output gate of
Full::forward, src/qwen.rs:581-643) in isolation through dg_attention_device:
the fast-mode tensor-core path (3 x TF32 tcgen05 products, softmax kernel)
and the CUDA-core kernel of reference-order mode, both against an FP64 torch
computation of the same attention, at the 2B head shapes (8 query heads, 2
KV heads, head_dim 256), with and without a prefix, across query-chunk and
tile edges. Bar: every output row within 1e-5 relative (norm of the
difference / norm of the row) of FP64, on both paths. (The tensor-core path
adds each 32-wide K chunk's products into FP32 register sums: the tensor
core's own FP32 accumulation does not round to nearest, and over a whole
256-wide score it drifted to 2.5e-5 of the row; chunk by chunk it measures
2.6e-6, below the CUDA-core kernel's 4.8e-6.)"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, KV, D = 8, 2, 256


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    return torch


def _reference(torch, q, k, v, gate, n, offset):
    q64, k64, v64 = q.double(), k.double(), v.double()
    out = torch.empty((n, H, D), dtype=torch.float64, device=q.device)
    t = torch.arange(n, device=q.device)[:, None] + offset
    keys = torch.arange(offset + n, device=q.device)[None, :]
    mask = keys <= t
    for h in range(H):
        kh = h // (H // KV)
        s = q64[:, h, :] @ k64[:, kh * D:(kh + 1) * D].T / 16.0
        s = s.masked_fill(~mask, float("-inf"))
        p = torch.softmax(s, dim=1)
        out[:, h, :] = p @ v64[:, kh * D:(kh + 1) * D]
    g = gate.double().view(n, H, 2 * D)[:, :, D:]
    return out * torch.sigmoid(g)


def _run(torch, q, k, v, gate, n, offset, tensor_cores):
    from decider_gpu._lib import check, load
    L = load()
    out = torch.full((n, H, D), float("nan"), dtype=torch.float32, device="cuda")
    ws_bytes = L.dg_attention_workspace_bytes(H, KV, D, n)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    check(L.dg_attention_device(q.data_ptr(), k.data_ptr(), v.data_ptr(), gate.data_ptr(), 2 * H * D, n, offset, H,
                                KV, D, out.data_ptr(), int(tensor_cores), ws.data_ptr(), ws_bytes,
                                C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return out


@pytest.mark.parametrize("n,offset", [(512, 0), (100, 0), (64, 1000), (33, 200), (1, 500), (300, 130), (1100, 0)])
def test_tensor_core_attention_matches_fp64(torch_cuda, n, offset):
    torch = torch_cuda
    gen = torch.Generator(device="cuda").manual_seed(n * 7 + offset)
    rn = lambda *s: torch.randn(*s, generator=gen, device="cuda", dtype=torch.float32)
    q = rn(n, H, D) * 1.5
    k = rn(offset + n, KV * D) * 1.5
    v = rn(offset + n, KV * D)
    gate = rn(n, 2 * H * D)
    ref = _reference(torch, q, k, v, gate, n, offset)
    for tc in (1, 0):
        got = _run(torch, q, k, v, gate, n, offset, tc).double()
        assert torch.isfinite(got).all()
        rows = ((got - ref).norm(dim=2) / ref.norm(dim=2).clamp_min(1e-30)).flatten()
        print(f"n={n} offset={offset} {'tensor cores' if tc else 'CUDA cores'}: max row error {rows.max():.2e}, "
              f"median {rows.median():.2e}")
        assert rows.max() <= 1e-5, (tc, float(rows.max()))
