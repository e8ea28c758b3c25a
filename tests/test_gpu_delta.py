"""Isolated gated delta rule (BASELINE config 3 shape family) against the
oracle's restatement of Recurrence::head's update (src/qwen.rs:846-866):
outputs and final states within 1e-4 relative (normwise), FP32 state."""
import numpy as np
import pytest

from model_util import rel_err

pytestmark = pytest.mark.gpu


def _inputs(seed, b, t, h, d=128):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((b, t, h, d)).astype(np.float32)
    k = rng.standard_normal((b, t, h, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q = (q / np.sqrt(np.float32(d))).astype(np.float32)
    v = rng.standard_normal((b, t, h, d)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, t, h))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((b, t, h))))).astype(np.float32)
    return q, k, v, g, beta


@pytest.mark.parametrize("chunked", [False, True])
@pytest.mark.parametrize("b,t,h", [(1, 1, 1), (2, 70, 3), (3, 257, 2)])
def test_gated_delta_rule_matches_oracle(oracle_mod, b, t, h, chunked):
    import torch
    from decider_gpu import gated_delta_chunk_workspace_bytes, gated_delta_rule, gated_delta_rule_chunked
    q, k, v, g, beta = _inputs(b * 1000 + t, b, t, h)
    rng = np.random.default_rng(1)
    s0 = (0.1 * rng.standard_normal((b, h, 128, 128))).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    tq, tk, tv, tg, tb, ts = map(dev, (q, k, v, g, beta, s0))
    to = torch.zeros((b, t, h, 128), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if chunked:
        nbytes = gated_delta_chunk_workspace_bytes(b, t, h)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        gated_delta_rule_chunked(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tg.data_ptr(), tb.data_ptr(), b, t, h,
                                 ts.data_ptr(), to.data_ptr(), ws.data_ptr(), nbytes, stream)
    else:
        gated_delta_rule(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tg.data_ptr(), tb.data_ptr(), b, t, h,
                         ts.data_ptr(), to.data_ptr(), stream)
    torch.cuda.synchronize()
    o_gpu, s_gpu = to.cpu().numpy(), ts.cpu().numpy()
    for bi in range(b):
        for hi in range(h):
            o, s = oracle_mod.gated_delta_rule(q[bi, :, hi], k[bi, :, hi], v[bi, :, hi], g[bi, :, hi],
                                               beta[bi, :, hi], s0[bi, hi])
            assert rel_err(o_gpu[bi, :, hi], o) < 1e-4
            assert rel_err(s_gpu[bi, hi], s) < 1e-4


@pytest.mark.parametrize("chunked", [False, True])
def test_config3_sequence_length_matches_oracle(oracle_mod, chunked):
    """BASELINE config 3 at its full sequence length and head count: 4096 tokens
    x 16 heads, chunk 64, zero initial state, inputs drawn as the config states
    (q, k L2-normalised N(0,1), v ~ N(0,1), beta = sigmoid(N(0,1)),
    g = -softplus(N(0,1))), the full batch of 64 sequences. Three (sequence,
    head) pairs, the last one included, are checked against the oracle's token
    recurrence, outputs and final states within 1e-4."""
    import torch
    from decider_gpu import gated_delta_chunk_workspace_bytes, gated_delta_rule, gated_delta_rule_chunked
    b, t, h, d = 64, 4096, 16, 128
    gen = torch.Generator(device="cuda").manual_seed(0)
    rn = lambda *shape: torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32)
    q, k, v = rn(b, t, h, d), rn(b, t, h, d), rn(b, t, h, d)
    q = q / q.norm(dim=-1, keepdim=True) / np.sqrt(np.float32(d))
    k = k / k.norm(dim=-1, keepdim=True)
    beta = torch.sigmoid(rn(b, t, h))
    g = -torch.nn.functional.softplus(rn(b, t, h))
    q, k, v, beta, g = (x.contiguous() for x in (q, k, v, beta, g))
    state = torch.zeros((b, h, d, d), dtype=torch.float32, device="cuda")
    o = torch.zeros((b, t, h, d), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if chunked:
        nbytes = gated_delta_chunk_workspace_bytes(b, t, h)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        gated_delta_rule_chunked(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), b, t, h,
                                 state.data_ptr(), o.data_ptr(), ws.data_ptr(), nbytes, stream)
    else:
        gated_delta_rule(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), b, t, h,
                         state.data_ptr(), o.data_ptr(), stream)
    torch.cuda.synchronize()
    s0 = np.zeros((d, d), np.float32)
    for bi, hi in ((0, 0), (29, 7), (63, 15)):
        host = lambda x: x[bi, :, hi].cpu().numpy()
        exp_o, exp_s = oracle_mod.gated_delta_rule(host(q), host(k), host(v), host(g), host(beta), s0)
        assert rel_err(o[bi, :, hi].cpu().numpy(), exp_o) < 1e-4, (bi, hi)
        assert rel_err(state[bi, hi].cpu().numpy(), exp_s) < 1e-4, (bi, hi)
