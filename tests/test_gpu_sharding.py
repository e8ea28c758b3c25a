"""Request sharding on two GPUs (one engine per device, no collective on the
data path): the same seeded request set, split over two engines by
decider_gpu.sharding.shard_requests (longest processing time first), gives
every request the logits, bit for bit in reference order, that one engine on
one device gives the whole set; the second device's engine runs two lanes.
Needs two GPUs; skipped on fewer."""
import numpy as np
import pytest

from model_util import random_tensors, small_config

pytestmark = pytest.mark.gpu


def test_sharded_requests_on_two_devices_match_one_device():
    import torch

    from decider_gpu import GpuModel
    from decider_gpu.sharding import RequestShape, request_cost, shard_requests
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = small_config()
    tensors = random_tensors(cfg, rank=32, pointer_dim=64, seed=51)

    def engine(device):
        m = GpuModel(cfg, "int8-compute", 32, 2.0, 64, device, 1024)
        m.set_tensors(tensors)
        m.finalize()
        m.set_exact(True)
        return m

    rng = np.random.default_rng(52)
    reqs = []
    for i in range(17):
        q = int(rng.integers(1, 4))
        L = int(rng.integers(40, 600))
        qs = [(rng.integers(0, cfg["vocab_size"], 32), [5, 9, 20]) for _ in range(q)]
        reqs.append({"state": rng.integers(0, cfg["vocab_size"], L), "questions": qs} if q > 1 else {"questions": qs})
    shapes = [RequestShape(len(r.get("state", ())), tuple(len(x[0]) for x in r["questions"])) for r in reqs]
    plan = shard_requests([request_cost(s) for s in shapes], 2)
    assert sorted(i for p in plan for i in p) == list(range(len(reqs))) and all(plan)
    one, st, _, err = engine(0).logits_batch(reqs)
    assert not st.any(), err
    engines = [engine(0), engine(1)]
    engines[1].set_lanes(2)  # lanes on a device other than the current one
    for rank, idx in enumerate(plan):
        got, st, _, err = engines[rank].logits_batch([reqs[i] for i in idx])
        assert not st.any(), err
        for j, i in enumerate(idx):
            for a, b in zip(got[j], one[i]):
                assert np.array_equal(a, b), (rank, i)
