"""Multi-rank host logic on the CPU: request sharding (one replica per rank,
no collective on the data path) checked with world-size-2 gloo process
groups, and the LPT plan's balance and determinism."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from decider_gpu.sharding import RequestShape, request_cost, run_sharded, shard_requests


def _shapes(n, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        q = int(rng.integers(1, 5))
        L = int(rng.integers(128, 4097))
        out.append(RequestShape(prefix=max(L - 64, 0), questions=tuple([64] * q)))
    return out


def test_plan_covers_every_request_once_and_is_deterministic():
    costs = [request_cost(s) for s in _shapes(257, 0)]
    for world in (1, 2, 3, 8):
        plan = shard_requests(costs, world)
        assert sorted(i for p in plan for i in p) == list(range(len(costs)))
        assert plan == shard_requests(list(costs), world)


def test_plan_meets_the_lpt_bound():
    costs = [request_cost(s) for s in _shapes(500, 1)]
    for world in (2, 4, 8):
        plan = shard_requests(costs, world)
        makespan = max(sum(costs[i] for i in p) for p in plan)
        lower = max(sum(costs) / world, max(costs))  # no schedule beats this
        assert makespan <= sum(costs) / world + max(costs)  # list-scheduling bound
        assert makespan <= 1.05 * lower  # LPT on many small jobs is near the optimum


def test_cost_grows_with_the_window():
    short = RequestShape(prefix=64, questions=(64,))
    long = RequestShape(prefix=4032, questions=(64,))
    assert request_cost(long) > request_cost(short) * 10
    # Each forward carries a fixed cost: four questions on a state cost more
    # than one question over the same window.
    many = RequestShape(prefix=1024, questions=(64, 64, 64, 64))
    one = RequestShape(prefix=1024 + 192, questions=(64,))
    assert many.forwards == 5 and one.forwards == 2
    assert request_cost(many) > request_cost(one) + 3 * 250


def _fake_engine(request):
    # Stand-in for a replica's decide call: deterministic in the request.
    return {"id": request["id"], "p": float(np.tanh(request["id"] * 0.37))}


def _worker(rank, world, port, n, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shapes = _shapes(n, 3)
        requests = [{"id": i} for i in range(n)]
        # Every rank derives the same plan without exchanging it.
        plan = shard_requests([request_cost(s) for s in shapes], world)
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        out = run_sharded(requests, shapes, _fake_engine, dist)
        q.put((rank, plans, out))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_gather_answers_in_request_order():
    world, n = 2, 37
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, plans, out = q.get(timeout=120)
        results[rank] = (plans, out)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0][0] == results[1][0]
    assert results[1][1] is None
    serial = [_fake_engine({"id": i}) for i in range(n)]
    assert results[0][1] == serial


def _failing_engine(request):
    if request["id"] == 5:
        raise ValueError("invalid encoding positions or window")
    return _fake_engine(request)


def _failing_worker(rank, world, port, n, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        try:
            out = run_sharded([{"id": i} for i in range(n)], _shapes(n, 3), _failing_engine, dist)
            q.put((rank, "ok", out))
        except RuntimeError as e:
            q.put((rank, "raised", str(e)))
        # Both ranks still agree on the next collective: nobody was left behind.
        t = torch_tensor(rank)
        dist.all_reduce(t)
        q.put((rank, "after", int(t.item())))
    finally:
        dist.destroy_process_group()


def torch_tensor(v):
    import torch
    return torch.tensor([v])


def test_a_failing_request_reaches_rank_0_without_stalling_the_gather():
    """A request that raises on one rank does not keep that rank from the
    gather: the failure travels with the answers, rank 0 re-raises it (naming
    the request), the other rank returns None, and both ranks go on to the
    next collective."""
    world, n = 2, 23
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(2 * world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    by = {(r, kind): v for r, kind, v in got}
    assert by[(0, "raised")].startswith("request 5 failed") and "invalid encoding" in by[(0, "raised")]
    assert by[(1, "ok")] is None
    assert by[(0, "after")] == by[(1, "after")] == 1
