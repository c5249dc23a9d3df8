"""Expert-parallel dispatch and combine (osm_b200.ep) on gloo ranks on the CPU:
pairs sorted by owner rank, rows and (local expert, weight) exchanged, a stand-in
expert applied on the owner, rows returned and summed per token in pick order.
With float32 rows the result equals a single-process computation exactly, for
even, skewed and empty destinations."""
import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "orbi-streammoe_b200"))

H, E, K = 16, 8, 3


def expert_mats():
    g = torch.Generator().manual_seed(5)
    return torch.randn(E, H, H, generator=g)


def make_inputs(rank, T, skew):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g)
    if skew == "one_rank":
        ids = torch.randint(0, E // 2, (T, K), generator=g)          # every pick on rank 0
    else:
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g)
    return x, ids.to(torch.int32), w


def reference(x, ids, w, M):
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        acc = None
        for p in range(K):
            y = w[t, p] * (x[t] @ M[int(ids[t, p])])
            acc = y if acc is None else acc + y
        out[t] = acc
    return out


def worker(rank, world, port, T, skew, q):
    from osm_b200 import ep

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M = expert_mats()
        e_local = E // world
        x, ids, w = make_inputs(rank, T, skew)
        rx, rid, rw, state = ep.dispatch_rows(x, ids, w, e_local, world, row_dtype=torch.float32)
        y = torch.empty_like(rx)
        for j in range(rx.shape[0]):
            y[j] = rw[j] * (rx[j] @ M[rank * e_local + int(rid[j])])
        got = ep.combine_rows(y, state, row_dtype=torch.float32)
        want = reference(x, ids, w, M)
        q.put((rank, bool(torch.equal(got, want)), int(rx.shape[0])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("skew", ["spread", "one_rank"])
def test_dispatch_combine_matches_single_process(skew):
    world, T = 2, 13
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    port = 29400 + (os.getpid() % 500) + (7 if skew == "one_rank" else 0)
    procs = [ctxm.Process(target=worker, args=(r, world, port, T, skew, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    res = sorted(q.get(timeout=5) for _ in range(world))
    assert all(ok for _, ok, _ in res), res
    if skew == "one_rank":
        assert res[1][2] == 0 and res[0][2] == world * T * K   # rank 1 received nothing


def test_dispatch_plan_orders_by_owner():
    from osm_b200 import ep

    ids = torch.tensor([[5, 0, 2], [1, 7, 4]], dtype=torch.int32)
    order, counts, local = ep.dispatch_plan(ids, 4, 2)
    assert counts.tolist() == [3, 3]
    owners = (ids.reshape(-1).long() // 4)[order]
    assert owners.tolist() == sorted(owners.tolist())
    assert order.tolist() == [1, 2, 3, 0, 4, 5]          # stable inside each owner
    assert local.tolist() == [1, 0, 2, 1, 3, 0]
    with pytest.raises(ValueError):
        ep.dispatch_plan(torch.tensor([[8]], dtype=torch.int32), 4, 2)
