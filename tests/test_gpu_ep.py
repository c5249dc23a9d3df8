"""Expert parallelism (osm_b200.ep: the exchange over NVLink peer memory,
osm_ep_forward): each rank owns E/N of the experts and routes T/N of the
tokens; ids match the oracle exactly and outputs agree with the fp32 oracle
within the prefill bound (2e-3, max|a-b| / max|b| per token), for a layer
with a shared expert (Qwen3-Next) and one without (Qwen3-30B-A3B), over two
consecutive calls (the receive slots are reused).  One rank runs the same
code on one GPU; two ranks need two visible GPUs (skipped otherwise).

A rank that skips a step: the other rank's device barriers give up after the
block's timeout (300 ms here) and its status word reports bit 7; the skipping
rank stays alive and joins the host barrier afterwards, so no mapped block
goes away while a peer can still write to it.  NVLS is off in NCCL."""
import os
import sys

import numpy as np
import pytest

from gpu_util import require_cuda

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
H, E, I, K, T, SEED = 256, 16, 256, 4, 160, 61


def _worker(rank, world, port, q, with_shared, skip_rank=-1):
    sys.path[:0] = [HERE, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "orbi-streammoe_b200")]
    import torch
    import torch.distributed as dist

    import osm_b200 as osm
    import pyoracle
    from osm_b200 import ep

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        port_o = pyoracle.Oracle("port")
        slots = np.stack([port_o.gen_expert_slot(SEED, 100 + 3 * e, 0.02, H, I) for e in range(E)])
        shared = port_o.gen_expert_slot(SEED, 90, 0.02, H, I)
        W = pyoracle.bf16_widen(port_o.bf16_round(port_o.gen_normal(SEED, 6, 0.02, E * H))).reshape(E, H)
        sg = pyoracle.bf16_widen(port_o.bf16_round(port_o.gen_normal(SEED, 7, 0.02, H)))
        x_all = port_o.gen_normal(SEED, 1, 1.0, T * H).reshape(T, H)
        e_count, t_count = E // world, T // world
        e0, t0 = rank * e_count, rank * t_count
        ctx = osm.Context(rank, max_tokens=ep.context_rows(world, t_count, K))
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        lay = osm.expert_layout(H, I)
        slab = osm.Slab(ctx, lay, e_count + (1 if with_shared else 0))
        pinned = torch.from_numpy(np.ascontiguousarray(slots[e0:e0 + e_count]).reshape(-1)).pin_memory()
        for e in range(e_count):
            slab.fill_async(e, pinned.data_ptr() + e * lay.stride)
        slab.fill_wait()
        timeout = 300 if skip_rank >= 0 else 2000
        if with_shared:
            moe = ep.ExpertParallelMoE(ctx, W, K, True, lay, slab, e0, e_count, shared, sg,
                                       tokens_per_rank=t_count, timeout_ms=timeout)
        else:
            moe = ep.ExpertParallelMoE(ctx, W, K, True, lay, slab, e0, e_count,
                                       tokens_per_rank=t_count, timeout_ms=timeout)
        x = torch.from_numpy(x_all[t0:t0 + t_count]).cuda()
        out = torch.empty(t_count, H, device="cuda")
        if skip_rank >= 0:
            if rank != skip_rank:
                moe.forward(x, out)
                torch.cuda.synchronize()
            q.put((rank, ctx.status()[0]))
            moe.close()
            return
        moe.forward(torch.zeros_like(x), out)   # a first call: the slots are reused below
        ids, _ = moe.forward(x, out)
        torch.cuda.synchronize()
        o, ih = out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32)
        deq = {}
        sh = port_o.dequant_slot(shared, H, I) if with_shared else None
        worst, ids_ok = 0.0, True
        for t in range(t_count):
            xt = x_all[t0 + t]
            _, rids, _, _ = port_o.route_qwen_top_k(xt, W, K, True)
            ids_ok &= bool(np.array_equal(ih[t], rids))
            for e in rids:
                if int(e) not in deq:
                    deq[int(e)] = port_o.dequant_slot(slots[int(e)], H, I)
            ref = port_o.moe_token(xt, W, K, True, {int(e): deq[int(e)] for e in rids}, shared=sh,
                                   scalar_gate=sg if with_shared else None)[0]
            worst = max(worst, float(np.abs(o[t] - ref).max()) / float(np.abs(ref).max()))
        q.put((rank, ids_ok, worst, ctx.status()[0]))
        moe.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("with_shared", [True, False])
def test_ep_ranks_match_oracle(world, with_shared):
    torch = require_cuda()
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = 29800 + os.getpid() % 100 + 2 * world + (1 if with_shared else 0)
    procs = [mpc.Process(target=_worker, args=(r, world, port, q, with_shared)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, ids_ok, worst, status in res:
        assert ids_ok, rank
        assert worst <= 2e-3, (rank, worst)
        assert status == 0, (rank, status)


def test_ep_rank_that_skips_a_step_times_out():
    torch = require_cuda()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = 29900 + os.getpid() % 90
    procs = [mpc.Process(target=_worker, args=(r, 2, port, q, True, 1)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert res[0][1] & (1 << 7), res   # rank 0 saw its barriers give up
    assert res[1][1] == 0, res


@pytest.mark.parametrize("with_extra", [True, False])
def test_gather_sum_rows_equals_the_torch_sum(with_extra):
    """osm_gather_sum_rows (the return step of the exchange) gives the bits of
    the torch path: rows gathered by position, summed in pick order in fp32,
    then the extra row."""
    torch = require_cuda()
    import osm_b200 as osm

    T, k, Hh = 300, 5, 512
    g = torch.Generator().manual_seed(7)
    rows = torch.randn(T * k, Hh, generator=g).half().cuda()
    pos = torch.randperm(T * k, generator=g).cuda()
    extra = torch.randn(T, Hh, generator=g).half().cuda() if with_extra else None
    ctx = osm.Context(0, max_tokens=8)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    out = torch.empty(T, Hh, device="cuda")
    ctx.gather_sum_rows(rows, pos, T, k, out, extra=extra)
    y = rows.index_select(0, pos).view(T, k, Hh)
    ref = y[:, 0].float()
    for p in range(1, k):
        ref = ref + y[:, p].float()
    if with_extra:
        ref = ref + extra.float()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
