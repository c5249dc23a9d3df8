"""The HBM expert cache on the GPU: two layers share a slab smaller than their
experts; each call routes, acquires its picks (copying misses from pinned host
memory, evicting by use count and recency) and runs the experts.  Outputs match
the oracle, the counts match the Python policy model, and every load moved one
slot of bytes host to device (the streaming mechanism of configs[4])."""
import numpy as np
import pytest

from gpu_util import MoeFixture, normwise_rel, require_cuda
from test_cache_policy import Model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


def test_cache_streams_experts_into_a_small_slab(torch):
    import osm_b200 as osm

    H, E, I, K, SLOTS = 256, 16, 128, 4, 6
    fx = [MoeFixture(torch, H, E, I, K, seed=70 + l) for l in range(2)]
    lay = osm.expert_layout(H, I)
    ctx = osm.Context(0, max_tokens=4)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    slab = osm.Slab(ctx, lay, SLOTS)
    pinned = [torch.from_numpy(np.ascontiguousarray(f.slots).reshape(-1)).pin_memory() for f in fx]
    layers = []
    for f in fx:
        L = osm.Layer(ctx, f.W, K, True, shared_slot=f.shared_slot, shared_layout=lay,
                      shared_gate=f.sg)
        L.bind_slab(slab, np.full(E, -1, np.int32))
        layers.append(L)
    cache = osm.ExpertCache(slab, SLOTS * lay.stride,
                            source=lambda l, e: pinned[l].data_ptr() + e * lay.stride)
    for l, L in enumerate(layers):
        cache.bind_layer(l, L)
    model = Model(SLOTS * lay.stride, lay.stride)
    for step in range(10):
        for l, (f, L) in enumerate(zip(fx, layers)):
            x = f.port.gen_normal(80 + l, step, 1.0, H).reshape(1, H)
            xd = torch.from_numpy(x).cuda()
            ids = torch.empty(1, K, dtype=torch.int32, device="cuda")
            w = torch.empty(1, K, device="cuda")
            L.route_qwen_top_k(xd, 1, ids, w)
            picks = ids.cpu().numpy().astype(np.uint32).reshape(-1)
            cache.acquire(l, picks)
            model.acquire(l, [int(e) for e in picks])
            out = torch.empty(1, H, device="cuda")
            L.run_experts(xd, 1, ids, w, out)
            torch.cuda.synchronize()
            ref, rids, _, _, _ = f.oracle_token(x[0])
            assert np.array_equal(picks, rids)
            assert normwise_rel(out.cpu().numpy()[0], ref) <= 1e-4
    s = cache.stats()
    assert s == model.stats()
    assert s["evictions"] > 0 and s["hits"] > 0
    assert osm.lib().osm_slab_h2d_bytes(slab.h) == s["loads"] * lay.stride
    assert ctx.status()[0] == 0
    cache.close()


@pytest.mark.parametrize("E,SLOTS,B", [(16, 6, 1), (24, 13, 3)])
def test_cached_forward_matches_oracle_and_policy(torch, E, SLOTS, B):
    """osm_moe_forward_cached (run_qwen_sparse_moe_vulkan_accum with its cache)
    in one call per layer: routing, the picks' residency and the experts.
    Outputs and ids match the oracle; the cache counts match the policy model
    acquiring each call's picks in token-major order; each load moved one
    slot of bytes."""
    import osm_b200 as osm

    H, I, K = 256, 128, 4
    fx = [MoeFixture(torch, H, E, I, K, seed=170 + l, max_tokens=B) for l in range(2)]
    lay = osm.expert_layout(H, I)
    ctx = osm.Context(0, max_tokens=B)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    slab = osm.Slab(ctx, lay, SLOTS)
    pinned = [torch.from_numpy(np.ascontiguousarray(f.slots).reshape(-1)).pin_memory() for f in fx]
    layers = []
    for f in fx:
        L = osm.Layer(ctx, f.W, K, True, shared_slot=f.shared_slot, shared_layout=lay,
                      shared_gate=f.sg)
        L.bind_slab(slab, np.full(E, -1, np.int32))
        layers.append(L)
    cache = osm.ExpertCache(slab, SLOTS * lay.stride,
                            source=lambda l, e: pinned[l].data_ptr() + e * lay.stride)
    for l, L in enumerate(layers):
        cache.bind_layer(l, L)
    model = Model(SLOTS * lay.stride, lay.stride)
    for step in range(8):
        for l, (f, L) in enumerate(zip(fx, layers)):
            x = f.port.gen_normal(180 + l, step, 1.0, B * H).reshape(B, H)
            xd = torch.from_numpy(x).cuda()
            ids = torch.empty(B, K, dtype=torch.int32, device="cuda")
            out = torch.empty(B, H, device="cuda")
            L.run_cached(cache, l, xd, B, out, ids=ids)
            torch.cuda.synchronize()
            got_ids = ids.cpu().numpy().astype(np.uint32)
            model.acquire(l, [int(e) for e in got_ids.reshape(-1)])
            o = out.cpu().numpy()
            for t in range(B):
                ref, rids, _, _, _ = f.oracle_token(x[t])
                assert np.array_equal(got_ids[t], rids)
                assert normwise_rel(o[t], ref) <= 1e-4
    s = cache.stats()
    assert s == model.stats()
    assert s["evictions"] > 0 and s["hits"] > 0
    assert osm.lib().osm_slab_h2d_bytes(slab.h) == s["loads"] * lay.stride
    assert ctx.status()[0] == 0
    cache.close()


@pytest.mark.parametrize("B", [1, 2])
def test_cached_forward_early_experts_match_the_ordinary_call(torch, B):
    """OSM_CACHED_EARLY: the one/two-token expert kernels are queued behind the
    router before the host has the picks and resolve them through the slot
    table as it stands; a call whose picks were all resident keeps that
    output, a call with a miss runs them again behind the copies.  Over a
    stream with hits, misses and evictions (two layers through a small slab),
    every output is bit-identical to the ordinary cached call's, the cache
    counts equal the policy model's, and the context status stays clean (the
    early run's non-resident picks go to a side word)."""
    import osm_b200 as osm

    H, I, K, E, SLOTS = 512, 256, 4, 20, 8
    fx = [MoeFixture(torch, H, E, I, K, seed=210 + l, max_tokens=B) for l in range(2)]
    lay = osm.expert_layout(H, I)
    runs = []
    for early in (False, True):
        ctx = osm.Context(0, max_tokens=B)
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        slab = osm.Slab(ctx, lay, SLOTS)
        pinned = [torch.from_numpy(np.ascontiguousarray(f.slots).reshape(-1)).pin_memory()
                  for f in fx]
        layers = []
        for f in fx:
            L = osm.Layer(ctx, f.W, K, True, shared_slot=f.shared_slot, shared_layout=lay,
                          shared_gate=f.sg)
            L.bind_slab(slab, np.full(E, -1, np.int32))
            layers.append(L)
        cache = osm.ExpertCache(slab, SLOTS * lay.stride,
                                source=lambda l, e, p=pinned: p[l].data_ptr() + e * lay.stride)
        for l, L in enumerate(layers):
            cache.bind_layer(l, L)
        model = Model(SLOTS * lay.stride, lay.stride)
        outs = []
        for step in range(12):
            for l, (f, L) in enumerate(zip(fx, layers)):
                x = f.port.gen_normal(220 + l, step, 1.0, B * H).reshape(B, H)
                xd = torch.from_numpy(x).cuda()
                ids = torch.empty(B, K, dtype=torch.int32, device="cuda")
                out = torch.empty(B, H, device="cuda")
                L.run_cached(cache, l, xd, B, out, ids=ids, early=early)
                torch.cuda.synchronize()
                got_ids = ids.cpu().numpy().astype(np.uint32)
                model.acquire(l, [int(e) for e in got_ids.reshape(-1)])
                outs.append(out.cpu().numpy())
                if step % 4 == 0:
                    for t in range(B):
                        ref, rids, _, _, _ = f.oracle_token(x[t])
                        assert np.array_equal(got_ids[t], rids)
                        assert normwise_rel(outs[-1][t], ref) <= 1e-4
        s = cache.stats()
        assert s == model.stats()
        assert s["evictions"] > 0 and s["hits"] > 0
        assert ctx.status()[0] == 0
        cache.close()
        runs.append(outs)
    for a, b in zip(*runs):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_cached_forward_rejects_an_unbound_layer(torch):
    import osm_b200 as osm

    H, E, I, K = 256, 8, 128, 2
    f = MoeFixture(torch, H, E, I, K, seed=190, max_tokens=1)
    lay = osm.expert_layout(H, I)
    slab = osm.Slab(f.ctx, lay, 4)
    L = osm.Layer(f.ctx, f.W, K, True)
    L.bind_slab(slab, np.full(E, -1, np.int32))
    cache = osm.ExpertCache(slab, 4 * lay.stride, source=lambda l, e: f.pinned.data_ptr())
    x = torch.zeros(1, H, device="cuda")
    out = torch.empty(1, H, device="cuda")
    with pytest.raises(osm.OsmError):
        L.run_cached(cache, 0, x, 1, out)   # layer 0 was never bound to the cache
    cache.bind_layer(0, L)
    with pytest.raises(osm.OsmError):
        L.run_cached(cache, 1, x, 1, out)   # bound as 0, called as 1
    L.run_cached(cache, 0, x, 1, out)
    torch.cuda.synchronize()
    assert cache.stats()["loads"] == K
    cache.close()


def test_failing_source_mid_acquire_keeps_slab_and_slot_table_consistent(torch):
    """A slab-backed cache whose host source fails on the third pick of an
    acquire: the first two picks are copied and bound, the failing expert is
    neither bound nor resident and frees or evicts nothing, and a later call
    with a working source loads it and computes the right output."""
    import osm_b200 as osm

    H, E, I, K, SLOTS = 256, 8, 128, 4, 4
    f = MoeFixture(torch, H, E, I, K, seed=191, max_tokens=1)
    lay = osm.expert_layout(H, I)
    slab = osm.Slab(f.ctx, lay, SLOTS)
    L = osm.Layer(f.ctx, f.W, K, True, shared_slot=f.shared_slot, shared_layout=lay,
                  shared_gate=f.sg)
    L.bind_slab(slab, np.full(E, -1, np.int32))
    broken = {6}

    def source(layer, expert):
        if expert in broken:
            raise RuntimeError("storage read failed")
        return f.pinned.data_ptr() + expert * lay.stride

    cache = osm.ExpertCache(slab, SLOTS * lay.stride, source=source)
    cache.bind_layer(0, L)
    model = Model(SLOTS * lay.stride, lay.stride)
    cache.acquire(0, [0, 1, 2, 3])
    model.acquire(0, [0, 1, 2, 3])
    with pytest.raises(osm.OsmError) as e:
        cache.acquire(0, [4, 5, 6])
    assert e.value.code == -2
    with pytest.raises(RuntimeError):
        model.acquire(0, [4, 5, 6], failing=broken)
    assert cache.stats() == model.stats()
    resident = [e for e in range(E) if cache.contains(0, e)]
    assert sorted(resident) == [2, 3, 4, 5]
    # the device slot table agrees with the policy: the resident experts give
    # the bits of the fully resident fixture layer, and a routing to 6 is
    # reported as not resident
    x = f.port.gen_normal(192, 0, 1.0, H).reshape(1, H)
    xd = torch.from_numpy(x).cuda()
    w = torch.full((1, K), 0.25, device="cuda")
    ids = torch.tensor([resident], dtype=torch.int32, device="cuda")
    out = torch.empty(1, H, device="cuda")
    ref = torch.empty(1, H, device="cuda")
    L.run_experts(xd, 1, ids, w, out)
    f.layer.run_experts(xd, 1, ids, w, ref)
    torch.cuda.synchronize()
    assert f.ctx.status()[0] == 0
    assert torch.equal(out, ref)
    L.run_experts(xd, 1, torch.tensor([[2, 3, 4, 6]], dtype=torch.int32, device="cuda"), w, out)
    torch.cuda.synchronize()
    assert f.ctx.status()[0] & 4
    # with the source working again the expert loads and routes normally
    broken.clear()
    ids = torch.empty(1, K, dtype=torch.int32, device="cuda")
    L.route_qwen_top_k(xd, 1, ids, w)
    picks = ids.cpu().numpy().astype(np.uint32).reshape(-1)
    cache.acquire(0, [6])
    assert cache.contains(0, 6)
    cache.acquire(0, picks)
    L.run_experts(xd, 1, ids, w, out)
    torch.cuda.synchronize()
    rout, rids, _, _, _ = f.oracle_token(x[0])
    assert np.array_equal(picks, rids)
    assert normwise_rel(out.cpu().numpy()[0], rout) <= 1e-4
    assert f.ctx.status()[0] == 0
    cache.close()


def test_slab_fill_wait_times_out_on_a_pending_fill(torch):
    """osm_slab_fill_wait with a 0 ms limit on a fill that cannot have landed
    (the context stream is held by a bounded spin that the fill is ordered
    after) returns OSM_ETIMEOUT; a longer limit then returns OK."""
    import osm_b200 as osm

    H, I = 256, 128
    lay = osm.expert_layout(H, I)
    ctx = osm.Context(0, max_tokens=1)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    slab = osm.Slab(ctx, lay, 2)
    host = torch.zeros(lay.stride, dtype=torch.uint8).pin_memory()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(400_000_000)   # a bounded spin, ~0.2 s at 1.9 GHz
    slab.fill_async(0, host.data_ptr())
    with pytest.raises(osm.OsmError) as e:
        slab.fill_wait(0)
    assert e.value.code == -6            # OSM_ETIMEOUT
    slab.fill_wait(10_000)
    stream.synchronize()
    slab.close()
    ctx.close()
