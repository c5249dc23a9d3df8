"""GPU parity on exactly the workloads bench.py times, through the C ABI.

* the Qwen3-Next sublayer (bench seeds, all 512 experts, Zipf(1.1)
  router bias) at every sweep batch B = 1, 8, 32, 64, 128, 256: every token's
  ids bit-exact against the oracle, weights within 1e-5 relative, outputs
  within 1e-4 normwise relative error (max|a-b| / max|b| per token).
* 4096 prefill tokens, no router bias, the tensor-core path: all
  4096 routings bit-exact, 64 tokens spread over the batch within 2e-3.
* The certified one/two-token router (the path of configs[0], of B = 1 in the
  sweep and of every configs[4] call): 2,000+ single- and two-token calls with
  and without the Zipf bias, plus constructed near-ties (router rows one bf16
  ulp apart; inputs moved so that the k-th and (k+1)-th logits nearly meet),
  every id bit-exact against route_qwen_top_k_cpu (src/model/qwen_router.cpp:
  11-94) compiled in place when available, else its C restatement.
* An fp32 router that is not bf16-representable (a Q8-dequantised checkpoint
  router, src/model/checkpoint_sparse_moe.cpp:159-162) at H 2048, E 512.

The oracle runs token-parallel on host threads (ctypes releases the GIL).
"""
import ctypes
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import pyoracle
from gpu_util import normwise_rel, require_cuda

pytestmark = pytest.mark.gpu

H, E, I, K = 2048, 512, 512, 10
THREADS = max(1, min(32, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


@pytest.fixture(scope="module")
def router_oracle():
    """route_qwen_top_k_cpu as the reference compiled it, when present."""
    return pyoracle.Oracle("reference") if pyoracle.ref_available() else pyoracle.Oracle("port")


@pytest.fixture(scope="module")
def q3n(torch):
    """The bench's own configs[1]/[2] sublayer (bench.build_sublayer), and its
    expert slots copied to the host for the oracle."""
    import bench
    import osm_b200 as osm

    ctx = osm.Context(0, max_tokens=bench.PF_T)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    layer_b, slab, W, sg, bias, shared = bench.build_sublayer(torch, ctx, osm, zipf=True)
    lay = osm.expert_layout(H, I)
    layer_u = osm.Layer(ctx, W, K, True, shared_slot=shared, shared_layout=lay, shared_gate=sg)
    layer_u.bind_slab(slab, np.arange(E, dtype=np.int32))
    ctx.synchronize()
    slots = np.zeros((E, lay.stride), np.uint8)
    ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(slots.ctypes.data),
                                     ctypes.c_void_p(slab.slot_ptr(0)), E * lay.stride))

    class NS:
        pass

    ns = NS()
    ns.ctx, ns.slab, ns.layer_b, ns.layer_u = ctx, slab, layer_b, layer_u
    ns.W, ns.sg, ns.bias, ns.shared, ns.slots, ns.bench = W, sg, bias, shared, slots, bench
    return ns


def _oracle_tokens(port, q, x, rows, bias):
    def one(t):
        return port.moe_token_slots(x[t], q.W, K, True, q.slots, I, shared_slot=q.shared,
                                    scalar_gate=q.sg, bias=bias)

    with ThreadPoolExecutor(THREADS) as ex:
        return list(ex.map(one, rows))


def _route_tokens(orc, W, x, rows, bias, k=K):
    def one(t):
        return orc.route_qwen_top_k(x[t], W, k, True, bias=bias)

    with ThreadPoolExecutor(THREADS) as ex:
        return list(ex.map(one, rows))


@pytest.mark.parametrize("B", [1, 8, 32, 64, 128, 256])
def test_decode_sweep_batches_every_token(torch, q3n, port, B):
    """configs[1] at the bench's own inputs (x = gen_normal(SEED, 5000 + B))."""
    ctx = q3n.ctx
    x = torch.empty(B, H, device="cuda")
    ctx.gen_normal(q3n.bench.SEED, 5000 + B, 1.0, x)
    out = torch.empty(B, H, device="cuda")
    ids = torch.empty(B, K, dtype=torch.int32, device="cuda")
    w = torch.empty(B, K, device="cuda")
    sgo = torch.empty(B, device="cuda")
    q3n.layer_b.run_qwen_sparse_moe(x, B, out, ids=ids, weights=w, shared_gate=sgo)
    torch.cuda.synchronize()
    assert ctx.status()[0] == 0
    xh = x.cpu().numpy()
    got, gids, gw, gsg = (out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32), w.cpu().numpy(),
                          sgo.cpu().numpy())
    refs = _oracle_tokens(port, q3n, xh, range(B), q3n.bias)
    worst = 0.0
    for t, (ref, rids, rw, _, rs) in enumerate(refs):
        assert np.array_equal(gids[t], rids), (B, t, gids[t], rids)
        np.testing.assert_allclose(gw[t], rw, rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(gsg[t], rs, rtol=1e-5, atol=1e-7)
        err = normwise_rel(got[t], ref)
        worst = max(worst, err)
        assert err <= 1e-4, (B, t, err)
        assert float(np.abs(got[t] - ref).max()) <= 0.03  # the reference's own gate
    print(f"B={B}: worst normwise error {worst:.3e}")


def test_prefill_4096_tokens_full_size(torch, q3n, port, router_oracle):
    """configs[2] at full size on the tensor-core path (x = gen_normal(SEED,
    7000), 4096 x 2048, no router bias): every routing bit-exact, 64 tokens
    spread over the batch within 2e-3 of the oracle."""
    T = q3n.bench.PF_T
    ctx = q3n.ctx
    x = torch.empty(T, H, device="cuda")
    ctx.gen_normal(q3n.bench.SEED, 7000, 1.0, x)
    out = torch.empty(T, H, device="cuda")
    ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
    w = torch.empty(T, K, device="cuda")
    q3n.layer_u.run_qwen_sparse_moe(x, T, out, ids=ids, weights=w, prefill=True)
    torch.cuda.synchronize()
    assert ctx.status()[0] == 0
    xh = x.cpu().numpy()
    gids = ids.cpu().numpy().astype(np.uint32)
    gw = w.cpu().numpy()
    routes = _route_tokens(router_oracle, q3n.W, xh, range(T), None)
    for t, (_, rids, rw, _) in enumerate(routes):
        assert np.array_equal(gids[t], rids), (t, gids[t], rids)
        np.testing.assert_allclose(gw[t], rw, rtol=1e-5, atol=1e-7)
    rows = list(range(0, T, T // 64))
    got = out.cpu().numpy()
    worst = 0.0
    for t, (ref, rids, _, _, _) in zip(rows, _oracle_tokens(port, q3n, xh, rows, None)):
        assert np.array_equal(gids[t], rids)
        err = normwise_rel(got[t], ref)
        worst = max(worst, err)
        assert err <= 2e-3, (t, err)
    print(f"prefill 4096: worst normwise error {worst:.3e} over {len(rows)} tokens")


def _single_calls(torch, layer, x, widths):
    """Route x in calls of `widths[i]` tokens each (1 or 2: the certified
    path), one call per slice, outputs gathered."""
    n = x.shape[0]
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    ids = torch.empty(n, K, dtype=torch.int32, device="cuda")
    w = torch.empty(n, K, device="cuda")
    t = 0
    i = 0
    while t < n:
        b = min(widths[i % len(widths)], n - t)
        layer.route_qwen_top_k(xd[t:t + b], b, ids[t:t + b], w[t:t + b])
        t += b
        i += 1
    torch.cuda.synchronize()
    return ids.cpu().numpy().astype(np.uint32), w.cpu().numpy()


def _check_routes(orc, W, x, bias, gids, gw):
    for t, (_, rids, rw, _) in enumerate(_route_tokens(orc, W, x, range(x.shape[0]), bias)):
        assert np.array_equal(gids[t], rids), (t, gids[t], rids)
        np.testing.assert_allclose(gw[t], rw, rtol=1e-5, atol=1e-7)


def test_certified_router_thousands_of_single_token_calls(torch, q3n, port, router_oracle):
    """2,400 one- and two-token calls at Q3N, with and without the Zipf bias."""
    n = 1200
    x = port.gen_normal(4242, 1, 1.0, n * H).reshape(n, H)
    total_exact = 0
    for layer, bias in ((q3n.layer_b, q3n.bias), (q3n.layer_u, None)):
        q3n.ctx.status()
        gids, gw = _single_calls(torch, layer, x, (1, 2, 1))
        st, ex = q3n.ctx.status()
        assert st == 0
        _check_routes(router_oracle, q3n.W, x, bias, gids, gw)
        total_exact += ex
    print(f"certified router: {2 * n} tokens, {total_exact} on the exact path")


def test_certified_router_constructed_near_ties(torch, q3n, port, router_oracle):
    """Inputs built to sit inside the certification bound: (1) the k-th and
    (k+1)-th logits of the oracle moved together along W[a] - W[b] until their
    gap is ~1e-6 of its size; (2) router rows one bf16 ulp apart pulled to the
    top of the ranking.  Every id stays bit-exact; these tokens go to the
    exact path."""
    import osm_b200 as osm

    rng = np.random.default_rng(77)
    W, bias = q3n.W, q3n.bias
    n = 200
    x = port.gen_normal(4243, 1, 1.0, n * H).reshape(n, H).astype(np.float64)
    for t in range(n):
        logits, rids, _, _ = router_oracle.route_qwen_top_k(x[t].astype(np.float32), W, K + 1,
                                                            True, bias=bias)
        a, b = int(rids[K - 1]), int(rids[K])
        d = W[a].astype(np.float64) - W[b].astype(np.float64)
        gap = float(logits[a]) - float(logits[b])
        x[t] -= (gap * (1.0 - 1e-6) / float(d @ d)) * d
    x = x.astype(np.float32)
    q3n.ctx.status()
    gids, gw = _single_calls(torch, q3n.layer_b, x, (1, 2))
    st, ex = q3n.ctx.status()
    assert st == 0
    _check_routes(router_oracle, W, x, bias, gids, gw)
    assert ex >= n // 2, ex  # the near-ties were sent to the exact path

    # (2) pairs of rows one bf16 ulp apart
    Wt = W.copy()
    pairs = []
    for p in range(24):
        i, j = 2 * p + 7, 2 * p + 300
        Wt[j] = Wt[i]
        m = int(rng.integers(H))
        bits = Wt[j, m:m + 1].view(np.uint32)
        bits += np.uint32(1 << 16)   # one bf16 ulp up
        pairs.append((i, j))
    ctx = osm.Context(0, max_tokens=2)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    layer = osm.Layer(ctx, Wt, K, True)
    m = 240
    xt = port.gen_normal(4244, 2, 1.0, m * H).reshape(m, H).astype(np.float64)
    for t in range(m):
        i, _ = pairs[t % len(pairs)]
        r = Wt[i].astype(np.float64)
        xt[t] += (6.0 / float(r @ r)) * r   # expert i and its twin lead by ~6
    xt = xt.astype(np.float32)
    gids, gw = _single_calls(torch, layer, xt, (1, 2))
    st, ex = ctx.status()
    assert st == 0
    _check_routes(router_oracle, Wt, xt, None, gids, gw)
    print(f"near ties: gap-closed {n} tokens ({ex} exact of the twins' {m})")


def _q8_dequantised_router(port, seed):
    """A router as a Q8 checkpoint delivers it after dequantisation: per row
    and group of 64, affine 8-bit (scale = range/255, bias = min) with fp32
    scale and bias, w = scale * q + bias rounded after each operation
    (cpu::dequantize_affine_rows with bits = 8, src/cpu/reference_ops.cpp:
    11-67).  The values are not bf16-representable."""
    w = port.gen_normal(seed, 1, 0.02, E * H).reshape(E * H // 64, 64)
    lo = w.min(axis=1, keepdims=True)
    hi = w.max(axis=1, keepdims=True)
    scale = ((hi - lo) / np.float32(255)).astype(np.float32)
    q = np.clip(np.rint((w - lo) / scale), 0, 255).astype(np.float32)
    deq = (scale * q).astype(np.float32) + lo
    deq = deq.astype(np.float32).reshape(E, H)
    assert np.any(deq.view(np.uint32) & 0xFFFF)
    return deq


def test_fp32_router_full_size(torch, port, router_oracle):
    """H 2048, E 512, top-10 with an fp32 (Q8-dequantised) router: 256 tokens
    in one call (the exact kernel on fp32 tiles) and 300 tokens in one- and
    two-token calls (the certified kernel on fp32 rows), ids bit-exact."""
    import osm_b200 as osm

    W = _q8_dequantised_router(port, 515)
    ctx = osm.Context(0, max_tokens=256)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    layer = osm.Layer(ctx, W, K, True)
    n = 256
    x = port.gen_normal(516, 1, 1.0, n * H).reshape(n, H)
    xd = torch.from_numpy(x).cuda()
    ids = torch.empty(n, K, dtype=torch.int32, device="cuda")
    w = torch.empty(n, K, device="cuda")
    layer.route_qwen_top_k(xd, n, ids, w)
    torch.cuda.synchronize()
    assert ctx.status()[0] == 0
    _check_routes(router_oracle, W, x, None, ids.cpu().numpy().astype(np.uint32), w.cpu().numpy())
    m = 300
    xs = port.gen_normal(517, 1, 1.0, m * H).reshape(m, H)
    gids, gw = _single_calls(torch, layer, xs, (1, 2))
    assert ctx.status()[0] == 0
    _check_routes(router_oracle, W, xs, None, gids, gw)
