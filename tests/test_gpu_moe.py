"""GPU parity of the router and the full routed-MoE sublayer, through the C ABI,
against the CPU oracle and the reference's own outputs (golden fixtures).

Criteria: top-k expert ids bit-exact (ties to the lower id) on every token;
routing weights and selected mass within 1e-6 (tests/
checkpoint_moe_sublayer_test.cpp:700-711) on the small fixtures and in exact
mode, within 1e-5 relative at hidden 2048 on the fast path; MoE outputs within 1e-4 normwise
relative error (max|a-b| / max|b| per token) and the reference's 0.02/0.03
absolute gates (tests/weighted_routed_moe_test.cpp:352-411,
tests/checkpoint_moe_sublayer_test.cpp:705-706).
"""
import json
import os

import numpy as np
import pytest

import pyoracle
from gpu_util import MoeFixture, normwise_rel, require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


def _route(torch, W, x, k, norm=True, bias=None, exact=False):
    import osm_b200 as osm

    B, H = x.shape
    ctx = osm.Context(0, max_tokens=max(B, 1))
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    layer = osm.Layer(ctx, W, k, norm, logit_bias=bias)
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    ids = torch.empty(B, k, dtype=torch.int32, device="cuda")
    w = torch.empty(B, k, device="cuda")
    m = torch.empty(B, device="cuda")
    layer.route_qwen_top_k(xd, B, ids, w, m, exact=exact)
    torch.cuda.synchronize()
    st, ex = ctx.status()
    return ids.cpu().numpy().astype(np.uint32), w.cpu().numpy(), m.cpu().numpy(), st, ex


def test_router_reference_kats(torch, golden_dir):
    with open(os.path.join(golden_dir, "reference_kats.json")) as f:
        kats = json.load(f)
    for exact in (False, True):
        k = kats["router_2_of_4"]
        W = np.array(k["weight"], np.float32).reshape(4, 1)
        ids, w, m, st, _ = _route(torch, W, np.array([k["hidden"]], np.float32), k["k"], exact=exact)
        assert st == 0
        assert list(ids[0]) == k["expected_ids"]
        np.testing.assert_allclose(w[0], k["expected_norm_weights"], atol=k["tol"])
        assert abs(m[0] - k["expected_mass"]) <= k["tol"]
        ids, w, m, st, _ = _route(torch, W, np.array([k["hidden"]], np.float32), k["k"],
                                  norm=False, exact=exact)
        np.testing.assert_allclose(w[0], k["expected_raw_weights"], atol=k["tol"])
        k = kats["router_tie"]
        W = np.array(k["weight"], np.float32).reshape(4, 1)
        ids, w, m, st, ex = _route(torch, W, np.array([k["hidden"]], np.float32), k["k"], exact=exact)
        assert list(ids[0]) == k["expected_ids"]
        np.testing.assert_allclose(w[0], k["expected_norm_weights"], atol=k["tol"])
        assert ex == 1  # an exact tie is never certified: the exact path decides it
        k = kats["router_512_top10"]
        W = (np.arange(k["experts"], dtype=np.float32) * np.float32(k["weight_step"])).reshape(-1, 1)
        ids, w, m, st, _ = _route(torch, W, np.array([k["hidden"]], np.float32), k["k"], exact=exact)
        assert list(ids[0]) == k["expected_ids"]
        assert abs(float(w[0].sum()) - 1.0) <= k["sum_tol"]


def test_router_rejects_bad_shapes(torch):
    import osm_b200 as osm

    ctx = osm.Context(0, max_tokens=4)
    with pytest.raises(osm.OsmError):
        osm.Layer(ctx, np.ones((4, 8), np.float32), 5)  # top_k > experts
    with pytest.raises(osm.OsmError):
        bad = np.ones((4, 8), np.float32)
        bad[1, 2] = np.inf
        osm.Layer(ctx, bad, 2)  # non-finite router weight (qwen_router.cpp:54-59)
    layer = osm.Layer(ctx, np.ones((4, 8), np.float32), 2)
    xd = torch.zeros(8, 8, device="cuda")
    ids = torch.empty(8, 2, dtype=torch.int32, device="cuda")
    w = torch.empty(8, 2, device="cuda")
    with pytest.raises(osm.OsmError):
        layer.route_qwen_top_k(xd, 5, ids, w)  # more tokens than max_tokens
    with pytest.raises(osm.OsmError):
        layer.route_qwen_top_k(xd, 0, ids, w)


def test_router_nonfinite_input_flagged(torch):
    W = np.random.default_rng(1).standard_normal((8, 16)).astype(np.float32)
    x = np.zeros((2, 16), np.float32)
    x[1, 3] = np.nan
    ids, w, m, st, _ = _route(torch, W, x, 2)
    assert st & 1  # non-finite hidden vector (qwen_router.cpp:49-53)


@pytest.mark.parametrize("exact", [False, True])
def test_router_golden_small(torch, golden_dir, exact):
    z = np.load(os.path.join(golden_dir, "router_small.npz"))
    ids, w, m, st, _ = _route(torch, z["W"], z["x"], int(z["k"]), exact=exact)
    assert st == 0
    assert np.array_equal(ids, z["ids"])
    np.testing.assert_allclose(w, z["weights"], atol=1e-6, rtol=0)
    np.testing.assert_allclose(m, z["mass"], atol=1e-6, rtol=0)


@pytest.mark.parametrize("exact", [False, True])
def test_router_golden_q3n_with_bias(torch, golden_dir, exact):
    z = np.load(os.path.join(golden_dir, "router_q3n.npz"))
    W = pyoracle.bf16_widen(z["Wbits"])
    x = z["x"]
    for sel, bias in ((slice(0, None, 2), None), (slice(1, None, 2), z["bias"])):
        ids, w, m, st, _ = _route(torch, W, x[sel], int(z["k"]), bias=bias, exact=exact)
        assert st == 0
        assert np.array_equal(ids, z["ids"][sel])
        np.testing.assert_allclose(w, z["weights"][sel], atol=1e-6, rtol=0)


def test_router_logits_q3n_match_reference(torch, golden_dir):
    """osm_moe_route_logits, the C++ drop-in's router: the logits the reference
    library returned (router_q3n.npz, with and without the Zipf bias) bit for
    bit, the same ids, weights and mass within 1e-6."""
    import osm_b200 as osm

    z = np.load(os.path.join(golden_dir, "router_q3n.npz"))
    W = pyoracle.bf16_widen(z["Wbits"])
    k = int(z["k"])
    for sel, bias in ((slice(0, None, 2), None), (slice(1, None, 2), z["bias"])):
        x = z["x"][sel]
        B, E = x.shape[0], W.shape[0]
        ctx = osm.Context(0, max_tokens=B)
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        layer = osm.Layer(ctx, W, k, True, logit_bias=bias)
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        logits = torch.empty(B, E, device="cuda")
        ids = torch.empty(B, k, dtype=torch.int32, device="cuda")
        w = torch.empty(B, k, device="cuda")
        m = torch.empty(B, device="cuda")
        layer.route_qwen_top_k_logits(xd, B, logits, ids, w, m)
        torch.cuda.synchronize()
        st, ex = ctx.status()
        assert st == 0 and ex == B
        assert np.array_equal(logits.cpu().numpy().view(np.uint32), z["logits"][sel].view(np.uint32))
        assert np.array_equal(ids.cpu().numpy().astype(np.uint32), z["ids"][sel])
        np.testing.assert_allclose(w.cpu().numpy(), z["weights"][sel], atol=1e-6, rtol=0)
        np.testing.assert_allclose(m.cpu().numpy(), z["mass"][sel], atol=1e-6, rtol=0)


def test_router_q3n_many_tokens_ids_bit_exact(torch, port):
    """Size-independent check at the decode batch size: every token's ids
    equal the oracle's (256 tokens, Zipf-biased and unbiased)."""
    H, E, K, B = 2048, 512, 10, 256
    W = pyoracle.bf16_widen(port.bf16_round(port.gen_normal(5, 1, 0.02, E * H))).reshape(E, H)
    x = port.gen_normal(5, 2, 1.0, B * H).reshape(B, H)
    r = np.arange(1, E + 1, dtype=np.float64)
    perm = np.random.default_rng(5).permutation(E)
    bias = np.zeros(E, np.float32)
    bias[perm] = np.log(r ** -1.1 / (r ** -1.1).sum()).astype(np.float32)
    for b in (None, bias):
        ids, w, m, st, ex = _route(torch, W, x, K, bias=b)
        assert st == 0
        for t in range(B):
            _, rid, rw, rm = port.route_qwen_top_k(x[t], W, K, True, bias=b)
            assert np.array_equal(ids[t], rid), (t, ids[t], rid)
            # A 2048-term logit summed in another order differs from the
            # reference's sequential sum by ~1e-6; weights follow within
            # 1e-5 relative (the fp32 output criterion is 1e-4).
            np.testing.assert_allclose(w[t], rw, rtol=1e-5, atol=1e-7)
            np.testing.assert_allclose(m[t], rm, rtol=1e-5, atol=1e-7)
        assert ex < B // 4  # the exact path is the exception, not the rule


def test_router_ties_take_exact_path(torch, port):
    """Duplicate router rows produce exact probability ties: lower id first."""
    rng = np.random.default_rng(3)
    H, E, K = 256, 64, 8
    W = rng.standard_normal((E, H)).astype(np.float32) * np.float32(0.05)
    W = pyoracle.bf16_widen(port.bf16_round(W)).reshape(E, H)
    for dst, src in ((40, 3), (41, 3), (17, 50), (9, 60)):
        W[dst] = W[src]
    x = rng.standard_normal((16, H)).astype(np.float32)
    x[:, :] += W[3] * 40  # make expert 3 (and its copies 40, 41) win
    ids, w, m, st, ex = _route(torch, W, x, K)
    for t in range(16):
        _, rid, rw, _ = port.route_qwen_top_k(x[t], W, K, True)
        assert np.array_equal(ids[t], rid)
        np.testing.assert_allclose(w[t], rw, atol=1e-6)
    assert ex >= 1


def test_moe_small_golden(torch, golden_dir):
    z = np.load(os.path.join(golden_dir, "moe_small.npz"))
    H, I = z["x"].shape[1], int(z["inter"])
    fx = MoeFixture(torch, H, z["slots"].shape[0], I, int(z["k"]), slots=z["slots"],
                    shared_slot=z["shared"], W=pyoracle.bf16_widen(z["Wbits"]),
                    sg=pyoracle.bf16_widen(z["sgbits"]))
    for exact in (False, True):
        out, ids, w, m, sg = fx.run(torch, z["x"], exact=exact)
        assert np.array_equal(ids, z["ids"])
        np.testing.assert_allclose(w, z["weights"], atol=1e-6, rtol=0)
        np.testing.assert_allclose(sg, z["shared_scale"], atol=1e-6, rtol=0)
        for b in range(out.shape[0]):
            assert normwise_rel(out[b], z["out"][b]) <= 1e-4
            assert float(np.abs(out[b] - z["out"][b]).max()) <= 0.03
    assert fx.ctx.status()[0] == 0


def test_moe_hash_fixture(torch, golden_dir):
    """tests/weighted_routed_moe_test.cpp: 3 experts, top-2, E1 then E2."""
    z = np.load(os.path.join(golden_dir, "hash_fixture.npz"))
    fx = MoeFixture(torch, 128, 3, 64, 2, slots=z["slots"], shared=False, W=z["router"])
    out, ids, w, m, _ = fx.run(torch, z["x"][None, :])
    assert list(ids[0]) == [1, 2]
    assert abs(float(w[0].sum()) - 1.0) <= 1e-6
    assert float(np.abs(out[0] - z["out"]).max()) <= 0.02
    assert normwise_rel(out[0], z["out"]) <= 1e-4


@pytest.mark.parametrize("B", [1, 2, 8, 33])
def test_moe_q3n_decode(torch, B):
    """Qwen3-Next shape (H 2048, E 512, k 10, I 512, shared 512), Zipf bias."""
    H, E, I, K = 2048, 512, 512, 10
    import osm_b200 as osm  # noqa: F401

    fx = _q3n_fixture(torch)
    x = fx.port.gen_normal(9, 100 + B, 1.0, B * H).reshape(B, H)
    out, ids, w, m, sg = fx.run(torch, x)
    assert fx.ctx.status()[0] == 0
    check = range(B) if B <= 8 else (0, B // 2, B - 1)
    for b in check:
        ref, rids, rw, rm, rs = fx.oracle_token(x[b])
        assert np.array_equal(ids[b], rids)
        np.testing.assert_allclose(w[b], rw, rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(sg[b], rs, rtol=1e-5, atol=1e-7)
        assert normwise_rel(out[b], ref) <= 1e-4, normwise_rel(out[b], ref)


_Q3N = {}


def _q3n_fixture(torch):
    """Generated once per process: 512 experts on the device generator are
    copied to host so the oracle sees the same bytes."""
    if "fx" in _Q3N:
        return _Q3N["fx"]
    import ctypes

    import osm_b200 as osm

    H, E, I, K = 2048, 512, 512, 10
    port = pyoracle.Oracle("port")
    ctx = osm.Context(0, max_tokens=8)
    lay = osm.expert_layout(H, I)
    gen = osm.Slab(ctx, lay, E + 1)
    gen.generate(2024, 1000, 0.02, 0, E + 1)
    ctx.synchronize()
    slots = np.zeros((E + 1, lay.stride), np.uint8)
    ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(slots.ctypes.data),
                                     ctypes.c_void_p(gen.slot_ptr(0)), (E + 1) * lay.stride))
    gen.close()
    r = np.arange(1, E + 1, dtype=np.float64)
    perm = np.random.default_rng(2024).permutation(E)
    bias = np.zeros(E, np.float32)
    bias[perm] = np.log(r ** -1.1 / (r ** -1.1).sum()).astype(np.float32)
    fx = MoeFixture(torch, H, E, I, K, seed=2024, slots=slots[:E], shared_slot=slots[E],
                    bias=bias, max_tokens=64)
    _Q3N["fx"] = fx
    return fx


@pytest.mark.parametrize("B", [1, 2, 5])
def test_moe_split_route_then_experts_matches_forward(torch, B):
    """osm_moe_route + osm_moe_experts (host cache between) == osm_moe_forward."""
    fx = _q3n_fixture(torch)
    H, K = fx.H, fx.K
    x = fx.port.gen_normal(9, 7, 1.0, B * H).reshape(B, H)
    out, ids, w, m, sg = fx.run(torch, x)
    xd = torch.from_numpy(x).cuda()
    ids2 = torch.empty(B, K, dtype=torch.int32, device="cuda")
    w2 = torch.empty(B, K, device="cuda")
    fx.layer.route_qwen_top_k(xd, B, ids2, w2)
    out2 = torch.empty(B, H, device="cuda")
    fx.layer.run_experts(xd, B, ids2, w2, out2)
    torch.cuda.synchronize()
    assert np.array_equal(ids2.cpu().numpy().astype(np.uint32), ids)
    assert np.array_equal(out2.cpu().numpy().view(np.uint32), out.view(np.uint32))


@pytest.mark.parametrize("shared,B", [(True, 1), (True, 2), (False, 1), (False, 2)])
def test_moe_decode_small_shapes(torch, shared, B):
    """The 1-2 token kernels at a small shape (H 256, I 128), with and without
    a shared expert, against the oracle."""
    H, E, I, K = 256, 16, 128, 4
    fx = MoeFixture(torch, H, E, I, K, seed=57, shared=shared)
    x = fx.port.gen_normal(57, 3 + B, 1.0, B * H).reshape(B, H)
    out, ids, w, m, sg = fx.run(torch, x)
    assert fx.ctx.status()[0] == 0
    for b in range(B):
        ref, rids, rw, rm, rs = fx.oracle_token(x[b])
        assert np.array_equal(ids[b], rids)
        assert normwise_rel(out[b], ref) <= 1e-4, normwise_rel(out[b], ref)


def test_moe_nonresident_expert_reported(torch):
    fx = _q3n_fixture(torch)
    x = fx.port.gen_normal(9, 8, 1.0, fx.H).reshape(1, fx.H)
    _, ids, _, _, _ = fx.run(torch, x)
    victim = int(ids[0][0])
    fx.layer.set_slot(victim, -1)
    fx.run(torch, x)
    st, _ = fx.ctx.status()
    fx.layer.set_slot(victim, victim)
    assert st & 4  # not resident
    out, ids2, _, _, _ = fx.run(torch, x)
    assert fx.ctx.status()[0] == 0


def test_sublayer_rmsnorm_residual(torch, port):
    """QwenCheckpointMoeSublayer::run: y = r + MoE(RMSNorm(r)); normalized is
    bit-exact in exact mode; the routing of the normalized vector equals the
    oracle's."""
    H, E, I, K = 256, 16, 64, 4
    nw = port.gen_normal(4, 4, 0.3, H) + np.float32(1.0)
    fx = MoeFixture(torch, H, E, I, K, seed=31, norm_weight=nw)
    B = 6
    r = port.gen_normal(31, 9, 2.0, B * H).reshape(B, H)
    rd = torch.from_numpy(r).cuda()
    for exact in (True, False):
        out = torch.empty(B, H, device="cuda")
        nrm = torch.empty(B, H, device="cuda")
        ids = torch.empty(B, K, dtype=torch.int32, device="cuda")
        w = torch.empty(B, K, device="cuda")
        fx.layer.run_sublayer(rd, B, out, normalized=nrm, ids=ids, weights=w,
                              exact_rmsnorm=exact)
        torch.cuda.synchronize()
        got_n = nrm.cpu().numpy()
        ref_n = port.rms_norm(r, nw, 1e-6)
        if exact:
            assert np.array_equal(got_n.view(np.uint32), ref_n.view(np.uint32))
        else:
            np.testing.assert_allclose(got_n, ref_n, atol=1e-5, rtol=0)
        got = out.cpu().numpy()
        gids = ids.cpu().numpy().astype(np.uint32)
        for b in range(B):
            ref, rids, _, _, _ = fx.oracle_token(got_n[b])
            assert np.array_equal(gids[b], rids)
            refy = r[b] + ref
            assert normwise_rel(got[b] - r[b], ref) <= 1e-4
            assert float(np.abs(got[b] - refy).max()) <= 0.03


def test_plan_replay_matches_direct_call(torch):
    """A captured plan (CUDA graph) gives bit-identical results to the direct
    call, with and without host buffers inside the plan.  With host buffers the
    plan itself must bring x in (the device input is cleared first) and out
    back, both for aligned pinned buffers (copied by the SMs through the
    mapping) and for buffers 4 bytes off alignment (copy-engine nodes)."""
    import osm_b200 as osm

    fx = _q3n_fixture(torch)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        fx.ctx.set_stream(stream.cuda_stream)
        try:
            for B in (1, 5):
                x = fx.port.gen_normal(9, 40 + B, 1.0, B * fx.H).reshape(B, fx.H)
                out_ref, ids_ref, _, _, _ = fx.run(torch, x)
                xd = torch.from_numpy(x).cuda()
                out = torch.empty(B, fx.H, device="cuda")
                ids = torch.empty(B, fx.K, dtype=torch.int32, device="cuda")
                plan = osm.Plan(fx.layer, B, xd, out, ids=ids)
                for _ in range(3):
                    plan.launch()
                torch.cuda.synchronize()
                assert np.array_equal(out.cpu().numpy().view(np.uint32), out_ref.view(np.uint32))
                assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_ref)
                plan.close()
                n = B * fx.H
                for off in (0, 1):  # element offset into the pinned buffers
                    xbuf = torch.zeros(n + 4).pin_memory()
                    obuf = torch.zeros(n + 4).pin_memory()
                    xh = xbuf[off:off + n].view(B, fx.H)
                    oh = obuf[off:off + n].view(B, fx.H)
                    xh.copy_(torch.from_numpy(x))
                    xd.zero_()
                    out.zero_()
                    torch.cuda.synchronize()
                    plan2 = osm.Plan(fx.layer, B, xd, out, x_host=xh, out_host=oh)
                    for _ in range(2):
                        plan2.launch()
                    torch.cuda.synchronize()
                    assert np.array_equal(xd.cpu().numpy(), x)
                    assert np.array_equal(out.cpu().numpy().view(np.uint32), out_ref.view(np.uint32))
                    assert np.array_equal(oh.numpy().view(np.uint32), out_ref.view(np.uint32))
                    assert float(obuf[:off].abs().sum()) == 0.0
                    assert float(obuf[off + n:].abs().sum()) == 0.0
                    plan2.close()
        finally:
            fx.ctx.set_stream(torch.cuda.current_stream().cuda_stream)


def test_plans_keep_their_scratch_when_a_larger_call_grows_it(torch):
    """Plans captured for growing batch sizes on one context (each capture
    grows the context's scratch) and all replayed afterwards: every plan still
    gives the direct call's bits, and the status word stays clean."""
    import osm_b200 as osm

    fx = _q3n_fixture(torch)
    ctx = osm.Context(0, max_tokens=64)       # fresh context: scratch not sized yet
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    slab = osm.Slab(ctx, fx.layout, fx.E)
    for e in range(fx.E):
        slab.fill_async(e, fx.pinned.data_ptr() + e * fx.layout.stride)
    slab.fill_wait()
    layer = osm.Layer(ctx, fx.W, fx.K, True, logit_bias=fx.bias, shared_slot=fx.shared_slot,
                      shared_layout=fx.layout, shared_gate=fx.sg)
    layer.bind_slab(slab, np.arange(fx.E, dtype=np.int32))
    plans, bufs = [], []
    with torch.cuda.stream(stream):
        for B in (1, 3, 40):
            x = fx.port.gen_normal(11, 70 + B, 1.0, B * fx.H).reshape(B, fx.H)
            xd = torch.from_numpy(x).cuda()
            out = torch.empty(B, fx.H, device="cuda")
            plans.append(osm.Plan(layer, B, xd, out))
            bufs.append((B, xd, out))
        for p in plans:
            p.launch()
        stream.synchronize()
        for (B, xd, out) in bufs:
            ref = torch.empty(B, fx.H, device="cuda")
            layer.run_qwen_sparse_moe(xd, B, ref)
            stream.synchronize()
            assert torch.equal(out, ref), B
    assert ctx.status()[0] == 0
    for p in plans:
        p.close()
