"""The warp-specialised tensor-core expert kernels (osm_tc.cu) against the oracle
and against the older kernels, through the C ABI.

* The precise (bf16 operand planes) variant serves fp32 calls of 3+ tokens when
  a context is created with OSM_TC_DECODE=1: every token of Qwen3-Next-shaped
  batches within the 1e-4 normwise bound of the fp32 path, ids bit-exact.
* The fast (fp16) variant serves every prefill call; with OSM_DISABLE_TC=1 the
  older prefill kernel runs instead.  Both
  stay within the 2e-3 bound of the oracle and within 4e-3 of each other.
"""
import ctypes
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import pyoracle
from gpu_util import normwise_rel, require_cuda

pytestmark = pytest.mark.gpu

H, E, I, K = 2048, 512, 512, 10


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


def _q3n(torch, monkeypatch, env, max_tokens):
    import bench
    import osm_b200 as osm

    for k, v in env.items():
        monkeypatch.setenv(k, v)
    ctx = osm.Context(0, max_tokens=max_tokens)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    layer, slab, W, sg, bias, shared = bench.build_sublayer(torch, ctx, osm, zipf=True)
    return ctx, layer, slab, W, sg, bias, shared


def _slots(osm, ctx, slab, stride):
    ctx.synchronize()
    slots = np.zeros((E, stride), np.uint8)
    ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(slots.ctypes.data),
                                     ctypes.c_void_p(slab.slot_ptr(0)), E * stride))
    return slots


def test_precise_tensor_core_path_matches_oracle(torch, monkeypatch, port):
    import bench
    import osm_b200 as osm

    ctx, layer, slab, W, sg, bias, shared = _q3n(torch, monkeypatch, {"OSM_TC_DECODE": "1"}, 64)
    lay = osm.expert_layout(H, I)
    slots = _slots(osm, ctx, slab, lay.stride)
    for B in (3, 8, 40):
        x = torch.empty(B, H, device="cuda")
        ctx.gen_normal(bench.SEED, 6100 + B, 1.0, x)
        out = torch.empty(B, H, device="cuda")
        ids = torch.empty(B, K, dtype=torch.int32, device="cuda")
        layer.run_qwen_sparse_moe(x, B, out, ids=ids)
        torch.cuda.synchronize()
        assert ctx.status()[0] == 0
        xh, got = x.cpu().numpy(), out.cpu().numpy()
        gids = ids.cpu().numpy().astype(np.uint32)

        def one(t):
            return port.moe_token_slots(xh[t], W, K, True, slots, I, shared_slot=shared,
                                        scalar_gate=sg, bias=bias)

        with ThreadPoolExecutor(16) as ex:
            refs = list(ex.map(one, range(B)))
        for t, (ref, rids, _, _, _) in enumerate(refs):
            assert np.array_equal(gids[t], rids), (B, t)
            assert normwise_rel(got[t], ref) <= 1e-4, (B, t, normwise_rel(got[t], ref))


@pytest.mark.parametrize("disable", ["0", "1"])
def test_fast_prefill_paths_match_oracle_and_each_other(torch, monkeypatch, port, disable):
    """200 tokens over 16 experts of hidden 512, inter 256, top-4 (50 pairs per
    expert): the tensor-core kernels by default, the older prefill kernel with
    OSM_DISABLE_TC=1."""
    from gpu_util import MoeFixture

    monkeypatch.setenv("OSM_DISABLE_TC", disable)
    Hs, Es, Is, Ks, T = 512, 16, 256, 4, 200
    f = MoeFixture(torch, Hs, Es, Is, Ks, seed=301, max_tokens=T)
    x = f.port.gen_normal(301, 1, 1.0, T * Hs).reshape(T, Hs)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(T, Hs, device="cuda")
    ids = torch.empty(T, Ks, dtype=torch.int32, device="cuda")
    f.layer.run_qwen_sparse_moe(xd, T, out, ids=ids, prefill=True)
    fp32 = torch.empty(T, Hs, device="cuda")
    f.layer.run_qwen_sparse_moe(xd, T, fp32)
    torch.cuda.synchronize()
    assert f.ctx.status()[0] == 0
    o, ref32 = out.cpu().numpy(), fp32.cpu().numpy()
    ih = ids.cpu().numpy().astype(np.uint32)
    for t in range(0, T, 7):
        ref, rids, _, _, _ = f.oracle_token(x[t])
        assert np.array_equal(ih[t], rids)
        assert normwise_rel(o[t], ref) <= 2e-3, (t, normwise_rel(o[t], ref))
    for t in range(T):
        assert normwise_rel(o[t], ref32[t]) <= 4e-3
