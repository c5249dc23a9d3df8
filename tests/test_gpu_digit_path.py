"""GPU parity of the int8 digit-plane tensor-core expert kernels (osm_tcd.cu)
at every token count, through the C ABI.

By default an fp32 call runs its experts on these kernels from 96 tokens on
(the bench sweep's B = 128 and 256, checked token by token in
test_gpu_bench_parity.py); here contexts created with OSM_DG_MIN_TOKENS=3 put
every call of three or more tokens on them, so the small chunks (one to
sixteen pairs per 16-pair chunk, partial row tiles, the shared expert, no
shared expert, the Qwen3-30B-A3B intermediate size 768) are all exercised.
Ids are bit-exact against the oracle and outputs within the fp32 path's 1e-4
normwise relative error; a context with OSM_DG_DECODE=0 keeps the older
mma.sync kernels for the same large batch and must agree to the same bound.
"""
import os

import numpy as np
import pytest

from gpu_util import MoeFixture, normwise_rel, require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


def _fixture(torch, env, **kw):
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        return MoeFixture(torch, **kw)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _check(fx, x, out, ids, tol=1e-4, rows=None):
    worst = 0.0
    for b in (range(x.shape[0]) if rows is None else rows):
        ref, rids, _, _, _ = fx.oracle_token(x[b])
        assert np.array_equal(ids[b], rids), (b, ids[b], rids)
        err = normwise_rel(out[b], ref)
        worst = max(worst, err)
        assert err <= tol, (b, err)
    return worst


@pytest.mark.parametrize("shared", [True, False])
@pytest.mark.parametrize("B", [3, 4, 17, 40])
def test_digit_path_small_shapes(torch, shared, B):
    """H 512, 16 experts, I 256 (two gate/up row tiles, four down row tiles)."""
    fx = _fixture(torch, {"OSM_DG_MIN_TOKENS": "3"}, H=512, E=16, I=256, K=4, seed=41 + B,
                  shared=shared, max_tokens=64)
    x = fx.port.gen_normal(5, 300 + B, 1.0, B * 512).reshape(B, 512)
    out, ids, _, _, _ = fx.run(torch, x)
    assert fx.ctx.status()[0] == 0
    _check(fx, x, out, ids)


_Q3N = {}


def _q3n(torch):
    """The Qwen3-Next sublayer (H 2048, E 512, k 10, I 512, shared 512, Zipf
    router bias) on a context that takes the digit-plane kernels from 3 tokens;
    the slots come from the device generator and are copied to the host so the
    oracle sees the same bytes."""
    if "fx" in _Q3N:
        return _Q3N["fx"]
    import ctypes

    import osm_b200 as osm

    H, E, I = 2048, 512, 512
    ctx = osm.Context(0, max_tokens=8)
    lay = osm.expert_layout(H, I)
    gen = osm.Slab(ctx, lay, E + 1)
    gen.generate(2025, 1000, 0.02, 0, E + 1)
    ctx.synchronize()
    slots = np.zeros((E + 1, lay.stride), np.uint8)
    ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(slots.ctypes.data),
                                     ctypes.c_void_p(gen.slot_ptr(0)), (E + 1) * lay.stride))
    gen.close()
    r = np.arange(1, E + 1, dtype=np.float64)
    perm = np.random.default_rng(2025).permutation(E)
    bias = np.zeros(E, np.float32)
    bias[perm] = np.log(r ** -1.1 / (r ** -1.1).sum()).astype(np.float32)
    fx = _fixture(torch, {"OSM_DG_MIN_TOKENS": "3"}, H=H, E=E, I=I, K=10, seed=2025,
                  slots=slots[:E], shared_slot=slots[E], bias=bias, max_tokens=256)
    _Q3N["fx"] = fx
    return fx


@pytest.mark.parametrize("B", [3, 8, 33, 64])
def test_digit_path_q3n_every_token(torch, B):
    fx = _q3n(torch)
    x = fx.port.gen_normal(11, 700 + B, 1.0, B * 2048).reshape(B, 2048)
    out, ids, _, _, _ = fx.run(torch, x)
    assert fx.ctx.status()[0] == 0
    worst = _check(fx, x, out, ids)
    print(f"B={B}: worst normwise error {worst:.3e}")


def test_digit_path_matches_mma_sync_path(torch):
    """The same 160-token call on the digit-plane kernels (the default at this
    size) and on the mma.sync grouped kernels (OSM_DG_DECODE=0)."""
    fx = _q3n(torch)
    B = 160
    x = fx.port.gen_normal(12, 900, 1.0, B * 2048).reshape(B, 2048)
    out_dg, ids_dg, _, _, _ = fx.run(torch, x)
    old = _fixture(torch, {"OSM_DG_DECODE": "0"}, H=2048, E=512, I=512, K=10, seed=2025,
                   slots=fx.slots, shared_slot=fx.shared_slot, W=fx.W, sg=fx.sg, bias=fx.bias,
                   max_tokens=256)
    out_mma, ids_mma, _, _, _ = old.run(torch, x)
    assert np.array_equal(ids_dg, ids_mma)
    for b in range(B):
        assert normwise_rel(out_dg[b], out_mma[b]) <= 1e-4, b
    _check(fx, x, out_dg, ids_dg, rows=(0, 1, 79, 158, 159))


@pytest.mark.parametrize("B", [5, 40])
def test_digit_path_q30_shape(torch, B):
    """Qwen3-30B-A3B shape: H 2048, 128 experts, top-8, I 768, no shared expert."""
    fx = _fixture(torch, {"OSM_DG_MIN_TOKENS": "3"}, H=2048, E=128, I=768, K=8, seed=37,
                  shared=False, max_tokens=64)
    x = fx.port.gen_normal(13, 40 + B, 1.0, B * 2048).reshape(B, 2048)
    out, ids, _, _, _ = fx.run(torch, x)
    assert fx.ctx.status()[0] == 0
    _check(fx, x, out, ids)
