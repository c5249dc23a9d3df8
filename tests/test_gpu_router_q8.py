"""The 8-bit router (osm_layer_set_router_q8): the router kept MLX-affine
8-bit on the device (group 64, bf16 scale and bias), dequantised as the
kernels read it.  Its routing must equal the reference's CPU router on the
fp32 matrix that cpu::dequantize_affine_rows gives for the same module
(src/model/checkpoint_sparse_moe.cpp:159-162): ids bit-exact and weights
the same, on every path -- the certified one-token logits with their fallbacks,
the exact logits of 3+ tokens at every kernel width, and the forced exact
path -- at the Qwen3-Next shape (512 experts x 2048, top-10).  Weights within
1e-5 relative (the device softmax), as for the bf16 and fp32 routers."""
import numpy as np
import pytest

import pyoracle
from gpu_util import require_cuda

pytestmark = pytest.mark.gpu

E, H, K = 512, 2048, 10


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


@pytest.fixture(scope="module")
def q8_router(port):
    rng = np.random.default_rng(808)
    q = rng.integers(0, 256, size=(E, H), dtype=np.uint8)
    # scales/biases around the range of an 8-bit quantised N(0, 0.02) router
    sc = port.bf16_round(rng.uniform(1e-4, 3e-4, size=E * (H // 64)).astype(np.float32))
    bi = port.bf16_round(rng.uniform(-0.04, -0.02, size=E * (H // 64)).astype(np.float32))
    packed = q.view(np.uint32).reshape(E, H // 4)
    W = port.dequantize_affine_rows(packed, E, H // 4, pyoracle.bf16_widen(sc), pyoracle.bf16_widen(bi),
                                    8, 64).reshape(E, H)
    return packed, sc.reshape(E, -1), bi.reshape(E, -1), W


@pytest.mark.parametrize("B,exact", [(1, False), (2, False), (1, True), (3, False), (8, False),
                                     (40, False), (200, False), (600, False)])
def test_q8_router_matches_reference_routing(torch, port, q8_router, B, exact):
    import osm_b200 as osm

    packed, sc, bi, W = q8_router
    ctx = osm.Context(0, max_tokens=max(B, 8))
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    layer = osm.Layer(ctx, W, K, True)
    layer.set_router_q8(packed, sc, bi)
    x = port.gen_normal(808, B, 1.0, B * H).reshape(B, H)
    xd = torch.from_numpy(x).cuda()
    ids = torch.empty(B, K, dtype=torch.int32, device="cuda")
    w = torch.empty(B, K, device="cuda")
    layer.route_qwen_top_k(xd, B, ids, w, exact=exact)
    torch.cuda.synchronize()
    assert ctx.status()[0] == 0
    gi, gw = ids.cpu().numpy().astype(np.uint32), w.cpu().numpy()
    for t in range(B):
        _, rids, rw, _ = port.route_qwen_top_k(x[t], W, K, True)
        assert np.array_equal(gi[t], rids), t
        np.testing.assert_allclose(gw[t], rw, rtol=1e-5, atol=1e-7)


def test_q8_router_rejects_misaligned_x(torch, port, q8_router):
    import osm_b200 as osm

    packed, sc, bi, W = q8_router
    ctx = osm.Context(0, max_tokens=8)
    layer = osm.Layer(ctx, W, K, True)
    layer.set_router_q8(packed, sc, bi)
    buf = torch.zeros(4 * H + 1, device="cuda")
    ids = torch.empty(4, K, dtype=torch.int32, device="cuda")
    w = torch.empty(4, K, device="cuda")
    with pytest.raises(osm.OsmError):
        layer.route_qwen_top_k(buf[1:], 4, ids, w)
