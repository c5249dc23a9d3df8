"""GPU parity of the element-wise replacements of the reference's Vulkan
kernels, through the C ABI (libosm_b200.so), against the CPU oracle.

Tolerances: dequantisation bit-exact; exact RMSNorm bit-exact; fast RMSNorm
1e-5 (tests/checkpoint_moe_sublayer_test.cpp:700-701); SwiGLU / weighted
accumulate 1e-6 (tests/vulkan_weighted_accumulate_test.cpp:104); Q4 GEMV
within 1e-4 normwise relative error (max|a-b| / max|b|) and the reference's
own 5e-4 absolute gate (tests/vulkan_q4_gemv_test.cpp:149-160).
"""
import numpy as np
import pytest

import pyoracle
from gpu_util import MoeFixture, normwise_rel, require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


@pytest.fixture(scope="module")
def ctx(torch):
    import osm_b200 as osm

    c = osm.Context(0, max_tokens=64)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    return c


def _proj(port, rows, cols, seed):
    vals = port.gen_normal(seed, 1, 0.02, rows * cols)
    pk, sc, bi = port.quantize_q4(vals, rows, cols, 64)
    sb = port.bf16_round(sc)
    bb = port.bf16_round(bi)
    return pk, sb.reshape(rows, -1), bb.reshape(rows, -1)


def test_q4_dequant_bit_exact(torch, ctx, port):
    for rows, cols in ((64, 128), (512, 2048), (2048, 512), (768, 2048)):
        pk, sb, bb = _proj(port, rows, cols, rows + cols)
        out = torch.empty(rows, cols, device="cuda")
        ctx.q4_dequant(torch.from_numpy(pk).cuda(), torch.from_numpy(sb).cuda(),
                       torch.from_numpy(bb).cuda(), rows, cols, out)
        torch.cuda.synchronize()
        ref = port.dequantize_affine_rows(pk, rows, cols // 8, pyoracle.bf16_widen(sb),
                                          pyoracle.bf16_widen(bb), 4, 64)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_q4_dequant_rejects_bad_group(torch, ctx):
    """A group that does not divide the row (tests/vulkan_q4_dequant_test.cpp:
    38-53 asks for group 3 on an 8-column row) is refused before any launch."""
    import osm_b200 as osm

    z = torch.zeros(64, dtype=torch.int32, device="cuda")
    with pytest.raises(osm.OsmError):
        ctx.q4_dequant(z, z, z, 1, 8, torch.empty(64, device="cuda"), group=3)
    with pytest.raises(osm.OsmError):
        ctx.q4_gemv(z, z, z, 1, 8, torch.zeros(8, device="cuda"), 1,
                    torch.empty(1, device="cuda"), group=3)


def _proj_g(port, rows, cols, group, seed):
    vals = port.gen_normal(seed, 1, 0.02, rows * cols)
    pk, sc, bi = port.quantize_q4(vals, rows, cols, group)
    return pk, port.bf16_round(sc).reshape(rows, -1), port.bf16_round(bi).reshape(rows, -1)


@pytest.mark.parametrize("rows,cols,group,tokens", [
    (8, 8, 4, 1),       # the checkpoint fixtures' geometry (hidden 8, group 4)
    (24, 96, 32, 3),    # rows not a multiple of 16, group 32
    (40, 8, 8, 2),
    (130, 64, 64, 70),  # more tokens than the context's max_tokens (64)
    (16, 4096, 64, 2),  # K above the row-tiled kernel's 2048
])
def test_q4_any_geometry(torch, ctx, port, rows, cols, group, tokens):
    """Shapes outside the row-tiled projection kernel run on the
    any-geometry dequant / GEMV kernels: dequant bit-exact, GEMV within the
    same bounds as above."""
    pk, sb, bb = _proj_g(port, rows, cols, group, rows * 7 + cols + group)
    W = port.dequantize_affine_rows(pk, rows, cols // 8, pyoracle.bf16_widen(sb),
                                    pyoracle.bf16_widen(bb), 4, group)
    pkd, sbd, bbd = (torch.from_numpy(a).cuda() for a in (pk, sb, bb))
    out = torch.empty(rows, cols, device="cuda")
    ctx.q4_dequant(pkd, sbd, bbd, rows, cols, out, group=group)
    x = port.gen_normal(6, rows + tokens, 1.0, tokens * cols).reshape(tokens, cols)
    y = torch.empty(tokens, rows, device="cuda")
    ctx.q4_gemv(pkd, sbd, bbd, rows, cols, torch.from_numpy(x).cuda(), tokens, y, group=group)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), W.view(np.uint32))
    got = y.cpu().numpy()
    for t in range(tokens):
        ref = port.matvec(W, x[t])
        assert normwise_rel(got[t], ref) <= 1e-4
        assert float(np.abs(got[t] - ref).max()) <= 5e-4


@pytest.mark.parametrize("rows,cols", [(64, 128), (512, 2048), (2048, 512), (2048, 768), (16, 64)])
@pytest.mark.parametrize("tokens", [1, 3, 8, 17])
def test_q4_gemv(torch, ctx, port, rows, cols, tokens):
    pk, sb, bb = _proj(port, rows, cols, 3 * rows + cols)
    x = port.gen_normal(5, rows + tokens, 1.0, tokens * cols).reshape(tokens, cols)
    y = torch.empty(tokens, rows, device="cuda")
    ctx.q4_gemv(torch.from_numpy(pk).cuda(), torch.from_numpy(sb).cuda(),
                torch.from_numpy(bb).cuda(), rows, cols, torch.from_numpy(x).cuda(), tokens, y)
    torch.cuda.synchronize()
    W = port.dequantize_affine_rows(pk, rows, cols // 8, pyoracle.bf16_widen(sb),
                                    pyoracle.bf16_widen(bb), 4, 64)
    got = y.cpu().numpy()
    for t in range(tokens):
        ref = port.matvec(W, x[t])
        assert normwise_rel(got[t], ref) <= 1e-4
        assert float(np.abs(got[t] - ref).max()) <= 5e-4


def test_swiglu_and_weighted_accumulate(torch, ctx, port):
    g = port.gen_normal(9, 1, 2.0, 4099)
    u = port.gen_normal(9, 2, 1.0, 4099)
    out = torch.empty(4099, device="cuda")
    ctx.swiglu(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda(), out)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), port.swiglu(g, u), atol=1e-6, rtol=0)
    acc0 = port.gen_normal(9, 3, 1.0, 4099)
    acc = torch.from_numpy(acc0.copy()).cuda()
    ctx.weighted_accumulate(torch.from_numpy(u).cuda(), 0.37, acc)
    torch.cuda.synchronize()
    ref = acc0 + np.float32(0.37) * u
    np.testing.assert_allclose(acc.cpu().numpy(), ref, atol=1e-6, rtol=0)


def test_rms_norm(torch, ctx, port):
    for rows, dim in ((1, 2048), (5, 2048), (3, 8)):
        v = port.gen_normal(11, dim, 1.5, rows * dim).reshape(rows, dim)
        w = port.gen_normal(12, dim, 1.0, dim)
        for exact in (True, False):
            d = torch.from_numpy(v.copy()).cuda()
            ctx.rms_norm(d, rows, dim, torch.from_numpy(w).cuda(), 1e-6, exact=exact)
            torch.cuda.synchronize()
            ref = port.rms_norm(v, w, 1e-6)
            got = d.cpu().numpy()
            if exact:
                assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
            else:
                np.testing.assert_allclose(got, ref, atol=1e-5, rtol=0)
    # reference KAT: [3, 4] with weight [2, 0.5], eps 0
    d = torch.tensor([3.0, 4.0], device="cuda")
    ctx.rms_norm(d, 1, 2, torch.tensor([2.0, 0.5], device="cuda"), 0.0, exact=True)
    torch.cuda.synchronize()
    base = np.sqrt(np.float32(12.5))
    np.testing.assert_allclose(d.cpu().numpy(), [3 / base * 2, 4 / base * 0.5], atol=1e-6)


def test_expert_forward_hash_fixture(torch, ctx, port, golden_dir):
    """The reference's integer-hash qpack fixture (hidden 128, inter 64): one
    resident expert at a time (VulkanResidentExpert::run_from_buffer)."""
    import os

    import osm_b200 as osm

    z = np.load(os.path.join(golden_dir, "hash_fixture.npz"))
    lay = osm.expert_layout(128, 64)
    import make_golden

    for e in range(3):
        slot = torch.from_numpy(z["slots"][e]).cuda()
        for seed in range(3):
            x = make_golden.hash_fixture_token(seed)
            out = torch.empty(1, 128, device="cuda")
            ctx.expert_forward(slot.data_ptr(), lay, torch.from_numpy(x).cuda(), 1, out)
            torch.cuda.synchronize()
            g, u, d = port.dequant_slot(z["slots"][e], 128, 64)
            ref = port.matvec(d, port.swiglu(port.matvec(g, x), port.matvec(u, x)))
            got = out.cpu().numpy()[0]
            assert float(np.abs(got - ref).max()) <= 0.01
            assert normwise_rel(got, ref) <= 1e-4


def test_expert_forward_q3n_batched(torch, ctx, port):
    import osm_b200 as osm

    H, I = 2048, 512
    slot = port.gen_expert_slot(21, 300, 0.02, H, I)
    lay = osm.expert_layout(H, I)
    x = port.gen_normal(21, 5, 1.0, 9 * H).reshape(9, H)
    out = torch.empty(9, H, device="cuda")
    ctx.expert_forward(torch.from_numpy(slot).cuda().data_ptr(), lay, torch.from_numpy(x).cuda(),
                       9, out)
    torch.cuda.synchronize()
    g, u, d = port.dequant_slot(slot, H, I)
    got = out.cpu().numpy()
    for t in range(9):
        ref = port.matvec(d, port.swiglu(port.matvec(g, x[t]), port.matvec(u, x[t])))
        assert normwise_rel(got[t], ref) <= 1e-4


def test_gpu_generator_matches_cpu_quantiser(torch, ctx, port):
    """The device generator restates the reference quantiser: same packed
    words and bf16 metadata as the C port on the same stream."""
    import osm_b200 as osm

    H, I = 256, 64
    lay = osm.expert_layout(H, I)
    slab = osm.Slab(ctx, lay, 2)
    slab.generate(5, 40, 0.02, 0, 2)
    torch.cuda.synchronize()
    import ctypes

    for i in range(2):
        host = np.zeros(lay.stride, np.uint8)
        ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(host.ctypes.data),
                                         ctypes.c_void_p(slab.slot_ptr(i)), lay.stride))
        cpu = port.gen_expert_slot(5, 40 + 3 * i, 0.02, H, I)
        mismatch = np.count_nonzero(host != cpu)
        assert mismatch <= 8, mismatch  # double-precision log/cos may differ in the last place


@pytest.mark.parametrize("rows,cols,group", [(64, 128, 64), (8, 8, 4), (33, 96, 32)])
def test_q4_fp32_metadata(torch, ctx, port, rows, cols, group):
    """fp32 scale and bias that bf16 cannot hold (the reference's own device
    format): dequant bit-exact with the oracle, GEMV within the bounds above."""
    vals = port.gen_normal(rows + 5 * cols, 1, 0.02, rows * cols)
    pk, sc, bi = port.quantize_q4(vals, rows, cols, group)  # fp32, not bf16-rounded
    assert not np.array_equal(sc, pyoracle.bf16_widen(port.bf16_round(sc)).reshape(sc.shape))
    W = port.dequantize_affine_rows(pk, rows, cols // 8, sc, bi, 4, group)
    pkd, scd, bid = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (pk, sc, bi))
    out = torch.empty(rows, cols, device="cuda")
    ctx.q4_dequant_f32(pkd, scd, bid, rows, cols, out, group=group)
    x = port.gen_normal(8, rows, 1.0, 2 * cols).reshape(2, cols)
    y = torch.empty(2, rows, device="cuda")
    ctx.q4_gemv_f32(pkd, scd, bid, rows, cols, torch.from_numpy(x).cuda(), 2, y, group=group)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), W.view(np.uint32))
    got = y.cpu().numpy()
    for t in range(2):
        ref = port.matvec(W, x[t])
        assert normwise_rel(got[t], ref) <= 1e-4
