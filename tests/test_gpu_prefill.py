"""Prefill path (OSM_PREFILL_BF16): the experts run as a 16-bit tcgen05 grouped
GEMM (fp16 operands, fp32 accumulation) over 128-pair chunks.  Routing stays
exact (ids bit-equal to the oracle's route_qwen_top_k); outputs are within
16-bit rounding of the fp32 oracle: the 2e-3 bound for tensor-core prefill, as
max|a - b| / max|b| per token.  Cases cover partial chunks and partial 128-row
tiles, a shared expert spanning several chunks, no shared expert, and the Q3N
hidden/intermediate sizes with top-10."""
import numpy as np
import pytest

from gpu_util import MoeFixture, normwise_rel, require_cuda

pytestmark = pytest.mark.gpu

TOL = 2e-3


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


@pytest.mark.parametrize("H,E,I,K,T,shared,seed", [
    (256, 16, 256, 4, 300, True, 91),
    (512, 8, 256, 2, 200, False, 92),
    (2048, 24, 512, 10, 96, True, 93),
])
def test_prefill_matches_oracle(torch, H, E, I, K, T, shared, seed):
    f = MoeFixture(torch, H, E, I, K, seed=seed, shared=shared, max_tokens=T)
    x = f.port.gen_normal(seed, 1, 1.0, T * H).reshape(T, H)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(T, H, device="cuda")
    ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
    w = torch.empty(T, K, device="cuda")
    f.layer.run_qwen_sparse_moe(xd, T, out, ids=ids, weights=w, prefill=True)
    torch.cuda.synchronize()
    o, ih = out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32)
    worst = 0.0
    for t in range(T):
        ref, rids, _, _, _ = f.oracle_token(x[t])
        assert np.array_equal(ih[t], rids), t
        worst = max(worst, normwise_rel(o[t], ref))
    assert worst <= TOL, worst
    assert f.ctx.status()[0] == 0


def test_prefill_agrees_with_the_fp32_path(torch):
    """The same call without the flag (fp32 grouped path) and with it agree to
    16-bit rounding; routing and the shared gate are identical."""
    H, E, I, K, T = 256, 12, 256, 3, 150
    f = MoeFixture(torch, H, E, I, K, seed=94, max_tokens=T)
    x = torch.from_numpy(f.port.gen_normal(94, 2, 1.0, T * H).reshape(T, H)).cuda()
    outs, idss, sgs = [], [], []
    for prefill in (False, True):
        out = torch.empty(T, H, device="cuda")
        ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
        sg = torch.empty(T, device="cuda")
        f.layer.run_qwen_sparse_moe(x, T, out, ids=ids, shared_gate=sg, prefill=prefill)
        outs.append(out.cpu().numpy())
        idss.append(ids.cpu().numpy())
        sgs.append(sg.cpu().numpy())
    assert np.array_equal(idss[0], idss[1])
    assert np.array_equal(sgs[0], sgs[1])
    for t in range(T):
        assert normwise_rel(outs[1][t], outs[0][t]) <= TOL


def test_prefill_experts_take_fp16_rows(torch):
    """osm_moe_experts with fp16 rows (OSM_INPUT_F16, as an expert-parallel
    exchange delivers them) equals the same call on fp32 rows, which the
    library rounds to fp16 itself."""
    H, E, I, K, T = 256, 8, 256, 2, 140
    f = MoeFixture(torch, H, E, I, K, seed=95, shared=False, max_tokens=T)
    x = torch.from_numpy(f.port.gen_normal(95, 3, 1.0, T * H).reshape(T, H)).cuda()
    rs = np.random.RandomState(3)
    ids = torch.from_numpy(np.stack([rs.permutation(E)[:K] for _ in range(T)]).astype(np.int32)).cuda()
    w = torch.from_numpy(rs.rand(T, K).astype(np.float32)).cuda()
    o32 = torch.empty(T, H, device="cuda")
    o16 = torch.empty(T, H, device="cuda")
    f.layer.run_experts(x, T, ids, w, o32, prefill=True)
    f.layer.run_experts(x.half(), T, ids, w, o16, prefill=True)
    torch.cuda.synchronize()
    assert torch.equal(o32, o16)
    assert f.ctx.status()[0] == 0


def test_prefill_experts_write_fp16_rows(torch):
    """With an fp16 output (OSM_OUTPUT_F16) each output element is the fp32
    result of the same call rounded to fp16 once."""
    H, E, I, K, T = 256, 8, 256, 2, 130
    f = MoeFixture(torch, H, E, I, K, seed=96, shared=False, max_tokens=T)
    x = torch.from_numpy(f.port.gen_normal(96, 4, 1.0, T * H).reshape(T, H)).cuda()
    rs = np.random.RandomState(4)
    ids = torch.from_numpy(np.stack([rs.permutation(E)[:K] for _ in range(T)]).astype(np.int32)).cuda()
    w = torch.from_numpy(rs.rand(T, K).astype(np.float32)).cuda()
    o32 = torch.empty(T, H, device="cuda")
    o16 = torch.empty(T, H, dtype=torch.float16, device="cuda")
    f.layer.run_experts(x, T, ids, w, o32, prefill=True)
    f.layer.run_experts(x.half(), T, ids, w, o16, prefill=True)
    torch.cuda.synchronize()
    assert torch.equal(o32.half(), o16)
    assert f.ctx.status()[0] == 0


def test_prefill_out_of_fp16_range_falls_back_to_fp32(torch):
    """Activations beyond the fp16 range (x scaled by 1e5): the checked
    prefill call (the default) re-runs on the fp32 path -- its output is that
    path's, bit for bit, and the status word reports bit 6, not bit 5; with
    the check off the call reports bit 5 (outputs invalid)."""
    H, E, I, K, T = 256, 12, 256, 3, 150
    f = MoeFixture(torch, H, E, I, K, seed=95, max_tokens=T)
    x = torch.from_numpy(f.port.gen_normal(95, 2, 1.0, T * H).reshape(T, H) * 1e5).cuda()
    f.ctx.status()
    ref = torch.empty(T, H, device="cuda")
    f.layer.run_qwen_sparse_moe(x, T, ref)
    assert f.ctx.status()[0] == 0
    out = torch.empty(T, H, device="cuda")
    f.layer.run_qwen_sparse_moe(x, T, out, prefill=True)
    st = f.ctx.status()[0]
    assert st == 1 << 6, st
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32))
    f.layer.run_qwen_sparse_moe(x, T, out, prefill=True, check_range=False)
    st = f.ctx.status()[0]
    assert st & (1 << 5) and not st & (1 << 6), st
    # in range, the checked call reports nothing and stays on the fp16 path
    xs = x / 1e5
    f.layer.run_qwen_sparse_moe(xs, T, out, prefill=True)
    assert f.ctx.status()[0] == 0
