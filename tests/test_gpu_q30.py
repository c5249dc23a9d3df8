"""Qwen3-30B-A3B shapes: hidden 2048, moe_intermediate 768,
top-8 renormalised, no shared expert, on every expert path: 1-2 tokens (the
bulk-copy decode kernels), 3+ tokens (grouped kernels) and the tensor-core
prefill path.  Ids bit-exact against the oracle; outputs within 1e-4 (fp32
paths) or 2e-3 (prefill), as max|a - b| / max|b| per token.  24 experts keep
the fixture small; the shapes per expert are the config's."""
import numpy as np
import pytest

from gpu_util import MoeFixture, normwise_rel, require_cuda

pytestmark = pytest.mark.gpu

H, I, K, E = 2048, 768, 8, 24


@pytest.fixture(scope="module")
def fx():
    torch = require_cuda()
    return torch, MoeFixture(torch, H, E, I, K, seed=31, shared=False, max_tokens=160)


@pytest.mark.parametrize("B", [1, 2, 5, 40])
def test_q30_fp32_paths_match_oracle(fx, B):
    torch, f = fx
    x = f.port.gen_normal(31, 100 + B, 1.0, B * H).reshape(B, H)
    out, ids, _, _, _ = f.run(torch, x)
    for t in range(B):
        ref, rids, _, _, _ = f.oracle_token(x[t])
        assert np.array_equal(ids[t], rids), (B, t)
        assert normwise_rel(out[t], ref) <= 1e-4, (B, t)
    assert f.ctx.status()[0] == 0


def test_q30_prefill_matches_oracle(fx):
    torch, f = fx
    T = 160
    x = f.port.gen_normal(31, 7, 1.0, T * H).reshape(T, H)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(T, H, device="cuda")
    ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
    f.layer.run_qwen_sparse_moe(xd, T, out, ids=ids, prefill=True)
    torch.cuda.synchronize()
    o, ih = out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32)
    worst = 0.0
    for t in range(T):
        ref, rids, _, _, _ = f.oracle_token(x[t])
        assert np.array_equal(ih[t], rids), t
        worst = max(worst, normwise_rel(o[t], ref))
    assert worst <= 2e-3, worst
    assert f.ctx.status()[0] == 0


@pytest.fixture(scope="module")
def fx128():
    """All 128 experts of the config, context sized for the 8192-token case."""
    torch = require_cuda()
    return torch, MoeFixture(torch, H, 128, I, K, seed=33, shared=False, max_tokens=8192)


def _check_sampled(f, x, out, ids, tol, tokens):
    for t in tokens:
        ref, rids, _, _, _ = f.oracle_token(x[t])
        assert np.array_equal(ids[t], rids), t
        assert normwise_rel(out[t], ref) <= tol, t


def test_q30_128_experts_64_tokens(fx128):
    """configs[3] at 64 tokens (the grouped decode path), every token checked."""
    torch, f = fx128
    B = 64
    x = f.port.gen_normal(33, 64, 1.0, B * H).reshape(B, H)
    out, ids, _, _, _ = f.run(torch, x)
    _check_sampled(f, x, out, ids, 1e-4, range(B))
    assert f.ctx.status()[0] == 0


def test_q30_128_experts_8192_token_prefill(fx128):
    """configs[3] at 8192 tokens on the tensor-core prefill path: 48 tokens
    spread over the batch checked against the oracle (ids exact, outputs
    within 2e-3); the routing of all 8192 equals the fp32 path's."""
    torch, f = fx128
    T = 8192
    x = f.port.gen_normal(33, 8192, 1.0, T * H).reshape(T, H)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(T, H, device="cuda")
    ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
    f.layer.run_qwen_sparse_moe(xd, T, out, ids=ids, prefill=True)
    ids32 = torch.empty(T, K, dtype=torch.int32, device="cuda")
    f.layer.route_qwen_top_k(xd, T, ids32, torch.empty(T, K, device="cuda"))
    torch.cuda.synchronize()
    o, ih = out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32)
    assert np.array_equal(ih, ids32.cpu().numpy().astype(np.uint32))
    sample = sorted(set(np.random.RandomState(5).randint(0, T, 46).tolist()) | {0, T - 1})
    _check_sampled(f, x, o, ih, 2e-3, sample)
    assert f.ctx.status()[0] == 0
