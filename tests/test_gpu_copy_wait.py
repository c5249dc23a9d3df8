"""The bounded waits on asynchronous weight copies (status bit 4), made to run
out safely: with osm_test_set_copy_wait_polls(device, 0) every first wait a
kernel makes on a copy gives up at once, sets status bit 4 and waits again
with the full bound.  The call must report bit 4 and still return the same
outputs, bit for bit, as with the default bound: the giving up is recorded,
nothing is read before it has landed, and no block exits with a copy in
flight.  Covers the one-token decode kernels, the grouped decode kernels, the
exact router's staged rows and the older prefill kernel."""
import numpy as np
import pytest

from gpu_util import MoeFixture, require_cuda

pytestmark = pytest.mark.gpu

COPY_TIMEOUT = 1 << 4


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


def _run(torch, f, x, T, prefill):
    out = torch.empty(T, f.H, device="cuda")
    ids = torch.empty(T, f.K, dtype=torch.int32, device="cuda")
    f.layer.run_qwen_sparse_moe(x, T, out, ids=ids, prefill=prefill, exact_route=T > 2)
    torch.cuda.synchronize()
    return out.cpu().numpy(), ids.cpu().numpy(), f.ctx.status()[0]


@pytest.mark.parametrize("T,prefill,disable_tc", [(1, False, "0"), (8, False, "0"),
                                                  (64, False, "0"), (200, True, "1")])
def test_copy_wait_gives_up_and_recovers(torch, monkeypatch, T, prefill, disable_tc):
    import osm_b200 as osm

    monkeypatch.setenv("OSM_DISABLE_TC", disable_tc)
    H, E, I, K = 2048, 24, 512, 10
    f = MoeFixture(torch, H, E, I, K, seed=131, max_tokens=max(T, 8))
    x = torch.from_numpy(f.port.gen_normal(131, T, 1.0, T * H).reshape(T, H)).cuda()
    f.ctx.status()
    ref, rids, st = _run(torch, f, x, T, prefill)
    assert st == 0
    lib = osm.lib()
    assert lib.osm_test_set_copy_wait_polls(0, 0) == 0
    try:
        got, gids, st = _run(torch, f, x, T, prefill)
    finally:
        assert lib.osm_test_set_copy_wait_polls(0, 0xFFFFFFFF) == 0
    assert st & COPY_TIMEOUT, st
    assert st & ~COPY_TIMEOUT == 0, st
    assert np.array_equal(gids, rids)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # the default bound is back
    _, _, st = _run(torch, f, x, T, prefill)
    assert st == 0
