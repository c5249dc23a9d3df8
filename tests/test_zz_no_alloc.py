"""osm_expert_forward_noalloc: the single-expert forward for hosts that cannot
call cudaMalloc where experts run (a server whose device memory belongs to a
pool allocator that forbids driver allocations after warm-up, or a plugin that
only borrows a CUDA context).  Its intermediates live in one fixed device array
of the library instead of a context's scratch.

Checked through the C ABI against osm_expert_forward (the context entry point)
on two calls in a row with different inputs, so that contents left in the
shared array by the first call cannot leak into the second.  This file is
collected last: a stop at the first failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest

from gpu_util import normwise_rel, require_cuda

pytestmark = pytest.mark.gpu

OSM_EINVAL = -1


@pytest.fixture(scope="module")
def torch():
    return require_cuda()


def _noalloc(lib, torch, slot, lay, x, tokens, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.osm_expert_forward_noalloc(ctypes.c_void_p(slot.data_ptr()), ctypes.byref(lay),
                                          ctypes.c_void_p(x.data_ptr()), tokens,
                                          ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))


@pytest.mark.parametrize("H,I,tokens", [(2048, 512, 5), (512, 256, 16), (2048, 768, 1)])
def test_noalloc_matches_context_entry_point(torch, H, I, tokens):
    import osm_b200 as osm
    import pyoracle
    from osm_b200 import _lib

    lib = _lib.load()
    port = pyoracle.Oracle("port")
    lay = osm.expert_layout(H, I)
    slot = torch.from_numpy(port.gen_expert_slot(33, 400 + H + I, 0.02, H, I)).cuda()
    ctx = osm.Context(0, max_tokens=16)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        x = torch.from_numpy(port.gen_normal(33, 50 + call, 1.0 + call, tokens * H)
                             .reshape(tokens, H)).cuda()
        ref = torch.empty(tokens, H, device="cuda")
        got = torch.full((tokens, H), float("nan"), device="cuda")
        ctx.expert_forward(slot.data_ptr(), lay, x, tokens, ref)
        assert _noalloc(lib, torch, slot, lay, x, tokens, got) == 0
        torch.cuda.synchronize()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        for t in range(tokens):
            assert normwise_rel(g[t], r[t]) <= 1e-4, (call, t, normwise_rel(g[t], r[t]))
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_limits(torch):
    import osm_b200 as osm
    from osm_b200 import _lib

    lib = _lib.load()
    lay = osm.expert_layout(2048, 512)
    slot = torch.zeros(lay.stride, dtype=torch.uint8, device="cuda")
    x = torch.zeros(17, 2048, device="cuda")
    out = torch.zeros(17, 2048, device="cuda")
    assert _noalloc(lib, torch, slot, lay, x, 17, out) == OSM_EINVAL
    assert _noalloc(lib, torch, slot, lay, x, 0, out) == OSM_EINVAL
    torch.cuda.synchronize()
    assert float(out.abs().max()) == 0.0  # nothing ran
