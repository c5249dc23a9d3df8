"""osm_expert_forward_noalloc: the single-expert forward for hosts that cannot
call cudaMalloc where experts run (a server whose device memory belongs to a
pool allocator that forbids driver allocations after warm-up, or a plugin that
only borrows a CUDA context).  Its intermediates live in one fixed device array
of the library instead of a context's scratch.

Checked through the C ABI against osm_expert_forward (the context entry point)
and against the CPU oracle's dequantised expert (gate, up, SwiGLU, down in the
reference's operation order), within the 1e-4 normwise tolerance of the fp32
path, on calls in a row with different inputs and token counts (a larger call
followed by a smaller one), so that contents left in the shared array by one
call cannot leak into the next.  This file is collected last: a stop at the
first failure has run every other test first.
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


def _oracle_expert(port, slot_bytes, H, I, x):
    gate, up, down = port.dequant_slot(slot_bytes, H, I)
    return np.stack([port.matvec(down, port.swiglu(port.matvec(gate, xt), port.matvec(up, xt)))
                     for xt in x])


@pytest.mark.parametrize("H,I,calls", [(2048, 512, (5, 2)), (512, 256, (16, 3)),
                                       (2048, 768, (1, 1))])
def test_noalloc_matches_context_entry_point_and_oracle(torch, H, I, calls):
    import osm_b200 as osm
    import pyoracle
    from osm_b200 import _lib

    lib = _lib.load()
    port = pyoracle.Oracle("port")
    lay = osm.expert_layout(H, I)
    slot_bytes = port.gen_expert_slot(33, 400 + H + I, 0.02, H, I)
    slot = torch.from_numpy(slot_bytes).cuda()
    ctx = osm.Context(0, max_tokens=16)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    for call, tokens in enumerate(calls):
        xh = port.gen_normal(33, 50 + call, 1.0 + call, tokens * H).reshape(tokens, H)
        x = torch.from_numpy(xh).cuda()
        ref = torch.empty(tokens, H, device="cuda")
        got = torch.full((tokens, H), float("nan"), device="cuda")
        ctx.expert_forward(slot.data_ptr(), lay, x, tokens, ref)
        assert _noalloc(lib, torch, slot, lay, x, tokens, got) == 0
        torch.cuda.synchronize()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        o = _oracle_expert(port, slot_bytes, H, I, xh)
        for t in range(tokens):
            assert normwise_rel(g[t], r[t]) <= 1e-4, (call, t, normwise_rel(g[t], r[t]))
            assert normwise_rel(g[t], o[t]) <= 1e-4, (call, t, normwise_rel(g[t], o[t]))
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_limits(torch):
    """16 tokens, hidden 2048 and inter 768 are the limits of the fixed array:
    anything beyond them is refused before any GPU work (out stays zero)."""
    import osm_b200 as osm
    from osm_b200 import _lib

    lib = _lib.load()
    for H, I, tokens in ((2048, 512, 17), (2048, 512, 0), (2304, 512, 1), (2048, 1024, 1)):
        lay = osm.expert_layout(H, I)
        slot = torch.zeros(lay.stride, dtype=torch.uint8, device="cuda")
        x = torch.zeros(max(tokens, 1), H, device="cuda")
        out = torch.zeros(max(tokens, 1), H, device="cuda")
        assert _noalloc(lib, torch, slot, lay, x, tokens, out) == OSM_EINVAL, (H, I, tokens)
        torch.cuda.synchronize()
        assert float(out.abs().max()) == 0.0  # nothing ran
