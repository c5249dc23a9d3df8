"""Expert parallelism for prefill-sized batches (configs 2 and 3): one process
per GPU, rank r owning experts [r E/N, (r+1) E/N) in its slab.

The exchange runs inside the library over NVLink peer memory, one call per
step with no host synchronisation (osm_ep_forward): each rank routes its own
tokens with the replicated router (ids exact as on one GPU; the shared
expert's gate comes from the same select kernel), stores each pick's fp16 row
straight into the owner's receive region, and after a device-side barrier the
owner runs its experts -- and this rank's own tokens on the shared expert,
held in the slab's spare last slot -- on the tensor-core prefill path, stores
each result times its routing weight (fp16) into the source's back rows, and
after a second barrier every rank sums its tokens' rows in pick order and then
the shared row, in fp32: the accumulation order of
run_qwen_sparse_moe_vulkan_accum (src/model/routed_moe.cpp:396-404).

The host part is the one-time setup done here: every rank creates its EP
block, exports it as a CUDA IPC handle, and the handles are gathered with the
rank geometry through torch.distributed (any backend; the checks run on gloo
ranks on the CPU), then every peer block is mapped."""
from __future__ import annotations

import ctypes as C
import datetime

import numpy as np
import torch
import torch.distributed as dist

IPC_HANDLE_BYTES = 64
STATUS_PEER_TIMEOUT = 1 << 7


def context_rows(world: int, tokens_per_rank: int, k: int) -> int:
    """Rows of the receive regions an owner runs its experts over: the
    context's max_tokens must be at least this."""
    return (world + 1) * tokens_per_rank * max(k, 1)


def exchange_handles(handle: bytes, geometry: tuple, group=None,
                     timeout: datetime.timedelta | None = None) -> list[bytes]:
    """Every rank's IPC handle in rank order.  All ranks must pass the same
    geometry (world, tokens per rank, k, hidden, experts per rank, shared);
    otherwise every rank raises ValueError.  A rank that does not take part
    makes the others fail with the process group's timeout (RuntimeError)."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("an IPC handle is 64 bytes")
    world = dist.get_world_size(group)
    gathered: list = [None] * world
    try:
        if timeout is None:
            dist.all_gather_object(gathered, (tuple(geometry), bytes(handle)), group=group)
        else:
            # a bounded exchange: monitored_barrier first, so a missing rank
            # is named after `timeout` instead of hanging the collective
            if dist.get_backend(group) == "gloo":
                dist.monitored_barrier(group=group, timeout=timeout, wait_all_ranks=True)
            dist.all_gather_object(gathered, (tuple(geometry), bytes(handle)), group=group)
    except RuntimeError as e:
        raise RuntimeError(f"expert parallel setup: a rank did not join the handle exchange ({e})") from e
    geos = {g for g, _ in gathered}
    if len(geos) != 1:
        raise ValueError(f"expert parallel setup: ranks disagree on the geometry: {sorted(geos)}")
    return [h for _, h in gathered]


class ExpertParallelMoE:
    """The Q4 routed-MoE sublayer with its experts spread over the ranks of a
    process group, one GPU per rank.  `slab` holds this rank's experts
    [e_first, e_first + e_count) in slots 0..e_count-1; for a layer with a
    shared expert (Qwen3-Next) it has one more slot, which receives it, and
    the shared expert and its gate row are replicated like the router weight.
    Layers without one (Qwen3-30B-A3B) pass shared_slot=None.  Each call
    routes at most `tokens_per_rank` tokens; the context's max_tokens must be
    at least context_rows(world, tokens_per_rank, k)."""

    def __init__(self, ctx, W: np.ndarray, k: int, norm: bool, layout, slab, e_first: int,
                 e_count: int, shared_slot=None, shared_gate=None, bias=None, group=None,
                 tokens_per_rank: int | None = None, timeout_ms: int = 2000):
        import osm_b200 as osm

        self.ctx, self.k, self.group = ctx, k, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e_first, self.e_count = e_first, e_count
        self.has_shared = shared_slot is not None
        if self.has_shared and shared_gate is None:
            raise ValueError("a shared expert needs its gate row")
        E, H = W.shape
        if E != e_count * self.world:
            raise ValueError("the router covers every rank's experts: E = e_count * world")
        n_local = e_count + (1 if self.has_shared else 0)
        if slab.slots < n_local:
            raise ValueError("the slab needs a slot per owned expert, plus one for a shared expert")
        if tokens_per_rank is None:
            tokens_per_rank = ctx.max_tokens // ((self.world + 1) * k)
        self.tokens_per_rank = int(tokens_per_rank)
        if ctx.max_tokens < context_rows(self.world, self.tokens_per_rank, k):
            raise ValueError("context max_tokens below context_rows(world, tokens_per_rank, k)")
        # the router computes the shared expert's gate in its select kernel
        self.router = osm.Layer(ctx, W, k, norm, logit_bias=bias,
                                shared_slot=shared_slot if self.has_shared else None,
                                shared_layout=layout if self.has_shared else None,
                                shared_gate=shared_gate if self.has_shared else None)
        if self.has_shared:
            self._sh_host = torch.from_numpy(np.ascontiguousarray(shared_slot).reshape(-1)).pin_memory()
            slab.fill_async(e_count, self._sh_host.data_ptr())
            slab.fill_wait()
        # local experts 0..e_count-1, then the shared expert as local id e_count
        self.experts = osm.Layer(ctx, np.zeros((n_local, H), np.float32), 1, False)
        self.experts.bind_slab(slab, np.arange(n_local, dtype=np.int32))
        lib = osm.lib()
        h = C.c_void_p()
        ctx.check(lib.osm_ep_create(ctx.h, self.world, self.rank, self.tokens_per_rank, k, H,
                                    e_count, 1 if self.has_shared else 0, C.byref(h)), "ep_create")
        self.h = h
        try:
            buf = C.create_string_buffer(IPC_HANDLE_BYTES)
            ctx.check(lib.osm_ep_ipc_handle(self.h, buf), "ep_ipc_handle")
            geometry = (self.world, self.tokens_per_rank, k, H, e_count, int(self.has_shared))
            handles = exchange_handles(buf.raw, geometry, group)
            if self.world > 1:
                ctx.check(lib.osm_ep_open_peers(self.h, b"".join(handles)), "ep_open_peers")
            ctx.check(lib.osm_ep_set_timeout(self.h, int(timeout_ms)), "ep_set_timeout")
        except Exception:
            lib.osm_ep_destroy(self.h)
            self.h = None
            raise

    def forward(self, x: torch.Tensor, out: torch.Tensor, ids: torch.Tensor | None = None,
                weights: torch.Tensor | None = None, exact_route: bool = False):
        """out[t] = the sublayer's output for x[t]; returns (ids, weights).  No
        host synchronisation; a rank that misses a barrier shows as status bit
        7 (STATUS_PEER_TIMEOUT) on the others."""
        import osm_b200 as osm

        T = x.shape[0]
        dev = x.device
        ids = ids if ids is not None else torch.empty(T, self.k, dtype=torch.int32, device=dev)
        w = weights if weights is not None else torch.empty(T, self.k, device=dev)
        flags = osm.OSM_ROUTE_EXACT if exact_route else 0
        self.ctx.check(osm.lib().osm_ep_forward(self.h, self.router.h, self.experts.h,
                                                C.c_void_p(x.data_ptr()), T,
                                                C.c_void_p(out.data_ptr()),
                                                C.c_void_p(ids.data_ptr()), C.c_void_p(w.data_ptr()),
                                                flags), "ep_forward")
        return ids, w

    def close(self):
        """Frees the EP block once every rank is done with every block."""
        import osm_b200 as osm

        if self.h is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        osm.lib().osm_ep_destroy(self.h)
        self.h = None
