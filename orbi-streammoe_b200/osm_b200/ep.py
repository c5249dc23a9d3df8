"""Expert parallelism for prefill-sized batches (configs 2 and 3): one process
per GPU, rank r owning experts [r E/N, (r+1) E/N) in its slab.

Each rank routes its own tokens with the replicated router (ids exact as the
single-GPU path), then:
  1. sorts its (token, pick) pairs by the rank that owns the picked expert;
  2. exchanges pair counts, then the pairs' activation rows (fp16) with the
     owner-local expert id and routing weight, in one all-to-all each;
  3. runs the owned experts on the rows it received, together with its own
     tokens routed to the shared expert when the layer has one (held in the
     slab's spare last slot, weighted by its sigmoid gate): one tensor-core
     prefill call on the fp16 rows, one pick per row, each row scaled by its
     weight, fp16 rows out;
  4. sends the weighted fp16 rows back with the reverse all-to-all;
  5. adds each token's rows in pick order, then the shared expert (replicated,
     computed locally for the rank's own tokens) scaled by its sigmoid gate --
     the accumulation order of run_qwen_sparse_moe_vulkan_accum
     (src/model/routed_moe.cpp:396-404).

The exchange steps are plain functions of tensors and a process group, so the
index arithmetic runs unchanged on gloo ranks on the CPU; ExpertParallelMoE
binds them to the library's kernels on CUDA ranks (NCCL over NVLink)."""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def dispatch_plan(ids: torch.Tensor, e_local: int, world: int):
    """Send order of the flattened (token, pick) pairs grouped by owner rank
    (stable: token-major, then pick, inside each destination), pairs per
    destination, and each pair's expert id local to its owner."""
    flat = ids.reshape(-1).long()
    owner = flat // e_local
    if flat.numel() and int(owner.max()) >= world:
        raise ValueError("expert id beyond the last rank's range")
    order = torch.sort(owner, stable=True).indices
    counts = torch.bincount(owner, minlength=world)
    return order, counts, (flat % e_local)


def exchange_counts(send_counts: torch.Tensor, group=None) -> torch.Tensor:
    recv = torch.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts, group=group)
    return recv


def dispatch_rows(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, e_local: int, world: int,
                  group=None, row_dtype=torch.float16, extra_rows: int = 0):
    """Steps 1-2: returns (received rows, their local expert ids, their routing
    weights, state for combine_rows).  The rows are gathered after one
    conversion of x to `row_dtype` (none when x has it already); the returned
    row buffer has `extra_rows` more rows after the received ones, left for
    the caller to fill."""
    T, k = ids.shape
    order, send_counts, local = dispatch_plan(ids, e_local, world)
    recv_counts = exchange_counts(send_counts.to(x.device), group).cpu()
    send_counts = send_counts.cpu()
    ss, rs = send_counts.tolist(), recv_counts.tolist()
    n_recv = int(sum(rs))
    tok = torch.div(order, k, rounding_mode="floor")
    xr = x if x.dtype == row_dtype else x.to(row_dtype)
    send_x = xr.index_select(0, tok)
    meta = torch.stack([local.index_select(0, order).to(torch.float32),
                        w.reshape(-1).index_select(0, order).to(torch.float32)], dim=1).contiguous()
    recv_x = torch.empty(n_recv + extra_rows, x.shape[1], dtype=row_dtype, device=x.device)
    recv_meta = torch.empty(n_recv, 2, dtype=torch.float32, device=x.device)
    dist.all_to_all_single(recv_x[:n_recv], send_x, rs, ss, group=group)
    dist.all_to_all_single(recv_meta, meta, rs, ss, group=group)
    state = (order, ss, rs, T, k)
    return recv_x, recv_meta[:, 0].to(torch.int32), recv_meta[:, 1].contiguous(), state


def combine_rows(y_recv: torch.Tensor, state, group=None, row_dtype=torch.float16, extra=None,
                 out=None, ctx=None):
    """Steps 4-5: the weighted rows back to their tokens (sent as `row_dtype`),
    each token's rows summed in pick order in fp32, then + extra[t] (the
    token's own shared-expert row) when given.  Returns [T, H] fp32 (`out`
    when given).  With a library context and fp16 CUDA rows the sum reads the
    returned rows in place through the inverse of the dispatch permutation
    (osm_gather_sum_rows); otherwise torch gathers them first: the same adds
    in the same order."""
    order, ss, rs, T, k = state
    H = y_recv.shape[1]
    back = torch.empty(len(order), H, dtype=row_dtype, device=y_recv.device)
    send = y_recv if y_recv.dtype == row_dtype else y_recv.to(row_dtype)
    dist.all_to_all_single(back, send.contiguous(), ss, rs, group=group)
    inv = torch.empty_like(order)
    inv[order] = torch.arange(len(order), device=order.device, dtype=order.dtype)
    if ctx is not None and back.is_cuda and row_dtype == torch.float16:
        res = out if out is not None else torch.empty(T, H, dtype=torch.float32, device=back.device)
        ctx.gather_sum_rows(back, inv, T, k, res, extra=extra)
        return res
    y = back.index_select(0, inv).view(T, k, H)
    acc = y[:, 0].to(torch.float32, copy=True)
    for p in range(1, k):
        acc.add_(y[:, p])
    if extra is not None:
        acc.add_(extra)
    if out is not None:
        out.copy_(acc)
        return out
    return acc


class ExpertParallelMoE:
    """The Q4 routed-MoE sublayer with its experts spread over the ranks of a
    process group (NCCL, one GPU per rank).  `slab` holds this rank's experts
    [e_first, e_first + e_count) in slots 0..e_count-1; for a layer with a
    shared expert (Qwen3-Next) it has one more slot, which receives it, and
    the shared expert and its gate row are replicated like the router weight.
    Layers without one (Qwen3-30B-A3B) pass shared_slot=None.  The context's
    max_tokens must cover the rows a rank can receive plus its own tokens."""

    def __init__(self, ctx, W: np.ndarray, k: int, norm: bool, layout, slab, e_first: int,
                 e_count: int, shared_slot=None, shared_gate=None, bias=None, group=None):
        import osm_b200 as osm

        self.ctx, self.k, self.group = ctx, k, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e_first, self.e_count = e_first, e_count
        self.has_shared = shared_slot is not None
        if self.has_shared and shared_gate is None:
            raise ValueError("a shared expert needs its gate row")
        H = W.shape[1]
        n_local = e_count + (1 if self.has_shared else 0)
        if slab.slots < n_local:
            raise ValueError("the slab needs a slot per owned expert, plus one for a shared expert")
        self.router = osm.Layer(ctx, W, k, norm, logit_bias=bias)
        if self.has_shared:
            self._sh_host = torch.from_numpy(np.ascontiguousarray(shared_slot).reshape(-1)).pin_memory()
            slab.fill_async(e_count, self._sh_host.data_ptr())
            slab.fill_wait()
            self.gate = torch.from_numpy(np.asarray(shared_gate, np.float32)).cuda()
        # local experts 0..e_count-1, then the shared expert as local id e_count
        self.experts = osm.Layer(ctx, np.zeros((n_local, H), np.float32), 1, False)
        self.experts.bind_slab(slab, np.arange(n_local, dtype=np.int32))

    def forward(self, x: torch.Tensor, out: torch.Tensor, ids: torch.Tensor | None = None,
                weights: torch.Tensor | None = None):
        T, H = x.shape
        dev = x.device
        ids = ids if ids is not None else torch.empty(T, self.k, dtype=torch.int32, device=dev)
        w = weights if weights is not None else torch.empty(T, self.k, device=dev)
        self.router.route_qwen_top_k(x, T, ids, w)
        x16 = x.to(torch.float16)
        ns = T if self.has_shared else 0
        # received rows, then this rank's own tokens for the shared expert
        rows, recv_ids, recv_w, state = dispatch_rows(x16, ids, w, self.e_count, self.world,
                                                      self.group, extra_rows=ns)
        n = rows.shape[0] - ns
        rid, rw = recv_ids, recv_w
        if self.has_shared:
            rows[n:].copy_(x16)
            rid = torch.cat([recv_ids, torch.full((T,), self.e_count, dtype=torch.int32, device=dev)])
            rw = torch.cat([recv_w, torch.sigmoid(x @ self.gate)]).contiguous()
        y = torch.empty(n + ns, H, dtype=torch.float16, device=dev)   # fp16 rows out
        if n + ns > 0:  # a rank may own no picked expert and have no shared expert
            self.experts.run_experts(rows, n + ns, rid.view(-1, 1).contiguous(), rw.view(-1, 1), y,
                                     prefill=True)
        # routed rows in pick order, then the shared expert's row
        combine_rows(y[:n], state, self.group, extra=y[n:] if self.has_shared else None, out=out,
                     ctx=self.ctx)
        return ids, w
