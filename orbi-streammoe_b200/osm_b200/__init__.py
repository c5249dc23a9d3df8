"""Python handle on the B200 routed-MoE sublayer (C ABI in include/osm_b200.h).

Device buffers are torch CUDA tensors (plumbing only: allocation, streams);
every computation is a call into libosm_b200.so.  Names follow the reference
(ingeniusvictor/orbi-streammoe): ``Context`` <-> VulkanComputeContext,
``Slab`` <-> the device side of VulkanResidentExpertCache, ``Layer`` <->
QwenCheckpointSparseMoeLayer, ``route_qwen_top_k`` <-> route_qwen_top_k_cpu,
``run_qwen_sparse_moe`` <-> run_qwen_sparse_moe_vulkan_accum, and so on.
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from ._lib import (OSM_ADD_RESIDUAL, OSM_CACHED_EARLY, OSM_INPUT_F16, OSM_OUTPUT_F16, OSM_PREFILL_BF16, OSM_RMSNORM_EXACT,  # noqa: F401
                   OSM_ROUTE_EXACT, ExpertLayout, LayerDesc)


class OsmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"osm error {code}: {msg}")
        self.code = code


def lib():
    return _lib.load()


def _ptr(t):
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


def expert_layout(hidden: int, inter: int, group: int = 64) -> ExpertLayout:
    L = ExpertLayout()
    rc = lib().osm_expert_layout_packed(hidden, inter, group, C.byref(L))
    if rc:
        raise OsmError(rc, "invalid expert geometry")
    return L


class Context:
    """One device, one stream, scratch for up to ``max_tokens`` rows."""

    def __init__(self, device: int = 0, max_tokens: int = 256):
        self.h = C.c_void_p()
        rc = lib().osm_context_create(device, max_tokens, C.byref(self.h))
        if rc:
            raise OsmError(rc, "context creation failed")
        self.device = device
        self.max_tokens = max_tokens

    def check(self, rc: int, what: str = ""):
        if rc:
            msg = lib().osm_last_error(self.h).decode()
            raise OsmError(rc, f"{what}: {msg}" if what else msg)

    def close(self):
        if self.h:
            lib().osm_context_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream_handle(self) -> int:
        return lib().osm_context_stream(self.h) or 0

    def set_stream(self, stream_handle: int):
        """Run on this CUDA stream (0 is the default stream, e.g. torch's
        default ``torch.cuda.current_stream().cuda_stream``)."""
        self.check(lib().osm_context_set_stream(self.h, C.c_void_p(stream_handle)))

    def reset_stream(self):
        self.check(lib().osm_context_reset_stream(self.h))

    def synchronize(self):
        self.check(lib().osm_context_synchronize(self.h))

    def status(self):
        st = C.c_uint32()
        ex = C.c_uint64()
        self.check(lib().osm_context_status(self.h, C.byref(st), C.byref(ex)))
        return st.value, ex.value

    @property
    def launches(self) -> int:
        return lib().osm_context_launches(self.h)

    def profile(self, enable: bool):
        self.check(lib().osm_context_profile(self.h, int(bool(enable))))

    def profile_read(self) -> dict:
        """{kernel kind: (total ms, launches)} since the last read."""
        n = _lib.KERNEL_KINDS
        ms = (C.c_double * n)()
        cnt = (C.c_uint64 * n)()
        self.check(lib().osm_context_profile_read(self.h, ms, cnt))
        return {lib().osm_kernel_kind_name(i).decode(): (ms[i], cnt[i]) for i in range(n)
                if cnt[i]}

    # ---- element-wise ops (Vulkan kernel replacements) ----
    def q4_dequant(self, packed, scales_bf16, biases_bf16, rows, in_dim, out, group=64):
        self.check(lib().osm_q4_dequant(self.h, _ptr(packed), _ptr(scales_bf16), _ptr(biases_bf16),
                                        rows, in_dim, group, _ptr(out)), "q4_dequant")

    def q4_gemv(self, packed, scales_bf16, biases_bf16, out_dim, in_dim, x, tokens, y, group=64):
        self.check(lib().osm_q4_gemv(self.h, _ptr(packed), _ptr(scales_bf16), _ptr(biases_bf16),
                                     out_dim, in_dim, group, _ptr(x), tokens, _ptr(y)), "q4_gemv")

    def q4_dequant_f32(self, packed, scales, biases, rows, in_dim, out, group=64):
        """q4_dequant with fp32 scale and bias."""
        self.check(lib().osm_q4_dequant_f32(self.h, _ptr(packed), _ptr(scales), _ptr(biases),
                                            rows, in_dim, group, _ptr(out)), "q4_dequant_f32")

    def q4_gemv_f32(self, packed, scales, biases, out_dim, in_dim, x, tokens, y, group=64):
        """q4_gemv with fp32 scale and bias."""
        self.check(lib().osm_q4_gemv_f32(self.h, _ptr(packed), _ptr(scales), _ptr(biases),
                                         out_dim, in_dim, group, _ptr(x), tokens, _ptr(y)),
                   "q4_gemv_f32")

    def swiglu(self, gate, up, out):
        self.check(lib().osm_swiglu(self.h, _ptr(gate), _ptr(up), _ptr(out), gate.numel()), "swiglu")

    def weighted_accumulate(self, src, weight, acc):
        self.check(lib().osm_weighted_accumulate(self.h, _ptr(src), float(weight), _ptr(acc),
                                                 src.numel()), "weighted_accumulate")

    def rms_norm(self, values, rows, dim, weight, eps, exact=False):
        self.check(lib().osm_rms_norm(self.h, _ptr(values), rows, dim, _ptr(weight), eps,
                                      OSM_RMSNORM_EXACT if exact else 0), "rms_norm")

    def expert_forward(self, slot_ptr: int, layout: ExpertLayout, x, tokens, out):
        self.check(lib().osm_expert_forward(self.h, C.c_void_p(slot_ptr), C.byref(layout), _ptr(x),
                                            tokens, _ptr(out)), "expert_forward")

    def gather_sum_rows(self, rows, pos, tokens, k, out, extra=None):
        """out[t] = sum over p < k of rows[pos[t k + p]] in pick order, then +
        extra[t] (fp16 rows, int64 positions, fp32 out): the return step of an
        expert-parallel exchange."""
        self.check(lib().osm_gather_sum_rows(self.h, _ptr(rows), _ptr(pos), tokens, k, out.shape[1],
                                             _ptr(extra), _ptr(out)), "gather_sum_rows")

    def gen_normal(self, seed, tensor, sigma, out, first=0):
        self.check(lib().osm_gen_normal(self.h, seed, tensor, sigma, _ptr(out), out.numel(), first),
                   "gen_normal")


class Slab:
    """Fixed-stride expert slots in HBM."""

    def __init__(self, ctx: Context, layout: ExpertLayout, slots: int):
        self.ctx = ctx
        self.layout = layout
        self.h = C.c_void_p()
        ctx.check(lib().osm_slab_create(ctx.h, C.byref(layout), slots, C.byref(self.h)), "slab")
        self.slots = slots

    def close(self):
        if self.h:
            lib().osm_slab_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def slot_ptr(self, slot: int) -> int:
        return lib().osm_slab_slot_ptr(self.h, slot) or 0

    def fill_async(self, slot: int, host_ptr: int):
        self.ctx.check(lib().osm_slab_fill_async(self.h, slot, C.c_void_p(host_ptr)), "slab fill")

    def fill_wait(self, timeout_ms: int = 5000):
        self.ctx.check(lib().osm_slab_fill_wait(self.h, timeout_ms), "slab fill wait")

    @property
    def h2d_bytes(self) -> int:
        return lib().osm_slab_h2d_bytes(self.h)

    def generate(self, seed: int, tensor_base: int, sigma: float, first: int, count: int):
        self.ctx.check(lib().osm_gen_expert_slots(self.h, seed, tensor_base, sigma, first, count),
                       "gen_expert_slots")


class Layer:
    """One MoE layer: router (+ optional logit bias), shared expert and its
    scalar gate, optional post-attention norm weight, and the expert slab."""

    def __init__(self, ctx: Context, router_weight, top_k: int, norm_topk_prob: bool = True,
                 logit_bias=None, shared_slot=None, shared_layout: ExpertLayout | None = None,
                 shared_gate=None, norm_weight=None, norm_eps: float = 1e-6):
        import numpy as np

        self.ctx = ctx
        rw = np.ascontiguousarray(router_weight, np.float32)
        E, H = rw.shape
        keep = [rw]
        d = LayerDesc()
        d.hidden, d.experts, d.top_k, d.norm_topk_prob = H, E, top_k, int(bool(norm_topk_prob))
        d.router_weight_host = rw.ctypes.data
        if logit_bias is not None:
            lb = np.ascontiguousarray(logit_bias, np.float32)
            keep.append(lb)
            d.logit_bias_host = lb.ctypes.data
        if shared_slot is not None:
            ss = np.ascontiguousarray(shared_slot, np.uint8)
            sg = np.ascontiguousarray(shared_gate, np.float32)
            keep += [ss, sg]
            d.shared_slot_host = ss.ctypes.data
            d.shared_layout = shared_layout
            d.shared_gate_host = sg.ctypes.data
        if norm_weight is not None:
            nw = np.ascontiguousarray(norm_weight, np.float32)
            keep.append(nw)
            d.norm_weight_host = nw.ctypes.data
        d.norm_eps = norm_eps
        self.h = C.c_void_p()
        ctx.check(lib().osm_layer_create(ctx.h, C.byref(d), C.byref(self.h)), "layer")
        self.hidden, self.experts, self.top_k = H, E, top_k
        self.has_shared = shared_slot is not None

    def close(self):
        if self.h:
            lib().osm_layer_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def bind_slab(self, slab: Slab, slot_of_expert):
        import numpy as np

        so = np.ascontiguousarray(slot_of_expert, np.int32)
        self.slab = slab
        self.ctx.check(lib().osm_layer_bind_slab(self.h, slab.h, C.c_void_p(so.ctypes.data)), "bind")

    def set_slot(self, expert: int, slot: int):
        self.ctx.check(lib().osm_layer_set_slot(self.h, expert, slot), "set_slot")

    def set_router_q8(self, packed, scales_bf16, biases_bf16, group=64):
        """Keeps the router 8-bit on the device (MLX affine: packed [E][H/4]
        uint32, bf16 scale and bias bits [E][H/64]); logits and ids are those
        of the fp32 router cpu::dequantize_affine_rows would give."""
        import numpy as np

        pk = np.ascontiguousarray(packed, np.uint32)
        sc = np.ascontiguousarray(scales_bf16, np.uint16)
        bi = np.ascontiguousarray(biases_bf16, np.uint16)
        self.ctx.check(lib().osm_layer_set_router_q8(self.h, C.c_void_p(pk.ctypes.data),
                                                     C.c_void_p(sc.ctypes.data),
                                                     C.c_void_p(bi.ctypes.data), group),
                       "set_router_q8")

    def route_qwen_top_k(self, x, tokens, ids, weights, mass=None, exact=False):
        self.ctx.check(lib().osm_moe_route(self.h, _ptr(x), tokens, _ptr(ids), _ptr(weights),
                                           _ptr(mass), OSM_ROUTE_EXACT if exact else 0), "route")

    def route_qwen_top_k_logits(self, x, tokens, logits, ids=None, weights=None, mass=None):
        """Every token on the reference's own arithmetic, with its logits
        (W x, plus the logit bias when the layer has one) in `logits`
        [tokens][experts] fp32."""
        self.ctx.check(lib().osm_moe_route_logits(self.h, _ptr(x), tokens, _ptr(logits), _ptr(ids),
                                                  _ptr(weights), _ptr(mass)), "route_logits")

    def run_qwen_sparse_moe(self, x, tokens, out, ids=None, weights=None, mass=None,
                            shared_gate=None, residual=None, exact_route=False, prefill=False,
                            check_range=True):
        """prefill=True: experts as the 16-bit tcgen05 grouped GEMM (outputs
        within 2e-3 of the fp32 path; for prefill-sized batches).  With
        check_range (the default) the call synchronises at its end and re-runs
        on the fp32 path when a value left the fp16 range (status bit 6)."""
        flags = ((OSM_ROUTE_EXACT if exact_route else 0) | (OSM_ADD_RESIDUAL if residual is not None else 0)
                 | (OSM_PREFILL_BF16 if prefill else 0)
                 | (0 if check_range else _lib.OSM_PREFILL_NO_CHECK))
        self.ctx.check(lib().osm_moe_forward(self.h, _ptr(x), tokens, _ptr(out), _ptr(ids),
                                             _ptr(weights), _ptr(mass), _ptr(shared_gate),
                                             _ptr(residual), flags), "moe_forward")

    def run_experts(self, x, tokens, ids, weights, out, shared_gate=None, residual=None,
                    prefill=False):
        """prefill=True: tensor-core path; an fp16 x (torch.float16) is passed
        as is (OSM_INPUT_F16, layers without a shared expert), and an fp16
        `out` receives fp16 rows (OSM_OUTPUT_F16)."""
        f16 = str(getattr(x, "dtype", "")) == "torch.float16"
        f16_out = str(getattr(out, "dtype", "")) == "torch.float16"
        flags = ((OSM_ADD_RESIDUAL if residual is not None else 0) | (OSM_PREFILL_BF16 if prefill else 0)
                 | (OSM_INPUT_F16 if f16 else 0) | (OSM_OUTPUT_F16 if f16_out else 0))
        self.ctx.check(lib().osm_moe_experts(self.h, _ptr(x), tokens, _ptr(ids), _ptr(weights),
                                             _ptr(out), _ptr(shared_gate), _ptr(residual), flags),
                       "moe_experts")

    def run_cached(self, cache: "ExpertCache", layer_id: int, x, tokens, out, ids=None,
                   weights=None, shared_gate=None, residual=None, exact_route=False,
                   prefill=False, early=False):
        """run_qwen_sparse_moe_vulkan_accum with its expert cache: route, make
        the picks resident through ``cache`` (this layer bound as
        ``layer_id``), run the experts.  early: one or two tokens, the
        experts are queued behind the router before the picks reach the host
        (OSM_CACHED_EARLY; same result)."""
        flags = ((OSM_ROUTE_EXACT if exact_route else 0) | (OSM_ADD_RESIDUAL if residual is not None else 0)
                 | (OSM_PREFILL_BF16 if prefill else 0) | (OSM_CACHED_EARLY if early else 0))
        rc = lib().osm_moe_forward_cached(self.h, cache.h, layer_id, _ptr(x), tokens, _ptr(out),
                                          _ptr(ids), _ptr(weights), _ptr(shared_gate),
                                          _ptr(residual), flags)
        self.ctx.check(rc, "moe_forward_cached")

    def run_sublayer(self, residual, tokens, out, normalized=None, ids=None, weights=None,
                     mass=None, shared_gate=None, exact_route=False, exact_rmsnorm=False,
                     prefill=False):
        flags = ((OSM_ROUTE_EXACT if exact_route else 0) | (OSM_RMSNORM_EXACT if exact_rmsnorm else 0)
                 | (OSM_PREFILL_BF16 if prefill else 0))
        self.ctx.check(lib().osm_moe_sublayer_forward(self.h, _ptr(residual), tokens, _ptr(out),
                                                      _ptr(normalized), _ptr(ids), _ptr(weights),
                                                      _ptr(mass), _ptr(shared_gate), flags),
                       "sublayer")


class Plan:
    """One sublayer call captured as a CUDA graph on fixed device buffers
    (optionally with the pinned-host H2D of x and D2H of out)."""

    def __init__(self, layer: Layer, tokens: int, x, out, ids=None, weights=None, x_host=None,
                 out_host=None, exact_route=False, sublayer=False, profile=False):
        self.layer = layer
        flags = ((_lib.OSM_ROUTE_EXACT if exact_route else 0)
                 | (_lib.OSM_PLAN_SUBLAYER if sublayer else 0)
                 | (_lib.OSM_PLAN_PROFILE if profile else 0))
        self.h = C.c_void_p()
        layer.ctx.check(lib().osm_plan_create(layer.h, tokens, _ptr(x), _ptr(out), _ptr(ids),
                                              _ptr(weights), _ptr(x_host), _ptr(out_host), flags,
                                              C.byref(self.h)), "plan")
        self.kernels = lib().osm_plan_kernels(self.h)

    def launch(self):
        self.layer.ctx.check(lib().osm_plan_launch(self.h), "plan launch")

    def profile_read(self) -> dict:
        n = _lib.KERNEL_KINDS
        ms = (C.c_double * n)()
        cnt = (C.c_uint64 * n)()
        self.layer.ctx.check(lib().osm_plan_profile_read(self.h, ms, cnt))
        return {lib().osm_kernel_kind_name(i).decode(): (ms[i], cnt[i]) for i in range(n)
                if cnt[i]}

    def close(self):
        if self.h:
            lib().osm_plan_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertCache:
    """HBM expert residency with the reference's LFU + recency policy
    (VulkanResidentExpertCache).  ``source(layer, expert)`` returns the
    address of the expert's slot bytes in (pinned) host memory; with
    ``slab=None`` only the policy runs (no copies)."""

    def __init__(self, slab, budget_bytes: int, accounted_bytes: int = 0, source=None):
        self._source = source

        def _cb(user, layer, expert, out):
            try:
                out[0] = int(self._source(layer, expert)) if self._source else 0
                return 0
            except Exception:  # the C side reports the failure
                return -1

        self._cb = _lib.CACHE_SOURCE_FN(_cb)
        self.h = C.c_void_p()
        rc = lib().osm_cache_create(slab.h if slab is not None else None, budget_bytes,
                                    accounted_bytes, self._cb, None, C.byref(self.h))
        if rc:
            raise OsmError(rc, "cache creation failed")

    def _check(self, rc, what):
        if rc:
            raise OsmError(rc, f"{what}: {lib().osm_cache_last_error(self.h).decode()}")

    def bind_layer(self, layer_id: int, layer: "Layer"):
        self._check(lib().osm_cache_bind_layer(self.h, layer_id, layer.h), "bind_layer")

    def get(self, layer_id: int, expert: int) -> int:
        slot = C.c_int32()
        self._check(lib().osm_cache_get(self.h, layer_id, expert, C.byref(slot)), "get")
        return slot.value

    def acquire(self, layer_id: int, experts) -> None:
        arr = (C.c_uint32 * len(experts))(*[int(e) for e in experts])
        self._check(lib().osm_cache_acquire(self.h, layer_id, arr, len(experts)), "acquire")

    def contains(self, layer_id: int, expert: int) -> bool:
        return bool(lib().osm_cache_contains(self.h, layer_id, expert))

    def stats(self) -> dict:
        c = _lib.CacheCounts()
        self._check(lib().osm_cache_stats(self.h, C.byref(c)), "stats")
        return {f: getattr(c, f) for f, _ in c._fields_}

    def time_copies(self, enable: bool):
        """Bracket each acquire's copies with compute-stream events."""
        self._check(lib().osm_cache_time_copies(self.h, int(bool(enable))), "time_copies")

    def exposed_read(self):
        """(ms the compute stream spent waiting on copies, number of waits)
        since the last read."""
        ms = C.c_double()
        n = C.c_uint64()
        self._check(lib().osm_cache_exposed_read(self.h, C.byref(ms), C.byref(n)), "exposed_read")
        return ms.value, n.value

    def close(self):
        if self.h:
            lib().osm_cache_destroy(self.h)
            self.h = C.c_void_p()

