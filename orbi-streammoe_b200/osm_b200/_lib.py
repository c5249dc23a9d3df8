"""ctypes declarations of include/osm_b200.h (libosm_b200.so, built in-tree).

Loading fails loudly when the library is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libosm_b200.so")

OSM_OK = 0
OSM_EINVAL = -1
OSM_ERUNTIME = -2
OSM_ECUDA = -3
OSM_ENOMEM = -4
OSM_ENOTRES = -5
OSM_ETIMEOUT = -6

OSM_ROUTE_EXACT = 0x1
OSM_RMSNORM_EXACT = 0x2
OSM_ADD_RESIDUAL = 0x4
OSM_PREFILL_BF16 = 0x8
OSM_INPUT_F16 = 0x10
OSM_OUTPUT_F16 = 0x20
OSM_PREFILL_NO_CHECK = 0x40
OSM_CACHED_EARLY = 0x80
OSM_PLAN_SUBLAYER = 0x100
OSM_PLAN_PROFILE = 0x200

KERNEL_KINDS = 8

STATUS_NONFINITE = 1
STATUS_BADMASS = 2
STATUS_NOTRESIDENT = 4
STATUS_BADSLOT = 8


class ExpertLayout(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("inter", C.c_uint32), ("group", C.c_uint32),
                ("reserved", C.c_uint32),
                ("gate_w", C.c_uint64), ("gate_s", C.c_uint64), ("gate_b", C.c_uint64),
                ("up_w", C.c_uint64), ("up_s", C.c_uint64), ("up_b", C.c_uint64),
                ("down_w", C.c_uint64), ("down_s", C.c_uint64), ("down_b", C.c_uint64),
                ("stride", C.c_uint64)]


class LayerDesc(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("experts", C.c_uint32), ("top_k", C.c_uint32),
                ("norm_topk_prob", C.c_uint32),
                ("router_weight_host", C.c_void_p), ("logit_bias_host", C.c_void_p),
                ("shared_slot_host", C.c_void_p), ("shared_layout", ExpertLayout),
                ("shared_gate_host", C.c_void_p), ("norm_weight_host", C.c_void_p),
                ("norm_eps", C.c_float)]


class CacheCounts(C.Structure):
    _fields_ = [("hits", C.c_uint64), ("misses", C.c_uint64), ("loads", C.c_uint64),
                ("evictions", C.c_uint64), ("resident_entries", C.c_uint64),
                ("resident_bytes", C.c_uint64), ("budget_bytes", C.c_uint64)]


# int source(void* user, uint32_t layer, uint32_t expert, const void** src)
CACHE_SOURCE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(C.c_void_p))

# name -> (restype, argtypes)
_P = C.c_void_p
_SIGS = {
    "osm_expert_layout_packed": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(ExpertLayout)]),
    "osm_context_create": (C.c_int, [C.c_int, C.c_uint32, C.POINTER(_P)]),
    "osm_device_info": (C.c_int, [C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_uint32),
                                  C.POINTER(C.c_uint32)]),
    "osm_context_destroy": (C.c_int, [_P]),
    "osm_last_error": (C.c_char_p, [_P]),
    "osm_context_device": (C.c_int, [_P]),
    "osm_context_stream": (_P, [_P]),
    "osm_context_set_stream": (C.c_int, [_P, _P]),
    "osm_context_reset_stream": (C.c_int, [_P]),
    "osm_context_synchronize": (C.c_int, [_P]),
    "osm_context_status": (C.c_int, [_P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)]),
    "osm_context_launches": (C.c_uint64, [_P]),
    "osm_context_profile": (C.c_int, [_P, C.c_int]),
    "osm_context_profile_read": (C.c_int, [_P, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "osm_kernel_kind_name": (C.c_char_p, [C.c_int]),
    "osm_device_alloc": (C.c_int, [_P, C.c_size_t, C.POINTER(_P)]),
    "osm_device_free": (C.c_int, [_P, _P]),
    "osm_upload": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "osm_download": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "osm_host_alloc_pinned": (C.c_int, [C.c_size_t, C.POINTER(_P)]),
    "osm_host_free_pinned": (C.c_int, [_P]),
    "osm_q4_dequant": (C.c_int, [_P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P]),
    "osm_q4_gemv": (C.c_int, [_P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P, C.c_uint32, _P]),
    "osm_test_set_copy_wait_polls": (C.c_int, [C.c_int, C.c_uint32]),
    "osm_layer_set_router_q8": (C.c_int, [_P, _P, _P, _P, C.c_uint32]),
    "osm_ep_create": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                C.c_uint32, C.c_int, C.POINTER(_P)]),
    "osm_ep_ipc_handle": (C.c_int, [_P, C.c_char_p]),
    "osm_ep_open_peers": (C.c_int, [_P, C.c_char_p]),
    "osm_ep_set_timeout": (C.c_int, [_P, C.c_uint32]),
    "osm_ep_destroy": (C.c_int, [_P]),
    "osm_ep_forward": (C.c_int, [_P, _P, _P, _P, C.c_uint32, _P, _P, _P, C.c_uint32]),
    "osm_q4_dequant_f32": (C.c_int, [_P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P]),
    "osm_q4_gemv_f32": (C.c_int, [_P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P, C.c_uint32, _P]),
    "osm_swiglu": (C.c_int, [_P, _P, _P, _P, C.c_size_t]),
    "osm_weighted_accumulate": (C.c_int, [_P, _P, C.c_float, _P, C.c_size_t]),
    "osm_rms_norm": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P, C.c_float, C.c_uint32]),
    "osm_expert_forward": (C.c_int, [_P, _P, C.POINTER(ExpertLayout), _P, C.c_uint32, _P]),
    "osm_expert_forward_noalloc": (C.c_int, [_P, C.POINTER(ExpertLayout), _P, C.c_uint32, _P, _P]),
    "osm_slab_create": (C.c_int, [_P, C.POINTER(ExpertLayout), C.c_uint32, C.POINTER(_P)]),
    "osm_slab_destroy": (C.c_int, [_P]),
    "osm_slab_slots": (C.c_uint32, [_P]),
    "osm_slab_layout": (C.c_int, [_P, _P]),
    "osm_slab_slot_ptr": (_P, [_P, C.c_uint32]),
    "osm_slab_fill_async": (C.c_int, [_P, C.c_uint32, _P]),
    "osm_slab_fill_wait": (C.c_int, [_P, C.c_uint32]),
    "osm_slab_h2d_bytes": (C.c_uint64, [_P]),
    "osm_layer_create": (C.c_int, [_P, C.POINTER(LayerDesc), C.POINTER(_P)]),
    "osm_layer_destroy": (C.c_int, [_P]),
    "osm_layer_bind_slab": (C.c_int, [_P, _P, _P]),
    "osm_layer_set_slot": (C.c_int, [_P, C.c_uint32, C.c_int32]),
    "osm_moe_route": (C.c_int, [_P, _P, C.c_uint32, _P, _P, _P, C.c_uint32]),
    "osm_moe_route_logits": (C.c_int, [_P, _P, C.c_uint32, _P, _P, _P, _P]),
    "osm_moe_forward": (C.c_int, [_P, _P, C.c_uint32, _P, _P, _P, _P, _P, _P, C.c_uint32]),
    "osm_moe_experts": (C.c_int, [_P, _P, C.c_uint32, _P, _P, _P, _P, _P, C.c_uint32]),
    "osm_gather_sum_rows": (C.c_int, [_P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P, _P]),
    "osm_moe_forward_cached": (C.c_int, [_P, _P, C.c_uint32, _P, C.c_uint32, _P, _P, _P, _P, _P,
                                         C.c_uint32]),
    "osm_moe_sublayer_forward": (C.c_int, [_P, _P, C.c_uint32, _P, _P, _P, _P, _P, _P, C.c_uint32]),
    "osm_plan_create": (C.c_int, [_P, C.c_uint32, _P, _P, _P, _P, _P, _P, C.c_uint32, C.POINTER(_P)]),
    "osm_plan_launch": (C.c_int, [_P]),
    "osm_plan_destroy": (C.c_int, [_P]),
    "osm_plan_profile_read": (C.c_int, [_P, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "osm_plan_kernels": (C.c_uint32, [_P]),
    "osm_gen_normal": (C.c_int, [_P, C.c_uint64, C.c_uint64, C.c_float, _P, C.c_size_t, C.c_size_t]),
    "osm_gen_expert_slots": (C.c_int, [_P, C.c_uint64, C.c_uint64, C.c_float, C.c_uint32, C.c_uint32]),
    "osm_cache_create": (C.c_int, [_P, C.c_uint64, C.c_uint64, CACHE_SOURCE_FN, _P, C.POINTER(_P)]),
    "osm_cache_destroy": (C.c_int, [_P]),
    "osm_cache_last_error": (C.c_char_p, [_P]),
    "osm_cache_bind_layer": (C.c_int, [_P, C.c_uint32, _P]),
    "osm_cache_get": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.POINTER(C.c_int32)]),
    "osm_cache_acquire": (C.c_int, [_P, C.c_uint32, _P, C.c_uint32]),
    "osm_cache_contains": (C.c_int, [_P, C.c_uint32, C.c_uint32]),
    "osm_cache_stats": (C.c_int, [_P, C.POINTER(CacheCounts)]),
    "osm_cache_time_copies": (C.c_int, [_P, C.c_int]),
    "osm_cache_exposed_read": (C.c_int, [_P, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
}

_lib = None


def load(path: str | None = None) -> C.CDLL:
    """Load libosm_b200.so (raises if it is missing: no fallback exists).
    OSM_LIB_PATH selects another build of the same library."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("OSM_LIB_PATH") or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with __graft_entry__.build() "
            "(the CUDA path has no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def declared_symbols() -> list[str]:
    return list(_SIGS)
