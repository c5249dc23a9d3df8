"""ctypes wrapper over the parity checkers (TEST INFRASTRUCTURE ONLY).

Two interchangeable back ends with identical Python signatures:

* ``Oracle("port")``      -- oracle/liboracle.so, the C restatement.
* ``Oracle("reference")`` -- oracle/_ref/libosm_ref.so, the reference's own
  CPU sources compiled in place (src/cpu/reference_ops.cpp,
  src/model/qwen_router.cpp, ...).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module; the product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libosm_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_sz = C.c_size_t


class OracleError(RuntimeError):
    """Raised for a non-zero oracle status (-1 invalid argument, -2 runtime)."""

    def __init__(self, rc: int, what: str):
        super().__init__(f"{what}: oracle status {rc}")
        self.rc = rc


def build() -> None:
    """Build liboracle.so (and _ref when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def _ptr_array(arrs):
    out = (C.c_void_p * len(arrs))()
    for i, a in enumerate(arrs):
        out[i] = None if a is None else a.ctypes.data
    return out


class Oracle:
    def __init__(self, kind: str = "port"):
        path = PORT_LIB if kind == "port" else REF_LIB
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.kind = kind
        self.lib = C.CDLL(path)
        p = "osm_oracle_" if kind == "port" else "osm_ref_"
        self.p = p
        L = self.lib
        self._dq = getattr(L, p + "dequantize_affine_rows")
        self._dq.argtypes = [_u32p, _sz, _sz, _f32p, _f32p, C.c_uint32, C.c_uint32, _f32p]
        self._mv = getattr(L, p + "matvec_row_major")
        self._mv.argtypes = [_f32p, _sz, _sz, _f32p, _f32p]
        self._rms = getattr(L, p + "rms_norm_inplace")
        self._rms.argtypes = [_f32p, _sz, _sz, C.c_void_p, C.c_float]
        self._sm = getattr(L, p + "softmax_inplace")
        self._sm.argtypes = [_f32p, _sz]
        self._tk = getattr(L, p + "route_top_k")
        self._tk.argtypes = [_f32p, _sz, _sz, C.c_int, _u32p, _f32p]
        self._sig = getattr(L, p + "sigmoid")
        self._sig.argtypes = [C.c_float]
        self._sig.restype = C.c_float
        self._silu = getattr(L, p + "silu")
        self._silu.argtypes = [C.c_float]
        self._silu.restype = C.c_float
        self._sw = getattr(L, p + "swiglu_inplace")
        self._sw.argtypes = [_f32p, _f32p, _sz]
        self._rq = getattr(L, p + "route_qwen_top_k")
        self._rq.argtypes = [_f32p, _f32p, C.c_void_p, _sz, _sz, _sz, C.c_int,
                             _f32p, _u32p, _f32p, C.POINTER(C.c_float)]
        self._qz = getattr(L, p + "quantize_affine_q4_rows")
        self._qz.argtypes = [_f32p, _sz, _sz, _sz, _u32p, _f32p, _f32p]
        self._sh = getattr(L, p + "shared_expert")
        self._sh.argtypes = [_f32p, _f32p, _f32p, _f32p, _sz, _sz, _f32p, _f32p,
                             C.POINTER(C.c_float)]
        if kind == "port":
            L.osm_oracle_dequant_slot.argtypes = [_u8p, _sz, _sz, _sz, _f32p, _f32p, _f32p]
            L.osm_oracle_gen_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_float, _f32p, _sz, _sz]
            L.osm_oracle_gen_expert_slot.argtypes = [C.c_uint64, C.c_uint64, C.c_float, _sz, _sz, _sz, _u8p]
            L.osm_oracle_bf16_narrow.argtypes = [_f32p, _u16p, _sz]
            L.osm_oracle_bf16_widen.argtypes = [_u16p, _f32p, _sz]
            L.osm_oracle_hash.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
            L.osm_oracle_hash.restype = C.c_uint64
            L.osm_oracle_add_residual.argtypes = [_f32p, _f32p, _f32p, _sz]
            L.osm_oracle_moe_token_slots.argtypes = [
                _f32p, _f32p, C.c_void_p, _sz, _sz, _sz, C.c_int, _sz, C.c_void_p, _sz,
                C.c_void_p, C.c_void_p, _f32p, _u32p, _f32p, C.POINTER(C.c_float),
                C.POINTER(C.c_float)]
        mt = getattr(L, p + "moe_token")
        mt.argtypes = [_f32p, _f32p, C.c_void_p, _sz, _sz, _sz, C.c_int, _sz,
                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                       C.c_void_p, C.c_void_p, _sz, _f32p, _u32p, _f32p,
                       C.POINTER(C.c_float), C.POINTER(C.c_float)]
        self._mt = mt
        if kind == "reference":
            L.osm_ref_moe_batch.argtypes = [
                _f32p, _sz, _f32p, C.c_void_p, _sz, _sz, _sz, C.c_int, _sz,
                C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                C.c_void_p, C.c_void_p, _sz, _f32p, _u32p, _f32p, C.c_int,
                C.POINTER(C.c_double)]
            L.osm_ref_cache_create.argtypes = [_sz, _sz, _sz]
            L.osm_ref_cache_create.restype = C.c_void_p
            L.osm_ref_cache_destroy.argtypes = [C.c_void_p]
            L.osm_ref_cache_fail_next.argtypes = [C.c_void_p]
            L.osm_ref_cache_fetch.argtypes = [C.c_void_p, C.c_uint32, _u32p, _sz,
                                              np.ctypeslib.ndpointer(np.uintp, flags="C_CONTIGUOUS")]
            L.osm_ref_cache_resident_slot.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32]
            L.osm_ref_cache_resident_slot.restype = C.c_longlong
            L.osm_ref_cache_stats.argtypes = [C.c_void_p, np.ctypeslib.ndpointer(np.uintp, flags="C_CONTIGUOUS")]

    # --- primitives (reference_ops.cpp) ------------------------------------
    def dequantize_affine_rows(self, packed, rows, packed_cols, scales, biases,
                               bits=4, group=64):
        packed = np.ascontiguousarray(packed, np.uint32)
        per_word = 32 // bits if bits in (4, 8) else 1
        out = np.zeros(max(rows * packed_cols * per_word, 1), np.float32)
        rc = self._dq(packed, rows, packed_cols,
                      np.ascontiguousarray(scales, np.float32),
                      np.ascontiguousarray(biases, np.float32), bits, group, out)
        if rc:
            raise OracleError(rc, "dequantize_affine_rows")
        return out.reshape(rows, packed_cols * per_word)

    def matvec(self, w, x):
        w = np.ascontiguousarray(w, np.float32)
        out_dim, in_dim = w.shape
        out = np.zeros(out_dim, np.float32)
        rc = self._mv(w.reshape(-1), out_dim, in_dim, np.ascontiguousarray(x, np.float32), out)
        if rc:
            raise OracleError(rc, "matvec")
        return out

    def rms_norm(self, values, weight, eps):
        v = np.array(values, np.float32, copy=True)
        rows, dim = v.shape if v.ndim == 2 else (1, v.shape[0])
        w = None if weight is None else np.ascontiguousarray(weight, np.float32)
        rc = self._rms(v.reshape(-1), rows, dim, None if w is None else w.ctypes.data, eps)
        if rc:
            raise OracleError(rc, "rms_norm")
        return v

    def softmax(self, values):
        v = np.array(values, np.float32, copy=True)
        rc = self._sm(v, v.size)
        if rc:
            raise OracleError(rc, "softmax")
        return v

    def route_top_k(self, logits, k, normalize):
        logits = np.ascontiguousarray(logits, np.float32)
        ids = np.zeros(max(k, 1), np.uint32)
        probs = np.zeros(max(k, 1), np.float32)
        rc = self._tk(logits, logits.size, k, int(normalize), ids, probs)
        if rc:
            raise OracleError(rc, "route_top_k")
        return ids[:k], probs[:k]

    def sigmoid(self, v):
        return self._sig(v)

    def silu(self, v):
        return self._silu(v)

    def swiglu(self, gate, up):
        g = np.array(gate, np.float32, copy=True)
        self._sw(g, np.ascontiguousarray(up, np.float32), g.size)
        return g

    def route_qwen_top_k(self, hidden, router_weight, k, norm, bias=None):
        hidden = np.ascontiguousarray(hidden, np.float32)
        router_weight = np.ascontiguousarray(router_weight, np.float32)
        E = router_weight.size // max(hidden.size, 1)
        logits = np.zeros(max(E, 1), np.float32)
        ids = np.zeros(max(k, 1), np.uint32)
        w = np.zeros(max(k, 1), np.float32)
        mass = C.c_float(0)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        rc = self._rq(hidden, router_weight.reshape(-1), None if b is None else b.ctypes.data,
                      hidden.size, E, k, int(norm), logits, ids, w, C.byref(mass))
        if rc:
            raise OracleError(rc, "route_qwen_top_k")
        return logits[:E], ids[:k], w[:k], mass.value

    def quantize_q4(self, values, rows, cols, group):
        v = np.ascontiguousarray(values, np.float32).reshape(-1)
        packed = np.zeros(rows * cols // 8, np.uint32)
        groups = rows * cols // group if group else 1
        s = np.zeros(max(groups, 1), np.float32)
        b = np.zeros(max(groups, 1), np.float32)
        rc = self._qz(v, rows, cols, group, packed, s, b)
        if rc:
            raise OracleError(rc, "quantize_affine_q4_rows")
        return packed.reshape(rows, cols // 8), s.reshape(rows, -1), b.reshape(rows, -1)

    def shared_expert(self, gate, up, down, scalar_gate, x):
        H = x.size
        I = gate.shape[0]
        out = np.zeros(H, np.float32)
        scale = C.c_float(0)
        rc = self._sh(np.ascontiguousarray(gate, np.float32).reshape(-1),
                      np.ascontiguousarray(up, np.float32).reshape(-1),
                      np.ascontiguousarray(down, np.float32).reshape(-1),
                      np.ascontiguousarray(scalar_gate, np.float32).reshape(-1),
                      H, I, np.ascontiguousarray(x, np.float32), out, C.byref(scale))
        if rc:
            raise OracleError(rc, "shared_expert")
        return out, scale.value

    def moe_token(self, x, router_weight, k, norm, experts, shared=None,
                  scalar_gate=None, bias=None):
        """experts: dict id -> (gate[I,H], up[I,H], down[H,I]) fp32 (only the
        picked ids are needed).  shared: (gate, up, down) or None."""
        x = np.ascontiguousarray(x, np.float32)
        router_weight = np.ascontiguousarray(router_weight, np.float32)
        H = x.size
        E = router_weight.size // H
        I = next(iter(experts.values()))[0].shape[0] if experts else 1
        keep = []
        g = [None] * E
        u = [None] * E
        d = [None] * E
        for e, (a, b_, c) in experts.items():
            a = np.ascontiguousarray(a, np.float32)
            b_ = np.ascontiguousarray(b_, np.float32)
            c = np.ascontiguousarray(c, np.float32)
            keep += [a, b_, c]
            g[e], u[e], d[e] = a, b_, c
        if shared is not None:
            sg, su, sd = (np.ascontiguousarray(t, np.float32) for t in shared)
            sgate = np.ascontiguousarray(scalar_gate, np.float32)
            SI = sg.shape[0]
            keep += [sg, su, sd, sgate]
        else:
            sg = su = sd = sgate = None
            SI = 0
        out = np.zeros(H, np.float32)
        ids = np.zeros(k, np.uint32)
        w = np.zeros(k, np.float32)
        mass = C.c_float(0)
        ss = C.c_float(0)
        bptr = None
        if bias is not None:
            bias = np.ascontiguousarray(bias, np.float32)
            bptr = bias.ctypes.data
        rc = self._mt(x, router_weight.reshape(-1), bptr, H, E, k, int(norm), I,
                      C.cast(_ptr_array(g), C.c_void_p), C.cast(_ptr_array(u), C.c_void_p),
                      C.cast(_ptr_array(d), C.c_void_p),
                      None if sg is None else sg.ctypes.data,
                      None if su is None else su.ctypes.data,
                      None if sd is None else sd.ctypes.data,
                      None if sgate is None else sgate.ctypes.data, SI,
                      out, ids, w, C.byref(mass), C.byref(ss))
        if rc:
            raise OracleError(rc, "moe_token")
        return out, ids, w, mass.value, ss.value

    # --- port-only helpers ---------------------------------------------------
    def moe_token_slots(self, x, router_weight, k, norm, slots, inter, shared_slot=None,
                        scalar_gate=None, bias=None):
        """moe_token with the experts given as Q4 slots: ``slots`` is a
        C-contiguous uint8 array [E][stride]; only the picked experts are
        dequantised.  Releases the GIL (ctypes), so threads run tokens in
        parallel."""
        x = np.ascontiguousarray(x, np.float32)
        W = np.ascontiguousarray(router_weight, np.float32)
        H = x.size
        E = W.size // H
        assert slots.flags["C_CONTIGUOUS"] and slots.dtype == np.uint8
        out = np.zeros(H, np.float32)
        ids = np.zeros(k, np.uint32)
        w = np.zeros(k, np.float32)
        mass = C.c_float(0)
        ss = C.c_float(0)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        sh = None if shared_slot is None else np.ascontiguousarray(shared_slot, np.uint8)
        sg = None if scalar_gate is None else np.ascontiguousarray(scalar_gate, np.float32)
        rc = self.lib.osm_oracle_moe_token_slots(
            x, W.reshape(-1), None if b is None else b.ctypes.data, H, E, k, int(norm), inter,
            slots.ctypes.data, slots.shape[1], None if sh is None else sh.ctypes.data,
            None if sg is None else sg.ctypes.data, out, ids, w, C.byref(mass), C.byref(ss))
        if rc:
            raise OracleError(rc, "moe_token_slots")
        return out, ids, w, mass.value, ss.value

    def dequant_slot(self, slot, H, I, group=64):
        gate = np.zeros((I, H), np.float32)
        up = np.zeros((I, H), np.float32)
        down = np.zeros((H, I), np.float32)
        rc = self.lib.osm_oracle_dequant_slot(np.ascontiguousarray(slot, np.uint8),
                                              H, I, group, gate, up, down)
        if rc:
            raise OracleError(rc, "dequant_slot")
        return gate, up, down

    def gen_normal(self, seed, tensor, sigma, n, first=0):
        out = np.zeros(n, np.float32)
        self.lib.osm_oracle_gen_normal(seed, tensor, sigma, out, n, first)
        return out

    def gen_expert_slot(self, seed, tensor_base, sigma, H, I, group=64):
        stride = slot_stride(H, I, group)
        slot = np.zeros(stride, np.uint8)
        rc = self.lib.osm_oracle_gen_expert_slot(seed, tensor_base, sigma, H, I, group, slot)
        if rc:
            raise OracleError(rc, "gen_expert_slot")
        return slot

    def bf16_round(self, values):
        v = np.ascontiguousarray(values, np.float32).reshape(-1)
        h = np.zeros(v.size, np.uint16)
        self.lib.osm_oracle_bf16_narrow(v, h, v.size)
        return h

    def hash(self, seed, tensor, index):
        return self.lib.osm_oracle_hash(seed, tensor, index)


def slot_layout(H: int, I: int, group: int = 64) -> dict:
    """Section offsets of one expert slot (U32 weights, BF16 metadata)."""
    gu_w = I * H // 2
    gu_m = I * (H // group) * 2
    dn_w = H * I // 2
    dn_m = H * (I // group) * 2
    off = {}
    o = 0
    for name, size in (("gate_w", gu_w), ("gate_s", gu_m), ("gate_b", gu_m),
                       ("up_w", gu_w), ("up_s", gu_m), ("up_b", gu_m),
                       ("down_w", dn_w), ("down_s", dn_m), ("down_b", dn_m)):
        off[name] = o
        o += size
    off["stride"] = o
    return off


def slot_stride(H: int, I: int, group: int = 64) -> int:
    return slot_layout(H, I, group)["stride"]


def bf16_widen(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)
