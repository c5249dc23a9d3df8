"""CPU baseline of the routed-MoE sublayer (TEST / MEASUREMENT INFRASTRUCTURE).

Runs the reference's own CPU code compiled in place (oracle/_ref, kind
"reference"), or the C restatement when that library is absent (kind
"port"), token-parallel over host threads: per token route_qwen_top_k_cpu
(or the biased-router harness), then per pick matvec/matvec/swiglu/matvec on
experts dequantised once beforehand (timed separately), the weighted sum in
pick order, then run_shared_expert_cpu.  Only bench.py's cpu_baseline leg and
its --impl reference arm use this module.
"""
from __future__ import annotations

import ctypes as C
import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

import pyoracle


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


class Sublayer:
    """Host copy of one sublayer: routed slots, shared slot, router, gate,
    bias; experts are dequantised on demand (in parallel)."""

    def __init__(self, slots: np.ndarray, shared_slot, W, sg, bias, H, I, k, threads):
        self.port = pyoracle.Oracle("port")
        self.kind = "reference" if pyoracle.ref_available() else "port"
        self.eng = pyoracle.Oracle(self.kind)
        self.slots, self.shared_slot = slots, shared_slot
        self.W = np.ascontiguousarray(W, np.float32)
        self.sg = None if sg is None else np.ascontiguousarray(sg, np.float32)
        self.bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.H, self.I, self.k, self.E = H, I, k, self.W.shape[0]
        self.threads = max(1, threads)
        self.deq = {}
        self.shared = None
        self.dequant_s = 0.0

    def route_ids(self, x: np.ndarray) -> set:
        ids = set()
        for t in range(x.shape[0]):
            _, i, _, _ = self.port.route_qwen_top_k(x[t], self.W, self.k, True, bias=self.bias)
            ids.update(int(v) for v in i)
        return ids

    def prepare(self, x: np.ndarray):
        need = sorted(e for e in self.route_ids(x) if e not in self.deq)
        t0 = time.perf_counter()
        with ThreadPoolExecutor(self.threads) as ex:
            for e, w in zip(need, ex.map(lambda e: self.port.dequant_slot(self.slots[e], self.H,
                                                                          self.I), need)):
                self.deq[e] = w
        if self.shared_slot is not None and self.shared is None:
            self.shared = self.port.dequant_slot(self.shared_slot, self.H, self.I)
        self.dequant_s += time.perf_counter() - t0

    def run(self, x: np.ndarray, threads: int | None = None) -> float:
        """Seconds for the whole batch x [T, H] on `threads` threads."""
        threads = threads or self.threads
        T, H = x.shape
        g = [None] * self.E
        u = [None] * self.E
        d = [None] * self.E
        for e, (a, b, c) in self.deq.items():
            g[e], u[e], d[e] = a, b, c
        out = np.zeros((T, H), np.float32)
        ids = np.zeros((T, self.k), np.uint32)
        w = np.zeros((T, self.k), np.float32)
        secs = C.c_double(0)
        sh = self.shared
        xs = np.ascontiguousarray(x, np.float32)
        if self.kind == "reference":
            L = self.eng.lib
            rc = L.osm_ref_moe_batch(
                xs, T, self.W.reshape(-1), None if self.bias is None else self.bias.ctypes.data,
                H, self.E, self.k, 1, self.I,
                C.cast(pyoracle._ptr_array(g), C.c_void_p), C.cast(pyoracle._ptr_array(u), C.c_void_p),
                C.cast(pyoracle._ptr_array(d), C.c_void_p),
                None if sh is None else sh[0].ctypes.data, None if sh is None else sh[1].ctypes.data,
                None if sh is None else sh[2].ctypes.data,
                None if self.sg is None else self.sg.ctypes.data, 0 if sh is None else self.I,
                out.reshape(-1), ids.reshape(-1), w.reshape(-1), threads, C.byref(secs))
            if rc:
                raise RuntimeError(f"reference batch failed: {rc}")
            self.last = (out, ids, w)
            return secs.value
        # port: a thread pool over tokens (ctypes releases the GIL)
        experts = self.deq
        t0 = time.perf_counter()

        def one(t):
            o, i, ww, _, _ = self.port.moe_token(xs[t], self.W, self.k, True, experts,
                                                 shared=sh, scalar_gate=self.sg, bias=self.bias)
            out[t], ids[t], w[t] = o, i, ww

        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(one, range(T)))
        self.last = (out, ids, w)
        return time.perf_counter() - t0
