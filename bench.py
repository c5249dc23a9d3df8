#!/usr/bin/env python
"""Benchmark of the B200 routed-MoE sublayer (Qwen3-Next-80B-A3B shape).

Workload: one sublayer with all 512 Q4 experts resident
in HBM (hidden 2048, top-10 renormalised, inter 512, shared expert 512,
sigmoid scalar gate), router logits biased by Zipf(1.1) over a seeded expert
permutation, decode batches B = 1, 8, 32, 64, 128, 256.  One step = one
sublayer call per batch size (489 tokens).  Synthetic seeded data.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Timing: L2 (126 MB) is flushed by a 256 MiB write before every call; each call
is bracketed by CUDA events on the stream it runs on; value = tokens / sum of
call intervals (max over ranks).  e2e = the same calls through pinned host
buffers, H2D of x and D2H of the output inside the intervals.  The roofline
names the kernel with the largest share of device time, timed by the
library's per-kernel events on its stream.  --gpus N > 1 runs N independent
replicas (the decode path does not shard): scaling "weak".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "orbi-streammoe_b200"))

import numpy as np  # noqa: E402

SWEEP = (1, 8, 32, 64, 128, 256)
H, E, I, K, SHI, GROUP = 2048, 512, 512, 10, 512, 64
SEED = 20241201
ZIPF_S = 1.1
METRIC = "routed-MoE sublayer tokens/s (Qwen3-Next-80B-A3B shape); decode µs/layer; HBM GB/s"
WORKLOAD = ("configs[1]: Qwen3-Next-80B-A3B routed-MoE sublayer, decode batches "
            "1,8,32,64,128,256, Zipf(1.1) router bias, all 512 Q4 experts in HBM")
# bytes of one Q4 expert slot (gate/up/down U32 + BF16 scale/bias)
S_EXPERT = 1769472
S_GATEUP = 1179648   # gate + up sections
S_DOWN = 589824
S_ROUTER = E * H * 2
S_SGATE = H * 2
# DRAM traffic (read + write) of one gate/up launch at B = 256 (the digit-plane
# tensor-core kernel, dg_kernel<0>), from the ncu capture summarised in
# profiles/dg_kernel_gateup_down_q3n_b256.md (algorithmic bytes of that
# launch: 105.8 MB).
NCU_GATEUP_TRAFFIC_B256 = 128_601_088 + 4_684_288


def bf16_round(v: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(v, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return r.astype(np.uint32).view(np.float32)


def zipf_bias(E: int, s: float, seed: int) -> np.ndarray:
    r = np.arange(1, E + 1, dtype=np.float64)
    perm = np.random.default_rng(seed).permutation(E)
    b = np.zeros(E, np.float32)
    b[perm] = np.log(r ** -s / (r ** -s).sum()).astype(np.float32)
    return b


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops", 1590.0),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi samples of this GPU while the timed work runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [s for s, p in zip(sm, power) if p > 200.0] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
def replicated_weights(torch, ctx, osm):
    """Router weight, shared-expert gate row and shared-expert slot bytes (the
    parts every rank holds), from the bench seeds."""
    lay = osm.expert_layout(H, I, GROUP)
    sh_slab = osm.Slab(ctx, lay, 1)
    sh_slab.generate(SEED, 1000 + 3 * E, 0.02, 0, 1)
    buf = torch.empty(E * H, device="cuda")
    ctx.gen_normal(SEED, 1, 0.02, buf)
    W = bf16_round(buf.cpu().numpy()).reshape(E, H)
    g = torch.empty(H, device="cuda")
    ctx.gen_normal(SEED, 2, 0.02, g)
    sg = bf16_round(g.cpu().numpy())
    ctx.synchronize()
    import ctypes

    shared = np.zeros(lay.stride, np.uint8)
    ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(shared.ctypes.data),
                                     ctypes.c_void_p(sh_slab.slot_ptr(0)), lay.stride))
    sh_slab.close()
    return W, sg, shared


def build_sublayer(torch, ctx, osm, zipf=True):
    """The Q3N sublayer of configs 0-2 (config 1 adds the Zipf router bias;
    config 2 routes without it)."""
    lay = osm.expert_layout(H, I, GROUP)
    slab = osm.Slab(ctx, lay, E)
    slab.generate(SEED, 1000, 0.02, 0, E)
    W, sg, shared = replicated_weights(torch, ctx, osm)
    bias = zipf_bias(E, ZIPF_S, SEED) if zipf else None
    layer = osm.Layer(ctx, W, K, True, logit_bias=bias, shared_slot=shared, shared_layout=lay,
                      shared_gate=sg)
    layer.bind_slab(slab, np.arange(E, dtype=np.int32))
    return layer, slab, W, sg, bias, shared


def sublayer_bytes(B: int, U: int) -> int:
    """Algorithmic bytes of one call (U distinct routed experts)."""
    return U * S_EXPERT + S_EXPERT + S_ROUTER + S_SGATE + B * H * 8


def kernel_bytes(kind: str, B: int, U: int) -> int:
    P = B * (K + 1)
    if kind == "proj_gate_up":
        return (U + 1) * S_GATEUP + B * H * 4 + P * I * 4
    if kind == "proj_down":
        return (U + 1) * S_DOWN + P * I * 4 + P * H * 4
    if kind == "router_logits":
        return S_ROUTER + B * H * 4 + B * E * 8
    if kind == "router_select":
        return B * E * 8 + B * H * 4 + B * H * 8
    if kind == "combine":
        return P * H * 4 + B * H * 4
    return 0


def run_ours(args, rank, world, local_rank):
    import torch

    import osm_b200 as osm

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    ctx = osm.Context(local_rank, max_tokens=max(SWEEP))
    ctx.set_stream(stream.cuda_stream)
    layer, slab, W, sg, bias, shared = build_sublayer(torch, ctx, osm)
    xs, outs, hx, hout = {}, {}, {}, {}
    ids_d = {}
    for B in SWEEP:
        x = torch.empty(B, H, device=dev)
        ctx.gen_normal(SEED, 5000 + B, 1.0, x)
        xs[B] = x
        outs[B] = torch.empty(B, H, device=dev)
        ids_d[B] = torch.empty(B, K, dtype=torch.int32, device=dev)
        hx[B] = x.cpu().pin_memory()
        hout[B] = torch.empty(B, H).pin_memory()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    # one CUDA-graph plan per batch size (osm_plan_create), the e2e ones with the
    # pinned-host copy of x in and of out back inside the graph
    # (largest batch first: the context's scratch is sized once)
    order = sorted(SWEEP, reverse=True)
    plans = {B: osm.Plan(layer, B, xs[B], outs[B], ids=ids_d[B]) for B in order} if args.graphs else {}
    plans_e2e = ({B: osm.Plan(layer, B, xs[B], outs[B], ids=ids_d[B], x_host=hx[B], out_host=hout[B])
                  for B in order} if args.graphs else {})

    def call(B, e2e, eager=False):
        if args.graphs and not eager:
            (plans_e2e if e2e else plans)[B].launch()
            return
        if e2e:
            xs[B].copy_(hx[B], non_blocking=True)
        layer.run_qwen_sparse_moe(xs[B], B, outs[B], ids=ids_d[B])
        if e2e:
            hout[B].copy_(outs[B], non_blocking=True)

    def timed_pass(steps, e2e, eager=False):
        evs = []
        for _ in range(steps):
            for B in SWEEP:
                flush.zero_()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                call(B, e2e, eager)
                b.record(stream)
                evs.append((B, a, b))
        return evs

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    gpu_uuid = str(getattr(torch.cuda.get_device_properties(dev), "uuid", local_rank))
    if gpu_uuid and not gpu_uuid.startswith("GPU-") and len(gpu_uuid) > 8:
        gpu_uuid = "GPU-" + gpu_uuid
    clocks = ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else str(local_rank))

    timed_pass(args.warmup, False)
    timed_pass(max(1, args.warmup // 2), True)
    timed_pass(max(1, args.warmup // 2), False, eager=True)
    torch.cuda.synchronize()
    ctx.status()
    clocks.start()
    # ---- value: inputs resident in HBM ----
    barrier()
    torch.cuda.synchronize()
    l0 = ctx.launches
    t_wall = time.perf_counter()
    evs = timed_pass(args.steps, False)
    torch.cuda.synchronize()
    barrier()
    bracket_s = time.perf_counter() - t_wall
    launches = ctx.launches - l0
    per_b = {B: 0.0 for B in SWEEP}
    for B, a, b in evs:
        per_b[B] += a.elapsed_time(b)
    total_ms = sum(per_b.values())
    # ---- e2e: host buffers, copies inside the intervals ----
    barrier()
    torch.cuda.synchronize()
    evs2 = timed_pass(args.steps, True)
    torch.cuda.synchronize()
    barrier()
    e2e_b = {B: 0.0 for B in SWEEP}
    for B, a, b in evs2:
        e2e_b[B] += a.elapsed_time(b)
    total_ms_e2e = sum(e2e_b.values())
    # ---- the same calls launched one by one (no graph), for comparison ----
    eager_b = {B: 0.0 for B in SWEEP}
    if args.graphs:
        evs3 = timed_pass(args.steps, False, eager=True)
        torch.cuda.synchronize()
        for B, a, b in evs3:
            eager_b[B] += a.elapsed_time(b)
    for p in list(plans.values()) + list(plans_e2e.values()):
        p.close()
    # ---- per-kernel profile pass (roofline) ----
    uniq = {}
    for B in SWEEP:
        layer.run_qwen_sparse_moe(xs[B], B, outs[B], ids=ids_d[B])
        torch.cuda.synchronize()
        uniq[B] = int(np.unique(ids_d[B].cpu().numpy()).size)
    ctx.profile_read()
    ctx.profile(True)
    prof_steps = max(1, min(args.steps, 50))
    kbytes = {}
    for _ in range(prof_steps):
        for B in SWEEP:
            flush.zero_()
            layer.run_qwen_sparse_moe(xs[B], B, outs[B], ids=ids_d[B])
            for kind in ("proj_gate_up", "proj_down", "router_logits", "router_select", "combine"):
                kbytes[kind] = kbytes.get(kind, 0) + kernel_bytes(kind, B, uniq[B])
    prof = ctx.profile_read()
    ctx.profile(False)
    clk = clocks.stop()
    status, exact_tokens = ctx.status()
    if status:
        raise RuntimeError(f"device status {status} during the benchmark")

    tokens_per_step = sum(SWEEP)
    total_ms = max_over_ranks(total_ms)
    total_ms_e2e = max_over_ranks(total_ms_e2e)
    value = world * tokens_per_step * args.steps / (total_ms / 1e3)
    e2e_value = world * tokens_per_step * args.steps / (total_ms_e2e / 1e3)
    peaks = load_peaks()
    dom = max(prof.items(), key=lambda kv: kv[1][0])
    dom_kind, (dom_ms, dom_n) = dom
    achieved = kbytes[dom_kind] / (dom_ms / 1e3) / 1e9
    sweep = {}
    for B in SWEEP:
        us = per_b[B] / args.steps * 1e3
        byt = sublayer_bytes(B, uniq[B])
        sweep[str(B)] = {"us_per_call": round(us, 2), "distinct_experts": uniq[B],
                         "alg_bytes": byt, "gbs": round(byt / us / 1e3, 1),
                         "frac_hbm": round(byt / us / 1e3 / peaks["hbm_gbs"], 3),
                         "e2e_us_per_call": round(e2e_b[B] / args.steps * 1e3, 2)}
        if args.graphs:
            sweep[str(B)]["eager_us_per_call"] = round(eager_b[B] / args.steps * 1e3, 2)
    kernels = {k: {"ms": round(v[0], 3), "launches": int(v[1]),
                   "share": round(v[0] / sum(x[0] for x in prof.values()), 3)} for k, v in prof.items()}
    traffic, traffic_note = None, None
    if dom_kind == "proj_gate_up":
        traffic = NCU_GATEUP_TRAFFIC_B256
        traffic_note = ("bytes of one B=256 launch (ncu); that launch's algorithmic bytes: "
                        f"{kernel_bytes('proj_gate_up', 256, uniq[256])}")
    h2d = sum(B * H * 4 for B in SWEEP)
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded N(0,0.02) weights, reference quantiser, bf16 scale/bias; x~N(0,1))",
        "config": {"workload": WORKLOAD, "tokens_per_step": tokens_per_step,
                   "hidden": H, "experts": E, "top_k": K, "moe_inter": I, "shared_inter": SHI,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "flushed before every call (256 MiB write, outside the timed intervals)",
                   "timing": "sum of per-call CUDA-event intervals on the launching stream",
                   "calls": ("one CUDA-graph plan launch per call (osm_plan_launch; e2e plans hold "
                             "the pinned-host copies, made by the SMs through the GPU's mapping of "
                             "the pinned buffers); eager_us_per_call: the same call through "
                             "osm_moe_forward, kernels launched one by one") if args.graphs
                            else "osm_moe_forward, kernels launched one by one",
                   "bracket_wall_s": round(bracket_s, 3),
                   "exact_route_tokens": int(exact_tokens),
                   "per_batch": sweep, "kernels": kernels},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": h2d},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": dom_kind, "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 3), "traffic": traffic,
                     "traffic_note": traffic_note,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)"},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_leg(torch, ctx, slab, W, sg, bias, shared, xs, osm)
    return line


# ----------------------------------------------------------------------------
# 4096-token prefill on the tensor-core path (--workload prefill)
# ----------------------------------------------------------------------------
PF_T = 4096
# expert GEMM flops per token: top-k routed gate/up/down + the shared expert
PF_FLOP_PER_TOKEN = K * 3 * 2 * H * I + 3 * 2 * H * SHI


def run_prefill(args, rank, world, local_rank):
    import torch

    import osm_b200 as osm

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    # N > 1: expert parallelism over the ranks (E/N experts each) on the same
    # 4096 tokens, T/N routed per rank (strong scaling)
    t_local = PF_T // world
    if args.ep:
        from osm_b200 import ep as osm_ep
    ctx = osm.Context(local_rank, max_tokens=osm_ep.context_rows(world, t_local, K) if args.ep else PF_T)
    ctx.set_stream(stream.cuda_stream)
    x_all = torch.empty(PF_T, H, device=dev)
    ctx.gen_normal(SEED, 7000, 1.0, x_all)
    x = x_all[rank * t_local:(rank + 1) * t_local].contiguous()
    del x_all
    out = torch.empty(t_local, H, device=dev)
    if args.ep:
        e_count = E // world
        e0 = rank * e_count
        lay = osm.expert_layout(H, I, GROUP)
        slab = osm.Slab(ctx, lay, e_count + 1)  # + the shared expert's slot
        slab.generate(SEED, 1000 + 3 * e0, 0.02, 0, e_count)
        W, sg, shared = replicated_weights(torch, ctx, osm)
        moe = osm_ep.ExpertParallelMoE(ctx, W, K, True, lay, slab, e0, e_count, shared, sg,
                                       tokens_per_rank=t_local)
    else:
        layer = build_sublayer(torch, ctx, osm, zipf=False)[0]
    hx = x.cpu().pin_memory()
    hout = torch.empty(t_local, H).pin_memory()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    def call(e2e):
        if e2e:
            x.copy_(hx, non_blocking=True)
        if args.ep:
            moe.forward(x, out)
        else:
            layer.run_qwen_sparse_moe(x, PF_T, out, prefill=True)
        if e2e:
            hout.copy_(out, non_blocking=True)

    def timed_pass(steps, e2e):
        ms = 0.0
        for _ in range(steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            call(e2e)
            b.record(stream)
            b.synchronize()
            ms += a.elapsed_time(b)
        return ms

    def barrier():
        if args.ep:
            torch.distributed.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    gpu_uuid = str(getattr(torch.cuda.get_device_properties(dev), "uuid", local_rank))
    if gpu_uuid and not gpu_uuid.startswith("GPU-") and len(gpu_uuid) > 8:
        gpu_uuid = "GPU-" + gpu_uuid
    clocks = ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else str(local_rank))
    timed_pass(args.warmup, False)
    timed_pass(max(1, args.warmup // 2), True)
    ctx.status()
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    l0 = ctx.launches
    total_ms = timed_pass(args.steps, False)
    barrier()
    launches = ctx.launches - l0
    total_ms_e2e = timed_pass(args.steps, True)
    barrier()
    ctx.profile_read()
    ctx.profile(True)
    prof_steps = max(1, min(args.steps, 10))
    for _ in range(prof_steps):
        flush.zero_()
        call(False)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    clk = clocks.stop()
    status, exact_tokens = ctx.status()
    if args.ep:
        moe.close()
    if status:
        raise RuntimeError(f"device status {status} during the prefill benchmark")
    total_ms = max_over_ranks(total_ms)
    total_ms_e2e = max_over_ranks(total_ms_e2e)
    value = PF_T * args.steps / (total_ms / 1e3)
    e2e_value = PF_T * args.steps / (total_ms_e2e / 1e3)
    peaks = load_peaks()
    gemm_ms = (prof.get("proj_gate_up", (0.0, 0))[0] + prof.get("proj_down", (0.0, 0))[0]) / prof_steps
    # this rank's expert GEMM work: its share of the routed pairs and the
    # shared expert for its own tokens
    tflops = t_local * PF_FLOP_PER_TOKEN / (gemm_ms / 1e3) / 1e12
    kernels = {k: {"ms_per_call": round(v[0] / prof_steps, 4), "launches": int(v[1]),
                   "share": round(v[0] / sum(x[0] for x in prof.values()), 3)} for k, v in prof.items()}
    return {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong" if args.ep else "weak",
        "vs_baseline": None,
        "dtype": "fp16 operands, fp32 accumulation (experts); fp32 exact routing",
        "data": "synthetic (seeded N(0,0.02) weights, reference quantiser, bf16 scale/bias; x~N(0,1))",
        "config": {"workload": "configs[2]: Qwen3-Next-80B-A3B routed-MoE sublayer, 4096-token prefill, "
                               "uniform routing (no router bias), tcgen05 grouped GEMM",
                   "tokens_per_step": PF_T, "hidden": H, "experts": E, "top_k": K,
                   "moe_inter": I, "shared_inter": SHI,
                   "parallelism": (f"expert parallel x{world} ({E // world} experts and "
                                   f"{t_local} tokens per rank, dispatch/combine by stores into "
                                   "peer memory over NVLink, device-side barriers)"
                                   if args.ep else "single GPU"),
                   "l2": "flushed before every call (256 MiB write, outside the timed intervals)",
                   "timing": "sum of per-call CUDA-event intervals on the launching stream",
                   "exact_route_tokens": int(exact_tokens), "kernels": kernels},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": t_local * H * 4, "d2h_bytes_per_step": t_local * H * 4},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "kernel": "pf_gemm (gate/up + down)",
                     "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(tflops / peaks["bf16_tflops"], 3), "traffic": None,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json bf16_tflops, burst)"},
        "clocks": clk,
    }


# ----------------------------------------------------------------------------
# Qwen3-30B-A3B-shaped sublayer at 1, 64 and 8192 tokens (--workload q30)
# ----------------------------------------------------------------------------
Q30_H, Q30_E, Q30_I, Q30_K = 2048, 128, 768, 8
Q30_T = (1, 64, 8192)


def run_q30_ep(args, rank, world, local_rank):
    """configs[3] 8192-token case, expert parallel: rank r owns experts
    [r 128/N, (r+1) 128/N) and routes 8192/N of the tokens (strong scaling);
    dispatch and combine by stores into peer memory (osm_b200.ep)."""
    import torch

    import osm_b200 as osm
    from osm_b200 import ep as osm_ep

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    T = Q30_T[-1]
    t_local, e_count = T // world, Q30_E // world
    e0 = rank * e_count
    # rows an owner runs its experts over: a receive region per rank
    ctx = osm.Context(local_rank, max_tokens=osm_ep.context_rows(world, t_local, Q30_K))
    ctx.set_stream(stream.cuda_stream)
    lay = osm.expert_layout(Q30_H, Q30_I, GROUP)
    slab = osm.Slab(ctx, lay, e_count)
    slab.generate(SEED + 3, 1000 + 3 * e0, 0.02, 0, e_count)  # the one-GPU leg's experts e0..
    buf = torch.empty(Q30_E * Q30_H, device=dev)
    ctx.gen_normal(SEED + 3, 1, 0.02, buf)
    W = bf16_round(buf.cpu().numpy()).reshape(Q30_E, Q30_H)
    moe = osm_ep.ExpertParallelMoE(ctx, W, Q30_K, True, lay, slab, e0, e_count,
                                   tokens_per_rank=t_local)
    x_all = torch.empty(T, Q30_H, device=dev)
    ctx.gen_normal(SEED + 3, 9000 + T, 1.0, x_all)
    x = x_all[rank * t_local:(rank + 1) * t_local].contiguous()
    del x_all
    out = torch.empty(t_local, Q30_H, device=dev)
    hx = x.cpu().pin_memory()
    hout = torch.empty(t_local, Q30_H).pin_memory()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    def call(e2e):
        if e2e:
            x.copy_(hx, non_blocking=True)
        moe.forward(x, out)
        if e2e:
            hout.copy_(out, non_blocking=True)

    def timed_pass(steps, e2e):
        ms = 0.0
        for _ in range(steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            call(e2e)
            b.record(stream)
            b.synchronize()
            ms += a.elapsed_time(b)
        return ms

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    gpu_uuid = str(getattr(torch.cuda.get_device_properties(dev), "uuid", local_rank))
    if gpu_uuid and not gpu_uuid.startswith("GPU-") and len(gpu_uuid) > 8:
        gpu_uuid = "GPU-" + gpu_uuid
    clocks = ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else str(local_rank))
    timed_pass(args.warmup, False)
    timed_pass(max(1, args.warmup // 2), True)
    ctx.status()
    clocks.start()
    torch.distributed.barrier()
    torch.cuda.synchronize()
    l0 = ctx.launches
    total_ms = timed_pass(args.steps, False)
    torch.distributed.barrier()
    launches = ctx.launches - l0
    total_e2e = timed_pass(args.steps, True)
    torch.distributed.barrier()
    ctx.profile_read()
    ctx.profile(True)
    prof_steps = max(1, min(args.steps, 10))
    for _ in range(prof_steps):
        flush.zero_()
        call(False)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    clk = clocks.stop()
    status, exact_tokens = ctx.status()
    moe.close()
    if status:
        raise RuntimeError(f"device status {status} during the q30 expert-parallel benchmark")
    total_ms = max_over_ranks(total_ms)
    total_e2e = max_over_ranks(total_e2e)
    peaks = load_peaks()
    gemm_ms = (prof.get("proj_gate_up", (0.0, 0))[0] + prof.get("proj_down", (0.0, 0))[0]) / prof_steps
    # this rank's share of the expert GEMM work (its tokens' picks, on average)
    tflops = t_local * Q30_K * 3 * 2 * Q30_H * Q30_I / (gemm_ms / 1e3) / 1e12
    kernels = {k: {"ms_per_call": round(v[0] / prof_steps, 4), "launches": int(v[1]),
                   "share": round(v[0] / sum(q[0] for q in prof.values()), 3)} for k, v in prof.items()}
    return {
        "metric": METRIC, "value": round(T * args.steps / (total_ms / 1e3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "fp16 operands, fp32 accumulation (experts); fp32 exact routing",
        "data": "synthetic (seeded N(0,0.02) weights, reference quantiser, bf16 scale/bias; x~N(0,1))",
        "config": {"workload": "configs[3]: Qwen3-30B-A3B-shaped routed-MoE sublayer, 8192-token "
                               "case, expert parallel",
                   "tokens_per_step": T,
                   "parallelism": (f"expert parallel x{world} ({e_count} experts and {t_local} "
                                   "tokens per rank, dispatch/combine by stores into peer "
                                   "memory over NVLink, device-side barriers)"),
                   "l2": "flushed before every call (256 MiB write, outside the timed intervals)",
                   "timing": "sum of per-call CUDA-event intervals on the launching stream, max "
                             "over ranks",
                   "exact_route_tokens": int(exact_tokens), "kernels": kernels},
        "e2e": {"value": round(T * args.steps / (total_e2e / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": t_local * Q30_H * 4, "d2h_bytes_per_step": t_local * Q30_H * 4},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "kernel": "pf_gemm (gate/up + down), this rank",
                     "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(tflops / peaks["bf16_tflops"], 3), "traffic": None,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json bf16_tflops, burst)"},
        "clocks": clk,
    }


def run_q30(args, rank, world, local_rank):
    import torch

    import osm_b200 as osm

    if args.ep:
        return run_q30_ep(args, rank, world, local_rank)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    ctx = osm.Context(local_rank, max_tokens=max(Q30_T))
    ctx.set_stream(stream.cuda_stream)
    lay = osm.expert_layout(Q30_H, Q30_I, GROUP)
    slab = osm.Slab(ctx, lay, Q30_E)
    slab.generate(SEED + 3, 1000, 0.02, 0, Q30_E)
    buf = torch.empty(Q30_E * Q30_H, device=dev)
    ctx.gen_normal(SEED + 3, 1, 0.02, buf)
    W = bf16_round(buf.cpu().numpy()).reshape(Q30_E, Q30_H)
    layer = osm.Layer(ctx, W, Q30_K, True)
    layer.bind_slab(slab, np.arange(Q30_E, dtype=np.int32))
    xs, outs, hx, hout = {}, {}, {}, {}
    for T in Q30_T:
        xs[T] = torch.empty(T, Q30_H, device=dev)
        ctx.gen_normal(SEED + 3, 9000 + T, 1.0, xs[T])
        outs[T] = torch.empty(T, Q30_H, device=dev)
        hx[T] = xs[T].cpu().pin_memory()
        hout[T] = torch.empty(T, Q30_H).pin_memory()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    dec = [T for T in Q30_T if T < 1024]
    plans = {T: osm.Plan(layer, T, xs[T], outs[T]) for T in sorted(dec, reverse=True)}
    plans_e2e = {T: osm.Plan(layer, T, xs[T], outs[T], x_host=hx[T], out_host=hout[T])
                 for T in sorted(dec, reverse=True)}

    def call(T, e2e):
        if T in plans:
            (plans_e2e if e2e else plans)[T].launch()
            return
        if e2e:
            xs[T].copy_(hx[T], non_blocking=True)
        layer.run_qwen_sparse_moe(xs[T], T, outs[T], prefill=True)
        if e2e:
            hout[T].copy_(outs[T], non_blocking=True)

    def timed_pass(steps, e2e):
        per = {T: 0.0 for T in Q30_T}
        for _ in range(steps):
            for T in Q30_T:
                flush.zero_()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                call(T, e2e)
                b.record(stream)
                b.synchronize()
                per[T] += a.elapsed_time(b)
        return per

    gpu_uuid = str(getattr(torch.cuda.get_device_properties(dev), "uuid", local_rank))
    if gpu_uuid and not gpu_uuid.startswith("GPU-") and len(gpu_uuid) > 8:
        gpu_uuid = "GPU-" + gpu_uuid
    clocks = ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else str(local_rank))
    timed_pass(args.warmup, False)
    timed_pass(max(1, args.warmup // 2), True)
    ctx.status()
    clocks.start()
    l0 = ctx.launches
    per = timed_pass(args.steps, False)
    launches = ctx.launches - l0
    per_e2e = timed_pass(args.steps, True)
    for p in list(plans.values()) + list(plans_e2e.values()):
        p.close()
    ctx.profile_read()
    ctx.profile(True)
    prof_steps = max(1, min(args.steps, 10))
    for _ in range(prof_steps):
        flush.zero_()
        call(Q30_T[-1], False)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    clk = clocks.stop()
    status, exact_tokens = ctx.status()
    if status:
        raise RuntimeError(f"device status {status} during the q30 benchmark")
    tokens = sum(Q30_T)
    total_ms, total_e2e = sum(per.values()), sum(per_e2e.values())
    value = tokens * args.steps / (total_ms / 1e3)
    peaks = load_peaks()
    Tp = Q30_T[-1]
    gemm_ms = (prof.get("proj_gate_up", (0.0, 0))[0] + prof.get("proj_down", (0.0, 0))[0]) / prof_steps
    tflops = Tp * Q30_K * 3 * 2 * Q30_H * Q30_I / (gemm_ms / 1e3) / 1e12
    cases = {str(T): {"us_per_call": round(per[T] / args.steps * 1e3, 2),
                      "tokens_per_s": round(T * args.steps / (per[T] / 1e3), 1),
                      "path": "graph plan, decode kernels" if T in plans else "tensor-core prefill"}
             for T in Q30_T}
    kernels = {k: {"ms_per_call": round(v[0] / prof_steps, 4), "launches": int(v[1]),
                   "share": round(v[0] / sum(x[0] for x in prof.values()), 3)} for k, v in prof.items()}
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (1 and 64 tokens); fp16 operands, fp32 accumulation (8192-token experts)",
        "data": "synthetic (seeded N(0,0.02) weights, reference quantiser, bf16 scale/bias; x~N(0,1))",
        "config": {"workload": "configs[3]: Qwen3-30B-A3B-shaped routed-MoE sublayer (hidden 2048, "
                               "128 experts, top-8, moe_inter 768, no shared expert), 1, 64 and 8192 "
                               "tokens per step",
                   "tokens_per_step": tokens, "parallelism": "single GPU",
                   "l2": "flushed before every call (256 MiB write, outside the timed intervals)",
                   "timing": "sum of per-call CUDA-event intervals on the launching stream",
                   "exact_route_tokens": int(exact_tokens), "per_case": cases,
                   "kernels_8192": kernels},
        "e2e": {"value": round(tokens * args.steps / (total_e2e / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": tokens * Q30_H * 4, "d2h_bytes_per_step": tokens * Q30_H * 4},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "kernel": "pf_gemm (gate/up + down), 8192 tokens",
                     "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(tflops / peaks["bf16_tflops"], 3), "traffic": None,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json bf16_tflops, burst)"},
        "clocks": clk,
    }


# ----------------------------------------------------------------------------
# 48-layer batch-1 decode streaming experts from pinned host memory
# into an 8 GB HBM cache (--workload stream)
# ----------------------------------------------------------------------------
STREAM_CACHE_BYTES = 8_000_000_000


def run_stream(args, rank, world, local_rank):
    import ctypes

    import torch

    import osm_b200 as osm

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    L = args.stream_layers
    ctx = osm.Context(local_rank, max_tokens=1)
    ctx.set_stream(stream.cuda_stream)
    lay = osm.expert_layout(H, I, GROUP)
    stride = lay.stride
    # every layer's experts in pinned host memory, generated on the GPU layer by layer
    host = torch.empty(L * E * stride, dtype=torch.uint8, pin_memory=True)
    stage = osm.Slab(ctx, lay, E)
    layers = []
    for l in range(L):
        seed = SEED + 7919 * (l + 1)
        stage.generate(seed, 1000, 0.02, 0, E)
        ctx.synchronize()
        ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(host.data_ptr() + l * E * stride),
                                         ctypes.c_void_p(stage.slot_ptr(0)), E * stride))
        sh = osm.Slab(ctx, lay, 1)
        sh.generate(seed, 1000 + 3 * E, 0.02, 0, 1)
        buf = torch.empty(E * H, device=dev)
        ctx.gen_normal(seed, 1, 0.02, buf)
        W = bf16_round(buf.cpu().numpy()).reshape(E, H)
        g = torch.empty(H, device=dev)
        ctx.gen_normal(seed, 2, 0.02, g)
        sg = bf16_round(g.cpu().numpy())
        ctx.synchronize()
        shared = np.zeros(stride, np.uint8)
        ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(shared.ctypes.data),
                                         ctypes.c_void_p(sh.slot_ptr(0)), stride))
        sh.close()
        layers.append(osm.Layer(ctx, W, K, True, logit_bias=zipf_bias(E, ZIPF_S, seed),
                                shared_slot=shared, shared_layout=lay, shared_gate=sg))
    stage.close()
    slots = STREAM_CACHE_BYTES // stride
    slab = osm.Slab(ctx, lay, slots)
    for layer in layers:
        layer.bind_slab(slab, np.full(E, -1, np.int32))
    base = host.data_ptr()
    cache = osm.ExpertCache(slab, slots * stride,
                            source=lambda l, e: base + (l * E + e) * stride)
    for l, layer in enumerate(layers):
        cache.bind_layer(l, layer)
    ones = torch.ones(H, device=dev)
    bufs = [torch.empty(1, H, device=dev), torch.empty(1, H, device=dev)]
    ctx.gen_normal(SEED, 9000, 1.0, bufs[0])

    def token():
        """One decode token through the stack: per layer one cached call
        (route, picks to the host, residency, experts), then the output
        RMS-normalised in place as the next layer's input.  Returns (ms,
        exposed H2D ms)."""
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for l, layer in enumerate(layers):
            x, out = bufs[l & 1], bufs[(l + 1) & 1]
            layer.run_cached(cache, l, x, 1, out, early=args.stream_early)
            ctx.rms_norm(out, 1, H, ones, 1e-6)
        if L & 1:
            bufs.reverse()
        t1.record(stream)
        t1.synchronize()
        return t0.elapsed_time(t1), cache.exposed_read()[0]

    cache.time_copies(True)
    for _ in range(args.warmup):
        token()
    s0 = cache.stats()
    h2d0 = osm.lib().osm_slab_h2d_bytes(slab.h)
    gpu_uuid = str(getattr(torch.cuda.get_device_properties(dev), "uuid", local_rank))
    if gpu_uuid and not gpu_uuid.startswith("GPU-") and len(gpu_uuid) > 8:
        gpu_uuid = "GPU-" + gpu_uuid
    clocks = ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else str(local_rank))
    clocks.start()
    l0 = ctx.launches
    tot_ms = exp_ms = 0.0
    for _ in range(args.steps):
        a, b = token()
        tot_ms += a
        exp_ms += b
    launches = ctx.launches - l0
    clk = clocks.stop()
    s1 = cache.stats()
    h2d = osm.lib().osm_slab_h2d_bytes(slab.h) - h2d0
    status, _ = ctx.status()
    if status:
        raise RuntimeError(f"device status {status} during the streaming benchmark")
    hits, misses = s1["hits"] - s0["hits"], s1["misses"] - s0["misses"]
    value = args.steps / (tot_ms / 1e3)
    peaks = load_peaks()
    alg = L * sublayer_bytes(1, K)
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tot_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (independently seeded layers, reference quantiser, bf16 scale/bias)",
        "config": {"workload": f"configs[4]: {L}-layer stack of Q3N sublayers, batch-1 decode, "
                               "output RMS-normalised and fed back, per-layer Zipf(1.1) bias, experts "
                               "in pinned host memory streamed into an HBM cache (LFU + recency)",
                   "layers": L, "host_expert_bytes": L * E * stride, "cache_bytes": slots * stride,
                   "cache_slots": int(slots),
                   "timing": "per-token CUDA events on the launching stream (the host's wait "
                             "for each layer's picks included); inputs: each token streams its "
                             "layers' weights (>1 GB) through HBM",
                   "expert_launch": ("early: queued behind the router before the picks reach "
                                     "the host, run again after a miss (OSM_CACHED_EARLY)"
                                     if args.stream_early else
                                     "after the picks are resident"),
                   "cache_hit_rate": round(hits / max(1, hits + misses), 4),
                   "cache_loads": int(s1["loads"] - s0["loads"]),
                   "cache_evictions": int(s1["evictions"] - s0["evictions"]),
                   "h2d_bytes_per_token": int(h2d // args.steps),
                   "exposed_h2d_ms_per_token": round(exp_ms / args.steps, 4),
                   "exposed_h2d_note": "compute-stream time from an acquire's copies being "
                                       "issued to the stream's wait for them ending, summed "
                                       "over layers (osm_cache_exposed_read)"},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d // args.steps),
                "d2h_bytes_per_step": L * K * 4},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": "whole token (all layers)",
                     "achieved": round(alg / (tot_ms / args.steps / 1e3) / 1e9, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(alg / (tot_ms / args.steps / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                     "traffic": None,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)"},
        "clocks": clk,
    }


def cpu_baseline_leg(torch, ctx, slab, W, sg, bias, shared, xs, osm):
    """The reference CPU path on the host cores on a bounded sample (the B=32
    batch of the sweep), token-parallel over all threads."""
    import ctypes

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as cb

    lay = osm.expert_layout(H, I, GROUP)
    slots = np.zeros((E, lay.stride), np.uint8)
    ctx.check(osm.lib().osm_download(ctx.h, ctypes.c_void_p(slots.ctypes.data),
                                     ctypes.c_void_p(slab.slot_ptr(0)), E * lay.stride))
    x = xs[32].cpu().numpy()
    threads = cb.cpu_count()
    sub = cb.Sublayer(slots, shared, W, sg, bias, H, I, K, threads)
    sub.prepare(x)
    secs, n = 0.0, 0
    while secs < 5.0 and n < 200:
        secs += sub.run(x, threads)
        n += 1
    st = sub.run(x[:4], 1)
    return {"value": round(n * x.shape[0] / secs, 2), "unit": "tokens/s", "cores": threads,
            "kind": sub.kind,
            "sample": f"the B=32 decode batch of the sweep, {n} passes, {threads} threads; "
                      f"dequantisation of {len(sub.deq)} experts excluded ({sub.dequant_s:.1f} s)",
            "single_thread_tokens_per_s": round(4 / st, 2), "cpu_model": cb.cpu_model()}


# ----------------------------------------------------------------------------
# reference arm
# ----------------------------------------------------------------------------
def run_reference(args, rank, world):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as cb
    import pyoracle

    if rank != 0:
        return None
    port = pyoracle.Oracle("port")
    threads = cb.cpu_count()
    W = bf16_round(port.gen_normal(SEED, 1, 0.02, E * H)).reshape(E, H)
    sg = bf16_round(port.gen_normal(SEED, 2, 0.02, H))
    bias = zipf_bias(E, ZIPF_S, SEED)
    shared = port.gen_expert_slot(SEED, 1000 + 3 * E, 0.02, H, I)
    # the whole sweep of our arm's step (B = 1, 8, 32, 64, 128, 256: 489
    # tokens, the same inputs), run token-parallel over all host threads
    x = np.concatenate([port.gen_normal(SEED, 5000 + B, 1.0, B * H).reshape(B, H)
                        for B in SWEEP])
    stride = pyoracle.slot_stride(H, I)
    slots = np.zeros((E, stride), np.uint8)
    sub = cb.Sublayer(slots, shared, W, sg, bias, H, I, K, threads)
    need = sorted(sub.route_ids(x))
    from concurrent.futures import ThreadPoolExecutor

    def gen(e):
        slots[e] = port.gen_expert_slot(SEED, 1000 + 3 * e, 0.02, H, I)

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(gen, need))
    sub.prepare(x)
    for _ in range(args.warmup):
        sub.run(x, threads)
    secs = sum(sub.run(x, threads) for _ in range(args.steps))
    value = args.steps * x.shape[0] / secs
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "impl": "reference",
        "data": "synthetic (same seeds as our arm)",
        "config": {"workload": WORKLOAD, "tokens_per_step": int(x.shape[0]),
                   "sample": "the full sweep (B=1,8,32,64,128,256) per step, all tokens "
                             "token-parallel over the host threads"},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads,
                         "kind": sub.kind,
                         "sample": f"{x.shape[0]} tokens per step (the whole sweep), "
                                   f"{len(sub.deq)} experts dequantised once "
                                   f"({sub.dequant_s:.1f} s, excluded)",
                         "cpu_model": cb.cpu_model()},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_single(B: int, reps: int, prefill: bool = False):
    """A few calls of one batch size on the bench sublayer: the small case
    for ncu captures of one kernel (prefill: the config-2 sublayer, no router
    bias, on the tensor-core prefill path)."""
    import torch

    import osm_b200 as osm

    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = osm.Context(0, max_tokens=max(SWEEP + (B,)))
    ctx.set_stream(stream.cuda_stream)
    layer = build_sublayer(torch, ctx, osm, zipf=not prefill)[0]
    x = torch.empty(B, H, device="cuda")
    ctx.gen_normal(SEED, 5000 + B, 1.0, x)
    out = torch.empty(B, H, device="cuda")
    for _ in range(reps):
        layer.run_qwen_sparse_moe(x, B, out, prefill=prefill)
    torch.cuda.synchronize()
    print(json.dumps({"single": B, "reps": reps, "status": list(ctx.status())}))


SUB_KEYS = ("value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "dtype",
            "e2e", "gpu_launches", "roofline", "clocks")


STREAM_SUB_TOKENS = 128   # configs[4] sub-run of the default line
STREAM_SUB_WARMUP = 8


def sub_workloads(args, rank, world, local_rank):
    """configs[2] (4096-token prefill) and configs[3] (Qwen3-30B-A3B shape)
    timed in the same run as the headline sweep, each with its own steps,
    timing rules and roofline; under torchrun both run expert parallel over
    the ranks (strong scaling), as the configs ask."""
    import copy

    sub = copy.copy(args)
    sub.steps = max(3, min(args.steps, 20))
    sub.warmup = 3
    out = {}
    for key, fn in (("configs[2]", run_prefill), ("configs[3]", run_q30)):
        line = fn(sub, rank, world, local_rank)
        d = {k: line[k] for k in SUB_KEYS if k in line}
        d["workload"] = line["config"]["workload"]
        d["parallelism"] = line["config"]["parallelism"]
        for extra in ("per_case", "kernels", "kernels_8192"):
            if extra in line["config"]:
                d[extra] = line["config"][extra]
        out[key] = d
    if world == 1 and args.stream_sub:
        # configs[4] on one GPU only: every rank would pin its own 43.5 GB
        # host copy of the 48 layers' experts
        s4 = copy.copy(args)
        s4.steps = STREAM_SUB_TOKENS
        s4.warmup = STREAM_SUB_WARMUP
        line = run_stream(s4, rank, world, local_rank)
        d = {k: line[k] for k in SUB_KEYS if k in line}
        for extra in ("workload", "layers", "cache_slots", "cache_hit_rate", "cache_loads",
                      "cache_evictions", "h2d_bytes_per_token", "exposed_h2d_ms_per_token",
                      "expert_launch"):
            d[extra] = line["config"][extra]
        d["sample"] = (f"{STREAM_SUB_TOKENS} decode tokens after {STREAM_SUB_WARMUP} warm-up "
                       "tokens (the cache fills during the warm-up and the first timed tokens)")
        out["configs[4]"] = d
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--single", type=int, default=0,
                    help="profiling driver: run REPS calls of this many tokens and exit")
    ap.add_argument("--prefill", action="store_true",
                    help="with --single: the config-2 sublayer on the tensor-core prefill path")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--workload", choices=("decode", "prefill", "q30", "stream"), default="decode",
                    help="decode: configs[1] sweep (the headline line); prefill: configs[2]; "
                         "q30: configs[3] (one GPU: 1, 64 and 8192 tokens; expert parallel: "
                         "8192 tokens); stream: configs[4]")
    ap.add_argument("--eager", dest="graphs", action="store_false",
                    help="decode sweep: launch each call's kernels one by one instead of "
                         "replaying a CUDA-graph plan")
    ap.add_argument("--ep", action="store_true",
                    help="prefill and q30 workloads: the expert-parallel path even on one rank "
                         "(a one-rank NCCL group); under torchrun with N > 1 it is always used")
    ap.add_argument("--no-sub", dest="sub", action="store_false",
                    help="decode workload: skip the configs[2], configs[3] (and configs[4]) sub-runs "
                         "whose results the line carries under 'workloads'")
    ap.add_argument("--no-stream-sub", dest="stream_sub", action="store_false",
                    help="decode workload on one GPU: skip the configs[4] streaming sub-run")
    ap.add_argument("--stream-late", dest="stream_early", action="store_false",
                    help="configs[4]: queue each layer's expert kernels only after its picks "
                         "are resident (default: early, OSM_CACHED_EARLY)")
    ap.add_argument("--stream-layers", type=int, default=48,
                    help="with --workload stream: layers in the stack")
    args = ap.parse_args()
    if args.single:
        run_single(args.single, args.reps, args.prefill)
        return
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    args.ep = args.ep or world > 1
    use_group = world > 1 or (args.ep and args.workload in ("prefill", "q30"))
    if use_group:
        import datetime

        import torch

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29531")
        os.environ.setdefault("RANK", str(rank))
        os.environ.setdefault("WORLD_SIZE", str(world))
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "prefill":
            line = run_prefill(args, rank, world, local_rank)
        elif args.workload == "stream":
            line = run_stream(args, rank, world, local_rank)
        elif args.workload == "q30":
            line = run_q30(args, rank, world, local_rank)
        else:
            line = run_ours(args, rank, world, local_rank)
            if args.sub:
                line["workloads"] = sub_workloads(args, rank, world, local_rank)
    finally:
        if use_group:
            import torch

            torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
