"""Generate the golden fixtures under tests/golden/ (run in the build
container, where the reference sources exist and oracle/_ref is built).

    python tests/golden/make_golden.py

Two kinds of fixture:

* ``reference_kats.json`` -- the known-answer tests that the reference's own
  test files hold for this path, restated as data: inputs, the closed-form
  expected values those tests assert, and their tolerances.  Sources:
  tests/cpu_reference_test.cpp:48-166, tests/qwen_router_test.cpp:51-191,
  tests/shared_expert_test.cpp:36-85, tests/affine_q4_quantizer_test.cpp:21-60,
  tests/expert_cache_test.cpp:80-192,
  tests/vulkan_resident_expert_cache_test.cpp:314-382.
* ``*.npz`` -- seeded inputs and the outputs of the reference's CPU code
  compiled in place (oracle/_ref/libosm_ref.so), so GPU tests on a box without
  the reference can compare against the reference itself.
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import pyoracle  # noqa: E402


def f32(v):
    return float(np.float32(v))


def kats() -> dict:
    e = [f32(math.exp(np.float32(i))) for i in range(5)]
    gsum = f32(np.float32(e[1]) + np.float32(e[2]) + np.float32(e[3]) + np.float32(e[4]))
    base = f32(np.sqrt(np.float32((9.0 + 16.0) / 2.0)))
    probs4 = np.exp(np.arange(4, dtype=np.float64) - 3.0)
    probs4 = probs4 / probs4.sum()
    return {
        "q4_affine": {  # cpu_reference_test.cpp:48-71
            "q": [0, 1, 2, 3, 4, 5, 6, 7], "scale": 2.0, "bias": -1.0, "group": 8,
            "expected": [2.0 * i - 1.0 for i in range(8)], "tol": 1e-6},
        "q8_affine": {  # cpu_reference_test.cpp:73-93
            "q": [2, 4, 6, 8], "scale": 0.5, "bias": 1.0, "group": 4,
            "expected": [2.0, 3.0, 4.0, 5.0], "tol": 1e-6},
        "matvec": {  # cpu_reference_test.cpp:95-106
            "w": [[1.0, 2.0], [-1.0, 3.0]], "x": [4.0, 5.0],
            "expected": [14.0, 11.0], "tol": 1e-6},
        "rmsnorm": {  # cpu_reference_test.cpp:107-113
            "values": [3.0, 4.0], "weight": [2.0, 0.5], "eps": 0.0,
            "expected": [f32(3.0 / base * 2.0), f32(4.0 / base * 0.5)], "tol": 1e-6},
        "top_k": {  # cpu_reference_test.cpp:115-136
            "logits": [0.0, 1.0, 2.0, 3.0], "k": 2, "expected_ids": [3, 2],
            "expected_raw_probs": [float(probs4[3]), float(probs4[2])],
            "normalized_sum": 1.0, "tol": 1e-6},
        "swiglu": {  # cpu_reference_test.cpp:138-147
            "gate": [-1.0, 0.0, 1.0], "up": [2.0, 3.0, 4.0],
            "expected": [f32(-1.0 / (1.0 + math.exp(1.0)) * 2.0), 0.0,
                         f32(1.0 / (1.0 + math.exp(-1.0)) * 4.0)], "tol": 1e-6},
        "invalid_bits": {"bits": 3, "group": 8},  # cpu_reference_test.cpp:149-166
        "router_2_of_4": {  # qwen_router_test.cpp:51-126
            "hidden": [1.0], "weight": [1.0, 2.0, 3.0, 4.0], "k": 2,
            "expected_ids": [3, 2],
            "expected_norm_weights": [f32(e[4] / (e[4] + e[3])), f32(e[3] / (e[4] + e[3]))],
            "expected_raw_weights": [f32(e[4] / gsum), f32(e[3] / gsum)],
            "expected_mass": f32((e[4] + e[3]) / gsum), "tol": 1e-6},
        "router_tie": {  # qwen_router_test.cpp:128-146
            "hidden": [1.0], "weight": [5.0, 5.0, 1.0, 0.0], "k": 1,
            "expected_ids": [0], "expected_norm_weights": [1.0], "tol": 1e-6},
        "router_512_top10": {  # qwen_router_test.cpp:151-179
            "hidden": [1.0], "weight_step": 0.01, "experts": 512, "k": 10,
            "expected_ids": [511 - i for i in range(10)], "sum_tol": 1e-5},
        "router_bad_shape": {  # qwen_router_test.cpp:181-191
            "hidden": [1.0], "weight": [1.0, 2.0], "experts": 4, "k": 2},
        "shared_expert": {  # shared_expert_test.cpp:36-85 (formula fixture)
            "hidden": 8, "inter": 4, "gate_tol": 1e-7, "out_tol": 1e-6},
        "quantizer": {  # affine_q4_quantizer_test.cpp:21-60
            "rows": 2, "cols": 8, "group": 4,
            "values": [-1.0, -0.5, 0.0, 0.5, 1.0, 1.5, 2.0, 2.5,
                       3.0, 3.0, 3.0, 3.0, -2.0, -1.0, 0.0, 1.0],
            "bad_group": 3},
        "expert_cache": {  # expert_cache_test.cpp:80-192
            "lfu": {"stride": 4, "slots": 2, "sequence": [[0], [0], [1], [2]],
                    "resident": [0, 2], "evicted": [1]},
            "recency_tie": {"stride": 4, "slots": 2, "sequence": [[0], [1], [2]],
                            "resident": [1, 2], "evicted": [0]},
            "batch_protect": {"stride": 8, "slots": 2, "sequence": [[0, 1], [2, 3]],
                              "resident": [2, 3]},
            "oversized": {"stride": 4, "slots": 2, "batch": [0, 1, 2]}},
        "resident_cache": {  # vulkan_resident_expert_cache_test.cpp:314-382
            "sequence": [0, 1, 0, 2], "budget_experts": 2,
            "resident": [0, 2], "evicted": [1],
            "stats_after": {"hits": 1, "misses": 3, "loads": 3, "evictions": 1},
            "accounted_bytes_hidden128_inter64": 17152,
            "out_tol": 0.01},
    }


def shared_fixture():
    """shared_expert_test.cpp:36-55 formula weights."""
    H, I = 8, 4
    x = np.array([(i - 3) * 0.25 for i in range(H)], np.float32)
    gate = np.array([((i % 9) - 4) * 0.0625 for i in range(I * H)], np.float32).reshape(I, H)
    up = np.array([(((i * 3) % 11) - 5) * 0.05 for i in range(I * H)], np.float32).reshape(I, H)
    down = np.array([(((i * 5) % 13) - 6) * 0.04 for i in range(H * I)], np.float32).reshape(H, I)
    scalar = np.array([((i % 5) - 2) * 0.125 for i in range(H)], np.float32)
    return x, gate, up, down, scalar


def hash_fixture_slot(expert: int) -> np.ndarray:
    """The integer-hash qpack fixture of tests/weighted_routed_moe_test.cpp:
    52-133 (hidden 128, inter 64, group 64, BF16 metadata by truncation)."""
    H, I = 128, 64
    lay = pyoracle.slot_layout(H, I, 64)
    slot = np.zeros(lay["stride"], np.uint8)

    def fill(seed, rows, packed_cols, groups, w_off, s_off, b_off):
        words = np.zeros((rows, packed_cols), np.uint32)
        for r in range(rows):
            for w in range(packed_cols):
                v = 0
                for lane in range(8):
                    q = (seed * 3 + expert * 5 + r * 7 + w * 2 + lane) & 0xF
                    v |= q << (lane * 4)
                words[r, w] = v
        sc = np.zeros((rows, groups), np.float32)
        bi = np.zeros((rows, groups), np.float32)
        for r in range(rows):
            for g in range(groups):
                sc[r, g] = ((seed + expert + r + g) % 6 + 1) * 0.125
                bi[r, g] = ((seed * 2 + expert + r + g) % 7 - 3) * 0.125
        slot[w_off:w_off + words.nbytes] = words.view(np.uint8).reshape(-1)
        trunc = lambda a: (a.view(np.uint32) >> 16).astype(np.uint16)  # noqa: E731
        slot[s_off:s_off + sc.size * 2] = trunc(sc).view(np.uint8).reshape(-1)
        slot[b_off:b_off + bi.size * 2] = trunc(bi).view(np.uint8).reshape(-1)

    fill(1, I, H // 8, H // 64, lay["gate_w"], lay["gate_s"], lay["gate_b"])
    fill(2, I, H // 8, H // 64, lay["up_w"], lay["up_s"], lay["up_b"])
    fill(3, H, I // 8, I // 64, lay["down_w"], lay["down_s"], lay["down_b"])
    return slot


def hash_fixture_token(seed: int) -> np.ndarray:
    """tests/weighted_routed_moe_test.cpp:271-279."""
    return np.array([((i * (seed + 5)) % 31 - 15) * 0.03125 for i in range(128)], np.float32)


def main() -> None:
    if not pyoracle.ref_available():
        sys.exit("oracle/_ref/libosm_ref.so missing: run make -C oracle first")
    ref = pyoracle.Oracle("reference")
    port = pyoracle.Oracle("port")
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(kats(), f, indent=1)

    rng_seed = 20240611

    # 1. router, small shape, many tokens, fp32 weights (bit-exact ids/logits)
    H, E, K, B = 64, 32, 4, 64
    x = port.gen_normal(rng_seed, 1, 1.0, B * H).reshape(B, H)
    W = port.gen_normal(rng_seed, 2, 0.5, E * H).reshape(E, H)
    logits = np.zeros((B, E), np.float32)
    ids = np.zeros((B, K), np.uint32)
    w = np.zeros((B, K), np.float32)
    mass = np.zeros(B, np.float32)
    for b in range(B):
        logits[b], ids[b], w[b], mass[b] = ref.route_qwen_top_k(x[b], W, K, True)
    np.savez_compressed(os.path.join(HERE, "router_small.npz"), x=x, W=W, k=K,
                        logits=logits, ids=ids, weights=w, mass=mass)

    # 2. router at the Qwen3-Next shape with bf16-valued weights and a Zipf
    #    logit bias on half the tokens
    H, E, K, B = 2048, 512, 10, 8
    x = port.gen_normal(rng_seed, 3, 1.0, B * H).reshape(B, H)
    Wbits = port.bf16_round(port.gen_normal(rng_seed, 4, 0.02, E * H)).reshape(E, H)
    W = pyoracle.bf16_widen(Wbits)
    perm = np.random.default_rng(rng_seed).permutation(E)
    r = np.arange(1, E + 1, dtype=np.float64)
    hz = (r ** -1.1).sum()
    bias = np.zeros(E, np.float32)
    bias[perm] = np.log(r ** -1.1 / hz).astype(np.float32)
    logits = np.zeros((B, E), np.float32)
    ids = np.zeros((B, K), np.uint32)
    w = np.zeros((B, K), np.float32)
    mass = np.zeros(B, np.float32)
    for b in range(B):
        bb = bias if b % 2 else None
        logits[b], ids[b], w[b], mass[b] = ref.route_qwen_top_k(x[b], W, K, True, bias=bb)
    np.savez_compressed(os.path.join(HERE, "router_q3n.npz"), x=x, Wbits=Wbits, bias=bias,
                        k=K, logits=logits, ids=ids, weights=w, mass=mass)

    # 3. quantizer (reference quantiser) on N(0, 0.02) rows
    vals = port.gen_normal(rng_seed, 5, 0.02, 8 * 256).reshape(8, 256)
    pk, sc, bi = ref.quantize_q4(vals, 8, 256, 64)
    np.savez_compressed(os.path.join(HERE, "quantizer.npz"), values=vals, packed=pk,
                        scales=sc, biases=bi)

    # 4. the reference's integer-hash routed-MoE fixture (3 experts, top-2)
    slots = np.stack([hash_fixture_slot(e) for e in range(3)])
    xt = hash_fixture_token(4)
    xt[0] = 1.0
    rw = np.zeros((3, 128), np.float32)
    rw[0, 0], rw[1, 0], rw[2, 0] = 1.0, 3.0, 2.0
    experts = {e: port.dequant_slot(slots[e], 128, 64) for e in range(3)}
    out, ids, w, mass, _ = ref.moe_token(xt, rw, 2, True, experts)
    np.savez_compressed(os.path.join(HERE, "hash_fixture.npz"), slots=slots, x=xt, router=rw,
                        out=out, ids=ids, weights=w, mass=np.float32(mass))

    # 5. a small complete sublayer: H=256, E=16, I=64, k=4, shared I=64
    H, E, I, K, B = 256, 16, 64, 4, 8
    slots = np.stack([port.gen_expert_slot(rng_seed, 100 + 3 * e, 0.02, H, I) for e in range(E)])
    shared = port.gen_expert_slot(rng_seed, 90, 0.02, H, I)
    Wbits = port.bf16_round(port.gen_normal(rng_seed, 6, 0.02, E * H)).reshape(E, H)
    sgbits = port.bf16_round(port.gen_normal(rng_seed, 7, 0.02, H))
    x = port.gen_normal(rng_seed, 8, 1.0, B * H).reshape(B, H)
    experts = {e: port.dequant_slot(slots[e], H, I) for e in range(E)}
    sh = port.dequant_slot(shared, H, I)
    outs = np.zeros((B, H), np.float32)
    ids = np.zeros((B, K), np.uint32)
    w = np.zeros((B, K), np.float32)
    ss = np.zeros(B, np.float32)
    for b in range(B):
        outs[b], ids[b], w[b], _, ss[b] = ref.moe_token(
            x[b], pyoracle.bf16_widen(Wbits), K, True, experts, shared=sh,
            scalar_gate=pyoracle.bf16_widen(sgbits))
    np.savez_compressed(os.path.join(HERE, "moe_small.npz"), slots=slots, shared=shared,
                        Wbits=Wbits, sgbits=sgbits, x=x, k=K, inter=I, out=outs, ids=ids,
                        weights=w, shared_scale=ss)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
