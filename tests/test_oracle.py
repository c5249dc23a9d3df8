"""Pins the C restatement (oracle/osm_oracle.c) before anything trusts it:

* against the known-answer tests of the reference's own test files
  (tests/golden/reference_kats.json), for both the port and the reference
  compiled in place;
* bit-for-bit against the reference's CPU code (oracle/_ref) on seeded inputs;
* against the committed golden vectors (reference outputs).
"""
import json
import math
import os

import numpy as np
import pytest

import pyoracle


@pytest.fixture(scope="module")
def kats(golden_dir):
    with open(os.path.join(golden_dir, "reference_kats.json")) as f:
        return json.load(f)


def both(port, request):
    out = [port]
    if pyoracle.ref_available():
        out.append(pyoracle.Oracle("reference"))
    return out


def test_kats_dequant_matvec_rmsnorm_topk_swiglu(port, kats, request):
    for o in both(port, request):
        k = kats["q4_affine"]
        word = sum(q << (4 * i) for i, q in enumerate(k["q"]))
        out = o.dequantize_affine_rows(np.array([word], np.uint32), 1, 1, [k["scale"]],
                                       [k["bias"]], 4, k["group"])
        np.testing.assert_allclose(out[0], k["expected"], atol=k["tol"])
        k = kats["q8_affine"]
        word = sum(q << (8 * i) for i, q in enumerate(k["q"]))
        out = o.dequantize_affine_rows(np.array([word], np.uint32), 1, 1, [k["scale"]],
                                       [k["bias"]], 8, k["group"])
        np.testing.assert_allclose(out[0], k["expected"], atol=k["tol"])
        k = kats["matvec"]
        np.testing.assert_allclose(o.matvec(np.array(k["w"], np.float32), k["x"]),
                                   k["expected"], atol=k["tol"])
        k = kats["rmsnorm"]
        np.testing.assert_allclose(o.rms_norm(np.array(k["values"], np.float32), k["weight"],
                                              k["eps"]), k["expected"], atol=k["tol"])
        k = kats["top_k"]
        ids, probs = o.route_top_k(k["logits"], k["k"], False)
        assert list(ids) == k["expected_ids"]
        np.testing.assert_allclose(probs, k["expected_raw_probs"], atol=k["tol"])
        ids, probs = o.route_top_k(k["logits"], k["k"], True)
        assert list(ids) == k["expected_ids"]
        assert abs(float(probs.sum()) - 1.0) <= k["tol"]
        k = kats["swiglu"]
        np.testing.assert_allclose(o.swiglu(k["gate"], k["up"]), k["expected"], atol=k["tol"])
        k = kats["invalid_bits"]
        with pytest.raises(pyoracle.OracleError) as ei:
            o.dequantize_affine_rows(np.zeros(1, np.uint32), 1, 1, [1.0], [0.0], k["bits"],
                                     k["group"])
        assert ei.value.rc == -1


def test_kats_router(port, kats, request):
    for o in both(port, request):
        k = kats["router_2_of_4"]
        _, ids, w, mass = o.route_qwen_top_k(k["hidden"], k["weight"], k["k"], True)
        assert list(ids) == k["expected_ids"]
        np.testing.assert_allclose(w, k["expected_norm_weights"], atol=k["tol"])
        assert abs(mass - k["expected_mass"]) <= k["tol"]
        _, ids, w, mass2 = o.route_qwen_top_k(k["hidden"], k["weight"], k["k"], False)
        assert list(ids) == k["expected_ids"]
        np.testing.assert_allclose(w, k["expected_raw_weights"], atol=k["tol"])
        assert abs(float(w.sum()) - mass2) <= k["tol"] and mass2 < 1.0
        k = kats["router_tie"]
        _, ids, w, _ = o.route_qwen_top_k(k["hidden"], k["weight"], k["k"], True)
        assert list(ids) == k["expected_ids"]
        np.testing.assert_allclose(w, k["expected_norm_weights"], atol=k["tol"])
        k = kats["router_512_top10"]
        W = (np.arange(k["experts"], dtype=np.float32) * np.float32(k["weight_step"]))
        _, ids, w, _ = o.route_qwen_top_k(k["hidden"], W, k["k"], True)
        assert list(ids) == k["expected_ids"]
        assert abs(float(w.sum()) - 1.0) <= k["sum_tol"]
        k = kats["router_bad_shape"]
        with pytest.raises(pyoracle.OracleError) as ei:
            o._rq(np.array(k["hidden"], np.float32), np.array(k["weight"], np.float32), None,
                  1, k["experts"], k["k"], 1, np.zeros(4, np.float32), np.zeros(2, np.uint32),
                  np.zeros(2, np.float32), pyoracle.C.byref(pyoracle.C.c_float()))
            raise pyoracle.OracleError(-1, "shape accepted")
        assert ei.value.rc == -1


def test_kats_shared_and_quantizer(port, kats, request):
    import make_golden

    for o in both(port, request):
        x, gate, up, down, scalar = make_golden.shared_fixture()
        out, scale = o.shared_expert(gate, up, down, scalar, x)
        g = port.matvec(gate, x)
        u = port.matvec(up, x)
        h = port.swiglu(g, u)
        expected = port.matvec(down, h)
        logit = np.float32(0)
        for i in range(8):
            logit = np.float32(logit + np.float32(scalar[i] * x[i]))
        es = np.float32(1.0) / (np.float32(1.0) + np.float32(math.exp(-float(logit))))
        assert abs(scale - es) <= kats["shared_expert"]["gate_tol"]
        np.testing.assert_allclose(out, expected * np.float32(scale),
                                   atol=kats["shared_expert"]["out_tol"])
        k = kats["quantizer"]
        pk, sc, bi = o.quantize_q4(np.array(k["values"], np.float32), k["rows"], k["cols"],
                                   k["group"])
        dq = o.dequantize_affine_rows(pk, k["rows"], k["cols"] // 8, sc, bi, 4, k["group"])
        err = np.abs(dq.reshape(-1) - np.array(k["values"], np.float32))
        assert np.all(err <= np.repeat(sc.reshape(-1), k["group"]) * 0.5001 + 1e-6)
        with pytest.raises(pyoracle.OracleError):
            o.quantize_q4(np.array(k["values"], np.float32), k["rows"], k["cols"],
                          k["bad_group"])


def test_port_matches_reference_bitwise(port, ref):
    rng = np.random.default_rng(7)
    for trial in range(20):
        rows = int(rng.integers(1, 9))
        pc = int(rng.integers(1, 9)) * 8
        bits = 4 if trial % 2 == 0 else 8
        per = 32 // bits
        group = 64 if bits == 4 else 32
        packed = rng.integers(0, 2**32, size=rows * pc, dtype=np.uint64).astype(np.uint32)
        g = rows * pc * per // group
        s = rng.standard_normal(g).astype(np.float32)
        b = rng.standard_normal(g).astype(np.float32)
        a = port.dequantize_affine_rows(packed, rows, pc, s, b, bits, group)
        r = ref.dequantize_affine_rows(packed, rows, pc, s, b, bits, group)
        assert np.array_equal(a.view(np.uint32), r.view(np.uint32))
        W = rng.standard_normal((13, 257)).astype(np.float32)
        x = rng.standard_normal(257).astype(np.float32)
        assert np.array_equal(port.matvec(W, x).view(np.uint32), ref.matvec(W, x).view(np.uint32))
        v = rng.standard_normal((3, 100)).astype(np.float32)
        w = rng.standard_normal(100).astype(np.float32)
        assert np.array_equal(port.rms_norm(v, w, 1e-6).view(np.uint32),
                              ref.rms_norm(v, w, 1e-6).view(np.uint32))
        assert np.array_equal(port.rms_norm(v, None, 1e-6).view(np.uint32),
                              ref.rms_norm(v, None, 1e-6).view(np.uint32))
        lg = (rng.standard_normal(64) * 3).astype(np.float32)
        assert np.array_equal(port.softmax(lg).view(np.uint32), ref.softmax(lg).view(np.uint32))
        for k in (1, 5, 64):
            for norm in (False, True):
                i1, p1 = port.route_top_k(lg, k, norm)
                i2, p2 = ref.route_top_k(lg, k, norm)
                assert np.array_equal(i1, i2) and np.array_equal(p1.view(np.uint32),
                                                                 p2.view(np.uint32))


def test_router_ties_and_bias_bitwise(port, ref):
    rng = np.random.default_rng(11)
    # many exact ties: logits drawn from a small set of values
    for trial in range(50):
        E = int(rng.integers(2, 80))
        k = int(rng.integers(1, E + 1))
        H = 4
        W = rng.integers(-2, 3, size=(E, H)).astype(np.float32)
        x = rng.integers(-1, 2, size=H).astype(np.float32)
        bias = rng.integers(-1, 2, size=E).astype(np.float32) if trial % 3 == 0 else None
        for norm in (False, True):
            a = port.route_qwen_top_k(x, W, k, norm, bias=bias)
            r = ref.route_qwen_top_k(x, W, k, norm, bias=bias)
            assert np.array_equal(a[0].view(np.uint32), r[0].view(np.uint32))
            assert np.array_equal(a[1], r[1]), (a[1], r[1])
            assert np.array_equal(a[2].view(np.uint32), r[2].view(np.uint32))
            assert np.float32(a[3]).view(np.uint32) == np.float32(r[3]).view(np.uint32)


def test_quantizer_and_shared_and_moe_bitwise(port, ref):
    vals = port.gen_normal(3, 9, 0.02, 16 * 256)
    a = port.quantize_q4(vals, 16, 256, 64)
    r = ref.quantize_q4(vals, 16, 256, 64)
    for x, y in zip(a, r):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
    H, I, E, K = 128, 64, 6, 3
    slots = [port.gen_expert_slot(5, 10 + 3 * e, 0.02, H, I) for e in range(E)]
    experts = {e: port.dequant_slot(slots[e], H, I) for e in range(E)}
    sh = port.dequant_slot(port.gen_expert_slot(5, 1, 0.02, H, I), H, I)
    sg = port.gen_normal(5, 2, 0.02, H)
    W = port.gen_normal(5, 3, 0.02, E * H).reshape(E, H)
    for t in range(4):
        x = port.gen_normal(5, 100 + t, 1.0, H)
        o1 = port.moe_token(x, W, K, True, experts, shared=sh, scalar_gate=sg)
        o2 = ref.moe_token(x, W, K, True, experts, shared=sh, scalar_gate=sg)
        assert np.array_equal(o1[0].view(np.uint32), o2[0].view(np.uint32))
        assert np.array_equal(o1[1], o2[1])
        s1 = port.shared_expert(*sh, sg, x)
        s2 = ref.shared_expert(*sh, sg, x)
        assert np.array_equal(s1[0].view(np.uint32), s2[0].view(np.uint32)) and s1[1] == s2[1]


def test_port_matches_golden_vectors(port, golden_dir):
    z = np.load(os.path.join(golden_dir, "router_small.npz"))
    for b in range(z["x"].shape[0]):
        lg, ids, w, m = port.route_qwen_top_k(z["x"][b], z["W"], int(z["k"]), True)
        assert np.array_equal(lg.view(np.uint32), z["logits"][b].view(np.uint32))
        assert np.array_equal(ids, z["ids"][b])
        assert np.array_equal(w.view(np.uint32), z["weights"][b].view(np.uint32))
        assert np.float32(m) == z["mass"][b]
    z = np.load(os.path.join(golden_dir, "router_q3n.npz"))
    W = pyoracle.bf16_widen(z["Wbits"])
    for b in range(z["x"].shape[0]):
        bias = z["bias"] if b % 2 else None
        lg, ids, w, m = port.route_qwen_top_k(z["x"][b], W, int(z["k"]), True, bias=bias)
        assert np.array_equal(lg.view(np.uint32), z["logits"][b].view(np.uint32))
        assert np.array_equal(ids, z["ids"][b])
        assert np.array_equal(w.view(np.uint32), z["weights"][b].view(np.uint32))
    z = np.load(os.path.join(golden_dir, "quantizer.npz"))
    pk, sc, bi = port.quantize_q4(z["values"], 8, 256, 64)
    assert np.array_equal(pk, z["packed"]) and np.array_equal(sc, z["scales"])
    assert np.array_equal(bi, z["biases"])
    z = np.load(os.path.join(golden_dir, "hash_fixture.npz"))
    experts = {e: port.dequant_slot(z["slots"][e], 128, 64) for e in range(3)}
    out, ids, w, m, _ = port.moe_token(z["x"], z["router"], 2, True, experts)
    assert list(ids) == [1, 2] and np.array_equal(ids, z["ids"])
    assert np.array_equal(out.view(np.uint32), z["out"].view(np.uint32))
    z = np.load(os.path.join(golden_dir, "moe_small.npz"))
    H, I = z["x"].shape[1], int(z["inter"])
    E = z["slots"].shape[0]
    experts = {e: port.dequant_slot(z["slots"][e], H, I) for e in range(E)}
    sh = port.dequant_slot(z["shared"], H, I)
    for b in range(z["x"].shape[0]):
        out, ids, w, _, ss = port.moe_token(z["x"][b], pyoracle.bf16_widen(z["Wbits"]),
                                            int(z["k"]), True, experts, shared=sh,
                                            scalar_gate=pyoracle.bf16_widen(z["sgbits"]))
        assert np.array_equal(ids, z["ids"][b])
        assert np.array_equal(out.view(np.uint32), z["out"][b].view(np.uint32))
        assert np.float32(ss) == z["shared_scale"][b]


def test_generator_is_deterministic_and_normal(port):
    a = port.gen_normal(1, 2, 1.0, 200000)
    b = port.gen_normal(1, 2, 1.0, 100, first=1000)
    assert np.array_equal(a[1000:1100], b)
    assert abs(float(a.mean())) < 0.01 and abs(float(a.std()) - 1.0) < 0.01
    s1 = port.gen_expert_slot(1, 2, 0.02, 256, 64)
    s2 = port.gen_expert_slot(1, 2, 0.02, 256, 64)
    assert np.array_equal(s1, s2) and s1.size == pyoracle.slot_stride(256, 64)
    assert pyoracle.slot_stride(2048, 512) == 1769472
    assert pyoracle.slot_stride(2048, 768) == 2654208


def test_moe_token_slots_equals_moe_token_bitwise(port):
    """The slot-based oracle entry (dequantise only the picked experts) gives
    the bits of moe_token on fully dequantised experts, with and without a
    shared expert and a logit bias."""
    H, E, I, K = 256, 12, 128, 4
    slots = np.stack([port.gen_expert_slot(9, 300 + 3 * e, 0.02, H, I) for e in range(E)])
    shared = port.gen_expert_slot(9, 290, 0.02, H, I)
    W = pyoracle.bf16_widen(port.bf16_round(port.gen_normal(9, 1, 0.05, E * H))).reshape(E, H)
    sg = port.gen_normal(9, 2, 0.02, H)
    bias = port.gen_normal(9, 3, 0.5, E)
    experts = {e: port.dequant_slot(slots[e], H, I) for e in range(E)}
    sh = port.dequant_slot(shared, H, I)
    for t in range(4):
        x = port.gen_normal(9, 10 + t, 1.0, H)
        for b, with_shared in ((None, True), (bias, False)):
            a = port.moe_token(x, W, K, True, experts, shared=sh if with_shared else None,
                               scalar_gate=sg if with_shared else None, bias=b)
            s = port.moe_token_slots(x, W, K, True, slots, I,
                                     shared_slot=shared if with_shared else None,
                                     scalar_gate=sg if with_shared else None, bias=b)
            assert np.array_equal(a[0].view(np.uint32), s[0].view(np.uint32))
            assert np.array_equal(a[1], s[1]) and np.array_equal(a[2], s[2])
            assert a[3] == s[3] and a[4] == s[4]
