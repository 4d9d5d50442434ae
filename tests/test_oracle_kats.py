"""The CPU oracle against the reference's own known-answer tests (no GPU).

Golden cases come from tests/golden/reference_kats.json (transcribed from the
reference's test files, see make_reference_kats.py), plus an independent numpy
restatement of the quantizers on seeded random data.
"""
import json
import os

import numpy as np
import pytest

import oracle
from tinybrain_b200.runtime import QuantizedTensor, SeededGenerator

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def np_round_half_away(x):
    x = np.asarray(x, dtype=np.float32)
    return np.where(x >= 0, np.floor(x + np.float32(0.5)), -np.floor(-x + np.float32(0.5))).astype(np.float32)


def unpack_pair(b):
    # QuantizedTensor.swift:322-331
    b = int(b) & 0xFF
    hi, lo = (b >> 4) & 0xF, b & 0xF
    return (hi - 16 if hi > 7 else hi), (lo - 16 if lo > 7 else lo)


def test_int4_pack_pairs_round_trip():
    g = GOLD["int4_pack_pairs"]
    for a, b in g["pairs"]:
        p, s, z = oracle.quantize_int4_group(np.array([a, b], dtype=np.float32) * 1.0, group_size=2)
        # a group of two values quantizes to +-7 at its abs-max: check the nibble order instead
        hi, lo = unpack_pair(p[0])
        deq = oracle.dequantize(QuantizedTensor((1, 2), p, s, "int4", 2, z)).ravel()
        assert np.allclose(deq, [a, b], atol=max(abs(a), abs(b)) / 7.0 / 2 + 1e-6)
        assert np.sign(hi) == np.sign(a) and np.sign(lo) == np.sign(b)


def test_int4_pack_nibble_layout_and_clamp():
    # values already on the integer grid with scale 1 (abs-max 7) round-trip exactly
    for a, b in GOLD["int4_pack_pairs"]["pairs"]:
        x = np.array([a, b, 7.0, 0.0], dtype=np.float32)
        p, s, z = oracle.quantize_int4_group(x, group_size=4)
        assert s[0] == np.float32(1.0)
        assert unpack_pair(p[0]) == (a, b)
    c = GOLD["int4_pack_pairs"]["clamp"]
    x = np.array(c["in"], dtype=np.float32)
    p, s, z = oracle.quantize_int4_group(x, group_size=2)
    assert unpack_pair(p[0]) == (7, -7)


def test_int4_odd_count_bytes():
    g = GOLD["int4_odd_count"]
    x = np.array(g["input"], dtype=np.float32)
    p, s, z = oracle.quantize_int4_group(x, group_size=g["group_size"])
    assert p.size == g["packed_len"]
    assert p.tolist() == g["packed"]
    assert s.tolist() == pytest.approx(g["scales"], rel=0, abs=0)
    deq = oracle.dequantize(QuantizedTensor((3, 3), p, s, "int4", g["group_size"], z)).ravel()
    assert np.linalg.norm(deq - x) / np.linalg.norm(x) < g["max_rel_error"]


def test_all_zero_groups():
    g4 = GOLD["int4_all_zero"]
    x = np.zeros(g4["shape"], dtype=np.float32)
    p, s, z = oracle.quantize_int4_group(x, group_size=g4["group_size"])
    assert np.all(s == g4["scale"]) and np.all(p == 0) and np.all(z == 0)
    g8 = GOLD["int8_all_zero"]
    q, s8 = oracle.quantize_int8_per_channel(np.zeros(g8["shape"], dtype=np.float32))
    assert np.all(s8 == g8["scale"]) and np.all(q == 0)


def test_int4_negative_constant():
    g = GOLD["int4_negative_constant"]
    x = np.full(g["shape"], g["value"], dtype=np.float32)
    p, s, z = oracle.quantize_int4_group(x, group_size=g["group_size"])
    deq = oracle.dequantize(QuantizedTensor(tuple(g["shape"]), p, s, "int4", g["group_size"], z))
    assert abs(deq[0, 0] - g["value"]) < g["tolerance"] and deq[0, 0] < 0


def test_int8_per_channel_scales():
    g = GOLD["int8_per_channel_scales"]
    w = np.array(g["input"], dtype=np.float32).reshape(g["shape"])
    q, s = oracle.quantize_int8_per_channel(w)
    assert s.size == g["num_scales"]
    assert q.tolist() == g["q"]
    assert s.tolist() == g["scales"]
    assert s[0] != s[1] and s[2] != s[3]


def test_quantizers_match_numpy_restatement_bit_exact():
    g = SeededGenerator(7)
    w = g.normal((96, 160), 0.0, 0.02)
    w[:, 3] = 0.0  # an all-zero column -> scale 1
    q, s = oracle.quantize_int8_per_channel(w)
    absmax = np.max(np.abs(w), axis=0)
    s_ref = np.where(absmax < np.float32(1.4e-45), np.float32(1), absmax / np.float32(127)).astype(np.float32)
    q_ref = np.clip(np_round_half_away(w / s_ref), -127, 127).astype(np.int8)
    assert np.array_equal(s, s_ref)
    assert np.array_equal(q.reshape(w.shape), q_ref)
    p, s4, z = oracle.quantize_int4_group(w, 32)
    flat = w.ravel()
    grp = flat.reshape(-1, 32)
    a = np.maximum(np.abs(grp.min(1)), np.abs(grp.max(1)))
    s4_ref = np.where(a < np.float32(1.4e-45), np.float32(1), a / np.float32(7)).astype(np.float32)
    assert np.array_equal(s4, s4_ref)
    q4 = np.clip(np_round_half_away(flat / np.repeat(s4_ref, 32)), -7, 7).astype(np.int8)
    p_ref = (((q4[0::2] & 0xF) << 4) | (q4[1::2] & 0xF)).astype(np.uint8)
    assert np.array_equal(p, p_ref)


def test_greedy_kats():
    for logits, want in GOLD["greedy"]["cases"]:
        assert oracle.greedy(np.array(logits, dtype=np.float32)) == want


def test_silu_rmsnorm_kats():
    g = GOLD["silu"]
    for x, y in zip(g["x"], g["y"]):
        if y is not None:
            assert abs(oracle.silu(x) - y) < g["atol"]
    r = GOLD["rmsnorm"]
    for case in r["cases"]:
        y = oracle.rmsnorm(np.array(case["x"], np.float32), np.array(case["w"], np.float32))
        assert np.allclose(y, case["y"], atol=r["atol"])


def test_softmax_has_reference_epsilon():
    y = oracle.softmax(np.array([0.0, -np.inf, -np.inf], dtype=np.float32))
    assert y[0] == np.float32(1.0) / (np.float32(1.0) + np.float32(1e-7))


def numpy_attention(q, K, V, H, Hkv, d):
    L = K.shape[0]
    rep = H // Hkv
    out = np.zeros(H * d, dtype=np.float64)
    for h in range(H):
        kh = h // rep
        qh = q[h * d:(h + 1) * d].astype(np.float64)
        s = K[:, kh * d:(kh + 1) * d].astype(np.float64) @ qh / np.sqrt(d)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * d:(h + 1) * d] = p @ V[:, kh * d:(kh + 1) * d]
    return out


@pytest.mark.parametrize("H,Hkv,d,L", [(4, 4, 16, 32), (8, 2, 16, 33), (32, 4, 64, 17)])
def test_attention_matches_numpy(H, Hkv, d, L):
    g = SeededGenerator(11)
    q = g.normal((H * d,))
    K = g.normal((L, Hkv * d))
    V = g.normal((L, Hkv * d))
    out = oracle.attention(q, K, V, H, Hkv, d)
    ref = numpy_attention(q, K, V, H, Hkv, d)
    tol = GOLD["attention_tolerance"]
    assert np.max(np.abs(out - ref) / np.maximum(np.abs(ref), tol["atol"])) < tol["rtol"]


def test_qmatmul_modes_agree():
    g = SeededGenerator(3)
    w = g.normal((256, 192), 0.0, 0.02)
    x = g.normal((2, 256))
    q, s = oracle.quantize_int8_per_channel(w)
    qt = QuantizedTensor((256, 192), q, s, "perChannel", 0, None)
    y0 = oracle.qmatmul(x, qt, 0)
    y1 = oracle.qmatmul(x, qt, 1)
    wd = oracle.dequantize(qt).astype(np.float64)
    ref = x.astype(np.float64) @ wd
    assert np.linalg.norm(y1 - ref) / np.linalg.norm(ref) < 1e-6
    assert np.linalg.norm(y0 - ref) / np.linalg.norm(ref) < 1e-5
    # quantization error vs fp32 within the reference's INT8 bound
    yf = x.astype(np.float64) @ w.astype(np.float64)
    assert np.linalg.norm(y1 - yf) / np.linalg.norm(yf) < GOLD["matmul_tolerance"]["int8_vs_fp32"]
    p, s4, z = oracle.quantize_int4_group(w, 32)
    qt4 = QuantizedTensor((256, 192), p, s4, "int4", 32, z)
    y4 = oracle.qmatmul(x, qt4, 1)
    assert np.linalg.norm(y4 - yf) / np.linalg.norm(yf) < GOLD["matmul_tolerance"]["int4_vs_fp32"]
