"""Kernel-level parity: the CUDA path (through the C ABI) against the CPU oracle.

Tolerances: quantizer bytes bit-exact; fp32 GEMV and attention outputs within
relative L2 <= 1e-3 of the oracle; attention also within
the reference test's element tolerance (atol 1e-5 or rel 5e-4,
FlashAttentionTests.swift:21-50).
"""
import numpy as np
import pytest

import oracle
from tests.helpers import rel_l2
from tinybrain_b200.runtime import QuantizedTensor, QuantizedWeight, SeededGenerator, attention_decode, quantize

pytestmark = pytest.mark.gpu
RTOL_L2 = 1e-3


def cfg1_inputs():
    # W [in 2048, out 4096] ~ N(0, 0.02) seed 0; x [1, 2048] ~ N(0, 1) seed 1
    w = SeededGenerator(0).normal((2048, 4096), 0.0, 0.02)
    x = SeededGenerator(1).normal((1, 2048), 0.0, 1.0)
    return w, x


def test_int8_quantizer_bit_exact_cfg1(ctx):
    w, _ = cfg1_inputs()
    qg = quantize(w, "perChannel", ctx=ctx)
    q, s = oracle.quantize_int8_per_channel(w)
    assert np.array_equal(qg.data, q)
    assert np.array_equal(qg.scales.view(np.uint32), s.view(np.uint32))


@pytest.mark.parametrize("gs", [32, 128])
def test_int4_quantizer_bit_exact(ctx, gs):
    w, _ = cfg1_inputs()
    qg = quantize(w, "int4", gs, ctx=ctx)
    p, s, z = oracle.quantize_int4_group(w, gs)
    assert np.array_equal(qg.data, p)
    assert np.array_equal(qg.scales.view(np.uint32), s.view(np.uint32))
    assert np.all(qg.zero_points == 0)


def test_quantizer_edge_cases(ctx):
    # all-zero columns/groups -> scale 1; odd element count; values exactly at .5 boundaries
    w = np.zeros((3, 3), np.float32)
    w.flat[:] = np.arange(1, 10)
    qg = quantize(w, "int4", 128, ctx=ctx)
    assert qg.data.tolist() == [0x12, 0x23, 0x45, 0x56, 0x70]
    z = np.zeros((10, 10), np.float32)
    q8 = quantize(z, ctx=ctx)
    assert np.all(q8.scales == 1.0) and np.all(q8.data == 0)
    h = (np.arange(-20, 20, dtype=np.float32) + 0.5).reshape(8, 5) / 127.0
    qa, sa = oracle.quantize_int8_per_channel(h)
    qb = quantize(h, ctx=ctx)
    assert np.array_equal(qa, qb.data) and np.array_equal(sa, qb.scales)


@pytest.mark.parametrize("mode", ["perChannel", "int4"])
def test_gemv_cfg1(ctx, mode):
    w, x = cfg1_inputs()
    qt = quantize(w, mode, 32, ctx=ctx)
    y = QuantizedWeight(qt, ctx).matmul(x)
    ref = oracle.qmatmul(x, qt, mode=1)
    assert rel_l2(y, ref) <= RTOL_L2
    assert rel_l2(y, ref) < 1e-5  # fp32 accumulation vs fp64: far inside the bar


@pytest.mark.parametrize("K,N,M", [(100, 70, 1), (48, 33, 3), (5632, 2048, 1), (2048, 5632, 2),
                                   (11008, 4096, 1), (4096, 32000, 1), (2048, 256, 8), (1024, 512, 5),
                                   (2048, 2560, 16), (5632, 2048, 33), (2048, 11264, 64), (200, 130, 17)])
def test_gemv_int8_shapes(ctx, K, N, M):
    g = SeededGenerator(K * 7 + N)
    w = g.normal((K, N), 0.0, 0.02)
    x = g.normal((M, K), 0.0, 1.0)
    q, s = oracle.quantize_int8_per_channel(w)
    qt = QuantizedTensor((K, N), q, s, "perChannel", 0, None)
    y = QuantizedWeight(qt, ctx).matmul(x)
    ref = oracle.qmatmul(x, qt, mode=1)
    assert y.shape == ref.shape
    assert rel_l2(y, ref) <= RTOL_L2


@pytest.mark.parametrize("K,N,M,gs", [(2048, 4096, 1, 32), (11008, 4096, 1, 32), (1000, 64, 1, 32),
                                      (4096, 256, 2, 128), (5632, 2048, 1, 32), (1024, 512, 7, 32),
                                      (100, 96, 3, 32), (4096, 22016, 1, 32), (2048, 2560, 16, 32),
                                      (1376, 4096, 33, 32), (2048, 1024, 64, 64), (4096, 32000, 4, 32)])
def test_gemv_int4_shapes(ctx, K, N, M, gs):
    g = SeededGenerator(K * 3 + N)
    w = g.normal((K, N), 0.0, 0.02)
    x = g.normal((M, K), 0.0, 1.0)
    p, s, z = oracle.quantize_int4_group(w, gs)
    qt = QuantizedTensor((K, N), p, s, "int4", gs, z)
    y = QuantizedWeight(qt, ctx).matmul(x)
    ref = oracle.qmatmul(x, qt, mode=1)
    assert rel_l2(y, ref) <= RTOL_L2


def test_gemv_rejects_unsupported_int4_layout(ctx):
    from tinybrain_b200._lib import TinyBrainError
    w = SeededGenerator(5).normal((64, 48), 0.0, 0.02)  # N not a multiple of the group
    p, s, z = oracle.quantize_int4_group(w, 32)
    with pytest.raises(TinyBrainError):
        QuantizedWeight(QuantizedTensor((64, 48), p, s, "int4", 32, z), ctx)


@pytest.mark.parametrize("H,Hkv,d,L", [(32, 4, 64, 1), (32, 4, 64, 15), (32, 4, 64, 16), (32, 4, 64, 17),
                                       (32, 4, 64, 384), (32, 4, 64, 2048), (32, 32, 128, 700),
                                       (4, 4, 16, 32), (8, 2, 16, 33), (4, 4, 32, 4224), (32, 4, 64, 4224)])
def test_decode_attention(ctx, H, Hkv, d, L):
    g = SeededGenerator(H * 1000 + L)
    q = g.normal((H * d,))
    K = g.normal((L, Hkv * d))
    V = g.normal((L, Hkv * d))
    out = attention_decode(q, K, V, H, Hkv, d, ctx)
    ref = oracle.attention(q, K, V, H, Hkv, d)
    assert rel_l2(out, ref) <= RTOL_L2
    diff = np.abs(out - ref)
    rel = diff / np.maximum(np.abs(ref), 1e-5)
    assert np.all((diff < 1e-5) | (rel < 5e-4))
