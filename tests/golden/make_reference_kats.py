"""Writes tests/golden/reference_kats.json.

The reference (vivekptnk/tinybrain) is a Swift package that cannot be built or
run on Linux, so its tests cannot be executed here.  This script records the
known-answer cases its own test files state (inputs and expected answers
transcribed with file:line citations, paths relative to the reference root),
and adds the exact expected bytes for the quantizer cases, derived with an
independent numpy float32 restatement of the quantizer formulas
(QuantizedTensor.swift:379-424 and :502-560).  Run: python make_reference_kats.py
"""
import json
import os

import numpy as np


def round_half_away(x):
    x = np.asarray(x, dtype=np.float32)
    return np.where(x >= 0, np.floor(x + np.float32(0.5)), -np.floor(-x + np.float32(0.5))).astype(np.float32)


def np_quantize_int8(w):
    w = np.asarray(w, dtype=np.float32)
    absmax = np.max(np.abs(w), axis=0).astype(np.float32)
    scales = np.where(absmax < np.float32(1.4e-45), np.float32(1.0), absmax / np.float32(127.0)).astype(np.float32)
    # exact float32 division then round-half-away; the x+0.5 floor trick is exact
    # for the magnitudes in these cases (< 2^22)
    q = np.clip(round_half_away((w / scales).astype(np.float32)), -127, 127).astype(np.int8)
    return q, scales


def np_quantize_int4(x, gs):
    x = np.asarray(x, dtype=np.float32).ravel()
    n = x.size
    ng = (n + gs - 1) // gs
    scales = np.zeros(ng, dtype=np.float32)
    packed = np.zeros((n + 1) // 2, dtype=np.uint8)
    for g in range(ng):
        grp = x[g * gs:(g + 1) * gs]
        a = max(abs(grp.min()), abs(grp.max()))
        scales[g] = np.float32(1.0) if a < np.float32(1.4e-45) else np.float32(a) / np.float32(7.0)
    for i in range(n):
        q = int(np.clip(round_half_away(np.float32(x[i]) / scales[i // gs]), -7, 7))
        if i % 2 == 0:
            packed[i // 2] = (q & 0xF) << 4
        else:
            packed[i // 2] |= q & 0xF
    return packed, scales


def main():
    kats = {"source": "vivekptnk/tinybrain test files (transcribed); expected bytes derived with numpy float32"}
    # INT4 pack/unpack pairs (Tests/TinyBrainRuntimeTests/INT4QuantizationTests.swift:37-48) and clamp (:50-58).
    kats["int4_pack_pairs"] = {
        "cite": "Tests/TinyBrainRuntimeTests/INT4QuantizationTests.swift:37-58",
        "pairs": [[0, 0], [7, -7], [-7, 7], [3, -3], [1, 2], [-1, -2], [5, -3]],
        "clamp": {"in": [10, -10], "out": [7, -7]},
    }
    # Odd element count 3x3 with group 128 -> 5 bytes (INT4QuantizationTests.swift:281-300).
    odd = np.arange(1, 10, dtype=np.float32).reshape(3, 3)
    p, s = np_quantize_int4(odd, 128)
    kats["int4_odd_count"] = {
        "cite": "Tests/TinyBrainRuntimeTests/INT4QuantizationTests.swift:281-300",
        "input": odd.ravel().tolist(), "group_size": 128, "packed_len": 5,
        "packed": p.tolist(), "scales": [float(v) for v in s], "max_rel_error": 0.15,
    }
    # All-zero INT4 64x64 / group 128 (INT4QuantizationTests.swift:258-267) and INT8 10x10 (QuantizationTests.swift:155-169).
    kats["int4_all_zero"] = {"cite": "Tests/TinyBrainRuntimeTests/INT4QuantizationTests.swift:258-267",
                             "shape": [64, 64], "group_size": 128, "scale": 1.0}
    kats["int8_all_zero"] = {"cite": "Tests/TinyBrainRuntimeTests/QuantizationTests.swift:155-169",
                             "shape": [10, 10], "scale": 1.0}
    # Negative constant (INT4QuantizationTests.swift:269-279).
    kats["int4_negative_constant"] = {"cite": "Tests/TinyBrainRuntimeTests/INT4QuantizationTests.swift:269-279",
                                      "shape": [32, 32], "value": -3.5, "group_size": 128, "tolerance": 1.0}
    # Per-column scales (QuantizationTests.swift:78-97).
    w = np.array([[1, 2, 3, 4], [100, 200, 300, 400], [0.01, 0.02, 0.03, 0.04]], dtype=np.float32)
    q, s = np_quantize_int8(w)
    kats["int8_per_channel_scales"] = {
        "cite": "Tests/TinyBrainRuntimeTests/QuantizationTests.swift:78-97",
        "input": w.ravel().tolist(), "shape": [3, 4], "num_scales": 4,
        "q": q.ravel().tolist(), "scales": [float(v) for v in s],
    }
    # Greedy argmax (Tests/TinyBrainRuntimeTests/SamplerTests.swift:25-46).
    kats["greedy"] = {
        "cite": "Tests/TinyBrainRuntimeTests/SamplerTests.swift:25-46",
        "cases": [[[0.1, 0.5, 0.2, 0.8, 0.3], 3], [[-2.0, -1.0, -3.0, -0.5], 3],
                  [[0.5, 0.8, 0.8, 0.3], 1]],
        "note": "the tie case accepts 1 or 2 in the reference test; Sampler.swift:126-138 (strict >) returns 1",
    }
    # SiLU (ConverterFixTests.swift:12-26) and RMSNorm (:37-89).
    kats["silu"] = {"cite": "Tests/TinyBrainRuntimeTests/ConverterFixTests.swift:12-26",
                    "x": [-2, -1, 0, 1, 2], "y": [None, -0.2689, 0.0, 0.7311, 1.7616], "atol": 1e-3}
    kats["rmsnorm"] = {"cite": "Tests/TinyBrainRuntimeTests/ConverterFixTests.swift:37-89",
                       "cases": [{"x": [1, 2, 3, 4], "w": [1, 1, 1, 1],
                                  "y": [float(v) for v in np.array([1, 2, 3, 4], np.float32) / np.sqrt(np.float32(7.5))]},
                                 {"x": [1, 2, 3, 4], "w": [2, 2, 2, 2],
                                  "y": [float(v) for v in 2 * np.array([1, 2, 3, 4], np.float32) / np.sqrt(np.float32(7.5))]},
                                 {"x": [10, 10, 10, 10], "w": [1, 1, 1, 1], "y": [1.0, 1.0, 1.0, 1.0]}],
                       "atol": 1e-3}
    # Attention tolerance contract (Tests/TinyBrainMetalTests/FlashAttentionTests.swift:21-50, 223-248).
    kats["attention_tolerance"] = {"cite": "Tests/TinyBrainMetalTests/FlashAttentionTests.swift:21-50,223-248",
                                   "atol": 1e-5, "rtol": 5e-4,
                                   "decode_case": {"num_heads": 4, "num_kv_heads": 4, "head_dim": 16, "kv_len": 32},
                                   "gqa_case": {"num_heads": 8, "num_kv_heads": 2}}
    # Quantized matmul tolerances (QuantizationTests.swift:117-151, INT4QuantizationTests.swift:189-254).
    kats["matmul_tolerance"] = {"cite": "QuantizationTests.swift:117-151; INT4QuantizationTests.swift:189-254",
                                "int8_vs_fp32": 0.01, "int4_vs_fp32": 0.15, "gpu_int4_vs_cpu": 0.01}
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(out, "w") as f:
        json.dump(kats, f, indent=1)
    print(out)


if __name__ == "__main__":
    main()
