"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute calls that need a GPU), plus host-only entry points."""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

from tinybrain_b200 import _lib
from tinybrain_b200.runtime import SeededGenerator, device_count

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"typedef[^;]*;", "", text, flags=re.S)
        for m in re.finditer(r"\b(tb_\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert "tb_matmul_quantized" in names and "tb_runner_generate" in names
    assert len(names) >= 40


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.tb_abi_version() == 1
    assert lib.tb_status_string(5) == b"KV page pool exhausted"


def test_rng_is_seeded_and_chunk_invariant():
    a = SeededGenerator(0).normal((300001,), 0.0, 1.0)
    b = SeededGenerator(0).normal((300001,), 0.0, 1.0)
    assert np.array_equal(a, b)
    # drawing in two pieces continues the same LCG stream (pairs of draws)
    g = SeededGenerator(0)
    c1 = g.normal((1000,), 0.0, 1.0)
    c2 = g.normal((299001,), 0.0, 1.0)
    assert np.array_equal(np.concatenate([c1, c2]), a)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    # seed 0 maps to 0xdeadbeef (ModelWeights.swift:21-23)
    assert np.array_equal(SeededGenerator(0xdeadbeef).normal((10,)), a[:10])


def test_rng_first_draws_follow_the_documented_formula():
    # LCG s' = a*s + 1, Float.random = (low 24 bits of the 32-bit truncation) * 2^-24,
    # Box-Muller with u1 clamped to the smallest subnormal.
    s = 42
    a = 6364136223846793005
    s = (a * s + 1) % 2**64
    u1 = np.float32((s & 0xFFFFFFFF) & 0xFFFFFF) * np.float32(2.0**-24)
    s = (a * s + 1) % 2**64
    u2 = np.float32((s & 0xFFFFFFFF) & 0xFFFFFF) * np.float32(2.0**-24)
    r = np.sqrt(np.float32(-2.0) * np.log(np.float32(u1)))
    th = np.float32(2.0 * np.float32(np.pi)) * u2
    x = SeededGenerator(42).normal((2,), 0.0, 1.0)
    assert abs(x[0] - r * np.cos(th)) < 1e-6 and abs(x[1] - r * np.sin(th)) < 1e-6


@pytest.mark.skipif(device_count() > 0, reason="checks the no-device error path")
def test_context_without_device_reports_error():
    h = C.c_void_p()
    st = _lib.load().tb_context_create(0, C.byref(h))
    assert st == 7  # TB_ERR_NO_DEVICE
    assert _lib.last_error()


def test_swift_binding_calls_only_exported_symbols():
    # The Swift target (Sources/TinyBrainCUDA) binds the header through the
    # module map; every tb_* function it calls must be declared and exported.
    src = os.path.join(ROOT, "Sources", "TinyBrainCUDA")
    used = set()
    for f in glob.glob(os.path.join(src, "*.swift")):
        used |= set(re.findall(r"\b(tb_[a-z0-9_]+)\(", open(f).read()))
    types = {"tb_model_config", "tb_sampler_config", "tb_qtensor_desc", "tb_status", "tb_projection",
             "tb_token_callback"}
    calls = used - types
    assert {"tb_matmul_quantized", "tb_runner_generate", "tb_runner_set_sampler", "tb_qweight_upload"} <= calls
    declared = set(declared_functions())
    assert calls <= declared, calls - declared
    lib = C.CDLL(_lib.LIB_PATH)
    assert all(hasattr(lib, n) for n in calls)
    mm = open(os.path.join(ROOT, "Sources", "CTinyBrainCUDA", "module.modulemap")).read()
    assert 'link "tinybrain_cuda"' in mm and "tinybrain_cuda.h" in mm
