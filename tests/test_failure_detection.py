"""Failure detection without a GPU fault.

Every device-side wait in the library is bounded (2 s of %globaltimer): when it
runs out the kernel records kDevWaitTimeout in the context's error word and
finishes, and tb_context_check_device reports TB_ERR_DEVICE_TIMEOUT.  Here a
probe kernel makes the two kinds of wait the kernels use run out on purpose --
an mbarrier wait that no thread arrives on, and the tensor-parallel pull's
spin on a tagged word that nothing writes -- and the context must report the
timeout and then keep working (a GEMV afterwards matches the oracle).
"""
import numpy as np
import pytest

import oracle
from tests.helpers import oracle_quantize, rel_l2
from tinybrain_b200 import _lib
from tinybrain_b200.runtime import QuantizedWeight, SeededGenerator

pytestmark = pytest.mark.gpu
TB_ERR_DEVICE_TIMEOUT = 8


@pytest.mark.parametrize("which", [0, 1], ids=["mbarrier", "tagged-word"])
def test_bounded_wait_runs_out_and_context_stays_usable(ctx, which):
    lib = _lib.load()
    ctx.check_device()
    _lib.check(lib.tb_debug_expire_wait(ctx.handle, which))
    assert lib.tb_context_check_device(ctx.handle) == TB_ERR_DEVICE_TIMEOUT
    assert lib.tb_context_check_device(ctx.handle) == 0  # the word was cleared
    w = SeededGenerator(1).normal((256, 384), 0.0, 0.02)
    x = SeededGenerator(2).normal((1, 256), 0.0, 1.0)
    q = oracle_quantize(w, "perChannel")
    got = QuantizedWeight(q, ctx).matmul(x)
    assert rel_l2(got, oracle.qmatmul(x, q, mode=1)) <= 1e-5
