"""tb_paged_attention_dev_noalloc: the allocation-free variant of the paged
decode attention, for callers that cannot allocate device memory (for example a
host that has handed all of HBM to its own pool, or a latency-critical path
where cudaMalloc/cudaFree would synchronise the device).  Its split partials
are combined inside each CTA cluster, so it needs no scratch memory at all.

Checked through the C ABI against tb_paged_attention_dev (the entry point whose
scratch the library allocates) on two calls in a row, within the relative-L2
tolerance the other kernel tests use.  This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

from tinybrain_b200 import _lib

pytestmark = pytest.mark.gpu
RTOL_L2 = 1e-3


def _rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _case(torch, seed, lens, H=32, Hkv=4, d=64, num_layers=2, layer=1):
    g = torch.Generator(device="cpu").manual_seed(seed)
    batch = len(lens)
    pages = [(n + 15) // 16 for n in lens]
    stride = max(pages) + 2
    total = sum(pages) + 3
    perm = torch.randperm(total, generator=g).tolist()
    ptab = torch.full((batch, stride), -1, dtype=torch.int32)
    k = 0
    for s, n in enumerate(pages):
        for p in range(n):
            ptab[s, p] = perm[k]
            k += 1
    if pages[0] > 2:
        ptab[0, 1] = -1  # an evicted page reads as zeros
    pool = torch.randn(total, num_layers, 2, Hkv, 16, d, generator=g).float()
    q = torch.randn(batch, H * d, generator=g).float()
    dev = torch.device("cuda", 0)
    return dict(q=q.to(dev), pool=pool.to(dev), ptab=ptab.to(dev),
                lens=torch.tensor(lens, dtype=torch.int32).to(dev), batch=batch, stride=stride,
                max_len=max(lens), H=H, Hkv=Hkv, d=d, num_layers=num_layers, layer=layer)


def _run(fn_name, first_arg, c, out):
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    st = _lib.load().__getattr__(fn_name)(first_arg, p(c["q"]), c["batch"], p(c["pool"]), p(c["ptab"]),
                                          c["stride"], p(c["lens"]), c["max_len"], c["layer"], c["num_layers"],
                                          c["H"], c["Hkv"], c["d"], p(out))
    _lib.check(st)


def test_noalloc_attention_matches_allocating_entry_point(ctx):
    torch = pytest.importorskip("torch")
    stream = _lib.load().tb_context_stream(ctx.handle)
    for seed, lens in ((1, [300, 37]), (2, [2048, 1, 16, 17])):
        c = _case(torch, seed, lens)
        torch.cuda.synchronize()
        ref = torch.zeros(c["batch"], c["H"] * c["d"], device="cuda")
        got = torch.full_like(ref, float("nan"))
        _run("tb_paged_attention_dev", ctx.handle, c, ref)
        _run("tb_paged_attention_dev_noalloc", C.c_void_p(stream), c, got)
        ctx.synchronize()
        ctx.check_device()
        err = _rel_l2(got.cpu().numpy(), ref.cpu().numpy())
        assert err <= RTOL_L2, (seed, err)


def test_noalloc_large_batch(ctx):
    # 1200 sequences x 4 KV heads: far beyond any fixed scratch; no limit applies
    torch = pytest.importorskip("torch")
    stream = _lib.load().tb_context_stream(ctx.handle)
    c = _case(torch, 3, [40] * 1200)
    torch.cuda.synchronize()
    ref = torch.zeros(c["batch"], c["H"] * c["d"], device="cuda")
    got = torch.full_like(ref, float("nan"))
    _run("tb_paged_attention_dev", ctx.handle, c, ref)
    _run("tb_paged_attention_dev_noalloc", C.c_void_p(stream), c, got)
    ctx.synchronize()
    ctx.check_device()
    assert _rel_l2(got.cpu().numpy(), ref.cpu().numpy()) <= RTOL_L2
