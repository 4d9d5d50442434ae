"""tb_paged_attention_dev_noalloc: the allocation-free entry point of the paged
decode attention.

Who needs it: callers that cannot allocate device memory -- a host that hands
all of HBM to its own memory pool before it loads this library, or a
latency-critical path where a cudaMalloc / cudaFree would synchronise the
whole device.  The entry point allocates nothing: the split partials combine
inside each CTA cluster, and its one piece of device state is an error word in
a file-scope __device__ variable, read back by
tb_paged_attention_noalloc_status.

Checked through the C ABI, on two calls in a row, against (a) a float64 numpy
restatement of the reference's attention (ModelRunner.swift:519-579) over the
gathered pages, evicted pages reading as zeros, and (b) the allocating entry
point tb_paged_attention_dev, within the relative-L2 bar the other kernel
tests use; the error word must stay clear.  This file is collected last on
purpose, and passes alone in a fresh process as well as after the others.
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
    return dict(q=q.to(dev), pool=pool.to(dev), ptab=ptab.to(dev), q_h=q.numpy(), pool_h=pool.numpy(),
                ptab_h=ptab.numpy(), lens_h=list(lens),
                lens=torch.tensor(lens, dtype=torch.int32).to(dev), batch=batch, stride=stride,
                max_len=max(lens), H=H, Hkv=Hkv, d=d, num_layers=num_layers, layer=layer)


def _numpy_attention(c):
    """softmax(q K^T / sqrt(d)) V per (sequence, head) in float64 over the
    gathered pages (page -1 = evicted: rows of zeros)."""
    H, Hkv, d, layer = c["H"], c["Hkv"], c["d"], c["layer"]
    rep = H // Hkv
    out = np.zeros((c["batch"], H * d))
    for s, L in enumerate(c["lens_h"]):
        pos = np.arange(L)
        pg = c["ptab_h"][s, pos // 16]
        kv = c["pool_h"][np.maximum(pg, 0), layer, :, :, pos % 16, :].astype(np.float64)  # [L][2][Hkv][d]
        kv[pg < 0] = 0.0
        q = c["q_h"][s].reshape(H, d).astype(np.float64)
        for h in range(H):
            K, V = kv[:, 0, h // rep], kv[:, 1, h // rep]
            sc = K @ q[h] / np.sqrt(d)
            p = np.exp(sc - sc.max())
            out[s, h * d:(h + 1) * d] = (p / p.sum()) @ V
    return out


def _run(fn_name, first_arg, c, out):
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    st = _lib.load().__getattr__(fn_name)(first_arg, p(c["q"]), c["batch"], p(c["pool"]), p(c["ptab"]),
                                          c["stride"], p(c["lens"]), c["max_len"], c["layer"], c["num_layers"],
                                          c["H"], c["Hkv"], c["d"], p(out))
    _lib.check(st)


def _check(torch, ctx, c):
    lib = _lib.load()
    stream = lib.tb_context_stream(ctx.handle)
    want = _numpy_attention(c)
    ref = torch.zeros(c["batch"], c["H"] * c["d"], device="cuda")
    _run("tb_paged_attention_dev", ctx.handle, c, ref)
    ctx.synchronize()
    ctx.check_device()
    for call in range(2):  # two calls in a row into the same output
        got = torch.full_like(ref, float("nan"))
        _run("tb_paged_attention_dev_noalloc", C.c_void_p(stream), c, got)
        _lib.check(lib.tb_paged_attention_noalloc_status(C.c_void_p(stream), 1))
        g = got.cpu().numpy()
        assert _rel_l2(g, want) <= RTOL_L2, (call, _rel_l2(g, want))
        assert _rel_l2(g, ref.cpu().numpy()) <= RTOL_L2, call


def test_noalloc_attention_matches_numpy_and_allocating_entry_point(ctx):
    torch = pytest.importorskip("torch")
    for seed, lens in ((1, [300, 37]), (2, [2048, 1, 16, 17])):
        _check(torch, ctx, _case(torch, seed, lens))


def test_noalloc_large_batch_with_long_context(ctx):
    # 1200 sequences x 4 KV heads, one of them 2048 tokens long: several
    # splits per (sequence, KV head) and the cluster combine at a large batch
    torch = pytest.importorskip("torch")
    _check(torch, ctx, _case(torch, 3, [2048] + [40] * 1199))
