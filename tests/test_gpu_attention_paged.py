"""Paged decode attention on device buffers (tb_paged_attention_dev) over a
batch of sequences with ragged lengths, scattered pages and an evicted page:
the GQA-8 / d = 64 kernel (the TinyLlama shape) against a float64 numpy
restatement of ModelRunner.swift:519-579 and against the generic kernel
(TB_ATTN_GENERIC=1), and the generic kernel on other head geometries."""
import ctypes as C

import numpy as np
import pytest

from tests.helpers import rel_l2
from tinybrain_b200 import _lib

pytestmark = pytest.mark.gpu


def _case(torch, seed, lens, H, Hkv, d, num_layers=2, layer=1):
    g = np.random.default_rng(seed)
    batch = len(lens)
    pages = [(n + 15) // 16 for n in lens]
    stride = max(pages) + 1
    total = sum(pages) + 2
    perm = g.permutation(total)
    ptab = np.full((batch, stride), -1, dtype=np.int32)
    k = 0
    for s, n in enumerate(pages):
        ptab[s, :n] = perm[k:k + n]
        k += n
    if pages[0] > 2:
        ptab[0, 1] = -1  # evicted: rows read as zeros
    pool = g.standard_normal((total, num_layers, 2, Hkv, 16, d)).astype(np.float32)
    q = g.standard_normal((batch, H * d)).astype(np.float32)
    return dict(q=q, pool=pool, ptab=ptab, lens=np.array(lens, dtype=np.int32), stride=stride, H=H, Hkv=Hkv, d=d,
                num_layers=num_layers, layer=layer)


def _numpy(c):
    H, Hkv, d, layer = c["H"], c["Hkv"], c["d"], c["layer"]
    rep = H // Hkv
    out = np.zeros((len(c["lens"]), H * d))
    for s, L in enumerate(c["lens"]):
        pos = np.arange(L)
        pg = c["ptab"][s, pos // 16]
        kv = c["pool"][np.maximum(pg, 0), layer, :, :, pos % 16, :].astype(np.float64)
        kv[pg < 0] = 0.0
        q = c["q"][s].reshape(H, d).astype(np.float64)
        for h in range(H):
            sc = kv[:, 0, h // rep] @ q[h] / np.sqrt(d)
            p = np.exp(sc - sc.max())
            out[s, h * d:(h + 1) * d] = (p / p.sum()) @ kv[:, 1, h // rep]
    return out


def _device(torch, ctx, c):
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(c[k]).to(dev) for k in ("q", "pool", "ptab", "lens")}
    out = torch.full((len(c["lens"]), c["H"] * c["d"]), float("nan"), device=dev)
    P = lambda x: C.c_void_p(x.data_ptr())  # noqa: E731
    _lib.check(_lib.load().tb_paged_attention_dev(ctx.handle, P(t["q"]), len(c["lens"]), P(t["pool"]), P(t["ptab"]),
                                                  c["stride"], P(t["lens"]), int(c["lens"].max()), c["layer"],
                                                  c["num_layers"], c["H"], c["Hkv"], c["d"], P(out)))
    ctx.synchronize()
    ctx.check_device()
    return out.cpu().numpy()


@pytest.mark.parametrize("lens", [[4224, 1, 15, 16, 17, 300], [40] * 70 + [2049], [7]])
def test_gqa8_kernel_matches_numpy_and_generic(ctx, monkeypatch, lens):
    torch = pytest.importorskip("torch")
    c = _case(torch, len(lens), lens, 32, 4, 64)
    want = _numpy(c)
    got = _device(torch, ctx, c)
    assert rel_l2(got, want) <= 1e-5
    monkeypatch.setenv("TB_ATTN_GENERIC", "1")
    gen = _device(torch, ctx, c)
    assert rel_l2(gen, want) <= 1e-5
    assert rel_l2(got, gen) <= 1e-5


@pytest.mark.parametrize("H,Hkv,d", [(32, 32, 128), (8, 2, 64), (16, 4, 32)])
def test_generic_kernel_paged_batch(ctx, H, Hkv, d):
    torch = pytest.importorskip("torch")
    c = _case(torch, H + d, [1000, 3, 64, 129], H, Hkv, d)
    assert rel_l2(_device(torch, ctx, c), _numpy(c)) <= 1e-5


@pytest.mark.parametrize("mode", ["perChannel", "int4"])
def test_runner_persistent_attention_matches_cluster_kernel_and_oracle(ctx, monkeypatch, mode):
    # GQA-8 / d 64 runners use the persistent chunked attention (chunk
    # partials merged by the last chunk of each (row, KV head)); contexts of
    # 1 to 40 pages, some rows a single chunk; the same batch through the
    # cluster kernel (TB_ATTN_CLUSTER=1) and the oracle must agree
    import oracle
    from tests.helpers import assert_same_tokens, small_llama
    from tinybrain_b200.runtime import ModelConfig, ModelRunner
    # 32 rows x 2 KV heads = 64 (row, KV head) pairs: the persistent kernel's range
    cfg = ModelConfig(num_layers=2, hidden_dim=1024, num_heads=16, vocab_size=512, max_seq_len=700, num_kv_heads=2,
                      intermediate_dim=512)
    w = small_llama(cfg, seed=21, mode=mode)
    rng = np.random.default_rng(3)
    lens = [640, 1, 17, 300, 33, 129] + [int(n) for n in rng.integers(1, 600, 26)]
    prompts = [rng.integers(0, 512, n).tolist() for n in lens]
    flat = ModelRunner(w, ctx, max_batch=len(prompts), max_positions=760).generate_batch(prompts, 10)
    monkeypatch.setenv("TB_ATTN_CLUSTER", "1")
    clus = ModelRunner(w, ctx, max_batch=len(prompts), max_positions=760).generate_batch(prompts, 10)
    for p, a, b in zip(prompts, flat, clus):
        want, gaps = oracle.OracleModel(w, mode=1).generate_greedy(p, 10)
        assert_same_tokens(a, want, gaps, w, p)
        assert_same_tokens(b, want, gaps, w, p)
