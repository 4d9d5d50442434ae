"""Tensor parallelism (the 7B-shaped configuration): weight sharding and the
per-rank decomposition of a decoder layer.

CPU: shards taken from the quantized bytes dequantize to exact slices of the
whole tensor; a world-size-2 gloo job runs one LLaMA layer as two ranks
(column-parallel q/k/v and gate/up, row-parallel o_proj/down_proj, all-reduce
of the partial sums) and matches the unsharded layer.
GPU (two devices): a small LLaMA model decoded by two ranks over NCCL gives
the oracle's greedy tokens.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import oracle
from tests.helpers import oracle_quantize, small_llama
from tinybrain_b200.runtime import ModelConfig, shard_quantized


@pytest.mark.parametrize("mode", ["perChannel", "int4"])
@pytest.mark.parametrize("axis", [0, 1])
@pytest.mark.parametrize("world", [2, 4])
def test_shards_are_exact_slices(mode, axis, world):
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((128, 256)) * 0.02).astype(np.float32)
    q = oracle_quantize(w, mode)
    full = oracle.dequantize(q)
    parts = [oracle.dequantize(shard_quantized(q, axis, r, world)) for r in range(world)]
    np.testing.assert_array_equal(np.concatenate(parts, axis=axis), full)
    if axis == 1 and mode == "perChannel":
        s = shard_quantized(q, 1, 1, world)
        np.testing.assert_array_equal(s.scales, q.scales[256 // world:2 * 256 // world])


def test_int4_shard_must_cut_whole_groups():
    w = np.zeros((64, 96), dtype=np.float32)
    q = oracle_quantize(w, "int4")
    with pytest.raises(ValueError):
        shard_quantized(q, 1, 0, 2)  # 48 columns: not whole groups of 32
    shard_quantized(q, 0, 1, 2)      # row shards keep whole groups


# ----------------------------------------------------------------- gloo --
H, NH, NKV, D, I, CTX = 128, 8, 4, 16, 128, 5


def _rms(x, w, eps=1e-5):
    return (x / np.sqrt(np.mean(x * x) + eps) * w).astype(np.float32)


def _layer_weights():
    rng = np.random.default_rng(11)
    shapes = {"q": (H, NH * D), "k": (H, NKV * D), "v": (H, NKV * D), "o": (NH * D, H),
              "gate": (H, I), "up": (H, I), "down": (I, H)}
    qw = {k: oracle_quantize((rng.standard_normal(s) * 0.05).astype(np.float32), "int4")
          for k, s in shapes.items()}
    kc = rng.standard_normal((NKV, CTX, D)).astype(np.float32)
    vc = rng.standard_normal((NKV, CTX, D)).astype(np.float32)
    h = rng.standard_normal(H).astype(np.float32)
    return qw, kc, vc, h


def _layer(h, w, kc, vc, nh, nkv, allreduce):
    """One decoder layer (ModelRunner.swift:320-495 order) on this rank's
    heads / intermediate rows; `allreduce` sums the row-parallel partials."""
    x = _rms(h, np.ones(H, np.float32))
    q = (x @ w["q"]).reshape(nh, D)
    k = (x @ w["k"]).reshape(nkv, D)
    v = (x @ w["v"]).reshape(nkv, D)
    G = nh // nkv
    ctx = np.empty((nh, D), np.float32)
    for hh in range(nh):
        K = np.concatenate([kc[hh // G], k[hh // G][None]])
        V = np.concatenate([vc[hh // G], v[hh // G][None]])
        s = K @ q[hh] / np.sqrt(D)
        p = np.exp(s - s.max())
        ctx[hh] = (p / p.sum()) @ V
    h1 = h + allreduce(ctx.ravel() @ w["o"])
    x2 = _rms(h1, np.ones(H, np.float32))
    g, u = x2 @ w["gate"], x2 @ w["up"]
    a = g / (1 + np.exp(-g)) * u
    return h1 + allreduce(a @ w["down"])


def _gloo_rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        qw, kc, vc, h = _layer_weights()
        axes = {"q": 1, "k": 1, "v": 1, "gate": 1, "up": 1, "o": 0, "down": 0}
        w = {k: oracle.dequantize(shard_quantized(q, axes[k], rank, world)) for k, q in qw.items()}
        nkv = NKV // world

        def allreduce(y):
            t = torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32))
            dist.all_reduce(t)
            return t.numpy()

        kvs = slice(rank * nkv, (rank + 1) * nkv)
        res = _layer(h, w, kc[kvs], vc[kvs], NH // world, nkv, allreduce)
        out.put((rank, res))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp2_layer_decomposition_gloo():
    qw, kc, vc, h = _layer_weights()
    ref = _layer(h, {k: oracle.dequantize(q) for k, q in qw.items()}, kc, vc, NH, NKV, lambda y: y)
    ctxm = mp.get_context("spawn")
    out = ctxm.Queue()
    port = _free_port()
    procs = [ctxm.Process(target=_gloo_rank, args=(r, 2, port, out), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank ends with the same residual stream, equal to the unsharded layer
    np.testing.assert_array_equal(res[0], res[1])
    np.testing.assert_allclose(res[0], ref, rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------------ GPU --
TP_CFG = dict(num_layers=2, hidden_dim=256, num_heads=4, num_kv_heads=2, vocab_size=512, intermediate_dim=512,
              max_seq_len=96)


def _gpu_rank(rank, world, uid, mode, prompt, n_new, out, peer, port):
    try:
        # torch first: its NCCL must be the process's libnccl.so.2 (the library
        # binds whichever copy is already loaded)
        import torch.distributed  # noqa: F401
        from tinybrain_b200.runtime import Context, ModelRunner
        cfg = ModelConfig(**TP_CFG)
        w = small_llama(cfg, seed=3, mode=mode)
        ctx = Context(rank)
        ctx.init_tensor_parallel(uid, rank, world)
        dm = w.upload(ctx, tp=(rank, world))
        r = ModelRunner(dm, ctx)
        if peer:  # all-reduce through peer memory: share the IPC handles over gloo
            import torch.distributed as dist
            os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
            dist.init_process_group("gloo", rank=rank, world_size=world)
            hs = [None] * world
            dist.all_gather_object(hs, r.tp_handle())
            r.tp_connect(hs)
            dist.barrier()
        toks = r.generate_batch([prompt], n_new)[0]
        out.put((rank, list(toks), None))
    except Exception as e:  # reported to the parent
        out.put((rank, None, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["perChannel", "int4"])
@pytest.mark.parametrize("peer", [False, True], ids=["nccl", "peer_memory"])
def test_tp2_greedy_matches_oracle(mode, peer):
    from tinybrain_b200.runtime import device_count, tp_unique_id
    if device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = ModelConfig(**TP_CFG)
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, cfg.vocab_size, 12)]
    n_new = 24
    om = oracle.OracleModel(small_llama(cfg, seed=3, mode=mode))
    expect, _ = om.generate_greedy(prompt, n_new)
    uid = tp_unique_id()
    ctxm = mp.get_context("spawn")
    out = ctxm.Queue()
    port = _free_port()
    procs = [ctxm.Process(target=_gpu_rank, args=(r, 2, uid, mode, prompt, n_new, out, peer, port), daemon=True)
             for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, toks, err = out.get(timeout=300)
        assert err is None, f"rank {rank}: {err}"
        res[rank] = toks
    for p in procs:
        p.join(timeout=60)
    assert res[0] == res[1]
    assert res[0] == list(expect)
