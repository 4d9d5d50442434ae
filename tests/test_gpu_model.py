"""Decode-step parity of the whole device path against the CPU oracle.

Logits within relative L2 <= 1e-3; greedy tokens identical to the oracle's
(the oracle accumulates in fp64; where its top-2 logit gap is below 1e-4 an
fp32 reordering could legitimately flip the argmax, and the test reports it).
"""
import numpy as np
import pytest

import oracle
from tests.helpers import assert_same_tokens, rel_l2, small_llama, toy_model
from tinybrain_b200.runtime import GenerationConfig, ModelConfig, ModelRunner, SamplerConfig

pytestmark = pytest.mark.gpu
RTOL_L2 = 1e-3


def small_cfg(**kw):
    base = dict(num_layers=2, hidden_dim=256, num_heads=8, vocab_size=1024, max_seq_len=128, num_kv_heads=2,
                intermediate_dim=512)
    base.update(kw)
    return ModelConfig(**base)


@pytest.mark.parametrize("mode,persistent", [("perChannel", True), ("perChannel", False), ("int4", False)])
def test_step_logits_and_kv_state(ctx, mode, persistent):
    w = small_llama(small_cfg(), seed=3, mode=mode)
    r = ModelRunner(w, ctx)
    r.persistent = persistent
    o = oracle.OracleModel(w, mode=1)
    for i, tok in enumerate([5, 17, 999, 0, 512, 3, 3, 77, 100, 42, 7, 8, 9, 10, 11, 12, 13, 14]):
        logits, am = r.step(tok)
        ref = o.step(tok)
        assert rel_l2(logits, ref) <= RTOL_L2, i
        assert am == int(np.argmax(logits))
        assert r.kv_cache.length == o.kv_length == i + 1
        assert r.current_position == o.position
        assert r.kv_cache.page_allocation_status() == o.page_status()
    r.reset()
    o.reset()
    assert r.kv_cache.length == 0 and r.current_position == 0
    l1, _ = r.step(5)
    assert rel_l2(l1, o.step(5)) <= RTOL_L2


def test_toy_model_greedy_identity(ctx):
    w = toy_model()
    r = ModelRunner(w, ctx)
    o = oracle.OracleModel(w, mode=1)
    prompt = [1, 2, 3, 4, 5]
    want, gaps = o.generate_greedy(prompt, 40)
    got = r.generate_batch([prompt], 40)[0]
    assert_same_tokens(got, want, gaps, w, prompt)


@pytest.mark.parametrize("mode,persistent", [("perChannel", "flow"), ("perChannel", "barrier"),
                                             ("perChannel", False), ("int4", False)])
def test_generate_greedy_identity(ctx, mode, persistent, monkeypatch):
    if persistent:
        monkeypatch.setenv("TB_STEP_KERNEL", persistent)
    w = small_llama(small_cfg(num_layers=3), seed=4, mode=mode)
    r = ModelRunner(w, ctx)
    r.persistent = bool(persistent)
    o = oracle.OracleModel(w, mode=1)
    prompt = [11, 22, 33, 44, 55, 66, 77, 88, 99, 111, 222, 333, 444, 555, 666, 777, 888]
    want, gaps = o.generate_greedy(prompt, 48)
    got = r.generate_batch([prompt], 48)[0]
    assert_same_tokens(got, want, gaps, w, prompt)
    assert r.kv_cache.length == len(prompt) - 1 + 48


def test_generate_stream_stop_token(ctx):
    w = small_llama(small_cfg(), seed=5)
    r = ModelRunner(w, ctx)
    o = oracle.OracleModel(w, mode=1)
    want, gaps = o.generate_greedy([1, 2, 3], 20)
    stop = want[5]
    outs = list(r.generate_stream([1, 2, 3], GenerationConfig(max_tokens=20, sampler=SamplerConfig(top_k=1),
                                                              stop_tokens=[stop])))
    ids = [t.token_id for t in outs]
    k = want.index(stop)
    assert ids == want[:k + 1]  # the stop token is yielded, then generation ends
    assert all(abs(t.probability - 0.9999999) < 1e-6 for t in outs)


@pytest.mark.parametrize("persistent", [True, False])
def test_kv_eviction_parity(ctx, persistent):
    cfg = small_cfg(max_seq_len=48)
    w = small_llama(cfg, seed=6)
    r = ModelRunner(w, ctx, max_positions=160)
    r.persistent = persistent
    o = oracle.OracleModel(w, mode=1)
    for i in range(120):
        tok = (i * 37) % cfg.vocab_size
        logits, _ = r.step(tok)
        ref = o.step(tok)
        assert rel_l2(logits, ref) <= RTOL_L2, i
        assert r.kv_cache.length == o.kv_length, i
        assert r.kv_cache.page_allocation_status() == o.page_status(), i


def test_batched_sequences_match_independent_runs(ctx):
    w = small_llama(small_cfg(), seed=7)
    r = ModelRunner(w, ctx, max_batch=4)
    prompts = [[1, 2, 3], [10] * 20, [5], [7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17, 18, 19, 20, 21, 22, 23, 24]]
    got = r.generate_batch(prompts, 24)
    for p, g in zip(prompts, got):
        o = oracle.OracleModel(w, mode=1)
        want, gaps = o.generate_greedy(p, 24)
        assert_same_tokens(g, want, gaps, w, p)


@pytest.mark.parametrize("mode", ["perChannel", "int4"])
def test_batch_of_twenty_sequences(ctx, mode):
    # more sequences than one GEMV CTA holds (INT8 16 rows, INT4 2): batch rows
    # are split over the grid; every sequence must match its own oracle run
    w = small_llama(small_cfg(num_layers=2), seed=12, mode=mode)
    r = ModelRunner(w, ctx, max_batch=20)
    rng = np.random.default_rng(77)
    prompts = [[int(v) for v in rng.integers(1, 200, size=1 + (i * 7) % 23)] for i in range(20)]
    got = r.generate_batch(prompts, 12)
    for p, gt in zip(prompts, got):
        o = oracle.OracleModel(w, mode=1)
        want, gaps = o.generate_greedy(p, 12)
        assert_same_tokens(gt, want, gaps, w, p)


def test_batched_eviction_parity(ctx):
    # two sequences whose contexts run past max_seq_len (reference FIFO page
    # eviction, KVCache.swift:157-224) next to a short one, decoded together
    cfg = small_cfg(max_seq_len=48)
    w = small_llama(cfg, seed=13)
    r = ModelRunner(w, ctx, max_batch=3, max_positions=128)
    prompts = [list(range(1, 41)), [7, 8, 9], list(range(50, 90))]
    got = r.generate_batch(prompts, 30)
    for p, gt in zip(prompts, got):
        o = oracle.OracleModel(w, mode=1)
        want, gaps = o.generate_greedy(p, 30)
        assert_same_tokens(gt, want, gaps, w, p)


def test_persistent_available_for_batch1_llama_only(ctx):
    from tinybrain_b200._lib import TinyBrainError
    w = small_llama(small_cfg(), seed=9)
    r = ModelRunner(w, ctx)
    assert not r.persistent  # the per-projection launch chain is the default
    r.persistent = True
    assert r.persistent
    # batch > 1, the toy architecture and INT4 weights keep the launch chain
    w4 = small_llama(small_cfg(), seed=9, mode="int4")
    for other in (ModelRunner(w, ctx, max_batch=2), ModelRunner(toy_model(), ctx), ModelRunner(w4, ctx)):
        with pytest.raises(TinyBrainError):
            other.persistent = True


@pytest.mark.parametrize("shape", [dict(hidden_dim=512, num_heads=8, num_kv_heads=8, intermediate_dim=1408),
                                   dict(hidden_dim=256, num_heads=4, num_kv_heads=4, intermediate_dim=704,
                                        num_layers=1),
                                   dict(hidden_dim=2048, num_heads=32, num_kv_heads=4, intermediate_dim=5632,
                                        vocab_size=32000)])
@pytest.mark.parametrize("mode,kernel", [("perChannel", "flow"), ("perChannel", "barrier")])
def test_persistent_other_shapes(ctx, shape, mode, kernel, monkeypatch):
    # MHA (G = 1), one layer with a short last slab, and the TinyLlama layer
    # shape; INT8 through both persistent kernels (dataflow and grid-barrier)
    monkeypatch.setenv("TB_STEP_KERNEL", kernel)
    cfg = small_cfg(**shape)
    w = small_llama(cfg, seed=10, mode=mode)
    r = ModelRunner(w, ctx)
    r.persistent = True
    o = oracle.OracleModel(w, mode=1)
    for i, tok in enumerate([3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8, 9, 7, 9, 3, 2, 3]):
        logits, _ = r.step(tok)
        assert rel_l2(logits, o.step(tok)) <= RTOL_L2, i


class _Recorder:
    """InferenceObserver (InferenceObserver.swift:40-84) that records every call."""

    def __init__(self):
        self.calls = []

    def did_enter_layer(self, layer, norm, position):
        self.calls.append(("enter", layer, position, norm))

    def did_compute_attention(self, layer, weights, position):
        self.calls.append(("attn", layer, position, weights))

    def did_compute_final_hidden_state(self, hidden, position):
        self.calls.append(("final", None, position, hidden))

    def did_compute_logits(self, logits, position):
        self.calls.append(("logits", None, position, logits))


@pytest.mark.parametrize("mode", ["perChannel", "int4"])
def test_observer_hooks_match_oracle(ctx, mode):
    cfg = small_cfg(num_layers=3)
    w = small_llama(cfg, seed=21, mode=mode)
    r = ModelRunner(w, ctx)
    rec = _Recorder()
    r.observer = rec
    o = oracle.OracleModel(w, mode=1)
    for i, tok in enumerate([5, 17, 3, 99, 42, 7, 11, 250, 1, 64, 33, 2, 8, 19, 600, 4, 12, 90]):
        rec.calls.clear()
        logits, _ = r.step(tok)
        ol, on, oa, of = o.step_observed(tok)
        kinds = [c[0] for c in rec.calls]
        assert kinds == ["enter", "attn"] * cfg.num_layers + ["final", "logits"]  # the reference's order
        assert all(c[2] == i for c in rec.calls)  # currentPosition
        norms = np.array([c[3] for c in rec.calls if c[0] == "enter"], dtype=np.float32)
        assert rel_l2(norms, on) <= 1e-5
        for l, c in enumerate([c for c in rec.calls if c[0] == "attn"]):
            assert c[3].shape == (cfg.num_heads * (i + 1),)
            assert np.allclose(c[3], oa[l], atol=1e-5, rtol=5e-4)
            assert np.allclose(c[3].reshape(cfg.num_heads, -1).sum(axis=1), 1.0, atol=1e-5)
        assert rel_l2(rec.calls[-2][3], of) <= 1e-5
        assert rel_l2(rec.calls[-1][3], ol) <= RTOL_L2
        assert rel_l2(logits, ol) <= RTOL_L2


def test_observer_generate_stream_same_tokens(ctx):
    w = small_llama(small_cfg(), seed=22)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    plain = [t.token_id for t in ModelRunner(w, ctx).generate_stream(prompt, GenerationConfig(max_tokens=12, sampler=SamplerConfig(top_k=1)))]
    r = ModelRunner(w, ctx)
    rec = _Recorder()
    r.observer = rec
    seen = [t.token_id for t in r.generate_stream(prompt, GenerationConfig(max_tokens=12, sampler=SamplerConfig(top_k=1)))]
    assert seen == plain
    # one didComputeLogits per step: 7 prefill steps + 12 decode steps
    assert sum(1 for c in rec.calls if c[0] == "logits") == len(prompt) - 1 + 12


@pytest.mark.parametrize("mode", ["perChannel", "int4"])
def test_chunked_prefill_matches_oracle_and_token_by_token(ctx, mode):
    from tinybrain_b200.runtime import KVCacheView
    w = small_llama(small_cfg(max_seq_len=256), seed=12, mode=mode, std=0.05)
    rng = np.random.default_rng(5)
    # 150 tokens span three chunks; 70 + 2 + 1 share chunks with it
    prompts = [rng.integers(0, 1024, n).tolist() for n in (150, 1, 70, 2)]
    chunked = ModelRunner(w, ctx, max_batch=4)
    stepped = ModelRunner(w, ctx, max_batch=4)
    stepped.set_chunked_prefill(False)
    a = chunked.generate_batch(prompts, 12)
    b = stepped.generate_batch(prompts, 12)
    for i, p in enumerate(prompts):
        want, gaps = oracle.OracleModel(w, mode=1).generate_greedy(p, 12)
        assert_same_tokens(a[i], want, gaps, w, p)
        assert_same_tokens(b[i], want, gaps, w, p)
        ka, kb = KVCacheView(chunked, i), KVCacheView(stepped, i)
        assert ka.length == kb.length == len(p) - 1 + 12 if p else True
        assert ka.page_allocation_status() == kb.page_allocation_status()


def test_chunked_prefill_then_step_logits(ctx):
    # the state a chunked prefill leaves (KV pages, positions) feeds later steps
    w = small_llama(small_cfg(max_seq_len=256), seed=13)
    prompt = np.random.default_rng(6).integers(0, 1024, 100).tolist()
    r = ModelRunner(w, ctx)
    r.generate_batch([prompt], 1)
    o = oracle.OracleModel(w, mode=1)
    for t in prompt:
        o.step(t)
    assert r.current_position == o.position
    nxt = [5, 900, 17]
    for t in nxt:
        logits, _ = r.step(t)
        assert rel_l2(logits, o.step(t)) <= RTOL_L2
