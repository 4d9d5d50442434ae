"""Perplexity harness (PerplexityHarness.swift:65-193) and QuantizedTensor.dequantize.

CPU: the oracle's computePerplexity restatement against a numpy evaluation of
its own step logits; the slice loader.  GPU: device dequantize and INT8->INT4
re-quantization bit-exact against the oracle; teacher-forced device
perplexity against the oracle (relative 2e-3: the logits themselves agree
within relative L2 1e-3), batched slices against single ones, errors.
"""
import json

import numpy as np
import pytest

import oracle
from tests.helpers import small_llama, toy_model
from tinybrain_b200.runtime import ModelConfig, PerplexitySlice, QuantizedTensor


def _cfg():
    return ModelConfig(num_layers=2, hidden_dim=256, num_heads=8, vocab_size=1024, max_seq_len=256, num_kv_heads=2,
                       intermediate_dim=512)


def _tokens(n, V, seed):
    rng = np.random.default_rng(seed)
    return [1] + rng.integers(0, V, n - 1).tolist()


def test_oracle_perplexity_is_exp_of_mean_negative_logprob():
    w = toy_model()
    o = oracle.OracleModel(w, mode=1)
    toks = _tokens(12, 100, 0)
    ppl, s = o.perplexity(toks)
    o.reset()
    acc = 0.0
    for i in range(len(toks) - 1):
        lg = o.step(toks[i])
        m = np.float64(lg.max())
        acc += np.float64(lg[toks[i + 1]]) - (np.log(np.exp(lg.astype(np.float64) - m).sum()) + m)
    assert s == pytest.approx(acc, rel=1e-12)
    assert ppl == float(np.float32(np.exp(-acc / (len(toks) - 1))))


def test_perplexity_slice_loader(tmp_path):
    d = {"source": "synthetic", "tokenizer": "none", "bos_token_id": 1, "seed": "s-1", "num_tokens": 4,
         "tokens": [1, 5, 6, 7], "notes": "made up"}
    p = tmp_path / "slice.json"
    p.write_text(json.dumps(d))
    s = PerplexitySlice.load(str(p))
    assert s.tokens == [1, 5, 6, 7] and s.bos_token_id == 1 and s.num_tokens == 4


@pytest.mark.gpu
def test_device_dequantize_bit_exact(ctx):
    rng = np.random.default_rng(4)
    K, N = 96, 160
    q8 = rng.integers(-127, 128, K * N).astype(np.int8)
    s8 = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    for zp in (None, rng.integers(-3, 4, N).astype(np.int8)):
        qt = QuantizedTensor((K, N), q8, s8, "perChannel", 0, zp)
        got = qt.dequantize(ctx)
        want = oracle.dequantize(qt) if zp is not None else \
            oracle.dequantize(QuantizedTensor((K, N), q8, s8, "perChannel", 0, np.zeros(N, np.int8)))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    K, N = 7, 9  # odd element count: the last byte holds one nibble
    cnt = K * N
    for gs in (32, 5):
        ng = (cnt + gs - 1) // gs
        p4 = rng.integers(0, 256, (cnt + 1) // 2).astype(np.uint8)
        s4 = rng.uniform(1e-3, 1e-1, ng).astype(np.float32)
        z4 = rng.integers(-2, 3, ng).astype(np.int8)
        qt = QuantizedTensor((K, N), p4, s4, "int4", gs, z4)
        assert np.array_equal(qt.dequantize(ctx).view(np.uint32), oracle.dequantize(qt).view(np.uint32))


@pytest.mark.gpu
def test_convert_to_int4_matches_oracle_composition(ctx):
    from tinybrain_b200.runtime import convert_to_int4
    w = small_llama(_cfg(), seed=2)
    w4 = convert_to_int4(w, 32, ctx)
    pairs = [(w.output, w4.output)] + [(getattr(a, n), getattr(b, n)) for a, b in zip(w.layers, w4.layers)
                                      for n in ("query", "key", "value", "output", "gate", "up", "down")]
    for lw8, lw4 in pairs:
        q8 = lw8.weights
        p, s, z = oracle.quantize_int4_group(oracle.dequantize(q8), 32)
        assert lw4.weights.mode == "int4" and lw4.weights.shape == q8.shape
        assert np.array_equal(lw4.weights.data, p)
        assert np.array_equal(lw4.weights.scales.view(np.uint32), s.view(np.uint32))
        assert np.array_equal(lw4.weights.zero_points, z)
    assert w4.token_embeddings is w.token_embeddings


@pytest.mark.gpu
@pytest.mark.parametrize("int4", [False, True])
def test_device_perplexity_matches_oracle(ctx, int4):
    from tinybrain_b200.runtime import compute_perplexity, convert_to_int4
    w = small_llama(_cfg(), seed=6, std=0.1)
    if int4:
        w = convert_to_int4(w, 32, ctx)
    toks = _tokens(65, 1024, 1)
    res = compute_perplexity(w, toks, ctx)
    ppl, s = oracle.OracleModel(w, mode=1).perplexity(toks)
    assert res.num_predictions == 64
    assert res.sum_log_prob == pytest.approx(s, rel=2e-3)
    assert res.perplexity == pytest.approx(ppl, rel=2e-3)


@pytest.mark.gpu
def test_batched_slices_match_single_and_errors(ctx):
    from tinybrain_b200._lib import TinyBrainError
    from tinybrain_b200.runtime import ModelRunner
    w = small_llama(_cfg(), seed=6, std=0.1)
    slices = [_tokens(40, 1024, 2), _tokens(17, 1024, 3), _tokens(2, 1024, 4)]
    rb = ModelRunner(w, ctx, max_batch=3)
    batched = rb.perplexity(slices)
    r1 = ModelRunner(w, ctx)
    for sl, b in zip(slices, batched):
        one = r1.perplexity([sl])[0]
        assert b.num_predictions == len(sl) - 1
        assert b.sum_log_prob == pytest.approx(one.sum_log_prob, rel=1e-4)
    with pytest.raises(TinyBrainError):
        r1.perplexity([[5]])
    with pytest.raises(TinyBrainError):
        r1.perplexity([[1, 1024]])
    # the runner still generates greedily afterwards
    r1.reset()
    assert len(r1.generate_batch([[1, 2, 3]], 4)[0]) == 4


@pytest.mark.gpu
def test_chunked_scoring_matches_token_by_token(ctx):
    from tinybrain_b200.runtime import ModelRunner
    w = small_llama(_cfg(), seed=9, std=0.1)
    slices = [_tokens(130, 1024, 7), _tokens(33, 1024, 8)]
    chunked = ModelRunner(w, ctx, max_batch=2).perplexity(slices)
    r = ModelRunner(w, ctx, max_batch=2)
    r.set_chunked_prefill(False)
    stepped = r.perplexity(slices)
    for a, b in zip(chunked, stepped):
        assert a.num_predictions == b.num_predictions
        assert a.sum_log_prob == pytest.approx(b.sum_log_prob, rel=1e-4)
