"""Sampler (Sampler.swift:401-473, sampleDetailed) parity.

CPU: the oracle restatement reproduces the behaviours the reference's
SamplerTests.swift checks (top-k / top-p support, repetition penalty,
seeded determinism, top-k = 1 is greedy).  GPU: the device sampler kernel
against the oracle on seeded logits, one draw at a time, with the same RNG
stream; then sampled generation end to end against the oracle model.
"""
from types import SimpleNamespace

import numpy as np
import pytest

import oracle


def cfg(temperature=1.0, top_k=None, top_p=None, repetition_penalty=1.0):
    return SimpleNamespace(temperature=temperature, top_k=top_k, top_p=top_p,
                           repetition_penalty=repetition_penalty)


L5 = np.array([0.1, 0.5, 0.2, 0.8, 0.3], dtype=np.float32)


def draws(logits, c, n, seed=7, history=()):
    st, out = seed, []
    for _ in range(n):
        t, p, e, st = oracle.sample_detailed(logits, c, list(history), st)
        out.append(t)
    return out


def test_lcg_matches_numerical_recipes_constants():
    st = 42
    for _ in range(3):
        st = (st * 6364136223846793005 + 1442695040888963407) % (1 << 64)
    _, _, _, got = oracle.sample_detailed(L5, cfg(), [], 42)
    _, _, _, got = oracle.sample_detailed(L5, cfg(), [], got)
    _, _, _, got = oracle.sample_detailed(L5, cfg(), [], got)
    assert got == st


def test_top_k_limits_support():
    assert set(draws(L5, cfg(top_k=2), 100)) <= {1, 3}


def test_top_k_one_is_greedy_with_reference_statistics():
    t, p, e, _ = oracle.sample_detailed(L5, cfg(top_k=1), [], 1)
    assert t == 3
    p32 = np.float32(1) / (np.float32(1) + np.float32(1e-7))
    assert p == pytest.approx(float(p32), rel=1e-7)
    assert e == pytest.approx(float(-p32 * np.log(p32)), rel=1e-5, abs=1e-12)


def test_top_k_larger_than_vocab_samples_broadly():
    assert len(set(draws(L5, cfg(temperature=1.5, top_k=10), 200))) > 2


def test_top_p_focuses_on_nucleus():
    lg = np.array([0.0, 1.0, 0.0, 2.0, 0.0], dtype=np.float32)
    s = set(draws(lg, cfg(top_p=0.9), 100))
    assert 3 in s and len(s) <= 4
    assert len(set(draws(L5, cfg(top_p=0.1), 50))) <= 2
    assert len(set(draws(L5, cfg(temperature=1.5, top_p=1.0), 200))) > 3


def test_repetition_penalty_is_sign_aware_and_per_history_entry():
    lg = np.array([0.8, 0.1, 0.1], dtype=np.float32)
    s = set(draws(lg, cfg(repetition_penalty=2.0), 50, history=[0, 0, 0]))
    assert s & {1, 2}
    # top_k=1 exposes the penalised argmax: each of the three history entries
    # divides again, 0.8 / 2^3 = 0.1 falls below token 1's 0.11
    lg2 = np.array([0.8, 0.11, 0.1], dtype=np.float32)
    t, _, _, _ = oracle.sample_detailed(lg2, cfg(top_k=1, repetition_penalty=2.0), [0, 0, 0], 1)
    assert t == 1
    neg = np.array([-0.1, -0.3], dtype=np.float32)
    t, _, _, _ = oracle.sample_detailed(neg, cfg(top_k=1, repetition_penalty=4.0), [0], 1)
    assert t == 1  # -0.1 * 4 = -0.4 < -0.3
    counts = np.bincount(draws(lg, cfg(repetition_penalty=1.0), 100, history=[0, 0, 0]), minlength=3)
    assert counts[0] > counts[1] and counts[0] > counts[2]


def test_seeded_determinism_and_diversity():
    a = draws(L5, cfg(), 5, seed=42)
    assert a == draws(L5, cfg(), 5, seed=42)
    assert len(set(a)) > 1


def test_uniform_and_single_token():
    assert len(set(draws(np.full(4, 0.5, np.float32), cfg(), 100))) >= 3
    assert draws(np.array([1.0], np.float32), cfg(), 5) == [0] * 5


def test_probability_and_entropy_of_final_distribution():
    c = cfg(temperature=0.8, top_k=3)
    t, p, e, _ = oracle.sample_detailed(L5, c, [], 3)
    x = L5.astype(np.float64) / 0.8
    keep = np.argsort(-L5, kind="stable")[:3]
    m = np.full(5, -np.inf)
    m[keep] = x[keep]
    q = np.exp(m - m.max())
    q /= q.sum()
    assert t in keep
    assert p == pytest.approx(q[t], rel=1e-5)
    assert e == pytest.approx(-(q[q > 0] * np.log(q[q > 0])).sum(), rel=1e-5)


# ----------------------------------------------------------------- device --
def _dev(c, seed=None):
    from tinybrain_b200.runtime import SamplerConfig
    return SamplerConfig(temperature=c.temperature, top_k=c.top_k, top_p=c.top_p,
                         repetition_penalty=c.repetition_penalty, seed=seed)


def _final_probs64(logits, c, history):
    """fp64 final distribution (for locating CDF boundaries in the checks)."""
    x = np.asarray(logits, dtype=np.float32).copy()
    if c.repetition_penalty != 1.0:
        for t in history:
            if 0 <= t < x.size:
                x[t] = x[t] / np.float32(c.repetition_penalty) if x[t] > 0 else x[t] * np.float32(c.repetition_penalty)
    order = np.argsort(-x, kind="stable")
    if c.top_k is not None and c.top_k > 0:
        keep = order[:c.top_k]
    elif c.top_p is not None:
        e = np.exp((x - x.max()).astype(np.float64))
        q = (e / (e.sum() + 1e-7)).astype(np.float32)
        order = np.argsort(-q, kind="stable")
        cum = np.cumsum(q[order], dtype=np.float32)
        hit = np.nonzero(cum >= np.float32(c.top_p))[0]
        keep = order[:(hit[0] + 1) if hit.size else x.size]
    else:
        keep = order
    m = np.full(x.size, -np.inf)
    m[keep] = x[keep]
    t = max(0.0, c.temperature)
    if t >= 0.01:
        m = m / t
    e = np.exp(m - m.max())
    return e / e.sum()


def _threshold(state):
    st = (state * 6364136223846793005 + 1442695040888963407) % (1 << 64)
    return float(np.float32(st) / np.float32(2.0 ** 64))


def _check_draws(ctx, V, c, logits_fn, n, seed, max_boundary_frac):
    from tinybrain_b200.runtime import sample_detailed as dev_sample
    rng = np.random.default_rng(seed)
    st = 1234 + seed
    boundary = 0
    for _ in range(n):
        logits = logits_fn(rng, V)
        hist = rng.integers(0, V, 24).tolist() + [int(np.argmax(logits))] * 3 + [-1, V + 5]
        t_d, p_d, e_d, st_d = dev_sample(logits, _dev(c), hist, st, ctx)
        t_o, p_o, e_o, st_o = oracle.sample_detailed(logits, c, hist, st)
        assert st_d == st_o
        thr = _threshold(st)
        st = st_o
        if t_d != t_o:
            # only where the reference's sequential fp32 CDF and the device's
            # parallel one straddle the threshold
            q = _final_probs64(logits, c, hist)
            lo = min(t_d, t_o)
            assert abs(np.cumsum(q)[lo] - thr) < 2e-4, (t_d, t_o)
            boundary += 1
            continue
        assert p_d == pytest.approx(p_o, rel=2e-3, abs=1e-7)
        assert e_d == pytest.approx(e_o, rel=1e-3, abs=1e-6)
    assert boundary <= max_boundary_frac * n


def _peaked(rng, V):
    x = rng.standard_normal(V).astype(np.float32)
    hot = rng.choice(V, 24, replace=False)
    x[hot] += rng.uniform(7.0, 12.0, hot.size).astype(np.float32)
    return x


def _flat(rng, V):
    return (rng.standard_normal(V) * 2.0).astype(np.float32)


DEVICE_CASES = [
    cfg(temperature=1.0),
    cfg(temperature=0.7, top_k=40),
    cfg(temperature=1.3, top_k=1),
    cfg(temperature=0.005, top_p=0.9),
    cfg(temperature=0.8, top_p=0.9, repetition_penalty=1.3),
    cfg(temperature=1.0, top_p=0.5),
    cfg(temperature=1.5, top_k=10 ** 6),
    cfg(temperature=0.9, top_k=100, top_p=0.5, repetition_penalty=0.8),
]


@pytest.mark.gpu
@pytest.mark.parametrize("V", [32000, 50021])
@pytest.mark.parametrize("ci", range(len(DEVICE_CASES)))
def test_device_sampler_peaked_logits_match_oracle(ctx, V, ci):
    # LLM-like rows (a few dominant tokens over a long tail; a high
    # temperature spreads the mass into the tail, where a draw can land on a
    # CDF boundary)
    _check_draws(ctx, V, DEVICE_CASES[ci], _peaked, 10, seed=ci, max_boundary_frac=0.2)


@pytest.mark.gpu
@pytest.mark.parametrize("ci", [0, 1, 4, 5])
def test_device_sampler_flat_logits_boundaries_only(ctx, ci):
    # a flat 32000-way distribution puts the threshold between tiny steps of
    # the CDF, where the sequential and parallel fp32 sums may disagree
    _check_draws(ctx, 32000, DEVICE_CASES[ci], _flat, 16, seed=10 + ci, max_boundary_frac=0.25)


@pytest.mark.gpu
def test_device_sampler_reference_examples(ctx):
    from tinybrain_b200.runtime import sample_detailed as dev_sample
    for c, lg, hist in [
        (cfg(top_k=2), L5, []),
        (cfg(top_k=1), L5, []),
        (cfg(temperature=1.5, top_p=1.0), L5, []),
        (cfg(top_p=0.1), L5, []),
        (cfg(repetition_penalty=2.0), np.array([0.8, 0.1, 0.1], np.float32), [0, 0, 0]),
        (cfg(temperature=0.8, top_k=3, top_p=0.95, repetition_penalty=1.2),
         np.array([0.5, 0.6, 0.7, 0.8, 0.9], np.float32), [4]),
        (cfg(), np.full(4, 0.5, np.float32), []),
        (cfg(top_k=2), np.full(6, 0.5, np.float32), []),          # ties: lowest indices kept
        (cfg(top_p=0.5), np.full(4, 0.5, np.float32), []),         # +1e-7 makes the nucleus 3 wide
        (cfg(), np.array([1.0], np.float32), []),
        (cfg(top_k=1, repetition_penalty=4.0), np.array([-0.1, -0.3], np.float32), [0]),
    ]:
        st_d = st_o = 42
        for _ in range(40):
            t_d, p_d, e_d, st_d = dev_sample(lg, _dev(c), hist, st_d, ctx)
            t_o, p_o, e_o, st_o = oracle.sample_detailed(lg, c, hist, st_o)
            assert (t_d, st_d) == (t_o, st_o)
            assert p_d == pytest.approx(p_o, rel=1e-5)
            assert e_d == pytest.approx(e_o, rel=1e-4, abs=1e-7)


def _model(std=0.1):
    from tests.helpers import small_llama
    from tinybrain_b200.runtime import ModelConfig
    c = ModelConfig(num_layers=2, hidden_dim=256, num_heads=8, vocab_size=1024, max_seq_len=128, num_kv_heads=2,
                    intermediate_dim=512)
    return small_llama(c, seed=5, std=std)


MODEL_CASES = [
    dict(temperature=0.5, top_k=50, seed=7),
    dict(temperature=0.7, top_p=0.9, repetition_penalty=1.2, seed=11),
    dict(temperature=0.6, seed=3),
    dict(temperature=1.0, top_k=1, repetition_penalty=1.5, seed=1),
]


@pytest.mark.gpu
@pytest.mark.parametrize("mi", range(len(MODEL_CASES)))
def test_generate_stream_sampled_teacher_forced_against_oracle(ctx, mi):
    from tinybrain_b200.runtime import GenerationConfig, ModelRunner, SamplerConfig
    w = _model()
    sc = SamplerConfig(**MODEL_CASES[mi])
    prompt = [3, 14, 15, 92, 65]
    outs = list(ModelRunner(w, ctx).generate_stream(prompt, GenerationConfig(max_tokens=24, sampler=sc)))
    assert len(outs) == 24
    assert outs[0].strategy == sc.strategy()
    o = oracle.OracleModel(w, mode=1)
    for t in prompt[:-1]:
        o.step(t)
    cur, hist, st = prompt[-1], list(prompt), sc.seed
    agree = 0
    for out in outs:
        logits = o.step(cur)
        t_o, p_o, e_o, st = oracle.sample_detailed(logits, sc, hist, st)
        if t_o == out.token_id:
            agree += 1
            assert out.probability == pytest.approx(p_o, rel=2e-2, abs=1e-6)
            assert out.entropy == pytest.approx(e_o, rel=2e-2, abs=1e-5)
        cur = out.token_id  # teacher forcing: follow the device's sequence
        hist.append(cur)
    assert agree >= 22


@pytest.mark.gpu
def test_sampled_generation_is_seeded_batched_and_observer_neutral(ctx):
    from tinybrain_b200.runtime import GenerationConfig, ModelRunner, SamplerConfig
    w = _model()
    sc = SamplerConfig(temperature=0.9, top_p=0.95, repetition_penalty=1.1, seed=99)
    gen = GenerationConfig(max_tokens=20, sampler=sc)
    prompt = [7, 8, 9]
    r = ModelRunner(w, ctx)
    a = list(r.generate_stream(prompt, gen))
    r.reset()
    b = list(r.generate_stream(prompt, gen))
    assert [t.token_id for t in a] == [t.token_id for t in b]
    assert [t.probability for t in a] == [t.probability for t in b]
    r.reset()
    other = [t.token_id for t in r.generate_stream(prompt, GenerationConfig(
        max_tokens=20, sampler=SamplerConfig(temperature=0.9, top_p=0.95, repetition_penalty=1.1, seed=100)))]
    assert other != [t.token_id for t in a]
    # every sequence of a batch runs generateStream with the same config
    rb = ModelRunner(w, ctx, max_batch=3)
    rb.set_sampler(sc)
    try:
        rows = rb.generate_batch([prompt, [1, 2, 3, 4, 5, 6], prompt], 20)
    finally:
        rb.set_sampler(None)
    assert rows[0] == rows[2] == [t.token_id for t in a]
    single = [t.token_id for t in ModelRunner(w, ctx).generate_stream([1, 2, 3, 4, 5, 6], gen)]
    assert rows[1] == single

    class Obs:
        def did_enter_layer(self, *a):
            pass

        def did_compute_attention(self, *a):
            pass

        def did_compute_logits(self, *a):
            pass

    ro = ModelRunner(w, ctx)
    ro.observer = Obs()
    c = list(ro.generate_stream(prompt, gen))
    assert [t.token_id for t in c] == [t.token_id for t in a]
    assert [t.probability for t in c] == pytest.approx([t.probability for t in a], rel=1e-6)
    assert [t.entropy for t in c] == pytest.approx([t.entropy for t in a], rel=1e-6)


@pytest.mark.gpu
def test_sampler_turns_the_persistent_step_off_and_back(ctx):
    from tinybrain_b200._lib import TinyBrainError
    from tinybrain_b200.runtime import ModelRunner, SamplerConfig
    w = _model()
    r = ModelRunner(w, ctx)
    r.persistent = True
    greedy = r.generate_batch([[1, 2, 3]], 8)[0]
    r.set_sampler(SamplerConfig(temperature=0.8, seed=5))
    assert not r.persistent
    with pytest.raises(TinyBrainError):
        r.persistent = True
    r.generate_batch([[1, 2, 3]], 8)
    r.set_sampler(None)
    assert r.persistent
    assert r.generate_batch([[1, 2, 3]], 8)[0] == greedy
