"""Greedy token identity at the BASELINE decode configurations.

The device decodes the seeded TinyLlama- and 7B-shaped models of configs 2-5
through the public API -- ModelRunner.generate_stream for one sequence,
ModelRunner.generate_batch for config 4's 64 sequences (the batched wide-GEMV
path the benchmark times) -- on the default per-projection launch chain, and
every token is compared with the oracle's list in tests/golden/config_tokens.json
(written on the CPU by tests/golden/make_config_tokens.py, oracle mode 1).  A
difference is tolerated only at a near-tie (oracle top-2 logit gap < 1e-4);
the rest of the run is then checked against the oracle teacher-forced on the
device's tokens (tests.helpers.assert_same_tokens).  Reference loop:
ModelRunner.swift:227-298.  These runs cover RoPE, KV append and attention up
to position 2047 (config 3) and 4223 (config 4) through the fused QKV epilogue.
"""
import json
import os

import numpy as np
import pytest

from tests.helpers import assert_same_tokens
from tinybrain_b200.runtime import GenerationConfig, ModelConfig, ModelRunner, SamplerConfig
from tinybrain_b200.synthetic import LLAMA2_7B, TINYLLAMA, make_llama_model, random_prompt

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "config_tokens.json")


def _fixture(name):
    with open(GOLD) as f:
        d = json.load(f)
    if name not in d:
        pytest.skip(f"{name} not in {os.path.basename(GOLD)}")
    return d[name]


def _oracle_teacher(cfg, mode, prompt):
    """Teacher-forced oracle check, built only if a near-tie flip happens."""
    def teach(got):
        from oracle.synthetic import llama_model
        from tests.helpers import teacher_forced
        return teacher_forced(llama_model(cfg, seed=0, mode=mode, group_size=32), prompt, got)
    return teach


def _stream(runner, prompt, n):
    cfg = GenerationConfig(max_tokens=n, sampler=SamplerConfig(top_k=1))
    return [t.token_id for t in runner.generate_stream(prompt, cfg)]


@pytest.mark.parametrize("name,cfg,mode,seed,plen", [
    ("config2", TINYLLAMA, "perChannel", 2, 128),
    ("config3", TINYLLAMA, "int4", 3, 1920),
    ("config5", {**LLAMA2_7B, "max_seq_len": 768}, "int4", 5, 512),
])
def test_single_sequence_config(ctx, name, cfg, mode, seed, plen):
    fx = _fixture(name)
    seq = fx["sequences"][0]
    prompt = random_prompt(plen, 32000, seed)
    assert prompt[:8] == seq["prompt_head"]
    w = make_llama_model(ModelConfig(**cfg), seed=0, mode=mode, group_size=32, ctx=ctx)
    r = ModelRunner(w, ctx, max_batch=1, max_positions=cfg["max_seq_len"] + 64)
    got = _stream(r, prompt, seq["new_tokens"])
    flips = assert_same_tokens(got, seq["tokens"], seq["gaps"], teacher=_oracle_teacher(cfg, mode, prompt))
    print(f"{name}: {len(got)} tokens identical to the oracle; tolerated flips {flips}")
    r.close()


def test_config4_batch_of_64(ctx):
    fx = _fixture("config4")
    cfg = {**TINYLLAMA, "max_seq_len": 4224}
    rng = np.random.default_rng(4)
    lens = rng.integers(512, 4097, size=64)
    prompts = [rng.integers(0, 32000, size=int(n)).tolist() for n in lens]
    w = make_llama_model(ModelConfig(**cfg), seed=0, mode="perChannel", ctx=ctx)
    r = ModelRunner(w, ctx, max_batch=64, max_positions=4224 + 64)
    n_new = fx["sequences"][0]["new_tokens"]
    got = r.generate_batch(prompts, n_new)
    assert len(got) == 64 and all(len(g) == n_new for g in got)
    for seq in fx["sequences"]:
        i = seq["key"]
        assert prompts[i][:8] == seq["prompt_head"]
        flips = assert_same_tokens(got[i], seq["tokens"], seq["gaps"],
                                   teacher=_oracle_teacher(cfg, "perChannel", prompts[i]))
        print(f"config4 sequence {i} (prompt {len(prompts[i])}): identical; tolerated flips {flips}")
    r.close()
