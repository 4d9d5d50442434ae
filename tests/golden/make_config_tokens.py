#!/usr/bin/env python3
"""Writes tests/golden/config_tokens.json: the oracle's greedy token sequences
for the BASELINE decode configurations, with each step's top-2 logit gap.

CPU only; uses the oracle alone (oracle/synthetic.py builds the seeded models
with the reference's SeededGenerator and quantizers).  The oracle runs in
mode 1 (fp64 GEMV accumulation), prompts chunked by orc_runner_prefill (the
same results as stepping token by token).  The -m gpu tests in
tests/test_config_tokens.py decode the same models on the device through the
public API and compare against these lists.

    python tests/golden/make_config_tokens.py [config ...]   # default: 2 3 4 5

Configurations (reference loop: ModelRunner.swift:227-298):
  2: TinyLlama-1.1B shape INT8, weights seed 0, prompt 128 ids (seed 2), 256 tokens
  3: TinyLlama INT4-g32, prompt 1920 ids (seed 3), 128 tokens (context 2048)
  4: TinyLlama INT8, max_seq_len 4224; the 64 prompts of config 4 (numpy PCG64
     seed 4: lengths U[512, 4096], then ids U[0, 32000) per sequence); the
     shortest, the median-length and the longest sequence, 16 tokens each
  5: Llama-2-7B shape INT4-g32, prompt 512 ids (seed 5), 32 tokens
"""
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import numpy as np  # noqa: E402

import oracle  # noqa: E402
from oracle.synthetic import LLAMA2_7B, TINYLLAMA, llama_model, random_prompt  # noqa: E402

OUT = os.path.join(HERE, "config_tokens.json")


def config4_prompts():
    rng = np.random.default_rng(4)
    lens = rng.integers(512, 4097, size=64)
    prompts = [rng.integers(0, 32000, size=int(n)).tolist() for n in lens]
    return lens, prompts


def config4_subset(lens):
    order = np.argsort(lens, kind="stable")
    return [int(order[0]), int(order[len(order) // 2]), int(order[-1])]


def run(cfg_id):
    t0 = time.time()
    if cfg_id == 2:
        w = llama_model(TINYLLAMA, seed=0, mode="perChannel")
        runs = [("seq", random_prompt(128, 32000, 2), 256)]
        meta = {"model": "TinyLlama-1.1B shape INT8 per-channel, seed 0", "prompt_seed": 2, "prompt_len": 128}
    elif cfg_id == 3:
        w = llama_model(TINYLLAMA, seed=0, mode="int4", group_size=32)
        runs = [("seq", random_prompt(1920, 32000, 3), 128)]
        meta = {"model": "TinyLlama-1.1B shape INT4 g32, seed 0", "prompt_seed": 3, "prompt_len": 1920}
    elif cfg_id == 4:
        w = llama_model({**TINYLLAMA, "max_seq_len": 4224}, seed=0, mode="perChannel")
        lens, prompts = config4_prompts()
        sub = config4_subset(lens)
        runs = [(i, prompts[i], 16) for i in sub]
        meta = {"model": "TinyLlama-1.1B shape INT8 per-channel, seed 0, max_seq_len 4224",
                "prompts": "numpy PCG64 seed 4: 64 lengths U[512,4096], then ids", "subset": sub,
                "lengths": [int(lens[i]) for i in sub]}
    elif cfg_id == 5:
        w = llama_model({**LLAMA2_7B, "max_seq_len": 768}, seed=0, mode="int4", group_size=32)
        runs = [("seq", random_prompt(512, 32000, 5), 32)]
        meta = {"model": "Llama-2-7B shape INT4 g32, seed 0, max_seq_len 768", "prompt_seed": 5,
                "prompt_len": 512}
    else:
        raise SystemExit(f"unknown config {cfg_id}")
    seqs = []
    for key, prompt, n_new in runs:
        o = oracle.OracleModel(w, mode=1)
        toks, gaps = o.generate_greedy(prompt, n_new)
        seqs.append({"key": key, "prompt_head": prompt[:8], "new_tokens": n_new, "tokens": toks,
                     "gaps": [float(g) for g in gaps]})
        del o
    meta["seconds"] = round(time.time() - t0, 1)
    return {**meta, "sequences": seqs}


def main():
    ids = [int(a) for a in sys.argv[1:]] or [2, 3, 4, 5]
    data = {}
    if os.path.exists(OUT):
        with open(OUT) as f:
            data = json.load(f)
    for c in ids:
        data[f"config{c}"] = run(c)
        with open(OUT, "w") as f:
            json.dump(data, f, indent=1)
        print(f"config {c}: {data[f'config{c}']['seconds']} s", flush=True)


if __name__ == "__main__":
    main()
