"""Seeded synthetic models for the benchmark configurations.

The reference builds test models with Tensor.random over its SeededGenerator
LCG (ModelWeights.swift:18-29, 171-244; Tensor.swift:1623-1644); the same
generator is exposed by libtinybrain_cuda (tb_rng_fill_normal), so the
weights here are a deterministic function of the seed.  Quantization runs on
the GPU with the reference's quantizer formulas (bit-exact).

Draw order: token embeddings [vocab, hidden]; then per layer q, k, v, o,
(gate), up, down weights (each [in, out]), each followed by its bias for the
toy model; then the output projection.  LLaMA-shaped models have unit norm
weights and no biases; the toy model follows makeToyModel exactly (biases on
every projection, zero LM-head bias, GELU FFN of width 4*hidden, no norms).
"""
from __future__ import annotations

from typing import Optional

import numpy as np

from .runtime import (TP_AXIS, Context, LinearLayerWeights, ModelConfig, ModelWeights, SeededGenerator,
                      TransformerLayerWeights, quantize, shard_linear)

TINYLLAMA = dict(num_layers=22, hidden_dim=2048, num_heads=32, num_kv_heads=4, vocab_size=32000,
                 intermediate_dim=5632, max_seq_len=2048)
LLAMA2_7B = dict(num_layers=32, hidden_dim=4096, num_heads=32, num_kv_heads=32, vocab_size=32000,
                 intermediate_dim=11008, max_seq_len=2048)
TOY = dict(num_layers=2, hidden_dim=128, num_heads=4, num_kv_heads=4, vocab_size=100,
           intermediate_dim=512, max_seq_len=256, architecture="toy")


_FIELD = {"q": "query", "k": "key", "v": "value", "o": "output", "gate": "gate", "up": "up", "down": "down"}


def _q(w, mode, group_size, ctx):
    return quantize(w, mode, group_size, ctx)


def make_llama_model(config: ModelConfig, seed: int = 0, mode: str = "perChannel", group_size: int = 32,
                     std: float = 0.02, ctx: Optional[Context] = None,
                     keep_float: bool = False, shard: Optional[tuple] = None) -> ModelWeights:
    """LLaMA-shaped decoder with N(0, std) weights drawn in the documented order.

    shard=(rank, world) keeps only that tensor-parallel rank's slice of every
    layer projection (the draws are the same; the model's .tp says so)."""
    ctx = ctx or Context.default()
    g = SeededGenerator(seed)
    H, I, V, kvd = config.hidden_dim, config.intermediate_dim, config.vocab_size, config.kv_dim
    emb = g.normal((V, H), 0.0, std)
    floats = {}
    layers = []
    for li in range(config.num_layers):
        proj = {}
        for name, shape in (("q", (H, H)), ("k", (H, kvd)), ("v", (H, kvd)), ("o", (H, H)),
                            ("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
            w = g.normal(shape, 0.0, std)
            if keep_float:
                floats[(li, name)] = w
            lw = LinearLayerWeights(_q(w, mode, group_size, ctx))
            if shard and shard[1] > 1:
                lw = shard_linear(lw, TP_AXIS[_FIELD[name]], shard[0], shard[1])
            proj[name] = lw
        ones = np.ones(H, dtype=np.float32)
        layers.append(TransformerLayerWeights(query=proj["q"], key=proj["k"], value=proj["v"], output=proj["o"],
                                              gate=proj["gate"], up=proj["up"], down=proj["down"],
                                              input_norm=ones, post_attention_norm=ones.copy()))
    wout = g.normal((H, V), 0.0, std)
    if keep_float:
        floats[("out",)] = wout
    model = ModelWeights(config, emb, layers, LinearLayerWeights(_q(wout, mode, group_size, ctx)),
                         final_norm=np.ones(H, dtype=np.float32))
    if keep_float:
        model.float_weights = floats
    if shard and shard[1] > 1:
        model.tp = tuple(shard)
    return model


def make_toy_model(config: Optional[ModelConfig] = None, seed: int = 42,
                   ctx: Optional[Context] = None) -> ModelWeights:
    """ModelWeights.makeToyModel (ModelWeights.swift:171-244), INT8 per-channel."""
    ctx = ctx or Context.default()
    config = config or ModelConfig(**TOY)
    g = SeededGenerator(seed)
    H, V, kvd = config.hidden_dim, config.vocab_size, config.kv_dim
    F = 4 * H
    emb = g.normal((V, H), 0.0, 0.02)

    def proj(n_in, n_out):
        w = g.normal((n_in, n_out), 0.0, 0.02)
        b = g.normal((n_out,), 0.0, 0.02)
        return LinearLayerWeights(_q(w, "perChannel", 32, ctx), b)

    layers = []
    for _ in range(config.num_layers):
        q, k, v, o = proj(H, H), proj(H, kvd), proj(H, kvd), proj(H, H)
        up = proj(H, F)
        down = proj(F, H)
        layers.append(TransformerLayerWeights(query=q, key=k, value=v, output=o, up=up, down=down))
    wout = g.normal((H, V), 0.0, 0.02)
    out = LinearLayerWeights(_q(wout, "perChannel", 32, ctx), np.zeros(V, dtype=np.float32))
    cfg = ModelConfig(config.num_layers, H, config.num_heads, V, config.max_seq_len, config.num_kv_heads, F,
                      "toy")
    return ModelWeights(cfg, emb, layers, out, final_norm=None)


def random_prompt(n: int, vocab: int, seed: int) -> list:
    """Uniform token ids in [0, vocab) from the same LCG (upper bits of next())."""
    s = SeededGenerator(seed)
    # draw uniform floats from the generator's normal stream's uniform source:
    # reuse the LCG directly for integers
    st = int(s.state.value)
    out = []
    a = 6364136223846793005
    for _ in range(n):
        st = (a * st + 1) & 0xFFFFFFFFFFFFFFFF
        out.append(int(((st >> 32) * vocab) >> 32))
    return out
