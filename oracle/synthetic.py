"""Seeded synthetic models built by the oracle alone (TEST INFRASTRUCTURE).

The benchmark configurations use random-init LLaMA-shaped models drawn with
the reference's SeededGenerator + Tensor.random (ModelWeights.swift:18-29,
Tensor.swift:1623-1644) in a fixed order: token embeddings [vocab, hidden];
per layer q, k, v, o, gate, up, down (each [in, out]); then the output
projection; unit norm weights, no biases.  Quantized with the oracle's
restatement of the reference quantizers (QuantizedTensor.swift:379-424,
502-560).  These builders use only oracle/libtb_oracle.so, so the CPU
reference arm of bench.py and the fixture scripts never load the product
library; tinybrain_b200.synthetic draws the same values on the product side.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from . import _p, load, quantize_int4_group, quantize_int8_per_channel

TINYLLAMA = dict(num_layers=22, hidden_dim=2048, num_heads=32, num_kv_heads=4, vocab_size=32000,
                 intermediate_dim=5632, max_seq_len=2048)
LLAMA2_7B = dict(num_layers=32, hidden_dim=4096, num_heads=32, num_kv_heads=32, vocab_size=32000,
                 intermediate_dim=11008, max_seq_len=2048)


class Generator:
    """SeededGenerator (ModelWeights.swift:18-29) driving Tensor.random."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(load().orc_rng_seed(C.c_uint64(seed)))

    def normal(self, shape, mean=0.0, std=1.0):
        n = int(np.prod(shape))
        out = np.empty(n, dtype=np.float32)
        load().orc_rng_fill_normal(C.byref(self.state), C.c_float(mean), C.c_float(std), n, _p(out))
        return out.reshape(shape)


@dataclass
class Config:
    num_layers: int
    hidden_dim: int
    num_heads: int
    vocab_size: int
    max_seq_len: int
    num_kv_heads: int
    intermediate_dim: int
    architecture: str = "llama"
    rms_eps: float = 1e-5

    @property
    def kv_dim(self):
        return self.hidden_dim // self.num_heads * self.num_kv_heads


@dataclass
class QTensor:
    shape: tuple
    data: np.ndarray
    scales: np.ndarray
    mode: str = "perChannel"
    group_size: int = 32
    zero_points: Optional[np.ndarray] = None

    @property
    def precision(self):
        return 4 if self.mode == "int4" else 8


@dataclass
class Linear:
    weights: QTensor
    bias: Optional[np.ndarray] = None


@dataclass
class Layer:
    query: Linear
    key: Linear
    value: Linear
    output: Linear
    gate: Optional[Linear]
    up: Linear
    down: Linear
    input_norm: Optional[np.ndarray] = None
    post_attention_norm: Optional[np.ndarray] = None


@dataclass
class Model:
    config: Config
    token_embeddings: np.ndarray
    layers: List[Layer]
    output: Linear
    final_norm: Optional[np.ndarray] = None
    extra: dict = field(default_factory=dict)


def quantize(w, mode="perChannel", group_size=32):
    if mode == "perChannel":
        q, s = quantize_int8_per_channel(w)
        return QTensor(tuple(w.shape), q, s, "perChannel", 0, None)
    p, s, z = quantize_int4_group(w, group_size)
    return QTensor(tuple(w.shape), p, s, "int4", group_size, z)


def llama_model(cfg: dict, seed=0, mode="perChannel", group_size=32, std=0.02) -> Model:
    c = Config(**cfg)
    g = Generator(seed)
    H, I, V, kvd = c.hidden_dim, c.intermediate_dim, c.vocab_size, c.kv_dim
    emb = g.normal((V, H), 0.0, std)
    layers = []
    for _ in range(c.num_layers):
        p = {}
        for name, shape in (("q", (H, H)), ("k", (H, kvd)), ("v", (H, kvd)), ("o", (H, H)),
                            ("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
            p[name] = Linear(quantize(g.normal(shape, 0.0, std), mode, group_size))
        ones = np.ones(H, dtype=np.float32)
        layers.append(Layer(p["q"], p["k"], p["v"], p["o"], p["gate"], p["up"], p["down"], ones, ones.copy()))
    out = Linear(quantize(g.normal((H, V), 0.0, std), mode, group_size))
    return Model(c, emb, layers, out, final_norm=np.ones(H, dtype=np.float32))


def random_prompt(n: int, vocab: int, seed: int) -> list:
    """Uniform ids in [0, vocab): (upper 32 bits of next()) * vocab >> 32 over
    the same LCG (seed 0 -> 0xdeadbeef)."""
    st = seed if seed != 0 else 0xDEADBEEF
    out = []
    a = 6364136223846793005
    for _ in range(n):
        st = (a * st + 1) & 0xFFFFFFFFFFFFFFFF
        out.append(int(((st >> 32) * vocab) >> 32))
    return out
