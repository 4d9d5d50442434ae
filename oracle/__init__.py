"""ctypes wrapper of the CPU oracle (oracle/libtb_oracle.so).

TEST INFRASTRUCTURE ONLY.  The oracle restates the reference's Swift CPU path
(see tb_oracle.c for the file:line each function follows) and is used solely
by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm as the checker.  The product (tinybrain_b200) never imports it.

Parity pinning: the reference cannot be built on Linux (Swift + Accelerate +
Metal), so the oracle is pinned by the known-answer tests found in the
reference's own test files (tests/golden/reference_kats.json); numeric parity
beyond those KATs is unpinned at the Accelerate sgemm boundary.
"""
import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtb_oracle.so")
_lib = None


def build():
    subprocess.check_call(["make", "-s", "-C", _HERE])
    return LIB_PATH


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    lib = C.CDLL(LIB_PATH)
    P, I64, I32, F = C.c_void_p, C.c_int64, C.c_int32, C.c_float
    sig = {
        "orc_quantize_int8_per_channel": ([P, I64, I64, P, P], None),
        "orc_quantize_int4_group": ([P, I64, I64, P, P, P], None),
        "orc_dequantize_int8_per_channel": ([P, P, P, I64, I64, P], None),
        "orc_dequantize_int4_group": ([P, P, P, I64, I64, P], None),
        "orc_qmatmul": ([P, I64, P, P, C.c_int], None),
        "orc_rmsnorm": ([P, P, I64, F, P], None),
        "orc_silu": ([F], F),
        "orc_gelu": ([F], F),
        "orc_softmax": ([P, I64, P], None),
        "orc_rope": ([P, I64, I64, I64, I64], None),
        "orc_attention": ([P, P, P, I64, I64, I64, I64, P, P], None),
        "orc_greedy": ([P, I64], I64),
        "orc_model_create": ([P], P),
        "orc_model_free": ([P], None),
        "orc_model_set_embedding": ([P, P], None),
        "orc_model_set_final_norm": ([P, P], None),
        "orc_model_set_output": ([P, P, P], None),
        "orc_model_set_layer_norms": ([P, I64, P, P], None),
        "orc_model_set_proj": ([P, I64, I32, P, P], None),
        "orc_runner_create": ([P, I32, I32], P),
        "orc_runner_free": ([P], None),
        "orc_runner_reset": ([P], None),
        "orc_runner_step": ([P, I64, P], None),
        "orc_runner_set_observer": ([P, P, P, I64, P], None),
        "orc_runner_position": ([P], I64),
        "orc_runner_kv_length": ([P], I64),
        "orc_runner_max_pages": ([P], I64),
        "orc_runner_page_status": ([P, I64, P], None),
        "orc_generate_greedy": ([P, P, I64, I64, P, P], I64),
        "orc_lcg_next": ([P], C.c_uint64),
        "orc_perplexity": ([P, P, I64, P], C.c_float),
        "orc_sample_detailed": ([P, I64, P, P, I64, P, P, P], I64),
        "orc_generate_sampled": ([P, P, I64, I64, P, P, P, P, P], I64),
        "orc_runner_prefill": ([P, P, I64], None),
        "orc_runner_fill_context": ([P, I64, C.c_uint64], None),
        "orc_rng_seed": ([C.c_uint64], C.c_uint64),
        "orc_rng_fill_normal": ([P, F, F, I64, P], None),
        "orc_set_threads": ([I32], None),
        "orc_get_threads": ([], I32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class _QT(C.Structure):
    _fields_ = [("precision", C.c_int32), ("K", C.c_int64), ("N", C.c_int64), ("group_size", C.c_int64),
                ("data", C.c_void_p), ("scales", C.c_void_p), ("zero_points", C.c_void_p)]


class _Cfg(C.Structure):
    _fields_ = [("num_layers", C.c_int64), ("hidden", C.c_int64), ("num_heads", C.c_int64),
                ("num_kv_heads", C.c_int64), ("vocab", C.c_int64), ("max_seq_len", C.c_int64),
                ("intermediate", C.c_int64), ("arch", C.c_int32), ("rms_eps", C.c_float)]


def set_threads(n):
    load().orc_set_threads(int(n))


def get_threads():
    return load().orc_get_threads()


def quantize_int8_per_channel(w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    K, N = w.shape
    q = np.empty(K * N, dtype=np.int8)
    s = np.empty(N, dtype=np.float32)
    load().orc_quantize_int8_per_channel(_p(w), K, N, _p(q), _p(s))
    return q, s


def quantize_int4_group(x, group_size=32):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    cnt = x.size
    ng = (cnt + group_size - 1) // group_size
    p = np.zeros((cnt + 1) // 2, dtype=np.uint8)
    s = np.empty(ng, dtype=np.float32)
    z = np.empty(ng, dtype=np.int8)
    load().orc_quantize_int4_group(_p(x), cnt, group_size, _p(p), _p(s), _p(z))
    return p, s, z


def dequantize(qt):
    K, N = qt.shape
    out = np.empty(K * N, dtype=np.float32)
    if qt.precision == 8:
        load().orc_dequantize_int8_per_channel(_p(qt.data), _p(qt.scales), _p(qt.zero_points), K, N, _p(out))
    else:
        load().orc_dequantize_int4_group(_p(qt.data), _p(qt.scales), _p(qt.zero_points), K * N,
                                         qt.group_size, _p(out))
    return out.reshape(K, N)


def _qt_struct(qt):
    s = _QT()
    s.precision = qt.precision
    s.K, s.N = qt.shape
    s.group_size = qt.group_size or 1
    s.data = qt.data.ctypes.data
    s.scales = qt.scales.ctypes.data
    s.zero_points = None if qt.zero_points is None else qt.zero_points.ctypes.data
    return s


def qmatmul(x, qt, mode=1):
    """mode 0: reference-faithful fp32 (dequantize + sequential sum); mode 1: fp64 accumulation."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    M = x.shape[0]
    y = np.empty((M, qt.shape[1]), dtype=np.float32)
    s = _qt_struct(qt)
    load().orc_qmatmul(_p(x), M, C.byref(s), _p(y), mode)
    return y


def rmsnorm(x, w, eps=1e-5):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    load().orc_rmsnorm(_p(x), _p(w), x.size, C.c_float(eps), _p(y))
    return y


def softmax(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    load().orc_softmax(_p(x), x.size, _p(y))
    return y


def silu(x):
    return load().orc_silu(C.c_float(x))


def gelu(x):
    return load().orc_gelu(C.c_float(x))


def rope(v, head_dim, num_heads, position, rotary_dims=None):
    v = np.array(v, dtype=np.float32)
    load().orc_rope(_p(v), head_dim, num_heads, position, rotary_dims or head_dim)
    return v


def attention(q, K, V, H, Hkv, d, want_probs=False):
    q = np.ascontiguousarray(q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    L = K.shape[0]
    ctx = np.empty(H * d, dtype=np.float32)
    probs = np.empty(H * L, dtype=np.float32) if want_probs else None
    load().orc_attention(_p(q), _p(K), _p(V), L, H, Hkv, d, _p(ctx), _p(probs))
    return (ctx, probs) if want_probs else ctx


class _Sampler(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int32), ("has_top_p", C.c_int32),
                ("top_p", C.c_float), ("repetition_penalty", C.c_float)]


def _sampler(cfg):
    """orc_sampler from an object with temperature, top_k, top_p, repetition_penalty."""
    return _Sampler(float(cfg.temperature), int(cfg.top_k or 0), 0 if cfg.top_p is None else 1,
                    float(cfg.top_p or 0.0), float(cfg.repetition_penalty))


def sample_detailed(logits, cfg, history, rng_state):
    """Sampler.sampleDetailed (Sampler.swift:401-473): (token, probability,
    entropy, next rng state)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    hist = np.ascontiguousarray(np.asarray(history, dtype=np.int64))
    st = C.c_uint64(rng_state)
    pr, en = C.c_float(0), C.c_float(0)
    sc = _sampler(cfg)
    tok = load().orc_sample_detailed(_p(logits), logits.size, C.byref(sc), _p(hist) if hist.size else None,
                                     hist.size, C.byref(st), C.byref(pr), C.byref(en))
    return int(tok), float(pr.value), float(en.value), int(st.value)


def greedy(logits):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    return int(load().orc_greedy(_p(logits), logits.size))


_PROJ = ("query", "key", "value", "output", "gate", "up", "down")


class OracleModel:
    """CPU restatement of ModelRunner over the same host weights (borrowed)."""

    def __init__(self, weights, mode=1, threads=0):
        lib = load()
        c = weights.config
        cfg = _Cfg(c.num_layers, c.hidden_dim, c.num_heads, c.num_kv_heads, c.vocab_size, c.max_seq_len,
                   c.intermediate_dim, 1 if c.architecture == "toy" else 0, c.rms_eps)
        self._keep = [weights]
        self._structs = []
        self.m = lib.orc_model_create(C.byref(cfg))
        self.emb = np.ascontiguousarray(weights.token_embeddings, dtype=np.float32)
        lib.orc_model_set_embedding(self.m, _p(self.emb))
        if weights.final_norm is not None:
            self.fn = np.ascontiguousarray(weights.final_norm, dtype=np.float32)
            lib.orc_model_set_final_norm(self.m, _p(self.fn))
        for li, ly in enumerate(weights.layers):
            lib.orc_model_set_layer_norms(self.m, li, _p(ly.input_norm), _p(ly.post_attention_norm))
            for wi, name in enumerate(_PROJ):
                lw = getattr(ly, name)
                if lw is None:
                    continue
                s = _qt_struct(lw.weights)
                self._structs.append(s)
                lib.orc_model_set_proj(self.m, li, wi, C.byref(s), _p(lw.bias))
        s = _qt_struct(weights.output.weights)
        self._structs.append(s)
        lib.orc_model_set_output(self.m, C.byref(s), _p(weights.output.bias))
        self.r = lib.orc_runner_create(self.m, mode, threads)
        self.vocab = c.vocab_size
        self.cfg = c

    def step(self, token):
        logits = np.empty(self.vocab, dtype=np.float32)
        load().orc_runner_step(self.r, int(token), _p(logits))
        return logits

    def prefill(self, tokens):
        """Steps every token of `tokens`, discarding the logits (chunked; the
        same results as stepping one token at a time)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64))
        load().orc_runner_prefill(self.r, _p(t), t.size)

    def fill_context(self, length, seed=1):
        """Position `length` with synthetic KV rows (benchmark samples: the
        next step costs what a decode step at that context costs)."""
        load().orc_runner_fill_context(self.r, int(length), seed)

    def step_observed(self, token):
        """step() plus the InferenceObserver values of this step:
        (logits, layer-entry norms [layers], attention weights per layer
        [layers][heads * L], final hidden state [hidden])."""
        c = self.cfg
        L = self.position + 1
        norms = np.empty(c.num_layers, dtype=np.float32)
        attn = np.empty((c.num_layers, c.num_heads * L), dtype=np.float32)
        fin = np.empty(c.hidden_dim, dtype=np.float32)
        lib = load()
        lib.orc_runner_set_observer(self.r, _p(norms), _p(attn), c.num_heads * L, _p(fin))
        try:
            logits = self.step(token)
        finally:
            lib.orc_runner_set_observer(self.r, None, None, 0, None)
        return logits, norms, attn, fin

    def reset(self):
        load().orc_runner_reset(self.r)

    @property
    def position(self):
        return load().orc_runner_position(self.r)

    @property
    def kv_length(self):
        return load().orc_runner_kv_length(self.r)

    def page_status(self, layer=0):
        n = load().orc_runner_max_pages(self.r)
        st = np.zeros(n, dtype=np.uint8)
        load().orc_runner_page_status(self.r, layer, _p(st))
        return [bool(x) for x in st]

    def generate_greedy(self, prompt, max_tokens):
        pr = np.ascontiguousarray(np.asarray(prompt, dtype=np.int64))
        out = np.zeros(max(1, max_tokens), dtype=np.int64)
        gap = np.zeros(max(1, max_tokens), dtype=np.float32)
        load().orc_generate_greedy(self.r, _p(pr), pr.size, max_tokens, _p(out), _p(gap))
        return out[:max_tokens].tolist(), gap[:max_tokens]

    def perplexity(self, tokens):
        """PerplexityHarness.computePerplexity from the current state (reset first):
        (perplexity, sum of log-probabilities)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64))
        s = C.c_double(0)
        ppl = load().orc_perplexity(self.r, _p(t), t.size, C.byref(s))
        return float(ppl), s.value

    def generate_sampled(self, prompt, max_tokens, cfg, seed):
        """generateStream with Sampler.sampleDetailed: (tokens, probabilities, entropies)."""
        pr = np.ascontiguousarray(np.asarray(prompt, dtype=np.int64))
        out = np.zeros(max(1, max_tokens), dtype=np.int64)
        prob = np.zeros(max(1, max_tokens), dtype=np.float32)
        ent = np.zeros(max(1, max_tokens), dtype=np.float32)
        st = C.c_uint64(seed)
        sc = _sampler(cfg)
        load().orc_generate_sampled(self.r, _p(pr), pr.size, max_tokens, C.byref(sc), C.byref(st), _p(out),
                                    _p(prob), _p(ent))
        return out[:max_tokens].tolist(), prob[:max_tokens], ent[:max_tokens]

    def __del__(self):
        try:
            lib = load()
            lib.orc_runner_free(self.r)
            lib.orc_model_free(self.m)
        except Exception:
            pass
