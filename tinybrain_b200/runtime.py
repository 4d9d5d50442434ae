"""Host-side mirror of TinyBrain's runtime API over libtinybrain_cuda.

Names and argument meanings follow the reference's Swift API
(Sources/TinyBrainRuntime): ModelConfig (ModelRunner.swift:27-121),
QuantizedTensor / Tensor.quantize (QuantizedTensor.swift:31-165, 359-560),
LinearLayerWeights / ModelWeights (ModelWeights.swift:32-244), ModelRunner
(ModelRunner.swift:127-298), KVCache.length / pageAllocationStatus
(KVCache.swift:138-356), SamplerConfig / GenerationConfig / TokenOutput
(Sampler.swift:46-104, GenerationConfig.swift:35-219).

Every numeric result comes from the CUDA library; nothing here computes a
projection, an attention or a sample on the CPU.  Unsupported requests
(e.g. stochastic sampling, which the device sampler does not implement yet)
raise instead of falling back.
"""
from __future__ import annotations

import atexit
import ctypes as C
import time
import weakref
from dataclasses import dataclass, field
from typing import Iterator, List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import QTensorDesc, TinyBrainError, call

ARCH_LLAMA, ARCH_TOY = 0, 1
PROJ_Q, PROJ_K, PROJ_V, PROJ_O, PROJ_GATE, PROJ_UP, PROJ_DOWN = range(7)


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# Live handles, released children-first when the interpreter exits so no CUDA
# object outlives its context or the CUDA runtime.
_LIVE = {"runner": weakref.WeakSet(), "model": weakref.WeakSet(), "qweight": weakref.WeakSet(),
         "context": weakref.WeakSet()}


@atexit.register
def _release_all():
    for kind in ("runner", "model", "qweight", "context"):
        for obj in list(_LIVE[kind]):
            try:
                obj.close()
            except Exception:
                pass


# ---------------------------------------------------------------- context --
class Context:
    """A CUDA device context (replaces `TinyBrainBackend.metalBackend = MetalBackend()`)."""

    _default = {}

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        call("tb_context_create", device, C.byref(h))
        self.handle = h
        self.device = device
        _LIVE["context"].add(self)

    @classmethod
    def default(cls, device: int = 0) -> "Context":
        if device not in cls._default:
            cls._default[device] = Context(device)
        return cls._default[device]

    def synchronize(self):
        call("tb_context_synchronize", self.handle)

    def check_device(self):
        call("tb_context_check_device", self.handle)

    def init_tensor_parallel(self, unique_id: bytes, rank: int, world: int):
        """Join the tensor-parallel communicator (`unique_id` from rank 0's
        tp_unique_id(), shared out of band, e.g. a torch.distributed broadcast)."""
        if len(unique_id) != 128:
            raise ValueError("unique_id must be 128 bytes")
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        call("tb_context_init_tp", self.handle, buf, int(rank), int(world))
        self.tp = (int(rank), int(world))

    def close(self):
        if self.handle:
            for kind in ("runner", "model", "qweight"):
                for obj in list(_LIVE[kind]):
                    if getattr(obj, "ctx", None) is self:
                        obj.close()
            _lib.load().tb_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_unique_id() -> bytes:
    """A fresh 128-byte NCCL communicator id (rank 0 draws it)."""
    buf = (C.c_uint8 * 128)()
    call("tb_tp_unique_id", buf)
    return bytes(buf)


def device_count() -> int:
    n = C.c_int32(0)
    st = _lib.load().tb_device_count(C.byref(n))
    return n.value if st == 0 else 0


# ------------------------------------------------------------- RNG / data --
class SeededGenerator:
    """ModelWeights.swift:18-29 LCG (seed 0 -> 0xdeadbeef) used by Tensor.random."""

    def __init__(self, seed: int):
        s = C.c_uint64(0)
        call("tb_rng_seed_state", C.c_uint64(seed), C.byref(s))
        self.state = s

    def normal(self, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
        """Tensor.random(shape:mean:std:using:) (Tensor.swift:1623-1644)."""
        n = int(np.prod(shape))
        out = np.empty(n, dtype=np.float32)
        call("tb_rng_fill_normal", C.byref(self.state), C.c_float(mean), C.c_float(std), n, _ptr(out))
        return out.reshape(shape)


# ------------------------------------------------------------ quantization --
@dataclass
class QuantizedTensor:
    """QuantizedTensor (QuantizedTensor.swift:62-165) in the reference layout.

    shape = (K in_features, N out_features), row-major, y = x @ dequant(W).
    mode 'perChannel': data int8 [K*N], scales [N].
    mode 'int4': data uint8 packed [ceil(K*N/2)] (even flat index = high
    nibble), scales / zero_points [ceil(K*N/group_size)].
    """

    shape: tuple
    data: np.ndarray
    scales: np.ndarray
    mode: str = "perChannel"
    group_size: int = 32
    zero_points: Optional[np.ndarray] = None

    @property
    def precision(self) -> int:
        return 4 if self.mode == "int4" else 8

    def desc(self) -> QTensorDesc:
        d = QTensorDesc()
        d.precision = self.precision
        d.in_features, d.out_features = int(self.shape[0]), int(self.shape[1])
        d.group_size = int(self.group_size)
        d.data = self.data.ctypes.data_as(C.c_void_p)
        d.data_bytes = self.data.nbytes
        d.scales = self.scales.ctypes.data_as(C.c_void_p)
        d.num_scales = self.scales.size
        if self.zero_points is not None:
            d.zero_points = self.zero_points.ctypes.data_as(C.c_void_p)
            d.num_zero_points = self.zero_points.size
        return d

    def dequantize(self, ctx: Optional[Context] = None) -> np.ndarray:
        """QuantizedTensor.dequantize (QuantizedTensor.swift:182-285) on the
        device: fp32 [K, N] = (q - zero_point) * scale."""
        ctx = ctx or Context.default()
        out = np.empty(self.shape, dtype=np.float32)
        d = self.desc()
        call("tb_dequantize", ctx.handle, C.byref(d), _ptr(out))
        return out

    def to_int4(self, group_size: int = 32, ctx: Optional[Context] = None) -> "QuantizedTensor":
        """dequantize() then quantize(mode='int4') in one device pass
        (the per-weight step of PerplexityHarness.convertToINT4)."""
        ctx = ctx or Context.default()
        cnt = int(self.shape[0]) * int(self.shape[1])
        ng = (cnt + group_size - 1) // group_size
        p = np.empty((cnt + 1) // 2, dtype=np.uint8)
        sc = np.empty(ng, dtype=np.float32)
        z = np.empty(ng, dtype=np.int8)
        d = self.desc()
        call("tb_requantize_int4", ctx.handle, C.byref(d), int(group_size), _ptr(p), _ptr(sc), _ptr(z))
        return QuantizedTensor(tuple(self.shape), p, sc, "int4", group_size, z)


def quantize(w: np.ndarray, mode: str = "perChannel", group_size: int = 32,
             ctx: Optional[Context] = None) -> QuantizedTensor:
    """Tensor.quantize(mode:groupSize:) (QuantizedTensor.swift:359-372) on the GPU."""
    ctx = ctx or Context.default()
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("quantize expects a 2-D [in, out] weight")
    K, N = w.shape
    if mode == "perChannel":
        q = np.empty(K * N, dtype=np.int8)
        s = np.empty(N, dtype=np.float32)
        call("tb_quantize_int8_per_channel", ctx.handle, _ptr(w), K, N, _ptr(q), _ptr(s))
        return QuantizedTensor((K, N), q, s, "perChannel", 0, None)
    if mode == "int4":
        cnt = K * N
        ng = (cnt + group_size - 1) // group_size
        p = np.empty((cnt + 1) // 2, dtype=np.uint8)
        s = np.empty(ng, dtype=np.float32)
        z = np.empty(ng, dtype=np.int8)
        call("tb_quantize_int4_group", ctx.handle, _ptr(w), cnt, group_size, _ptr(p), _ptr(s), _ptr(z))
        return QuantizedTensor((K, N), p, s, "int4", group_size, z)
    raise TinyBrainError(4, f"quantization mode {mode!r} is not on the decode path")


def _unpack_nibbles(q: "QuantizedTensor") -> np.ndarray:
    n = q.shape[0] * q.shape[1]
    nib = np.empty(2 * q.data.size, dtype=np.uint8)
    nib[0::2] = q.data >> 4
    nib[1::2] = q.data & 0x0F
    return nib[:n]


def _pack_nibbles(nib: np.ndarray) -> np.ndarray:
    if nib.size % 2:
        nib = np.concatenate([nib, np.zeros(1, dtype=np.uint8)])
    return ((nib[0::2] << 4) | nib[1::2]).astype(np.uint8)


def shard_quantized(q: QuantizedTensor, axis: int, rank: int, world: int) -> QuantizedTensor:
    """Slice of a quantized [in, out] weight for tensor-parallel rank `rank`:
    axis 1 = a column shard (out features), axis 0 = a row shard (in features).

    The slice is taken from the quantized bytes, so every kept element,
    scale and zero point is bit-identical to the unsharded tensor.  INT4
    groups run along the out dimension of the row-major [in][out] data
    (QuantizedTensor.swift:502-560, groups of consecutive flat elements):
    a shard must cut whole groups."""
    K, N = q.shape
    if axis not in (0, 1):
        raise ValueError("axis must be 0 (rows) or 1 (columns)")
    D = N if axis == 1 else K
    if D % world:
        raise ValueError(f"dimension {D} does not split over {world} ranks")
    w = D // world
    a, b = rank * w, (rank + 1) * w
    if q.mode == "perChannel":
        m = q.data.reshape(K, N)
        if axis == 1:
            return QuantizedTensor((K, w), np.ascontiguousarray(m[:, a:b]).ravel(),
                                   np.ascontiguousarray(q.scales[a:b]), q.mode, q.group_size, None)
        return QuantizedTensor((w, N), np.ascontiguousarray(m[a:b]).ravel(), q.scales.copy(), q.mode,
                               q.group_size, None)
    if q.mode != "int4":
        raise TinyBrainError(4, f"cannot shard mode {q.mode!r}")
    gs = q.group_size
    if N % gs or (axis == 1 and w % gs):
        raise ValueError(f"INT4 shard must cut whole groups of {gs} out features")
    nib = _unpack_nibbles(q).reshape(K, N)
    sc = q.scales[:K * N // gs].reshape(K, N // gs)
    zp = q.zero_points[:K * N // gs].reshape(K, N // gs)
    if axis == 1:
        nb, s2, z2, shape = nib[:, a:b], sc[:, a // gs:b // gs], zp[:, a // gs:b // gs], (K, w)
    else:
        nb, s2, z2, shape = nib[a:b], sc[a:b], zp[a:b], (w, N)
    return QuantizedTensor(shape, _pack_nibbles(np.ascontiguousarray(nb).ravel()),
                           np.ascontiguousarray(s2).ravel(), "int4", gs, np.ascontiguousarray(z2).ravel())


class QuantizedWeight:
    """A quantized weight resident in HBM (cachedQuantizedBuffers replacement)."""

    def __init__(self, q: QuantizedTensor, ctx: Optional[Context] = None):
        self.ctx = ctx or Context.default()
        self.q = q
        h = C.c_void_p()
        d = q.desc()
        call("tb_qweight_upload", self.ctx.handle, C.byref(d), C.byref(h))
        self.handle = h
        _LIVE["qweight"].add(self)

    def matmul(self, x: np.ndarray) -> np.ndarray:
        """QuantizedMatMulBackend.matmulQuantized (Backend.swift:173-175)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x[None, :]
        M = x.shape[0]
        y = np.empty((M, self.q.shape[1]), dtype=np.float32)
        call("tb_matmul_quantized", self.ctx.handle, _ptr(x), M, self.handle, _ptr(y))
        return y

    def close(self):
        if self.handle:
            _lib.load().tb_qweight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemv_stream_time(weights: Sequence["QuantizedWeight"], x_dev: int, M: int, y_dev: int, reps: int = 20,
                     pdl: bool = True) -> float:
    """Milliseconds per pass of one GEMV per weight (device pointers x [M][K],
    y [M][max N]); the single-GEMV HBM measurement of BASELINE config 1.
    pdl: 0 / False stream order, 1 / True dependent chain, 2 independent
    (overlapping) GEMVs."""
    if not weights:
        raise ValueError("no weights")
    ctx = weights[0].ctx
    arr = (C.c_void_p * len(weights))(*[w.handle for w in weights])
    ms = C.c_float(0.0)
    call("tb_qgemv_stream_time", ctx.handle, arr, len(weights), C.c_void_p(x_dev), M, C.c_void_p(y_dev), reps,
         int(pdl), C.byref(ms))
    return float(ms.value)


def attention_decode(q, keys, values, num_heads, num_kv_heads, head_dim, ctx=None) -> np.ndarray:
    """Single-query decode attention (ModelRunner.swift:519-579 semantics)."""
    ctx = ctx or Context.default()
    q = np.ascontiguousarray(q, dtype=np.float32)
    keys = np.ascontiguousarray(keys, dtype=np.float32)
    values = np.ascontiguousarray(values, dtype=np.float32)
    L = keys.shape[0]
    out = np.empty(num_heads * head_dim, dtype=np.float32)
    call("tb_attention_decode", ctx.handle, _ptr(q), _ptr(keys), _ptr(values), L, num_heads, num_kv_heads,
         head_dim, _ptr(out))
    return out


# ------------------------------------------------------------------ model --
@dataclass
class ModelConfig:
    """ModelConfig (ModelRunner.swift:27-121)."""

    num_layers: int
    hidden_dim: int
    num_heads: int
    vocab_size: int
    max_seq_len: int = 2048
    num_kv_heads: Optional[int] = None
    intermediate_dim: Optional[int] = None
    architecture: str = "llama"
    rms_eps: float = 1e-5

    def __post_init__(self):
        if self.num_kv_heads is None:
            self.num_kv_heads = self.num_heads
        if self.intermediate_dim is None:
            self.intermediate_dim = 4 * self.hidden_dim

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.num_heads

    @property
    def kv_dim(self) -> int:
        return self.head_dim * self.num_kv_heads

    def to_c(self) -> _lib.ModelConfigC:
        c = _lib.ModelConfigC()
        c.num_layers, c.hidden_dim, c.num_heads = self.num_layers, self.hidden_dim, self.num_heads
        c.num_kv_heads, c.vocab_size, c.max_seq_len = self.num_kv_heads, self.vocab_size, self.max_seq_len
        c.intermediate_dim = self.intermediate_dim
        c.architecture = ARCH_TOY if self.architecture == "toy" else ARCH_LLAMA
        c.rms_eps = self.rms_eps
        return c


@dataclass
class LinearLayerWeights:
    """LinearLayerWeights (ModelWeights.swift:32-69): quantized weight + optional bias."""

    weights: QuantizedTensor
    bias: Optional[np.ndarray] = None


@dataclass
class TransformerLayerWeights:
    """TransformerLayerWeights (ModelWeights.swift:98-134)."""

    query: LinearLayerWeights
    key: LinearLayerWeights
    value: LinearLayerWeights
    output: LinearLayerWeights
    up: LinearLayerWeights
    down: LinearLayerWeights
    gate: Optional[LinearLayerWeights] = None
    input_norm: Optional[np.ndarray] = None
    post_attention_norm: Optional[np.ndarray] = None


@dataclass
class ModelWeights:
    """ModelWeights (ModelWeights.swift:137-168)."""

    config: ModelConfig
    token_embeddings: np.ndarray  # [vocab, hidden] fp32
    layers: List[TransformerLayerWeights]
    output: LinearLayerWeights
    final_norm: Optional[np.ndarray] = None

    def upload(self, ctx: Optional[Context] = None, tp: Optional[tuple] = None) -> "DeviceModel":
        return DeviceModel(self, ctx, tp)

    @staticmethod
    def load(path: str, int4_layout: str = "runtime", ctx: Optional["Context"] = None) -> "ModelWeights":
        """ModelWeights.load(from:) -- a .tbf file (ModelWeights.swift:496-798).
        int4_layout: what to do with INT4 tensors of a file written by
        Scripts/convert_model.py (see tbf.load)."""
        from . import tbf
        return tbf.load(path, int4_layout=int4_layout, ctx=ctx)

    def save(self, path: str) -> None:
        """ModelWeights.save(to:) -- a .tbf file (ModelWeights.swift:260-490)."""
        from . import tbf
        tbf.save(self, path)


# Which axis of each projection a tensor-parallel rank keeps: 1 = column
# shard (heads / intermediate rows), 0 = row shard (partial sums).
TP_AXIS = {"query": 1, "key": 1, "value": 1, "gate": 1, "up": 1, "output": 0, "down": 0}


def convert_to_int4(weights: "ModelWeights", group_size: int = 32, ctx: Optional[Context] = None
                    ) -> "ModelWeights":
    """PerplexityHarness.convertToINT4 (PerplexityHarness.swift:65-126): every
    linear weight re-quantized to INT4 groups on the device; embeddings, norms
    and biases unchanged."""
    def q4(lw):
        return None if lw is None else LinearLayerWeights(lw.weights.to_int4(group_size, ctx), lw.bias)

    layers = [TransformerLayerWeights(query=q4(ly.query), key=q4(ly.key), value=q4(ly.value), output=q4(ly.output),
                                      up=q4(ly.up), down=q4(ly.down), gate=q4(ly.gate), input_norm=ly.input_norm,
                                      post_attention_norm=ly.post_attention_norm) for ly in weights.layers]
    return ModelWeights(weights.config, weights.token_embeddings, layers, q4(weights.output),
                        final_norm=weights.final_norm)


def shard_linear(lw: "LinearLayerWeights", axis: int, rank: int, world: int) -> "LinearLayerWeights":
    """Tensor-parallel slice of a projection; a row shard's bias stays on rank 0
    (the partial sums of all ranks are added up once)."""
    b = lw.bias
    if b is not None:
        if axis == 1:
            w = b.size // world
            b = np.ascontiguousarray(b[rank * w:(rank + 1) * w])
        elif rank != 0:
            b = None
    return LinearLayerWeights(shard_quantized(lw.weights, axis, rank, world), b)


def shard_layer(ly: "TransformerLayerWeights", rank: int, world: int) -> "TransformerLayerWeights":
    kw = {}
    for name, axis in TP_AXIS.items():
        lw = getattr(ly, name)
        kw[name] = None if lw is None else shard_linear(lw, axis, rank, world)
    return TransformerLayerWeights(input_norm=ly.input_norm, post_attention_norm=ly.post_attention_norm, **kw)


class DeviceModel:
    """ModelWeights uploaded to HBM (fused QKV and gate/up, GPU tile layout).

    tp=(rank, world): this GPU's tensor-parallel shard.  `w` holds either the
    whole model (sliced here) or layers already sharded for this rank
    (w.tp == tp, as make_llama_model(shard=...) builds them); the context
    must have joined the communicator (Context.init_tensor_parallel)."""

    def __init__(self, w: ModelWeights, ctx: Optional[Context] = None, tp: Optional[tuple] = None):
        self.ctx = ctx or Context.default()
        self.config = w.config
        self.tp = tuple(tp) if tp else (0, 1)
        cfg = w.config.to_c()
        h = C.c_void_p()
        call("tb_model_create", self.ctx.handle, C.byref(cfg), C.byref(h))
        self.handle = h
        _LIVE["model"].add(self)
        rank, world = self.tp
        pre_sharded = getattr(w, "tp", (0, 1)) == self.tp and world > 1
        if world > 1:
            call("tb_model_set_tensor_parallel", h, rank, world)
        emb = np.ascontiguousarray(w.token_embeddings, dtype=np.float32)
        call("tb_model_set_embedding", h, _ptr(emb))
        if w.final_norm is not None:
            fn = np.ascontiguousarray(w.final_norm, dtype=np.float32)
            call("tb_model_set_final_norm", h, _ptr(fn))
        for i, ly in enumerate(w.layers):
            if world > 1 and not pre_sharded:
                ly = shard_layer(ly, rank, world)
            ni = None if ly.input_norm is None else np.ascontiguousarray(ly.input_norm, dtype=np.float32)
            npn = None if ly.post_attention_norm is None else np.ascontiguousarray(ly.post_attention_norm,
                                                                                    dtype=np.float32)
            call("tb_model_set_layer_norms", h, i, _ptr(ni), _ptr(npn))
            for which, lw in ((PROJ_Q, ly.query), (PROJ_K, ly.key), (PROJ_V, ly.value), (PROJ_O, ly.output),
                              (PROJ_GATE, ly.gate), (PROJ_UP, ly.up), (PROJ_DOWN, ly.down)):
                if lw is None:
                    continue
                d = lw.weights.desc()
                b = None if lw.bias is None else np.ascontiguousarray(lw.bias, dtype=np.float32)
                call("tb_model_set_projection", h, i, which, C.byref(d), _ptr(b))
        d = w.output.weights.desc()
        b = None if w.output.bias is None else np.ascontiguousarray(w.output.bias, dtype=np.float32)
        call("tb_model_set_output", h, C.byref(d), _ptr(b))
        call("tb_model_finalize", h)

    @property
    def weight_bytes(self) -> int:
        v = C.c_int64(0)
        call("tb_model_weight_bytes", self.handle, C.byref(v))
        return v.value

    def close(self):
        if self.handle:
            for r in list(_LIVE["runner"]):
                if r.model is self:
                    r.close()
            _lib.load().tb_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- sampling --
@dataclass
class SamplerConfig:
    """SamplerConfig (Sampler.swift:46-104)."""

    temperature: float = 0.7
    top_k: Optional[int] = None
    top_p: Optional[float] = None
    repetition_penalty: float = 1.0
    seed: Optional[int] = None

    def is_greedy(self) -> bool:
        return self.top_k == 1

    def uses_argmax(self) -> bool:
        """top_k = 1 without a penalty draws the argmax: the LM-head epilogue
        decodes it without a sampler launch."""
        return self.top_k == 1 and self.repetition_penalty == 1.0

    def strategy(self) -> str:
        """TokenOutput.strategy text (ModelRunner.swift:262-269)."""
        parts = [f"temp={self.temperature:.2f}"]
        if self.top_k is not None:
            parts.append(f"topK={self.top_k}")
        if self.top_p is not None:
            parts.append(f"topP={self.top_p:.2f}")
        if self.repetition_penalty != 1.0:
            parts.append(f"penalty={self.repetition_penalty:.2f}")
        return ", ".join(parts)

    def to_c(self) -> "_lib.SamplerConfigC":
        return _lib.SamplerConfigC(float(self.temperature), int(self.top_k) if self.top_k is not None else 0,
                                   0 if self.top_p is None else 1, float(self.top_p or 0.0),
                                   float(self.repetition_penalty), 0 if self.seed is None else 1,
                                   int(self.seed or 0) & 0xFFFFFFFFFFFFFFFF)


@dataclass
class GenerationConfig:
    """GenerationConfig (GenerationConfig.swift:35-119)."""

    max_tokens: int = 100
    sampler: SamplerConfig = field(default_factory=SamplerConfig)
    stop_tokens: Sequence[int] = ()


@dataclass
class TokenOutput:
    """TokenOutput (GenerationConfig.swift:149-219)."""

    token_id: int
    probability: float
    entropy: float
    timestamp: float
    strategy: Optional[str] = None


def sample_detailed(logits, sampler: SamplerConfig, history: Sequence[int] = (), rng_state: int = 0,
                    ctx: Optional[Context] = None):
    """Sampler.sampleDetailed (Sampler.swift:401-473) on the device for one
    logits row: (token, probability, entropy, next LCG state)."""
    ctx = ctx or Context.default()
    lg = np.ascontiguousarray(np.asarray(logits, dtype=np.float32).reshape(-1))
    h = np.ascontiguousarray(np.asarray(list(history), dtype=np.int32))
    c = sampler.to_c()
    st = C.c_uint64(int(rng_state) & 0xFFFFFFFFFFFFFFFF)
    tok, pr, en = C.c_int32(0), C.c_float(0), C.c_float(0)
    call("tb_sample_detailed", ctx.handle, _ptr(lg), lg.size, C.byref(c), _ptr(h) if h.size else None, int(h.size),
         C.byref(st), C.byref(tok), C.byref(pr), C.byref(en))
    return tok.value, pr.value, en.value, st.value


def _greedy_topk1_stats():
    # Sampler.sampleDetailed with topK = 1: softmax over one finite logit with
    # the +1e-7 denominator (Tensor.swift:1293), entropy -p*log(p), in fp32.
    p = np.float32(1.0) / (np.float32(1.0) + np.float32(1e-7))
    ent = -p * np.log(p, dtype=np.float32)
    return float(p), float(ent)


@dataclass
class PerplexitySlice:
    """PerplexitySlice (PerplexityHarness.swift:15-46): a pinned, pre-tokenized
    slice; the first token is the BOS id."""

    source: str
    tokenizer: str
    bos_token_id: int
    seed: str
    num_tokens: int
    tokens: List[int]
    notes: str = ""

    @classmethod
    def load(cls, path: str) -> "PerplexitySlice":
        import json
        with open(path) as f:
            d = json.load(f)
        return cls(d["source"], d["tokenizer"], int(d["bos_token_id"]), str(d["seed"]), int(d["num_tokens"]),
                   [int(t) for t in d["tokens"]], d.get("notes", ""))


@dataclass
class PerplexityResult:
    """PerplexityHarness.Result (PerplexityHarness.swift:127-133)."""

    perplexity: float
    num_predictions: int
    elapsed_seconds: float
    sum_log_prob: float = 0.0


def compute_perplexity(weights, tokens, ctx: Optional[Context] = None) -> PerplexityResult:
    """PerplexityHarness.computePerplexity (PerplexityHarness.swift:141-193):
    a fresh runner, teacher-forced over the slice, fp64 log-probabilities
    summed on the device; perplexity = Float(exp(-mean))."""
    toks = tokens.tokens if isinstance(tokens, PerplexitySlice) else list(tokens)
    r = ModelRunner(weights, ctx, max_batch=1, max_positions=max(len(toks), 1))
    try:
        return r.perplexity([toks])[0]
    finally:
        r.close()


class KVCacheView:
    """The runner's KVCache as the reference exposes it (KVCache.swift:138-356)."""

    def __init__(self, runner: "ModelRunner", seq: int = 0):
        self._r, self._seq = weakref.proxy(runner), seq

    @property
    def length(self) -> int:
        v = C.c_int64(0)
        call("tb_runner_kv_length", self._r.handle, self._seq, C.byref(v))
        return v.value

    @property
    def max_pages(self) -> int:
        v = C.c_int64(0)
        call("tb_runner_max_pages", self._r.handle, C.byref(v))
        return v.value

    def page_allocation_status(self, layer: int = 0) -> List[bool]:
        n = self.max_pages
        st = np.zeros(n, dtype=np.uint8)
        call("tb_runner_page_status", self._r.handle, self._seq, _ptr(st), n)
        return [bool(x) for x in st]


class ModelRunner:
    """ModelRunner (ModelRunner.swift:127-298) on one GPU.

    `max_batch` > 1 decodes that many independent sequences together
    (generate_batch); step() drives sequence 0 of a batch-1 runner.
    """

    def __init__(self, weights, ctx: Optional[Context] = None, max_batch: int = 1,
                 max_positions: Optional[int] = None):
        self.model = weights if isinstance(weights, DeviceModel) else DeviceModel(weights, ctx)
        self.ctx = self.model.ctx
        self.config = self.model.config
        self.max_batch = max_batch
        h = C.c_void_p()
        call("tb_runner_create", self.model.handle, max_batch, int(max_positions or self.config.max_seq_len),
             C.byref(h))
        self.handle = h
        _LIVE["runner"].add(self)
        self.kv_cache = KVCacheView(self, 0)
        self.observer = None

    # -- ModelRunner.step / reset / currentPosition --
    def step(self, token_id: int, want_logits: bool = True):
        """One forward step; returns (logits or None, greedy token).  With an
        observer attached (``runner.observer``, the InferenceObserver of
        InferenceObserver.swift:40-84) the step reports its internals through
        the observer's methods, in the reference's order: per layer
        ``did_enter_layer(layer, hidden_state_norm, position)`` and
        ``did_compute_attention(layer, weights, position)`` (weights flattened
        num_heads x L), then ``did_compute_final_hidden_state(hidden, position)``
        (optional method) and ``did_compute_logits(logits, position)``."""
        if self.observer is not None:
            return self._step_observed(int(token_id))
        logits = np.empty(self.config.vocab_size, dtype=np.float32) if want_logits else None
        am = C.c_int32(0)
        call("tb_runner_step", self.handle, int(token_id), _ptr(logits), C.byref(am))
        return logits, am.value

    def _step_observed(self, token_id: int):
        c = self.config
        pos = self.current_position
        L = pos + 1
        logits = np.empty(c.vocab_size, dtype=np.float32)
        norms = np.empty(c.num_layers, dtype=np.float32)
        attn = np.empty((c.num_layers, c.num_heads * L), dtype=np.float32)
        fin = np.empty(c.hidden_dim, dtype=np.float32)
        am = C.c_int32(0)
        call("tb_runner_step_observed", self.handle, token_id, _ptr(logits), C.byref(am), _ptr(norms), _ptr(attn),
             c.num_heads * L, _ptr(fin))
        ob = self.observer
        for layer in range(c.num_layers):
            ob.did_enter_layer(layer, float(norms[layer]), pos)
            ob.did_compute_attention(layer, attn[layer].copy(), pos)
        if hasattr(ob, "did_compute_final_hidden_state"):
            ob.did_compute_final_hidden_state(fin, pos)
        ob.did_compute_logits(logits.copy(), pos)
        return logits, am.value

    def reset(self):
        call("tb_runner_reset", self.handle)

    @property
    def current_position(self) -> int:
        v = C.c_int64(0)
        call("tb_runner_position", self.handle, 0, C.byref(v))
        return v.value

    # -- generation --
    def generate_batch(self, prompts: Sequence[Sequence[int]], max_new_tokens: int,
                       stop_tokens: Sequence[int] = (), callback=None) -> List[List[int]]:
        """Greedy generation for independent sequences (generateStream semantics each)."""
        n = len(prompts)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.int64) for p in prompts])
                                    .astype(np.int32) if n and sum(len(p) for p in prompts) else
                                    np.zeros(1, dtype=np.int32))
        offs = np.zeros(n + 1, dtype=np.int64)
        offs[1:] = np.cumsum([len(p) for p in prompts])
        out = np.zeros((n, max(1, max_new_tokens)), dtype=np.int32)
        counts = np.zeros(n, dtype=np.int32)
        stops = np.asarray(list(stop_tokens), dtype=np.int32)
        cb = _lib.TOKEN_CALLBACK(0) if callback is None else _lib.TOKEN_CALLBACK(
            lambda user, seq, idx, tok: int(bool(callback(seq, idx, tok))))
        call("tb_runner_generate", self.handle, _ptr(flat), _ptr(offs), n, max_new_tokens,
             _ptr(stops) if stops.size else None, int(stops.size), _ptr(out), _ptr(counts), cb, None)
        return [out[i, :counts[i]].tolist() for i in range(n)]

    def perplexity(self, slices: Sequence[Sequence[int]]) -> List[PerplexityResult]:
        """computePerplexity for up to max_batch slices decoded together (each
        teacher-forced on its own sequence)."""
        n = len(slices)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(t, dtype=np.int32) for t in slices]))
        offs = np.zeros(n + 1, dtype=np.int64)
        offs[1:] = np.cumsum([len(t) for t in slices])
        acc = np.zeros(n, dtype=np.float64)
        cnt = np.zeros(n, dtype=np.int64)
        t0 = time.perf_counter()
        call("tb_runner_perplexity", self.handle, _ptr(flat), _ptr(offs), n, _ptr(acc), _ptr(cnt))
        el = time.perf_counter() - t0
        return [PerplexityResult(float(np.float32(np.exp(-acc[i] / cnt[i]))), int(cnt[i]), el, float(acc[i]))
                for i in range(n)]

    def set_sampler(self, sampler: Optional[SamplerConfig]):
        """Device sampler for generate_batch / step (Sampler.sampleDetailed);
        None restores greedy argmax decoding.  The LCG restarts from the
        config's seed at every generate call."""
        if sampler is None:
            call("tb_runner_set_sampler", self.handle, None)
        else:
            c = sampler.to_c()
            call("tb_runner_set_sampler", self.handle, C.byref(c))

    def set_step_history(self, tokens: Sequence[int]):
        """Penalty history (prompt + generated tokens) of the next sampled step()."""
        h = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.int32))
        call("tb_runner_set_step_history", self.handle, _ptr(h) if h.size else None, int(h.size))

    def step_stats(self):
        """(probability, entropy) of the last sampled step()."""
        p, e = C.c_float(0), C.c_float(0)
        call("tb_runner_step_stats", self.handle, C.byref(p), C.byref(e))
        return p.value, e.value

    def token_stats(self, n_seqs: int, max_new_tokens: int):
        """Per generated token of the last sampled generate: (probabilities, entropies), [n_seqs][max_new]."""
        pr = np.zeros((n_seqs, max(1, max_new_tokens)), dtype=np.float32)
        en = np.zeros_like(pr)
        call("tb_runner_token_stats", self.handle, n_seqs, max_new_tokens, _ptr(pr), _ptr(en))
        return pr[:, :max_new_tokens], en[:, :max_new_tokens]

    def generate_stream(self, prompt: Sequence[int], config: Optional[GenerationConfig] = None
                        ) -> Iterator[TokenOutput]:
        """ModelRunner.generateStream (ModelRunner.swift:227-298): every token is
        drawn on the device -- by the LM-head argmax for top_k = 1 without a
        penalty, else by the sampler kernel after the LM head."""
        config = config or GenerationConfig()
        sc = config.sampler
        strategy = sc.strategy()
        V = self.config.vocab_size
        hist = [min(max(int(t), 0), V - 1) for t in prompt]  # ModelRunner.swift:236
        stops = set(config.stop_tokens)
        argmax = sc.uses_argmax()
        if self.observer is not None:
            # observed generation runs step by step so every step reports to the
            # observer (ModelRunner.swift:236-298: clamp, prefill all but the
            # last prompt token, then step + sample; a stop token is yielded)
            ids = hist or [0]
            for t in ids[:-1]:
                self.step(t)  # prompt steps draw nothing (the sampler is set after them)
            cur = ids[-1]
            if not argmax:
                self.set_sampler(sc)
            try:
                for _ in range(config.max_tokens):
                    if not argmax:
                        self.set_step_history(hist)
                    _, nxt = self.step(cur)
                    p, ent = _greedy_topk1_stats() if argmax else self.step_stats()
                    yield TokenOutput(nxt, p, ent, time.time(), strategy)
                    if nxt in stops:
                        break
                    hist.append(nxt)
                    cur = nxt
            finally:
                if not argmax:
                    self.set_sampler(None)
            return
        if not argmax:
            self.set_sampler(sc)
        try:
            toks: List[int] = []

            def cb(seq, idx, tok):
                toks.append(tok)
                return False

            self.generate_batch([list(prompt)], config.max_tokens, config.stop_tokens, cb)
            if argmax:
                p, ent = _greedy_topk1_stats()
                stats = [(p, ent)] * len(toks)
            else:
                pr, en = self.token_stats(1, config.max_tokens)
                stats = [(float(pr[0, i]), float(en[0, i])) for i in range(len(toks))]
        finally:
            if not argmax:
                self.set_sampler(None)
        for t, (p, ent) in zip(toks, stats):
            yield TokenOutput(t, p, ent, time.time(), strategy)

    # -- benchmark hooks --
    def prefill_device(self, prompts: Sequence[Sequence[int]], max_new_tokens: int):
        n = len(prompts)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.int32) for p in prompts]))
        offs = np.zeros(n + 1, dtype=np.int64)
        offs[1:] = np.cumsum([len(p) for p in prompts])
        call("tb_runner_prefill_device", self.handle, _ptr(flat), _ptr(offs), n, max_new_tokens)

    def decode_device(self, n_steps: int) -> float:
        ms = C.c_float(0)
        call("tb_runner_decode_device", self.handle, n_steps, C.byref(ms))
        return ms.value

    def read_tokens(self, n_seqs: int, max_new_tokens: int) -> List[List[int]]:
        out = np.zeros((self.max_batch, max(1, max_new_tokens)), dtype=np.int32)
        counts = np.zeros(self.max_batch, dtype=np.int32)
        call("tb_runner_read_tokens", self.handle, _ptr(out), _ptr(counts))
        return [out[i, :counts[i]].tolist() for i in range(n_seqs)]

    def set_chunked_prefill(self, enable: bool):
        """Prefill prompts up to 64 tokens per pass of the layers (default) or
        one token per step as the reference does."""
        call("tb_runner_set_chunked_prefill", self.handle, int(bool(enable)))

    @property
    def persistent(self) -> bool:
        """True when each decode step is one persistent cooperative kernel."""
        v = C.c_int32(0)
        call("tb_runner_get_persistent", self.handle, C.byref(v))
        return bool(v.value)

    @persistent.setter
    def persistent(self, enable: bool):
        call("tb_runner_set_persistent", self.handle, int(bool(enable)))

    def debug_read(self, which: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        call("tb_runner_debug_read", self.handle, which, _ptr(out), n)
        return out

    def io_bytes(self, reset: bool = False):
        a, b = C.c_int64(0), C.c_int64(0)
        call("tb_runner_io_bytes", self.handle, C.byref(a), C.byref(b), int(reset))
        return a.value, b.value

    def profile_step(self):
        cap = 4096
        t = np.zeros(cap, dtype=np.float32)
        k = np.zeros(cap, dtype=np.int32)
        b = np.zeros(cap, dtype=np.int64)
        n = C.c_int32(cap)
        call("tb_runner_profile_step", self.handle, _ptr(t), _ptr(k), _ptr(b), C.byref(n))
        return t[:n.value].copy(), k[:n.value].copy(), b[:n.value].copy()

    def tp_handle(self) -> bytes:
        """Tensor parallel: this rank's all-reduce buffer as a 64-byte CUDA IPC
        handle, to be shared with the other ranks (then tp_connect)."""
        buf = (C.c_uint8 * 64)()
        call("tb_runner_tp_handle", self.handle, buf)
        return bytes(buf)

    def tp_connect(self, handles: Sequence[bytes]):
        """Map every rank's all-reduce buffer (handles in rank order); from then
        on the residual all-reduce runs through peer memory inside the GEMV
        launches instead of NCCL."""
        blob = b"".join(handles)
        if len(blob) != 64 * len(handles):
            raise ValueError("handles must be 64 bytes each")
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        call("tb_runner_tp_connect", self.handle, buf)

    def trace_launches(self):
        """Device timeline of one decode step: (stamps [n][16], kinds [n])."""
        cap = 4096
        st = np.zeros((cap, 16), dtype=np.uint64)
        k = np.zeros(cap, dtype=np.int32)
        n = C.c_int32(cap)
        call("tb_runner_trace_launches", self.handle, _ptr(st), _ptr(k), C.byref(n))
        return st[:n.value].copy(), k[:n.value].copy()

    def close(self):
        if self.handle:
            _lib.load().tb_runner_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
