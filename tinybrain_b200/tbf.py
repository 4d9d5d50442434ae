"""TinyBrain Binary Format (.tbf): ModelWeights.load / ModelWeights.save.

Restates the reference's reader and writer
(Sources/TinyBrainRuntime/ModelWeights.swift:246-490 save, 496-798 load; the
same layout is written by Scripts/convert_model.py:462-710):

  header    "TBFM", u32 version (1), u32 length + ModelConfig JSON
            (camelCase keys), zero-padded to 4 KB
  metadata  u32 count; per quantized tensor: u32 name length + name, u8
            precision (1 INT8, 2 INT4), u8 mode (2 per-channel, 3 INT4 per
            group), u32 group size, u32 + f32[] scales, u32 + i8[] zero points;
            padded to 4 KB
  index     u32 count; per tensor: u32 name length + name, u32 rank + i32[]
            dims, u64 absolute data offset, u64 data size; padded to 4 KB
  data      one blob per tensor (quantized bytes or fp32), each padded to 4 KB

All integers little-endian.  Tensor names: "embeddings", "layer_{i}_attn_{q,k,v,o}",
"layer_{i}_ffn_{gate,up,down}", "layer_{i}_ln_{input,post}", optional
"layer_{i}_ln_input_bias", "layer_{i}_attn_{q,k,v,o}_bias",
"layer_{i}_ffn_{up,down}_bias", "final_norm", "final_norm_bias", "output",
"output_bias".

The file is memory-mapped and tensors are views into it until uploaded (the
reference reads the whole file; mmap gives the same bytes).

Converter-written INT4 files.  Scripts/convert_model.py:489-502 quantizes an
INT4 weight as the flattened PyTorch [out, in] tensor (groups of 32
consecutive inputs of one output) without transposing the data, but records
the shape as [in, out]; the runtime reads every INT4 tensor as row-major
[in, out] (QuantizedTensor.swift:195-216, DequantINT4.metal:95-137), so such
a file decodes to a different matrix than the one converted.  The writer is
recognisable from the header: the converter writes the config with Python's
json.dumps default separators (", " and ": ", convert_model.py:57-68) while
Swift's JSONEncoder (ModelWeights.swift:273) writes compact JSON.  load()
flags such files (ModelWeights.tbf_info["converter_int4"]) and, by
`int4_layout`, keeps the reference's runtime reading ("runtime", the default:
what the reference itself computes, with a warning), refuses the file
("reject", TB_ERR_FORMAT), or rebuilds each INT4 tensor as the converted
matrix ("requantize": dequantize in [out, in] order, transpose to [in, out],
quantize again with the runtime's INT4 quantizer on the device -- a second
rounding, since the two layouts group different elements).
"""
from __future__ import annotations

import json
import mmap
import struct
import warnings
from typing import Dict, List, Optional, Tuple

import numpy as np

from ._lib import TinyBrainError
from .runtime import (LinearLayerWeights, ModelConfig, ModelWeights, QuantizedTensor,
                      TransformerLayerWeights)

MAGIC = b"TBFM"
VERSION = 1
_PAGE = 4096

# TBFError cases (ModelWeights.swift:6-20) as status-style messages
_ERR_FORMAT = 6


def _pad(n: int) -> int:
    return (n + _PAGE - 1) // _PAGE * _PAGE


class _Reader:
    def __init__(self, buf):
        self.buf = buf
        self.off = 0

    def take(self, n: int) -> bytes:
        if self.off + n > len(self.buf):
            raise TinyBrainError(_ERR_FORMAT, "tbf: truncated file")
        b = self.buf[self.off:self.off + n]
        self.off += n
        return b

    def u8(self) -> int:
        return self.take(1)[0]

    def u32(self) -> int:
        return struct.unpack("<I", self.take(4))[0]

    def i32(self) -> int:
        return struct.unpack("<i", self.take(4))[0]

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def name(self) -> str:
        return self.take(self.u32()).decode("utf-8")

    def align(self):
        self.off = _pad(self.off)


def _config_from_json(d: dict) -> ModelConfig:
    # ModelConfig.init(from:) defaults (ModelRunner.swift:95-106)
    arch = d.get("architecture", "llama")
    if arch not in ("llama", "toy"):
        raise TinyBrainError(4, f"tbf: architecture {arch!r} is outside the decode path (llama)")
    if float(d.get("partialRotaryFactor", 1.0)) != 1.0:
        raise TinyBrainError(4, "tbf: partial RoPE is outside the decode path")
    return ModelConfig(num_layers=int(d["numLayers"]), hidden_dim=int(d["hiddenDim"]),
                       num_heads=int(d["numHeads"]), vocab_size=int(d["vocabSize"]),
                       max_seq_len=int(d["maxSeqLen"]),
                       num_kv_heads=int(d.get("numKVHeads", d["numHeads"])),
                       intermediate_dim=int(d.get("intermediateDim", 4 * int(d["hiddenDim"]))),
                       architecture=arch)


class ConverterInt4Warning(UserWarning):
    """An INT4 tensor of a converter-written file is read with the runtime's
    [in, out] semantics, not as the matrix that was converted."""


def written_by_converter(config_json: bytes) -> bool:
    """True for a header written by Scripts/convert_model.py (json.dumps with
    its default ", " / ": " separators); Swift's JSONEncoder writes none."""
    return b'": ' in config_json or b'", "' in config_json


def load(path: str, int4_layout: str = "runtime", ctx=None) -> ModelWeights:
    """ModelWeights.load(from:) (ModelWeights.swift:496-798).  int4_layout is
    "runtime", "reject" or "requantize" (module docstring)."""
    if int4_layout not in ("runtime", "reject", "requantize"):
        raise ValueError("int4_layout must be 'runtime', 'reject' or 'requantize'")
    f = open(path, "rb")
    try:
        buf = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    except ValueError:
        f.close()
        raise TinyBrainError(_ERR_FORMAT, "tbf: file too small")
    f.close()
    if len(buf) < 12:
        raise TinyBrainError(_ERR_FORMAT, "tbf: file too small")
    r = _Reader(buf)
    if r.take(4) != MAGIC:
        raise TinyBrainError(_ERR_FORMAT, "tbf: invalid magic bytes")
    version = r.u32()
    if version != VERSION:
        raise TinyBrainError(_ERR_FORMAT, f"tbf: unsupported version {version}")
    cj = r.take(r.u32())
    config = _config_from_json(json.loads(cj.decode("utf-8")))
    from_converter = written_by_converter(cj)
    r.align()

    meta: Dict[str, Tuple[int, int, int, np.ndarray, Optional[np.ndarray]]] = {}
    for _ in range(r.u32()):
        name = r.name()
        precision, mode, gs = r.u8(), r.u8(), r.u32()
        ns = r.u32()
        scales = np.frombuffer(r.take(4 * ns), dtype="<f4").astype(np.float32)
        nz = r.u32()
        zps = np.frombuffer(r.take(nz), dtype=np.int8).copy() if nz else None
        meta[name] = (precision, mode, gs, scales, zps)
    r.align()

    index: Dict[str, Tuple[List[int], int, int]] = {}
    for _ in range(r.u32()):
        name = r.name()
        dims = [r.i32() for _ in range(r.u32())]
        off, size = r.u64(), r.u64()
        if off + size > len(buf):
            raise TinyBrainError(_ERR_FORMAT, f"tbf: tensor {name} runs past the end of the file")
        index[name] = (dims, off, size)

    def blob(name: str) -> Tuple[List[int], np.ndarray]:
        dims, off, size = index[name]
        return dims, np.frombuffer(buf, dtype=np.uint8, count=size, offset=off)

    def f32(name: str) -> Optional[np.ndarray]:
        if name not in index:
            return None
        dims, raw = blob(name)
        return raw.view("<f4").astype(np.float32).reshape(dims)

    def quant(name: str) -> QuantizedTensor:
        if name not in index:
            raise TinyBrainError(_ERR_FORMAT, f"tbf: missing tensor {name}")
        if name not in meta:
            raise TinyBrainError(_ERR_FORMAT, f"tbf: missing metadata for {name}")
        dims, raw = blob(name)
        precision, mode, gs, scales, zps = meta[name]
        if len(dims) != 2:
            raise TinyBrainError(_ERR_FORMAT, f"tbf: {name} is not a matrix")
        if precision == 2:  # INT4 per group (ModelWeights.swift:672-679)
            q = QuantizedTensor((dims[0], dims[1]), raw.copy(), scales, "int4", int(gs),
                                zps if zps is not None else np.zeros(scales.size, dtype=np.int8))
            if from_converter:
                converter_int4.append(name)
                if int4_layout == "reject":
                    raise TinyBrainError(_ERR_FORMAT, f"tbf: {name} is an INT4 tensor written by convert_model.py "
                                                      "([out, in] data recorded as [in, out])")
                if int4_layout == "requantize":
                    return _requantize_converter_int4(q, ctx)
            return q
        if mode != 2:
            raise TinyBrainError(4, f"tbf: {name}: INT8 mode {mode} (symmetric) is outside the decode path")
        return QuantizedTensor((dims[0], dims[1]), raw.view(np.int8).copy(), scales, "perChannel", 0, zps)

    def linear(name: str, bias: str) -> LinearLayerWeights:
        return LinearLayerWeights(quant(name), f32(bias))

    converter_int4: List[str] = []
    emb = f32("embeddings")
    if emb is None:
        raise TinyBrainError(_ERR_FORMAT, "tbf: missing tensor embeddings")
    layers = []
    for i in range(config.num_layers):
        p = f"layer_{i}_"
        if f32(p + "ln_input_bias") is not None:
            raise TinyBrainError(4, "tbf: LayerNorm biases (Phi-2) are outside the decode path")
        layers.append(TransformerLayerWeights(
            query=linear(p + "attn_q", p + "attn_q_bias"), key=linear(p + "attn_k", p + "attn_k_bias"),
            value=linear(p + "attn_v", p + "attn_v_bias"), output=linear(p + "attn_o", p + "attn_o_bias"),
            gate=LinearLayerWeights(quant(p + "ffn_gate")) if p + "ffn_gate" in index else None,
            up=linear(p + "ffn_up", p + "ffn_up_bias"), down=linear(p + "ffn_down", p + "ffn_down_bias"),
            input_norm=f32(p + "ln_input"), post_attention_norm=f32(p + "ln_post")))
    if f32("final_norm_bias") is not None:
        raise TinyBrainError(4, "tbf: LayerNorm biases (Phi-2) are outside the decode path")
    out = linear("output", "output_bias")
    weights = ModelWeights(config, emb, layers, out, final_norm=f32("final_norm"))
    weights.tbf_info = {"writer": "convert_model.py" if from_converter else "ModelWeights.save",
                        "converter_int4": bool(converter_int4), "int4_layout": int4_layout,
                        "int4_tensors": converter_int4}
    if converter_int4 and int4_layout == "runtime":
        warnings.warn(f"{path}: {len(converter_int4)} INT4 tensors written by convert_model.py are read with the "
                      "runtime's [in, out] semantics, as the reference does (int4_layout='requantize' rebuilds "
                      "the converted matrices)", ConverterInt4Warning, stacklevel=3)
    return weights


def _requantize_converter_int4(q: QuantizedTensor, ctx) -> QuantizedTensor:
    """The converted matrix of a converter-written INT4 tensor: its flat data
    is the PyTorch [out, in] weight, so dequantize flat, view as [out, in],
    transpose to [in, out] and quantize with the runtime INT4 quantizer (same
    group size) on the device."""
    from .runtime import quantize
    K, N = q.shape  # recorded [in, out]
    flat = q.dequantize(ctx).reshape(-1)  # element order of the converter's flat [out, in] data
    w = np.ascontiguousarray(flat.reshape(N, K).T)
    return quantize(w, "int4", q.group_size, ctx)


def save(weights: ModelWeights, path: str) -> None:
    """ModelWeights.save(to:) (ModelWeights.swift:260-490), same tensor order."""
    c = weights.config
    cfg = {"numLayers": c.num_layers, "hiddenDim": c.hidden_dim, "numHeads": c.num_heads,
           "numKVHeads": c.num_kv_heads, "vocabSize": c.vocab_size, "maxSeqLen": c.max_seq_len,
           "intermediateDim": c.intermediate_dim, "architecture": c.architecture, "partialRotaryFactor": 1.0}
    entries: List[Tuple[str, Optional[QuantizedTensor], Optional[np.ndarray], Tuple[int, ...]]] = []

    def add_f(name, arr):
        if arr is not None:
            a = np.ascontiguousarray(arr, dtype=np.float32)
            entries.append((name, None, a, a.shape))

    def add_q(name, q):
        entries.append((name, q, None, tuple(q.shape)))

    add_f("embeddings", weights.token_embeddings)
    for i, ly in enumerate(weights.layers):
        p = f"layer_{i}_"
        add_q(p + "attn_q", ly.query.weights)
        add_q(p + "attn_k", ly.key.weights)
        add_q(p + "attn_v", ly.value.weights)
        add_q(p + "attn_o", ly.output.weights)
        if ly.gate is not None:
            add_q(p + "ffn_gate", ly.gate.weights)
        add_q(p + "ffn_up", ly.up.weights)
        add_q(p + "ffn_down", ly.down.weights)
        add_f(p + "ln_input", ly.input_norm)
        add_f(p + "ln_post", ly.post_attention_norm)
        for proj, lw in (("q", ly.query), ("k", ly.key), ("v", ly.value), ("o", ly.output)):
            add_f(p + f"attn_{proj}_bias", lw.bias)
        for proj, lw in (("up", ly.up), ("down", ly.down)):
            add_f(p + f"ffn_{proj}_bias", lw.bias)
    add_f("final_norm", weights.final_norm)
    add_q("output", weights.output.weights)
    add_f("output_bias", weights.output.bias)

    out = bytearray()
    cj = json.dumps(cfg, separators=(",", ":")).encode("utf-8")
    out += MAGIC + struct.pack("<I", VERSION) + struct.pack("<I", len(cj)) + cj
    out += b"\0" * (_pad(len(out)) - len(out))
    quants = [(n, q) for n, q, _, _ in entries if q is not None]
    out += struct.pack("<I", len(quants))
    for n, q in quants:
        nb = n.encode("utf-8")
        out += struct.pack("<I", len(nb)) + nb
        int4 = q.mode == "int4"
        out += struct.pack("<BBI", 2 if int4 else 1, 3 if int4 else 2, q.group_size if int4 else 0)
        sc = np.ascontiguousarray(q.scales, dtype="<f4")
        out += struct.pack("<I", sc.size) + sc.tobytes()
        zp = q.zero_points
        if zp is None:
            out += struct.pack("<I", 0)
        else:
            zp = np.ascontiguousarray(zp, dtype=np.int8)
            out += struct.pack("<I", zp.size) + zp.tobytes()
    out += b"\0" * (_pad(len(out)) - len(out))
    blobs = [(q.data.tobytes() if q is not None else f.tobytes()) for _, q, f, _ in entries]
    index = bytearray(struct.pack("<I", len(entries)))
    patch = []
    for (n, _, _, shape), b in zip(entries, blobs):
        nb = n.encode("utf-8")
        index += struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(shape))
        index += b"".join(struct.pack("<i", int(d)) for d in shape)
        patch.append(len(index))
        index += struct.pack("<QQ", 0, len(b))
    index_start = len(out)
    data_start = _pad(index_start + len(index))
    pos = data_start
    for at, b in zip(patch, blobs):
        index[at:at + 8] = struct.pack("<Q", pos)
        pos += _pad(len(b))
    out += index
    out += b"\0" * (data_start - len(out))
    for b in blobs:
        out += b
        out += b"\0" * (_pad(len(out)) - len(out))
    with open(path, "wb") as fh:
        fh.write(out)
