"""The .tbf model format (ModelWeights.load / save): the golden files were
written by the reference's own converter (tests/golden/make_tbf_fixtures.py);
their contents are checked against a restatement of that converter's
quantizers on the same seeded weights (Scripts/convert_model.py:370-460)."""
import hashlib
import json
import os

import numpy as np
import pytest

from tests.golden.make_tbf_fixtures import CFG, weights
from tinybrain_b200._lib import TinyBrainError
from tinybrain_b200.runtime import ModelWeights

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _q8(t):  # per output channel of [out, in], symmetric, round half to even (numpy)
    s = np.abs(t).max(axis=1) / np.float32(127.0)
    s = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
    return np.round(t / s[:, None]).astype(np.int8), s


def _q4(t, gs=32):  # flattened groups of gs, clipped to [-7, 7], even index = high nibble
    flat = t.flatten().astype(np.float32)
    g = flat.reshape(-1, gs)
    s = np.abs(g).max(axis=1) / np.float32(7.0)
    s = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.round(g / s[:, None]), -7, 7).astype(np.int8).ravel()
    nib = (q & 0x0F).astype(np.uint8)
    return ((nib[0::2] << 4) | nib[1::2]).astype(np.uint8), s


def test_fixture_files_unchanged():
    meta = json.load(open(os.path.join(GOLD, "tbf_fixtures.json")))
    for name, m in meta["files"].items():
        data = open(os.path.join(GOLD, name), "rb").read()
        assert len(data) == m["size"] and hashlib.sha256(data).hexdigest() == m["sha256"]


@pytest.mark.parametrize("mode", ["int8", "int4"])
def test_load_reference_written_file(mode):
    w = ModelWeights.load(os.path.join(GOLD, f"tiny_{mode}.tbf"))
    c = w.config
    assert (c.num_layers, c.hidden_dim, c.num_heads, c.num_kv_heads, c.vocab_size, c.intermediate_dim,
            c.max_seq_len) == tuple(CFG[k] for k in ("num_layers", "hidden_dim", "num_heads", "num_kv_heads",
                                                      "vocab_size", "intermediate_dim", "max_seq_len"))
    src = weights(7)
    np.testing.assert_array_equal(w.token_embeddings, src["embeddings"])
    np.testing.assert_array_equal(w.final_norm, src["final_norm"])
    pairs = [("query", "q_proj"), ("key", "k_proj"), ("value", "v_proj"), ("output", "o_proj"),
             ("gate", "gate_proj"), ("up", "up_proj"), ("down", "down_proj")]
    mats = [(getattr(ly, a).weights, src["layers"][i][b]) for i, ly in enumerate(w.layers) for a, b in pairs]
    mats.append((w.output.weights, src["lm_head"]))
    for i, ly in enumerate(w.layers):
        np.testing.assert_array_equal(ly.input_norm, src["layers"][i]["input_layernorm"])
        np.testing.assert_array_equal(ly.post_attention_norm, src["layers"][i]["post_attention_layernorm"])
    for qt, t in mats:
        assert qt.shape == (t.shape[1], t.shape[0])  # stored [in, out]
        if mode == "int8":
            q, s = _q8(t)
            assert qt.mode == "perChannel"
            np.testing.assert_array_equal(qt.data.reshape(qt.shape), q.T)
            np.testing.assert_array_equal(qt.scales, s)
        else:
            p, s = _q4(t)
            assert qt.mode == "int4" and qt.group_size == 32
            np.testing.assert_array_equal(qt.data, p)
            np.testing.assert_array_equal(qt.scales, s)
            assert not np.any(qt.zero_points)


@pytest.mark.parametrize("mode", ["int8", "int4"])
def test_save_load_round_trip(tmp_path, mode):
    w = ModelWeights.load(os.path.join(GOLD, f"tiny_{mode}.tbf"))
    path = str(tmp_path / "rt.tbf")
    w.save(path)
    assert os.path.getsize(path) % 4096 == 0
    v = ModelWeights.load(path)
    assert vars(v.config) == vars(w.config)
    np.testing.assert_array_equal(v.token_embeddings, w.token_embeddings)
    for a, b in zip(v.layers, w.layers):
        for f in ("query", "key", "value", "output", "gate", "up", "down"):
            x, y = getattr(a, f).weights, getattr(b, f).weights
            assert x.shape == y.shape and x.mode == y.mode
            np.testing.assert_array_equal(x.data, y.data)
            np.testing.assert_array_equal(x.scales, y.scales)
    np.testing.assert_array_equal(v.output.weights.data, w.output.weights.data)


def test_rejects_bad_files(tmp_path):
    bad = tmp_path / "bad.tbf"
    bad.write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(TinyBrainError, match="magic"):
        ModelWeights.load(str(bad))
    data = bytearray(open(os.path.join(GOLD, "tiny_int8.tbf"), "rb").read())
    data[4:8] = (2).to_bytes(4, "little")
    bad.write_bytes(bytes(data))
    with pytest.raises(TinyBrainError, match="version"):
        ModelWeights.load(str(bad))
    bad.write_bytes(bytes(data[:5000]))
    with pytest.raises(TinyBrainError):
        ModelWeights.load(str(bad))
    bad.write_bytes(b"TBFM")
    with pytest.raises(TinyBrainError, match="small"):
        ModelWeights.load(str(bad))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["int8", "int4"])
def test_tbf_model_decodes_like_oracle(ctx, mode):
    import oracle
    from tests.helpers import assert_same_tokens
    from tinybrain_b200.runtime import ModelRunner
    w = ModelWeights.load(os.path.join(GOLD, f"tiny_{mode}.tbf"))
    got = ModelRunner(w, ctx).generate_batch([[1, 2, 3, 4, 5]], 20)[0]
    want, gaps = oracle.OracleModel(w, mode=1).generate_greedy([1, 2, 3, 4, 5], 20)
    assert_same_tokens(got, want, gaps, w, [1, 2, 3, 4, 5])


def test_converter_int4_files_are_flagged():
    from tinybrain_b200 import tbf
    w8 = ModelWeights.load(os.path.join(GOLD, "tiny_int8.tbf"))
    assert w8.tbf_info["writer"] == "convert_model.py" and not w8.tbf_info["converter_int4"]
    with pytest.warns(tbf.ConverterInt4Warning):
        w4 = ModelWeights.load(os.path.join(GOLD, "tiny_int4.tbf"))
    assert w4.tbf_info["converter_int4"] and len(w4.tbf_info["int4_tensors"]) == 2 * 7 + 1
    with pytest.raises(TinyBrainError, match="convert_model"):
        ModelWeights.load(os.path.join(GOLD, "tiny_int4.tbf"), int4_layout="reject")


def test_files_written_by_save_are_not_flagged(tmp_path):
    w4 = ModelWeights.load(os.path.join(GOLD, "tiny_int4.tbf"))
    path = str(tmp_path / "saved.tbf")
    w4.save(path)
    v = ModelWeights.load(path, int4_layout="reject")  # compact JSON header: ModelWeights.save
    assert v.tbf_info["writer"] == "ModelWeights.save" and not v.tbf_info["converter_int4"]


@pytest.mark.gpu
def test_converter_int4_requantize_rebuilds_the_converted_matrix(ctx):
    # int4_layout="requantize": each INT4 tensor becomes the runtime-layout
    # quantization of the matrix the converter was given ([in, out] = W.T)
    w = ModelWeights.load(os.path.join(GOLD, "tiny_int4.tbf"), int4_layout="requantize", ctx=ctx)
    src = weights(7)
    qt = w.layers[0].query.weights
    assert qt.shape == (CFG["hidden_dim"], CFG["hidden_dim"]) and qt.mode == "int4"
    deq = qt.dequantize(ctx)
    t = src["layers"][0]["q_proj"].T  # [in, out]
    # two roundings (converter groups, then runtime groups): within ~2 steps of 1/7 of the group max
    assert np.max(np.abs(deq - t)) <= 2.0 * np.abs(t).max() / 7.0
    assert np.corrcoef(deq.ravel(), t.ravel())[0, 1] > 0.95
