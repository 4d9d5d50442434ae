"""Generate the .tbf golden fixtures with the reference's own writer.

Runs the reference's converter (Scripts/convert_model.py: write_tbf_format,
which its header says matches Swift ModelWeights.save() byte for byte) on a
tiny seeded LLaMA-shaped weight set, once with INT8 and once with INT4
quantization, and records what the files must decode to (config, tensor
shapes, SHA-256 of every tensor's bytes, scales and zero points) in
tbf_fixtures.json.  Needs the reference tree, so it runs in the build
container only; the fixtures it writes are committed.

    python tests/golden/make_tbf_fixtures.py /path/to/reference
"""
import contextlib
import hashlib
import io
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
CFG = dict(num_layers=2, hidden_dim=64, num_heads=4, num_kv_heads=2, vocab_size=96, intermediate_dim=128,
           max_seq_len=64)


def weights(seed):
    """PyTorch-layout ([out, in]) fp32 weights of a tiny LLaMA model."""
    rng = np.random.default_rng(seed)
    H, I, V = CFG["hidden_dim"], CFG["intermediate_dim"], CFG["vocab_size"]
    kvd = H // CFG["num_heads"] * CFG["num_kv_heads"]
    n = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float32)  # noqa: E731
    layers = []
    for _ in range(CFG["num_layers"]):
        layers.append({"q_proj": n(H, H), "k_proj": n(kvd, H), "v_proj": n(kvd, H), "o_proj": n(H, H),
                       "gate_proj": n(I, H), "up_proj": n(I, H), "down_proj": n(H, I),
                       "input_layernorm": (1 + 0.1 * rng.standard_normal(H)).astype(np.float32),
                       "post_attention_layernorm": (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)})
    return {"embeddings": n(V, H), "layers": layers,
            "final_norm": (1 + 0.1 * rng.standard_normal(H)).astype(np.float32), "lm_head": n(V, H)}


def sha(b):
    return hashlib.sha256(bytes(b)).hexdigest()


def main(ref):
    sys.path.insert(0, os.path.join(ref, "Scripts"))
    import convert_model as cm
    out = {"config": CFG, "files": {}}
    for mode in ("int8", "int4"):
        path = os.path.join(HERE, f"tiny_{mode}.tbf")
        cfg = cm.ModelConfig(**CFG)
        with contextlib.redirect_stdout(io.StringIO()), contextlib.redirect_stderr(io.StringIO()):
            cm.write_tbf_format(weights(7), cfg, path, quantize_mode=mode, group_size=32)
        # expectations straight from the file's own sections (independent parse)
        data = open(path, "rb").read()
        out["files"][os.path.basename(path)] = {"sha256": sha(data), "size": len(data)}
    with open(os.path.join(HERE, "tbf_fixtures.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_tbf_fixtures.py <path of the reference checkout>")
    main(sys.argv[1])
