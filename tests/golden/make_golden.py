"""Regenerate the committed golden vectors (run from the repo root):

    python tests/golden/make_golden.py [CASE ...]

(with case names, only those are regenerated and replaced in manifest.json; the others stay
byte-identical)

Each case writes a seeded synthetic GGUF (glypr_b200.synth), embeds a fixed batch of token
ids with the CPU oracle in both matmul modes (M1 candle-faithful, M2 exact dequant) and
stores ids, lengths and embeddings in a small .npz next to this script, listed in
manifest.json.  The model files themselves are regenerated from the seed by the tests.
"""
from __future__ import annotations

import dataclasses
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from glypr_b200 import synth  # noqa: E402

CASES = [
    # name, config overrides, batch lengths, max_len, out_dim
    ("tiny_cond", dict(n_layers=2, vocab=512, qk_gain_scale=0.25), [96, 33, 1], 96, 768),
    ("tiny_cond_mrl", dict(n_layers=2, vocab=512, qk_gain_scale=0.25), [64, 20], 64, 256),
    ("one_layer_baseline_init", dict(n_layers=1, vocab=512), [128, 5], 128, 768),
    ("global_layer_window", dict(n_layers=6, vocab=512, qk_gain_scale=0.25), [600], 600, 768),
    # the EmbeddingGemma 2 structure: hidden 512, 4 query heads over 2 KV heads (1 on the global
    # layer), per-layer embeddings; the second also with the 512-wide global heads
    ("embeddinggemma2_shape", dict(n_layers=6, hidden=512, n_heads=4, n_kv_heads=2, global_kv_heads=1, ffn=1024,
                                   head_dims=(768,), ple_dim=256, vocab=512, qk_gain_scale=0.25), [200, 17], 200, 768),
    ("embeddinggemma2_global_d512", dict(n_layers=6, hidden=512, n_heads=4, n_kv_heads=2, global_kv_heads=1,
                                         global_head_dim=512, ffn=1024, head_dims=(768,), ple_dim=256, vocab=512,
                                         qk_gain_scale=0.25), [200, 17], 200, 768),
]


def main(only=()) -> None:
    manifest = {"seed": synth.MASTER_SEED, "generator": "tests/golden/make_golden.py", "cases": []}
    mpath = os.path.join(HERE, "manifest.json")
    old = {}
    if only and os.path.exists(mpath):
        old = {c["name"]: c for c in json.load(open(mpath))["cases"]}
    with tempfile.TemporaryDirectory() as tmp:
        for name, over, lengths, max_len, out_dim in CASES:
            if only and name not in only:
                if name in old:
                    manifest["cases"].append(old[name])
                continue
            cfg = synth.EncoderConfig(**over)
            path = synth.write_gguf(os.path.join(tmp, name + ".gguf"), cfg, synth.MASTER_SEED)
            m = oracle.OracleModel(path)
            ids, lens = synth.make_batch(len(lengths), max_len, cfg.vocab, lengths=lengths)
            m1 = m.embed(ids, lens, oracle.M1_CANDLE, out_dim=out_dim)
            m2 = m.embed(ids, lens, oracle.M2_EXACT, out_dim=out_dim)
            fname = name + ".npz"
            np.savez_compressed(os.path.join(HERE, fname), ids=ids, lengths=lens, m1=m1, m2=m2)
            cfg_dict = {k: v for k, v in dataclasses.asdict(cfg).items() if k in over}
            manifest["cases"].append({"name": name, "config": cfg_dict, "seed": synth.MASTER_SEED,
                                      "file": fname, "out_dim": out_dim, "lengths": lengths})
            print(name, "cos(m1, m2) =", (m1 * m2).sum(1))
    with open(mpath, "w") as fh:
        json.dump(manifest, fh, indent=1)


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
