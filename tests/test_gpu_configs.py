"""GPU parity at the sizes and shapes BASELINE's configs name, against the CPU oracle.

* config 4: BF16 weights, ONE 8,192-token sequence, six layers with a global layer attending
  over all 8,192 keys and sliding layers with the 512 window (chunked.rs:56-172,
  model.rs:634-638), pooled over 16 segments of 512 tokens;
* config 3: 256 right-padded sequences with lengths uniform in [64, 512], 768-d output and the
  256-d Matryoshka output (model.rs:691-698), one call;
* the full 262,144-row token table, with ids drawn across the whole range (0, 1, 2 and
  262,143 included): the embedding gather's addressing of high rows;
* the CTA-pair variant of every 256-wide GEMM (GLP_GEMM=pair, in a child process since the
  engine choice is read once per process), on per-layer-embedding models -- the PLE gate GEMM
  with its GeGLU epilogue included.

Gates as in test_gpu_model: cosine >= 0.9999 and max |delta| <= 2e-3 (scaled by sqrt(768/d)
for d-wide MRL outputs) against the exact oracle (M2), and against the candle-faithful oracle
(M1) for sequences of >= 16 tokens; all models are the well-conditioned variant (q/k gains
x0.25), for the reason test_oracle_kat.test_baseline_init_is_ill_conditioned shows.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from glypr_b200 import api, synth
from glypr_b200.api import GlyprEmbedder

from .conftest import ROOT, cosine_rows
from .test_gpu_model import ABS_GATE, _check, _check_both

pytestmark = pytest.mark.gpu


def _model(gguf_dir, name, cfg):
    return synth.ensure_gguf(os.path.join(str(gguf_dir), name), cfg)


def test_config4_one_8192_token_sequence_bf16(gguf_dir):
    cfg = synth.small_config(n_layers=6, weight_type="bf16", qk_gain_scale=0.25)
    assert not cfg.layer_is_sliding(5)  # layer 5 attends over every key
    path = _model(gguf_dir, "c4_bf16_6l.gguf", cfg)
    ids, lens = synth.make_batch(1, 8192, cfg.vocab, lengths=[8192], seed=synth.MASTER_SEED + 44)
    with GlyprEmbedder.load_gguf(path, [0]) as emb:
        got = emb.embed_tokens(ids, lens)
        got256 = emb.embed_tokens(ids, lens, out_dim=256)
        assert emb.device_status() == 0
    orc = oracle.OracleModel(path)
    want = orc.embed(ids, lens, oracle.M2_EXACT)
    cos, err = _check(got, want)
    print(f"config 4 (8192 tokens, BF16, 6 layers): cosine {cos[0]:.7f}, max|d| {err[0]:.2e}")
    _check(got256, np.stack([api.truncate_mrl(w, 256) for w in want]), abs_gate=ABS_GATE * np.sqrt(3.0))


def test_config3_256_ragged_sequences_and_mrl(gguf_dir):
    cfg = synth.small_config(n_layers=2, qk_gain_scale=0.25)
    path = _model(gguf_dir, "small_cond.gguf", cfg)
    rng = np.random.default_rng(synth.MASTER_SEED + 33)
    lens = rng.integers(64, 513, size=256).astype(np.int32)
    ids, lens = synth.make_batch(256, 512, cfg.vocab, seed=synth.MASTER_SEED + 34, lengths=list(lens))
    with GlyprEmbedder.load_gguf(path, [0]) as emb:
        got = emb.embed_tokens(ids, lens)
        got256 = emb.embed_tokens(ids, lens, out_dim=256)
        assert emb.device_status() == 0
    # one call, 256 sequences; the oracle checks every fourth (across the batch; batch
    # invariance covers the rest), at both widths
    sel = np.arange(0, 256, 4)
    m1, m2 = _check_both(got[sel], oracle.OracleModel(path), ids[sel], lens[sel])
    _check(got256[sel], np.stack([api.truncate_mrl(w, 256) for w in m2]), abs_gate=ABS_GATE * np.sqrt(3.0))
    np.testing.assert_allclose(got256, np.stack([api.truncate_mrl(g, 256) for g in got]), atol=2e-6)
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)


def test_full_262144_row_token_table(gguf_dir):
    cfg = synth.small_config(n_layers=1, vocab=262144, qk_gain_scale=0.25)
    path = _model(gguf_dir, "vocab262144_1l.gguf", cfg)
    rng = np.random.default_rng(7)
    n, L = 6, 300
    ids = rng.integers(0, 262144, size=(n, L)).astype(np.int32)
    ids[0, :4] = [0, 1, 2, 262143]
    ids[1, :] = 262143 - np.arange(L)          # the table's last rows
    ids[2, :] = np.arange(L) * 873 + 3         # spread over the whole table
    lens = np.array([L, L, L, 200, 17, 1], np.int32)
    ids[5, 0] = 262143
    with GlyprEmbedder.load_gguf(path, [0]) as emb:
        assert emb.info.vocab == 262144
        got = emb.embed_tokens(ids, lens)
        with pytest.raises(api.GlyprError):
            emb.embed_tokens(np.array([[262144]], np.int32), np.array([1], np.int32))
    _check_both(got, oracle.OracleModel(path), ids, lens)


_CHILD = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from glypr_b200.api import GlyprEmbedder
spec = json.loads(sys.argv[2])
ids = np.array(spec["ids"], np.int32); lens = np.array(spec["lens"], np.int32)
with GlyprEmbedder.load_gguf(spec["path"], [0]) as emb:
    out = emb.embed_tokens(ids, lens)
    assert emb.device_status() == 0
np.save(spec["out"], out)
"""


def _embed_in_child(path, ids, lens, out, engine):
    env = dict(os.environ, GLP_GEMM=engine)
    spec = json.dumps({"path": path, "ids": ids.tolist(), "lens": lens.tolist(), "out": out})
    subprocess.run([sys.executable, "-c", _CHILD, ROOT, spec], env=env, check=True, timeout=600)
    return np.load(out)


@pytest.mark.parametrize("kw", [
    dict(n_layers=6, hidden=512, n_heads=4, n_kv_heads=2, global_kv_heads=1, ffn=2048, head_dims=(2048, 512),
         ple_dim=256),
    dict(n_layers=2, ple_dim=512),
])
def test_cta_pair_gemms_on_ple_models(gguf_dir, tmp_path, kw):
    """GLP_GEMM=pair: every 256-wide GEMM on CTA pairs, including the PLE gate GEMM's GeGLU
    epilogue (kEpiMulGeglu), which the default engine only pairs on full-size launch chunks."""
    cfg = synth.small_config(qk_gain_scale=0.25, **kw)
    path = _model(gguf_dir, f"ple_{cfg.hidden}_{cfg.ple_dim}.gguf", cfg)
    ids, lens = synth.make_batch(4, 600, cfg.vocab, lengths=[600, 513, 64, 1])
    pair = _embed_in_child(path, ids, lens, str(tmp_path / "pair.npy"), "pair")
    single = _embed_in_child(path, ids, lens, str(tmp_path / "single.npy"), "single")
    _check_both(pair, oracle.OracleModel(path), ids, lens)
    # pair and single-CTA tiles round differently; on a single token (no pooling to average the
    # rounding) they stay within the gate of each other (measured 1 - cos 3e-5)
    assert cosine_rows(pair, single).min() >= 0.9999
