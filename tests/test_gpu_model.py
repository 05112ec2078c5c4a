"""End-to-end parity of the GPU embedding path against the CPU oracle, plus the
size-independent properties the reference's own tests assert (batch == single,
L2 norm 1, MRL renormalisation, context-limit errors).

Tolerances: cosine >= 0.9999 per vector and max |delta| <= 2e-3 after
L2 normalisation, against the reference CPU path (oracle mode M1, candle-faithful).  The
cosine gate is applied to the well-conditioned variants (q/k gains x0.25): with the
BASELINE init (unit q/k gains, attention scale 1.0) the 24-layer model amplifies any
1e-7 perturbation chaotically, so no two implementations that round differently agree
there (measured: oracle f32- vs f64-accumulation cos 0.97, M1 vs M2 cos 0.62); that model
is checked through the properties below instead.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from glypr_b200 import api, synth
from glypr_b200.api import GlyprEmbedder, GlyprError

from .conftest import cosine_rows

pytestmark = pytest.mark.gpu

COS_GATE = 0.9999
ABS_GATE = 2e-3


@pytest.fixture(scope="module")
def small_emb(small_cond_gguf):
    e = GlyprEmbedder.load_gguf(small_cond_gguf, [0])
    yield e
    e.close()


@pytest.fixture(scope="module")
def small_oracle(small_cond_gguf):
    return oracle.OracleModel(small_cond_gguf)


def _check(got, want, cos_gate=COS_GATE, abs_gate=ABS_GATE):
    cos = cosine_rows(got, want)
    err = np.abs(got - want).max(axis=1)
    assert cos.min() >= cos_gate, (cos, err)
    assert err.max() <= abs_gate, (cos, err)
    return cos, err


def _check_both(got, orc, ids, lens, out_dim=None):
    """Gate against the exact-dequant oracle (M2) for every sequence, and against the
    candle-faithful reference path (M1) for sequences of >= 16 tokens.  M1 quantises every
    activation row to int8 blocks; for a very short sequence that noise is not averaged by
    the mean-pool and M1 itself sits ~1.6e-4 (cosine) from the exact result (single-token
    golden case), so there the M1 check allows the M1-vs-exact gap."""
    m1 = orc.embed(ids, lens, oracle.M1_CANDLE, out_dim=out_dim)
    m2 = orc.embed(ids, lens, oracle.M2_EXACT, out_dim=out_dim)
    # MRL renormalises the first out_dim values: element magnitudes (and absolute errors)
    # grow by ~sqrt(E / out_dim), so the 768-d absolute gate scales with it
    abs_gate = ABS_GATE * np.sqrt(got.shape[1] and 768.0 / got.shape[1])
    _check(got, m2, abs_gate=abs_gate)
    long_ = np.asarray(lens) >= 16
    if long_.any():
        _check(got[long_], m1[long_], abs_gate=abs_gate)
    gap = 1.0 - cosine_rows(m1, m2)
    cos1 = cosine_rows(got, m1)
    assert (cos1 >= np.minimum(COS_GATE, 1.0 - 2.0 * gap - 2e-5)).all(), (cos1, gap)
    return m1, m2


def test_small_parity_ragged(small_emb, small_oracle):
    ids, lens = synth.make_batch(6, 700, small_oracle.vocab, lengths=[700, 513, 512, 64, 1, 300])
    got = small_emb.embed_tokens(ids, lens)
    _check_both(got, small_oracle, ids, lens)
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)


def test_small_parity_mrl(small_emb, small_oracle):
    ids, lens = synth.make_batch(4, 256, small_oracle.vocab, len_range=(16, 256))
    got256 = small_emb.embed_tokens(ids, lens, out_dim=256)
    full = small_emb.embed_tokens(ids, lens)
    # MRL on the device == truncate + renormalise of the 768-d output (model.rs:691-698)
    np.testing.assert_allclose(got256, np.stack([api.truncate_mrl(f, 256) for f in full]), atol=2e-6)
    _check_both(got256, small_oracle, ids, lens, out_dim=256)


def test_deterministic_and_batch_invariant(small_emb, small_oracle):
    ids, lens = synth.make_batch(5, 400, small_oracle.vocab, len_range=(1, 400))
    a = small_emb.embed_tokens(ids, lens)
    b = small_emb.embed_tokens(ids, lens)
    np.testing.assert_array_equal(a, b)  # bit-identical reruns (no atomics in reductions)
    # batch vs single (tests/batch_equivalence.rs asserts >= 0.9999; rows here are exact)
    for i in range(len(lens)):
        one = small_emb.embed_tokens(ids[i:i + 1, : lens[i]], lens[i:i + 1])
        np.testing.assert_array_equal(one[0], a[i])
    # permutation of the batch permutes the output
    perm = np.array([3, 0, 4, 1, 2])
    c = small_emb.embed_tokens(ids[perm], lens[perm])
    np.testing.assert_array_equal(c, a[perm])


def test_empty_and_zero_length(small_emb):
    assert small_emb.embed_batch([]) == []
    ids = np.zeros((2, 8), dtype=np.int32)
    ids[1, :3] = [5, 6, 7]
    out = small_emb.embed_tokens(ids, np.array([0, 3], dtype=np.int32))
    np.testing.assert_array_equal(out[0], 0.0)  # mean over no tokens -> 0 (model.rs:676-679)
    assert abs(np.linalg.norm(out[1]) - 1.0) < 1e-5


def test_errors(small_emb):
    info = small_emb.info
    ids = np.full((1, info.max_position + 1), 5, dtype=np.int32)
    with pytest.raises(GlyprError) as e:
        small_emb.embed_tokens(ids, np.array([info.max_position + 1], dtype=np.int32))
    assert e.value.code == api.GLP_ERR_CONTEXT_LIMIT
    assert "exceeds model max_position_embeddings" in e.value.message
    with pytest.raises(GlyprError) as e:
        small_emb.embed_tokens(np.array([[info.vocab]], dtype=np.int32), np.array([1], dtype=np.int32))
    assert e.value.code == api.GLP_ERR_INVALID_ARG
    with pytest.raises(GlyprError) as e:
        small_emb.embed_tokens(np.array([[3]], dtype=np.int32), np.array([1], dtype=np.int32), out_dim=769)
    assert e.value.code == api.GLP_ERR_INVALID_ARG
    assert small_emb.device_status() == 0


def test_bf16_weights(bf16_gguf):
    orc = oracle.OracleModel(bf16_gguf)
    with GlyprEmbedder.load_gguf(bf16_gguf, [0]) as emb:
        ids, lens = synth.make_batch(3, 600, orc.vocab, lengths=[600, 200, 33])
        got = emb.embed_tokens(ids, lens)
    want = orc.embed(ids, lens, oracle.M2_EXACT)
    _check(got, want)


def test_deep_parity(deep_cond_gguf):
    """24 layers (4 global), conditioned: the full BASELINE depth end to end."""
    orc = oracle.OracleModel(deep_cond_gguf)
    with GlyprEmbedder.load_gguf(deep_cond_gguf, [0]) as emb:
        ids, lens = synth.make_batch(4, 1024, orc.vocab, lengths=[512, 1024, 77, 300])
        got = emb.embed_tokens(ids, lens)
    _check_both(got, orc, ids, lens)


def test_chaotic_baseline_init_properties(deep_gguf):
    """BASELINE init, 24 layers: outputs are finite unit vectors, deterministic and
    batch-invariant (the end-to-end value is chaotic in any rounding, see module doc)."""
    orc = oracle.OracleModel(deep_gguf)
    with GlyprEmbedder.load_gguf(deep_gguf, [0]) as emb:
        ids, lens = synth.make_batch(3, 512, orc.vocab, lengths=[512, 200, 31])
        a = emb.embed_tokens(ids, lens)
        b = emb.embed_tokens(ids[1:2], lens[1:2])
    np.testing.assert_allclose(np.linalg.norm(a, axis=1), 1.0, atol=1e-5)
    np.testing.assert_array_equal(a[1], b[0])
    assert np.isfinite(a).all()


def test_baseline_init_one_layer(gguf_dir):
    """BASELINE init, one layer: the GPU path stays as close to the exact result as the
    reference's own candle-faithful path does (the amplification starts in layer 1)."""
    import os
    path = synth.ensure_gguf(os.path.join(str(gguf_dir), "one_layer.gguf"), synth.EncoderConfig(n_layers=1, vocab=4096))
    orc = oracle.OracleModel(path)
    ids, lens = synth.make_batch(4, 512, orc.vocab, lengths=[512, 300, 100, 40])
    with GlyprEmbedder.load_gguf(path, [0]) as emb:
        got = emb.embed_tokens(ids, lens)
    m1 = orc.embed(ids, lens, oracle.M1_CANDLE)
    m2 = orc.embed(ids, lens, oracle.M2_EXACT)
    gpu_gap = 1.0 - cosine_rows(got, m2)
    ref_gap = 1.0 - cosine_rows(m1, m2)
    print("1-layer BASELINE init: 1-cos(gpu, exact) =", gpu_gap, " 1-cos(M1, exact) =", ref_gap)
    assert (gpu_gap <= np.maximum(2.0 * ref_gap, 1e-4)).all()


@pytest.mark.parametrize("hidden,n_heads,n_kv,ffn,head_dims,weight_type,n_layers", [
    (512, 4, 2, 2048, (2048, 1024, 512), "q8_0", 6),  # EmbeddingGemma 2 widths; a head stage wider than H
    (1536, 6, 2, 1536, (768,), "q8_0", 2),
    (1024, 4, 1, 1536, (1024,), "bf16", 2),
    (2048, 8, 2, 2048, (2048,), "q8_0", 2),
])
def test_other_hidden_sizes(gguf_dir, hidden, n_heads, n_kv, ffn, head_dims, weight_type, n_layers):
    """Hidden sizes other than 768 (the row kernels instantiated per width, the post-norm as a
    row kernel after the O and down GEMMs): parity with the oracle on ragged sequences (one
    longer than a pooling segment), a six-layer model with its global layer, and batch == single."""
    import os
    cfg = synth.small_config(n_layers=n_layers, hidden=hidden, n_heads=n_heads, n_kv_heads=n_kv, ffn=ffn,
                             head_dims=head_dims, weight_type=weight_type, qk_gain_scale=0.25)
    path = synth.ensure_gguf(os.path.join(str(gguf_dir), f"h{hidden}_{weight_type}.gguf"), cfg)
    orc = oracle.OracleModel(path)
    ids, lens = synth.make_batch(4, 600, orc.vocab, lengths=[600, 513, 64, 1])
    with GlyprEmbedder.load_gguf(path, [0]) as emb:
        assert emb.info.hidden == hidden and emb.info.embedding_dim == head_dims[-1]
        got = emb.embed_tokens(ids, lens)
        one = emb.embed_tokens(ids[2:3, : lens[2]], lens[2:3])
        mrl = emb.embed_tokens(ids, lens, out_dim=128)
        assert emb.device_status() == 0
    np.testing.assert_array_equal(one[0], got[2])
    np.testing.assert_allclose(mrl, np.stack([api.truncate_mrl(g, 128) for g in got]), atol=2e-6)
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    _check_both(got, orc, ids, lens)


@pytest.mark.parametrize("kw", [
    # EmbeddingGemma 2 widths (hidden 512, FFN 2048, 4 query heads over 2 KV heads on the sliding
    # layers and 1 on the global one) with 256-wide per-layer inputs, six layers
    dict(n_layers=6, hidden=512, n_heads=4, n_kv_heads=2, global_kv_heads=1, ffn=2048, head_dims=(2048, 512),
         ple_dim=256),
    # BASELINE widths (the fused row-norm O projection) with 512-wide per-layer inputs
    dict(n_layers=2, ple_dim=512),
])
def test_per_layer_embeddings(gguf_dir, kw):
    """Per-layer embeddings (ple.rs:48-145): the per-layer inputs from the embedding rows, and
    after each FFN block the gate, GeGLU with the layer's slice, projection, post-norm,
    residual and layer scalar.  Parity with the oracle, batch == single."""
    import os
    cfg = synth.small_config(qk_gain_scale=0.25, **kw)
    path = synth.ensure_gguf(os.path.join(str(gguf_dir), f"ple_{cfg.hidden}_{cfg.ple_dim}.gguf"), cfg)
    orc = oracle.OracleModel(path)
    ids, lens = synth.make_batch(4, 600, orc.vocab, lengths=[600, 513, 64, 1])
    with GlyprEmbedder.load_gguf(path, [0]) as emb:
        got = emb.embed_tokens(ids, lens)
        one = emb.embed_tokens(ids[2:3, : lens[2]], lens[2:3])
        assert emb.device_status() == 0
    np.testing.assert_array_equal(one[0], got[2])
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    _check_both(got, orc, ids, lens)
    # the block is not the identity: the same weights without PLE tensors embed differently
    plain = synth.small_config(qk_gain_scale=0.25, **{k: v for k, v in kw.items() if k != "ple_dim"})
    ppath = synth.ensure_gguf(os.path.join(str(gguf_dir), f"nople_{plain.hidden}.gguf"), plain)
    with GlyprEmbedder.load_gguf(ppath, [0]) as emb:
        base = emb.embed_tokens(ids, lens)
    assert cosine_rows(got, base).max() < 0.999


def test_committed_golden_vectors(gguf_dir):
    """The GPU path against the committed oracle fixtures (tests/golden/manifest.json) with the
    gates above, for the conditioned cases (the head_dim-512 global layers included)."""
    import json
    import os
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    man = json.load(open(os.path.join(golden, "manifest.json")))
    checked = 0
    for case in man["cases"]:
        cfg = synth.EncoderConfig(**case["config"])
        path = synth.ensure_gguf(os.path.join(str(gguf_dir), "golden_" + case["name"] + ".gguf"), cfg, case["seed"])
        if cfg.qk_gain_scale == 1.0:
            continue  # BASELINE init: chaotic under rounding (module doc), checked by properties
        data = np.load(os.path.join(golden, case["file"]))
        with GlyprEmbedder.load_gguf(path, [0]) as emb:
            got = emb.embed_tokens(data["ids"], data["lengths"], out_dim=int(case["out_dim"]))
        m1, m2 = data["m1"], data["m2"]
        _check(got, m2, abs_gate=ABS_GATE * np.sqrt(768.0 / got.shape[1]))
        # against the reference path: within twice its own distance from the exact result (a
        # 17-token sequence of the hidden-512 model has M1 1.2e-4 from exact, cosine)
        gap = 1.0 - cosine_rows(m1, m2)
        assert (cosine_rows(got, m1) >= np.minimum(COS_GATE, 1.0 - 2.0 * gap - 2e-5)).all(), case["name"]
        checked += 1
    assert checked >= 5


@pytest.mark.parametrize("kw", [
    # EmbeddingGemma 2's structure: hidden 512, 4 query heads over 2 KV heads on sliding layers,
    # 1 KV head of 512 dims on the global layer, per-layer embeddings
    dict(n_layers=6, hidden=512, n_heads=4, n_kv_heads=2, global_kv_heads=1, global_head_dim=512, ffn=2048,
         head_dims=(768,), ple_dim=256),
    # BASELINE widths with 512-wide global heads (3 query heads, 1 KV head), no PLE
    dict(n_layers=6, global_head_dim=512),
])
def test_global_layers_head_dim_512(gguf_dir, kw):
    """Global layers with 512-wide heads: the QKV GEMM plus the 512-wide norm/RoPE row kernel,
    the two-CTA tcgen05 attention, the wider O projection; parity with the oracle and
    batch == single."""
    import os
    cfg = synth.small_config(qk_gain_scale=0.25, **kw)
    path = synth.ensure_gguf(os.path.join(str(gguf_dir), f"d512_{cfg.hidden}_{cfg.ple_dim}.gguf"), cfg)
    orc = oracle.OracleModel(path)
    ids, lens = synth.make_batch(4, 600, orc.vocab, lengths=[600, 513, 64, 1])
    with GlyprEmbedder.load_gguf(path, [0]) as emb:
        got = emb.embed_tokens(ids, lens)
        one = emb.embed_tokens(ids[1:2, : lens[1]], lens[1:2])
        assert emb.device_status() == 0
    np.testing.assert_array_equal(one[0], got[1])
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    _check_both(got, orc, ids, lens)
