"""Pin the CPU oracle against every known answer the reference's own tests hold for this
path (no GPU needed).

* util.rs:258-306       MRL / L2 known answers
* tests/test_cpu_simd.rs RMSNorm and GeGLU against the candle formula, max diff < 1e-5
* metal_kernels/mod.rs:1924-1979  the Q8_0 GEMM recipe: candle-faithful (M1) within 1e-2 of
                        the exact dequantised product
* corpus_parity.rs:420-494  long-context pooling precision recipe (f32 accumulation)
* rope.rs:14-87         RoPE tables (f64 inv_freq -> f32, f32 freqs)
* ggml quantize_row_q8_0 / dequantize_row_q8_0 (the synthetic writer's pinned quantiser)
* the llama.cpp ``gguf`` reader accepts the synthetic files (independent format check)
* committed golden vectors (tests/golden/, made by tests/golden/make_golden.py)
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import oracle
from glypr_b200 import api, synth

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ------------------------------------------------------------------ util.rs:258-306
def test_mrl_and_norm_known_answers():
    n = api.l2_normalize(np.array([3.0, 4.0], dtype=np.float32))
    assert abs(n[0] - 0.6) < 1e-6 and abs(n[1] - 0.8) < 1e-6
    v4 = api.l2_normalize(np.ones(4, dtype=np.float32))
    t = api.truncate_mrl(v4, 2)
    assert t.shape == (2,)
    assert abs(api.cosine_similarity(t, t) - 1.0) < 1e-6
    with pytest.raises(ValueError):
        api.truncate_mrl(v4, 0)
    with pytest.raises(ValueError):
        api.truncate_mrl(v4, 5)
    # the oracle's pooling path on a one-token "sequence" is L2 (+ MRL) of that row
    row = np.array([[3.0, 4.0] + [0.0] * 30], dtype=np.float32)
    p = oracle.pool_normalize(row)
    assert abs(p[0] - 0.6) < 1e-6 and abs(p[1] - 0.8) < 1e-6
    p2 = oracle.pool_normalize(np.ones((1, 4), dtype=np.float32), out_dim=2)
    np.testing.assert_allclose(p2, [2 ** -0.5] * 2, atol=1e-7)


# ------------------------------------------------------------------ tests/test_cpu_simd.rs
def test_rmsnorm_matches_candle_formula():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 8, 256)).astype(np.float32)
    w = (1.0 + 0.2 * rng.standard_normal(256)).astype(np.float32)
    eps = 1e-6
    mean_sq = (x.astype(np.float32) ** 2).mean(-1, keepdims=True)
    expected = x * (mean_sq + np.float32(eps)) ** np.float32(-0.5) * w
    got = oracle.rmsnorm(x, w, eps)
    assert np.abs(got - expected).max() < 1e-5
    got_now = oracle.rmsnorm(x, None, eps)  # v-norm: no weight (model.rs:373)
    assert np.abs(got_now - x * (mean_sq + np.float32(eps)) ** np.float32(-0.5)).max() < 1e-5


def test_geglu_matches_candle_formula():
    rng = np.random.default_rng(2)
    gate = (2.0 * rng.standard_normal((1, 16, 512))).astype(np.float32)
    up = rng.standard_normal((1, 16, 512)).astype(np.float32)
    g = gate.astype(np.float64)
    expected = 0.5 * g * (1.0 + np.tanh(0.7978845608028654 * (g + 0.044715 * g ** 3))) * up
    got = oracle.geglu(gate, up)
    assert np.abs(got - expected).max() < 1e-5
    # the +-10 clamp of cpu_simd/geglu.rs:7-10
    out = oracle.geglu(np.array([-10.0, -12.0, 10.0, 11.0], np.float32), np.full(4, 2.0, np.float32))
    np.testing.assert_array_equal(out, [0.0, 0.0, 20.0, 22.0])


# ------------------------------------------------------------------ Q8_0 quantiser / dequant
def test_q8_0_quantiser_pinned():
    # known answer: block 0..31 -> d = 31/127 (fp16), q = round(i * 127/31)
    x = np.arange(32, dtype=np.float32)
    b = synth.quantize_q8_0(x.reshape(1, 32))[0, 0]
    assert b["d"] == np.float16(np.float32(31.0) / np.float32(127.0))
    inv = np.float32(1.0) / (np.float32(31.0) / np.float32(127.0))
    want_q = np.floor(x * inv + np.float32(0.5)).astype(np.int8)
    np.testing.assert_array_equal(b["qs"], want_q)
    assert b["qs"][31] == 127
    # zero block -> d = 0, q = 0
    z = synth.quantize_q8_0(np.zeros((1, 32), np.float32))[0, 0]
    assert z["d"] == 0 and not z["qs"].any()
    # writer quantiser == oracle's ggml restatement, bit for bit
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 768)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0
    w[5, 5] = 1e-30
    ours = synth.quantize_q8_0(w).view(np.uint8).reshape(-1)
    theirs = oracle.q8_0_quantize(w)
    np.testing.assert_array_equal(ours, theirs)


def test_q8_0_dequant_oracle_vs_numpy():
    rng = np.random.default_rng(4)
    blocks = synth.quantize_q8_0((rng.standard_normal((16, 256)) * 0.5).astype(np.float32))
    a = oracle.q8_0_dequant(blocks)
    b = synth.dequantize_q8_0(blocks).reshape(-1)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    np.testing.assert_array_equal(a, (blocks["qs"].astype(np.float32) *
                                      blocks["d"].astype(np.float32)[..., None]).reshape(-1))


# ------------------------------------------------------------------ metal_kernels/mod.rs:1924-1979
def test_q8_0_gemm_recipe_m1_vs_exact():
    n, k = 128, 256
    i = np.arange(n * k, dtype=np.float32)
    w = (np.sin(i * np.float32(0.031)) * np.float32(1.5)).astype(np.float32).reshape(n, k)
    blocks = synth.quantize_q8_0(w)
    wd = synth.dequantize_q8_0(blocks).astype(np.float64)
    for m in (1, 19, 64):
        j = np.arange(m * k, dtype=np.float32)
        x = (np.cos(j * np.float32(0.059)) * np.float32(3.0)).astype(np.float32).reshape(m, k)
        m1 = oracle.q8_0_matmul(blocks, n, k, x, oracle.M1_CANDLE)
        m2 = oracle.q8_0_matmul(blocks, n, k, x, oracle.M2_EXACT)
        exact = x.astype(np.float64) @ wd.T
        assert np.abs(m2 - exact).max() <= 1e-4 * np.abs(exact).max()
        # the reference's 1e-2 bound between its Q8_0 paths, scaled to this recipe's range
        assert np.abs(m1 - exact).max() <= 1e-2 * np.abs(exact).max()


# ------------------------------------------------------------------ corpus_parity.rs:420-494
@pytest.mark.parametrize("seq_len", [1024, 2048, 4096, 8192])
def test_long_context_pooling_precision(seq_len):
    t = np.arange(seq_len)[:, None]
    c = np.arange(768)[None, :]
    raw = (((t * 7919 + c * 104729) % 10000).astype(np.float64) / 5000.0 - 1.0).astype(np.float32)
    ref = raw.astype(np.float64).mean(0)
    ref = ref / max(np.linalg.norm(ref), 1e-12)
    got = oracle.pool_normalize(raw)
    cos = float((got * ref).sum() / np.linalg.norm(got))
    assert cos >= 0.99999  # f32 accumulation (the reference gate for bf16 input is 0.95)


# ------------------------------------------------------------------ rope.rs:14-87
@pytest.mark.parametrize("theta", [1e4, 1e6])
def test_rope_tables(theta):
    d, s = 256, 300
    c, sn = oracle.rope_tables(d, theta, s)
    inv = (1.0 / theta ** (np.arange(0, d, 2, dtype=np.float64) / d)).astype(np.float32)
    freqs = np.arange(s, dtype=np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([freqs, freqs], axis=1)
    np.testing.assert_allclose(c, np.cos(emb.astype(np.float64)), atol=2e-7)
    np.testing.assert_allclose(sn, np.sin(emb.astype(np.float64)), atol=2e-7)
    np.testing.assert_array_equal(c[:, :128], c[:, 128:])


# ------------------------------------------------------------------ GGUF format cross-check
def test_gguf_readable_by_llama_cpp_reader(small_gguf):
    gguf = pytest.importorskip("gguf")
    r = gguf.GGUFReader(small_gguf)
    names = {t.name: t for t in r.tensors}
    cfg = synth.small_config()
    assert len(names) == 1 + 13 * cfg.n_layers + 1 + len(cfg.head_dims)
    te = names["token_embd.weight"]
    assert list(te.shape) == [cfg.hidden, cfg.vocab]
    assert int(te.tensor_type) == synth.GGML_Q8_0
    q = names["blk.1.attn_q.weight"]
    assert list(q.shape) == [cfg.hidden, cfg.n_heads * cfg.head_dim]
    # raw Q8_0 bytes match the writer's generator for that tensor
    order = [n for n, _, _ in synth._tensor_order(cfg)]
    idx = order.index("blk.1.attn_q.weight")
    _, raw, _ = synth.generate_tensor(cfg, synth.MASTER_SEED, idx, (cfg.n_heads * cfg.head_dim, cfg.hidden), "mat")
    assert np.asarray(q.data).tobytes() == raw
    f = r.fields["gemma-embedding2.block_count"]
    assert int(f.parts[f.data[0]][0]) == cfg.n_layers
    pat = r.fields["gemma-embedding2.attention.sliding_window_pattern"]
    assert [bool(pat.parts[i][0]) for i in pat.data] == [cfg.layer_is_sliding(i) for i in range(cfg.n_layers)]


def test_oracle_reads_config(small_gguf):
    m = oracle.OracleModel(small_gguf)
    cfg = synth.small_config()
    assert (m.n_layers, m.hidden, m.ffn, m.n_heads, m.vocab, m.emb_out, m.max_pos, m.head_dim, m.n_kv,
            m.window) == (cfg.n_layers, 768, 1152, 3, cfg.vocab, 768, cfg.context_length, 256, 1, 512)
    with pytest.raises(RuntimeError, match="exceeds model max_position_embeddings"):
        m.embed(np.zeros((1, cfg.context_length + 1), np.int32), np.array([1], np.int32))


# ------------------------------------------------------------------ committed golden vectors
def _golden():
    with open(os.path.join(GOLDEN, "manifest.json")) as fh:
        return json.load(fh)


def test_golden_vectors_reproduce(gguf_dir):
    man = _golden()
    for case in man["cases"]:
        cfg = synth.EncoderConfig(**case["config"])
        path = os.path.join(str(gguf_dir), case["name"] + ".gguf")
        synth.ensure_gguf(path, cfg, case["seed"])
        data = np.load(os.path.join(GOLDEN, case["file"]))
        m = oracle.OracleModel(path)
        for mode_name, mode in (("m1", oracle.M1_CANDLE), ("m2", oracle.M2_EXACT)):
            got = m.embed(data["ids"], data["lengths"], mode, out_dim=int(case["out_dim"]))
            want = data[mode_name]
            # same restatement, same seed: reproducible to f32 round-off of the thread split
            assert np.abs(got - want).max() <= 1e-5, (case["name"], mode_name)


# ------------------------------------------------------------------ ple.rs:48-145, layer.rs:44-49
def _tensor(cfg, name):
    """The synthetic writer's tensor `name` of `cfg`: Q8_0 blocks [n, k/32] or an f32 gain."""
    order = synth._tensor_order(cfg)
    idx = [n for n, _, _ in order].index(name)
    shape, kind = order[idx][1], order[idx][2]
    _, raw, logical = synth.generate_tensor(cfg, synth.MASTER_SEED, idx, shape, kind)
    if logical is not None:
        return logical
    return np.frombuffer(raw, dtype=synth.Q8_0_DTYPE).reshape(shape[0], shape[1] // 32)


@pytest.mark.parametrize("mode", [oracle.M1_CANDLE, oracle.M2_EXACT])
def test_ple_block_restated(gguf_dir, mode):
    """The oracle's per-layer-embedding path against a composition of the pinned primitives:
    a one-layer model with PLE tensors equals the same model without them (identical other
    tensors) followed by P = RMSNorm(proj(x0) * H^-0.5) * w (ple.rs:48-93) and
    h = (h + RMSNorm(proj(geglu(gate(h), P))) * w) * s (ple.rs:118-145, norm.rs:65-94)."""
    base = dict(n_layers=1, hidden=512, n_heads=2, n_kv_heads=1, ffn=1024, head_dims=(512,), vocab=512,
                qk_gain_scale=0.25)
    cfg_a = synth.small_config(**base)
    cfg_b = synth.small_config(ple_dim=256, **base)
    pa = synth.ensure_gguf(os.path.join(str(gguf_dir), "ple_off.gguf"), cfg_a)
    pb = synth.ensure_gguf(os.path.join(str(gguf_dir), "ple_on.gguf"), cfg_b)
    ids = np.random.default_rng(5).integers(2, 512, size=37).astype(np.int32)
    h2 = oracle.OracleModel(pa).hidden_after(ids, 0, mode)
    got = oracle.OracleModel(pb).hidden_after(ids, 0, mode)
    H, D = 512, 256
    x0 = synth.dequantize_q8_0(_tensor(cfg_b, "token_embd.weight")[ids]) * np.float32(np.sqrt(H))
    p = oracle.q8_0_matmul(_tensor(cfg_b, "per_layer_model_proj.weight"), D, H, x0, mode)
    p = oracle.rmsnorm(p * np.float32(H ** -0.5), _tensor(cfg_b, "per_layer_proj_norm.weight"))
    g = oracle.q8_0_matmul(_tensor(cfg_b, "blk.0.inp_gate.weight"), D, H, h2, mode)
    y = oracle.q8_0_matmul(_tensor(cfg_b, "blk.0.proj.weight"), H, D, oracle.geglu(g, p), mode)
    y = oracle.rmsnorm(y, _tensor(cfg_b, "blk.0.post_norm.weight"))
    s = _tensor(cfg_b, "blk.0.layer_output_scale.weight")[0]
    want = (h2 + y) * s
    assert s != 1.0 and np.abs(y).max() > 0.1
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------------ config.rs:141-160, rope.rs, model.rs:279-300
def _rope(x, cos, sin):
    """NeoX rotate_half RoPE (rope.rs:90-106) on rows [t, n, d] with tables [t, d]."""
    d = x.shape[-1]
    rot = np.concatenate([-x[..., d // 2:], x[..., :d // 2]], axis=-1)
    return (x * cos[:, None, :] + rot * sin[:, None, :]).astype(np.float32)


@pytest.mark.parametrize("mode", [oracle.M1_CANDLE, oracle.M2_EXACT])
def test_global_layer_head_dim_512_restated(gguf_dir, mode):
    """The oracle's global layer of the real EmbeddingGemma 2 (head_dim 512 from key_length, its
    own KV-head count, RoPE over 512 dims with the global theta) against a composition of the
    pinned primitives.  The CUDA library rejects such files; this pins the checker for them."""
    H, NH, KV, D = 512, 4, 1, 512
    cfg = synth.small_config(n_layers=1, global_every=1, hidden=H, n_heads=NH, n_kv_heads=2, global_kv_heads=KV,
                             global_head_dim=D, ffn=1024, head_dims=(512,), vocab=512, qk_gain_scale=0.25)
    path = synth.ensure_gguf(os.path.join(str(gguf_dir), "global_d512.gguf"), cfg)
    m = oracle.OracleModel(path)
    assert (m.head_dim, m.n_kv) == (D, KV)
    ids = np.random.default_rng(9).integers(2, 512, size=41).astype(np.int32)
    t = ids.size
    got = m.hidden_after(ids, 0, mode)

    def lin(name, n, k, x):
        return oracle.q8_0_matmul(_tensor(cfg, name), n, k, x, mode)

    h = synth.dequantize_q8_0(_tensor(cfg, "token_embd.weight")[ids]) * np.float32(np.sqrt(H))
    x = oracle.rmsnorm(h, _tensor(cfg, "blk.0.attn_norm.weight"))
    q = oracle.rmsnorm(lin("blk.0.attn_q.weight", NH * D, H, x).reshape(t, NH, D), _tensor(cfg, "blk.0.attn_q_norm.weight"))
    k = oracle.rmsnorm(lin("blk.0.attn_k.weight", KV * D, H, x).reshape(t, KV, D), _tensor(cfg, "blk.0.attn_k_norm.weight"))
    v = oracle.rmsnorm(lin("blk.0.attn_v.weight", KV * D, H, x).reshape(t, KV, D), None)
    cos, sin = oracle.rope_tables(D, cfg.rope_theta_full, t)
    q, k = _rope(q, cos, sin), _rope(k, cos, sin)
    a = oracle.attention(q.reshape(t, -1), k.reshape(t, -1), v.reshape(t, -1), NH, KV, D, 512, False)
    y = oracle.rmsnorm(lin("blk.0.attn_output.weight", H, NH * D, a), _tensor(cfg, "blk.0.post_attention_norm.weight"))
    h = h + y
    x = oracle.rmsnorm(h, _tensor(cfg, "blk.0.ffn_norm.weight"))
    g = oracle.geglu(lin("blk.0.ffn_gate.weight", 1024, H, x), lin("blk.0.ffn_up.weight", 1024, H, x))
    y = oracle.rmsnorm(lin("blk.0.ffn_down.weight", H, 1024, g), _tensor(cfg, "blk.0.post_ffw_norm.weight"))
    want = h + y
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5)


def test_baseline_init_is_ill_conditioned(deep_gguf, deep_cond_gguf):
    """Why the end-to-end cosine gate runs on the well-conditioned variant.  On the BASELINE
    init (unit q/k gains, attention scale 1.0: logits with std ~16) the reference's own two
    arithmetic forms -- M1, candle's int8 activation blocks, and M2, exact f32 dequantisation --
    disagree after 24 layers (cosine ~0.55-0.65 here), so no implementation that rounds
    differently from M1 can meet cosine >= 0.9999 there.  With the q/k gains x0.25 (logits / 16)
    the same two forms agree to better than 1e-4.  Both are the oracle (no GPU involved)."""
    ids, lens = synth.make_batch(2, 256, 4096, lengths=[256, 128], seed=7)
    chaotic = oracle.OracleModel(deep_gguf)
    a = chaotic.embed(ids, lens, oracle.M1_CANDLE)
    b = chaotic.embed(ids, lens, oracle.M2_EXACT)
    cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    assert (cos < 0.9).all(), cos
    cond = oracle.OracleModel(deep_cond_gguf)
    a = cond.embed(ids, lens, oracle.M1_CANDLE)
    b = cond.embed(ids, lens, oracle.M2_EXACT)
    cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    assert (cos >= 0.9999).all(), cos


@pytest.mark.parametrize("mode", [oracle.M1_CANDLE, oracle.M2_EXACT])
def test_simd_paths_bit_identical(small_cond_gguf, mode):
    """The oracle's AVX2 paths (int8 block dots of M1, attention with transposed keys) give
    the scalar loops' results bit for bit: the timed CPU baseline computes exactly what the
    checker computes."""
    m = oracle.OracleModel(small_cond_gguf)
    ids, lens = synth.make_batch(3, 700, m.vocab, lengths=[700, 37, 1], seed=11)
    try:
        oracle.set_simd(False)
        slow = m.embed(ids, lens, mode)
        oracle.set_simd(True)
        fast = m.embed(ids, lens, mode)
    finally:
        oracle.set_simd(True)
    np.testing.assert_array_equal(fast.view(np.uint32), slow.view(np.uint32))
