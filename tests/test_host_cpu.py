"""Host-side checks of libglypr_cuda.so that need no GPU: the library loads, exports every
function include/glypr_cuda.h declares, and rejects malformed GGUF files (host-side fault
injection: corrupt, truncated, missing keys/tensors, unsupported layouts) before it touches a
device -- the reference's anyhow errors from config.rs:79-95 / model.rs:251-473."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from glypr_b200 import api, synth

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "glypr_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(glp_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = api.load_library()
    names = declared_functions()
    assert len(names) >= 13
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(api.EXPORTED_SYMBOLS)
    assert lib.glp_last_error() is not None


def _open(path):
    L = api.load_library()
    out = ctypes.c_void_p()
    rc = L.glp_open(path.encode(), None, 0, None, ctypes.byref(out))
    msg = L.glp_last_error().decode()
    if rc == api.GLP_OK:
        L.glp_close(out)
    return rc, msg


@pytest.fixture(scope="module")
def tiny_cfg():
    return synth.small_config(n_layers=1, vocab=256)


def test_open_missing_file(tmp_path):
    rc, msg = _open(str(tmp_path / "nope.gguf"))
    assert rc == api.GLP_ERR_IO and "cannot open" in msg


def test_open_not_gguf(tmp_path):
    p = tmp_path / "junk.gguf"
    p.write_bytes(os.urandom(4096))
    rc, msg = _open(str(p))
    assert rc == api.GLP_ERR_FORMAT and "magic" in msg


@pytest.mark.parametrize("keep", [40, 300, 0.5])
def test_open_truncated(tmp_path, tiny_cfg, keep):
    full = synth.write_gguf(str(tmp_path / "full.gguf"), tiny_cfg)
    data = open(full, "rb").read()
    n = int(len(data) * keep) if isinstance(keep, float) else keep
    p = tmp_path / "cut.gguf"
    p.write_bytes(data[:n])
    rc, msg = _open(str(p))
    assert rc == api.GLP_ERR_FORMAT, msg
    assert "truncated" in msg or "out of file bounds" in msg or "too small" in msg


def test_open_missing_metadata(tmp_path, tiny_cfg):
    p = synth.write_gguf(str(tmp_path / "m.gguf"), tiny_cfg, drop={"gemma-embedding2.block_count"})
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_FORMAT and msg == "Missing gemma-embedding2.block_count"


def test_open_missing_tensor(tmp_path, tiny_cfg):
    p = synth.write_gguf(str(tmp_path / "t.gguf"), tiny_cfg, drop={"blk.0.ffn_up.weight"})
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_FORMAT and "blk.0.ffn_up.weight" in msg


def test_open_ple_block_without_projection(tmp_path, tiny_cfg):
    """A layer's PLE block without the model-level projection (model.rs:257-275 loads both)."""
    p = synth.write_gguf(str(tmp_path / "ple.gguf"), tiny_cfg, extra_f32=[("blk.0.proj.weight", (768, 256))])
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_FORMAT and msg == "missing tensor per_layer_model_proj.weight"


@pytest.mark.parametrize("drop,want", [
    ("blk.0.layer_output_scale.weight", "missing tensor blk.0.layer_output_scale.weight"),
    ("blk.0.inp_gate.weight", "missing tensor blk.0.inp_gate.weight"),
    ("per_layer_proj_norm.weight", "missing tensor per_layer_proj_norm.weight"),
])
def test_open_ple_missing_tensor(tmp_path, drop, want):
    cfg = synth.small_config(n_layers=1, vocab=256, ple_dim=256)
    p = synth.write_gguf(str(tmp_path / "ple.gguf"), cfg, drop={drop})
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_FORMAT and msg == want


def test_open_ple_width(tmp_path):
    cfg = synth.small_config(n_layers=1, vocab=256, ple_dim=96)
    rc, msg = _open(synth.write_gguf(str(tmp_path / "p96.gguf"), cfg))
    assert rc == api.GLP_ERR_UNSUPPORTED and "per_layer_input" in msg
    cfg = synth.small_config(n_layers=2, vocab=256, ple_dim=256)
    rc, msg = _open(synth.write_gguf(str(tmp_path / "p256.gguf"), cfg))
    assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg


def test_open_rejects_f32_linear(tmp_path, tiny_cfg):
    p = synth.write_gguf(str(tmp_path / "f32.gguf"), tiny_cfg, f32_mats={"blk.0.attn_k.weight"})
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_UNSUPPORTED and "attn_k" in msg


@pytest.mark.parametrize("hidden", [640, 2304])
def test_open_rejects_other_hidden(tmp_path, hidden):
    cfg = synth.small_config(n_layers=1, vocab=256, hidden=hidden, head_dims=(hidden,))
    p = synth.write_gguf(str(tmp_path / f"h{hidden}.gguf"), cfg)
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_UNSUPPORTED and msg == "hidden size must be a multiple of 256 up to 2048"


@pytest.mark.parametrize("hidden", [256, 512, 1024, 2048])
def test_open_accepts_hidden_multiples_of_256(tmp_path, hidden):
    """Hidden sizes the row kernels are compiled for pass the config checks; without a GPU the
    open then stops at the first CUDA call, never at a format or support check."""
    cfg = synth.small_config(n_layers=1, vocab=256, hidden=hidden, head_dims=(hidden,))
    p = synth.write_gguf(str(tmp_path / f"h{hidden}.gguf"), cfg)
    rc, msg = _open(p)
    assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg


def test_open_accepts_global_kv_heads(tmp_path):
    """Global layers with their own KV-head count (head_count_kv[i], config.rs:141-160) load."""
    cfg = synth.small_config(n_layers=6, vocab=256, n_heads=4, n_kv_heads=2, global_kv_heads=1)
    rc, msg = _open(synth.write_gguf(str(tmp_path / "kv.gguf"), cfg))
    assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg
    cfg = synth.small_config(n_layers=6, vocab=256, n_heads=4, n_kv_heads=2, global_kv_heads=3)
    rc, msg = _open(synth.write_gguf(str(tmp_path / "kv3.gguf"), cfg))
    assert rc == api.GLP_ERR_FORMAT and msg == "head_count must be a multiple of head_count_kv"


def test_open_accepts_global_head_dim_512(tmp_path):
    """The real EmbeddingGemma 2's head_dim-512 global layers (config.rs:141-160, 512-wide RoPE
    at model.rs:279) pass every format and support check; without a GPU the open then stops
    at the first CUDA call."""
    cfg = synth.small_config(n_layers=6, vocab=256, hidden=512, n_heads=4, n_kv_heads=2, global_kv_heads=1,
                             global_head_dim=512, head_dims=(512,))
    rc, msg = _open(synth.write_gguf(str(tmp_path / "d512.gguf"), cfg))
    assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg


def test_open_rejects_head_dim_other_than_256_or_512(tmp_path):
    cfg = synth.small_config(n_layers=6, vocab=256, global_head_dim=384)
    rc, msg = _open(synth.write_gguf(str(tmp_path / "d384.gguf"), cfg))
    assert rc == api.GLP_ERR_UNSUPPORTED and msg == "head_dim must be 256 (512 is supported on global layers)"


def test_open_head_dim_default_512_needs_512_wide_tensors(tmp_path):
    cfg = synth.small_config(n_layers=6, vocab=256)
    p = synth.write_gguf(str(tmp_path / "hd.gguf"), cfg, drop={"gemma-embedding2.attention.key_length"})
    # key_length defaults to 512 for the global layer (config.rs:143-144); this file's global
    # layer has 256-wide tensors, so its shapes do not match
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_FORMAT and msg == "bad shape for blk.5.attn_q_norm.weight"


def test_util_mirrors():
    v = api.l2_normalize(np.zeros(4, np.float32))
    np.testing.assert_array_equal(v, 0)  # util.rs:24-25 returns the zero vector unchanged
    assert api.cosine_similarity(np.zeros(3), np.ones(3)) == 0.0
    assert abs(api.cosine_similarity([1, 0], [0, 1])) < 1e-7


def test_make_batch_padding():
    ids, lens = synth.make_batch(5, 40, 1000, len_range=(3, 40))
    assert ids.shape == (5, 40) and lens.min() >= 3 and lens.max() <= 40
    for i, L in enumerate(lens):
        assert (ids[i, L:] == 0).all() and (ids[i, :L] >= 2).all() and (ids[i, :L] < 1000).all()


@pytest.mark.parametrize("global_kv,ok", [(1, True), (2, False)])
def test_open_kv_heads_defaults(tmp_path, global_kv, ok):
    """Without head_count_kv the sliding layers take 2 KV heads and the global ones 1
    (config.rs:141-160): a file whose tensors agree opens, one whose global layer has 2 fails on
    that layer's shapes."""
    cfg = synth.small_config(n_layers=6, vocab=256, n_heads=4, n_kv_heads=2, global_kv_heads=global_kv)
    p = synth.write_gguf(str(tmp_path / "kv.gguf"), cfg, drop={"gemma-embedding2.attention.head_count_kv"})
    rc, msg = _open(p)
    if ok:
        assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg
    else:
        assert rc == api.GLP_ERR_FORMAT and msg == "bad shape for blk.5.attn_k.weight"


@pytest.mark.parametrize("ple_dim,ok", [(512, True), (256, False)])
def test_open_ple_width_default(tmp_path, ple_dim, ok):
    """Without embedding_length_per_layer_input the per-layer width is 512 (config.rs:100-102)."""
    cfg = synth.small_config(n_layers=2, vocab=256, ple_dim=ple_dim)
    p = synth.write_gguf(str(tmp_path / "ple.gguf"), cfg,
                         drop={"gemma-embedding2.embedding_length_per_layer_input"})
    rc, msg = _open(p)
    if ok:
        assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg
    else:
        assert rc == api.GLP_ERR_FORMAT and msg == "bad shape for per_layer_model_proj.weight"


def test_kv_heads_non_integer_elements_take_the_defaults(tmp_path):
    """head_count_kv elements that are not integers yield no value in the reference's get_u32
    (config.rs:253-265), so the defaults apply: 2 for the sliding layers, 1 for global ones.
    An f32 array therefore behaves like a missing key."""
    cfg = synth.small_config(n_layers=6, vocab=256, n_heads=4, n_kv_heads=2, global_kv_heads=1)
    key = "gemma-embedding2.attention.head_count_kv"
    p = synth.write_gguf(str(tmp_path / "kvf.gguf"), cfg, drop={key},
                         extra_kv=[synth.gguf_kv(key, "arr_f32", [2.0] * 5 + [1.0])])
    rc, msg = _open(p)
    assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg
    # f32 elements [3, ..] would give 3 KV heads if they were read; the defaults (2, 1) fit the tensors
    p = synth.write_gguf(str(tmp_path / "kvf3.gguf"), cfg, drop={key},
                         extra_kv=[synth.gguf_kv(key, "arr_f32", [3.0] * 6)])
    rc, msg = _open(p)
    assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg


def test_scalar_keys_follow_the_reference_types(tmp_path):
    """An f32 context_length is not an integer for the reference's get_u32 (config.rs:253-265):
    the default 262144 (config.rs:95-96) applies instead of a truncated 300, so the model
    still opens (without a GPU: up to the first CUDA call)."""
    cfg = synth.small_config(n_layers=1, vocab=256)
    key = "gemma-embedding2.context_length"
    p = synth.write_gguf(str(tmp_path / "ctx.gguf"), cfg, drop={key}, extra_kv=[synth.gguf_kv(key, "f32", 300.5)])
    rc, msg = _open(p)
    assert rc not in (api.GLP_ERR_UNSUPPORTED, api.GLP_ERR_FORMAT), msg


def test_layer_output_scale_checked_before_allocation(tmp_path):
    """A malformed per-layer scalar is a format error found while validating the file, before
    any device work (so it fails the same way with or without a GPU)."""
    cfg = synth.small_config(n_layers=2, vocab=256, ple_dim=256)
    p = synth.write_gguf(str(tmp_path / "los.gguf"), cfg, f32_scalars={"blk.1.layer_output_scale.weight"})
    rc, msg = _open(p)
    assert rc == api.GLP_ERR_FORMAT and msg == "bad layer_output_scale"


def _open_opts(path, limit_mib):
    L = api.load_library()
    out = ctypes.c_void_p()
    opt = api.GlpOptions(device_memory_limit_mib=limit_mib)
    rc = L.glp_open(path.encode(), None, 0, ctypes.byref(opt), ctypes.byref(out))
    msg = L.glp_last_error().decode()
    if rc == api.GLP_OK:
        L.glp_close(out)
    assert not out.value or rc == api.GLP_OK
    return rc, msg


def test_device_memory_limit_fails_before_any_device_work(tmp_path):
    """glp_options.device_memory_limit_mib: a plan above the limit fails with GLP_ERR_OOM
    before the library touches a device (so this runs without one) and no context comes back;
    a limit above the plan passes the check (without a GPU the open then stops at the first
    CUDA call)."""
    cfg = synth.small_config(n_layers=1, vocab=256)
    p = synth.write_gguf(str(tmp_path / "cap.gguf"), cfg)
    rc, msg = _open_opts(p, 16)
    assert rc == api.GLP_ERR_OOM, msg
    assert "above the limit of 16 MiB" in msg
    need = int(msg.split("the model needs ")[1].split(" MiB")[0])
    assert need > 16
    rc, msg = _open_opts(p, need)
    assert rc != api.GLP_ERR_OOM, msg


def test_status_texts():
    """Every device status code the kernels record has its own text (glp_status_text)."""
    texts = {c: api.status_text(c) for c in range(0, 7)}
    assert texts[0] == "no device error"
    assert len(set(texts.values())) == 7
    assert "self-test" in texts[6]
    assert api.status_text(99) == "unknown device status code"
