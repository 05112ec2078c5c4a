"""Seeded synthetic GGUF writer for the EmbeddingGemma-style text encoder.

The reference only *reads* GGUF files (candle's ``gguf_file::Content``, called from
``crates/glypr-core/src/model.rs:229-488`` and ``src/config.rs:76-213``); there are no
real weights in this environment, so every weight file used by the tests and the bench
is produced here from one master seed.  The writer emits exactly the key and tensor
schema the reference loader looks up:

* metadata ``gemma-embedding2.*`` keys (``config.rs:79-189``) plus ``tokenizer.ggml.tokens``
  whose length is the vocabulary size (``config.rs:107-110``);
* tensors ``token_embd.weight`` and ``blk.N.{attn_norm, attn_q, attn_k, attn_v,
  attn_output, attn_q_norm, attn_k_norm, post_attention_norm, ffn_norm, ffn_gate, ffn_up,
  ffn_down, post_ffw_norm}.weight`` and ``output_norm.weight`` (``model.rs:251-473``);
* the two-stage dense head as ``dense.0.weight`` [3072, 768] and ``dense.1.weight``
  [768, 3072] (a documented extension: the reference has a single ``output.weight``,
  ``model.rs:472-473``, which is also accepted by the loader when ``head_dims`` is
  ``(embedding_out,)``).

Per-layer-embedding tensors (``ple.rs``) are written only when ``ple_dim > 0``: absent PLE is
the identity (zero ``proj`` weight and a layer scalar of 1 give ``h' = (h + RMSNorm(0)) * 1 =
h``, ``ple.rs:118-145``).  With ``ple_dim = D`` the file carries the reference's PLE schema
(``model.rs:257-275, 418-453``): metadata ``embedding_length_per_layer_input`` = D,
``per_layer_model_proj.weight`` [L*D, H], ``per_layer_proj_norm.weight`` [D] and per layer
``inp_gate.weight`` [D, H], ``proj.weight`` [H, D], ``post_norm.weight`` [H] and
``layer_output_scale.weight`` [1].  They follow every other tensor, so the other tensors'
seeds (their index in the order) are the same with or without PLE.

Quantiser (pinned here; the reference only reads the blocks): per 32-element block,
``d = absmax / 127`` in f32, stored as IEEE fp16 (round to nearest even);
``q = round_half_away_from_zero(w * (1/d))`` clamped to [-127, 127]; ``d == 0`` gives
``q == 0``.  This is the ggml ``quantize_row_q8_0`` recipe.  Block layout is
``{fp16 d; int8 qs[32]}`` = 34 bytes, row-major over the input dimension
(``metal_kernels/fused_ops.metal:568-572``).

Norm gains are written as F32 ``1 + g`` with ``g ~ N(0, 0.1)``: Gemma's ``(1 + w)``
convention folded at conversion time, so the loader computes plain ``x_hat * w``
(``norm.rs:47-53``).
"""
from __future__ import annotations

import dataclasses
import os
import struct
from typing import Iterable, List, Optional, Sequence, Tuple

import numpy as np

MASTER_SEED = 20261201

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian
GGUF_VERSION = 3
ALIGNMENT = 32

# ggml tensor type ids
GGML_F32 = 0
GGML_F16 = 1
GGML_Q8_0 = 8
GGML_BF16 = 30

# gguf metadata value type ids
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)

Q8_0_BLOCK = 32
Q8_0_BYTES = 34
Q8_0_DTYPE = np.dtype([("d", "<f2"), ("qs", "i1", (Q8_0_BLOCK,))])
assert Q8_0_DTYPE.itemsize == Q8_0_BYTES


@dataclasses.dataclass(frozen=True)
class EncoderConfig:
    """Shape of the synthetic encoder (defaults = the BASELINE shape)."""

    n_layers: int = 24
    hidden: int = 768
    ffn: int = 1152
    n_heads: int = 3
    n_kv_heads: int = 1
    head_dim: int = 256
    vocab: int = 262144
    context_length: int = 8192
    eps: float = 1e-6
    rope_theta_swa: float = 10000.0
    rope_theta_full: float = 1000000.0
    head_dims: Tuple[int, ...] = (3072, 768)  # dense head stages; (E,) = reference output.weight
    weight_type: str = "q8_0"  # "q8_0" or "bf16" (matrices incl. token table)
    weight_std: float = 0.02
    gain_std: float = 0.1
    # global (full-attention) layers: (i+1) % 6 == 0, the reference default (config.rs:131-139)
    global_every: int = 6
    # multiplier on the q/k norm gains: 1.0 = BASELINE init.  0.25 scales every attention
    # logit by 1/16 (a well-conditioned variant used for end-to-end parity tests; the
    # reference attention scale stays 1.0, standard.rs:62).
    qk_gain_scale: float = 1.0
    # per-layer-embedding width D (0 = no PLE tensors)
    ple_dim: int = 0
    # KV heads of the global layers (0 = n_kv_heads, as on the sliding layers)
    global_kv_heads: int = 0
    # head_dim of the global layers (0 = head_dim; the real EmbeddingGemma 2 has 512 there)
    global_head_dim: int = 0

    def head_dim_of(self, i: int) -> int:
        return self.head_dim if self.layer_is_sliding(i) or not self.global_head_dim else self.global_head_dim

    def kv_heads(self, i: int) -> int:
        return self.n_kv_heads if self.layer_is_sliding(i) or not self.global_kv_heads else self.global_kv_heads

    @property
    def embedding_out(self) -> int:
        return self.head_dims[-1]

    def layer_is_sliding(self, i: int) -> bool:
        return (i + 1) % self.global_every != 0


BASELINE = EncoderConfig()


def small_config(**kw) -> EncoderConfig:
    """A reduced encoder for fast parity tests (same per-layer shapes, fewer layers)."""
    base = dict(n_layers=2, vocab=4096, context_length=8192)
    base.update(kw)
    return EncoderConfig(**base)


# ---------------------------------------------------------------------------------------
# quantisation helpers
# ---------------------------------------------------------------------------------------

def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """Quantise an f32 matrix [N, K] (K % 32 == 0) to Q8_0 blocks -> structured [N, K/32]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if k % Q8_0_BLOCK:
        raise ValueError("Q8_0 needs the input dimension to be a multiple of 32")
    blocks = w.reshape(-1, Q8_0_BLOCK)
    amax = np.abs(blocks).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    x = blocks * inv[:, None]
    q = np.sign(x) * np.floor(np.abs(x) + np.float32(0.5))  # round half away from zero
    q = np.clip(q, -127, 127).astype(np.int8)
    out = np.empty(blocks.shape[0], dtype=Q8_0_DTYPE)
    out["d"] = d.astype(np.float16)
    out["qs"] = q
    return out.reshape(n, k // Q8_0_BLOCK)


def dequantize_q8_0(blocks: np.ndarray) -> np.ndarray:
    """Exact f32 dequantisation f32(d) * q (candle/ggml ``dequantize_row_q8_0``)."""
    d = blocks["d"].astype(np.float32)
    q = blocks["qs"].astype(np.float32)
    return (q * d[..., None]).reshape(blocks.shape[0], -1)


def to_bf16_bits(w: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns (round to nearest even), as uint16."""
    u = np.ascontiguousarray(w, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------------------
# GGUF serialisation
# ---------------------------------------------------------------------------------------

def _gstr(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, value) -> bytes:
    out = _gstr(key) + struct.pack("<I", vtype)
    if vtype == _U32:
        out += struct.pack("<I", value)
    elif vtype == _F32:
        out += struct.pack("<f", value)
    elif vtype == _F64:
        out += struct.pack("<d", value)
    elif vtype == _STR:
        out += _gstr(value)
    elif vtype == _BOOL:
        out += struct.pack("<B", 1 if value else 0)
    elif vtype == _ARR:
        etype, items = value
        out += struct.pack("<IQ", etype, len(items))
        if etype == _U32:
            out += np.asarray(items, dtype="<u4").tobytes()
        elif etype == _BOOL:
            out += np.asarray(items, dtype=np.uint8).tobytes()
        elif etype == _F32:
            out += np.asarray(items, dtype="<f4").tobytes()
        elif etype == _STR:
            out += b"".join(_gstr(s) for s in items)
        else:
            raise ValueError(etype)
    else:
        raise ValueError(vtype)
    return out


def gguf_kv(key: str, vtype: str, value) -> bytes:
    """One encoded GGUF key/value for write_gguf's ``extra_kv``: vtype "u32", "f32", "f64",
    "str", "bool", or "arr_u32" / "arr_f32" / "arr_bool" with a list value."""
    if vtype.startswith("arr_"):
        et = {"u32": _U32, "f32": _F32, "bool": _BOOL}[vtype[4:]]
        return _kv(key, _ARR, (et, value))
    return _kv(key, {"u32": _U32, "f32": _F32, "f64": _F64, "str": _STR, "bool": _BOOL}[vtype], value)


def _kv_key(kv: bytes) -> str:
    (n,) = struct.unpack_from("<Q", kv, 0)
    return kv[8:8 + n].decode()


def _tensor_order(cfg: EncoderConfig) -> List[Tuple[str, Tuple[int, ...], str]]:
    """(name, shape [rows, cols] or [n], kind) in the fixed sub-stream order."""
    h, f = cfg.hidden, cfg.ffn
    order: List[Tuple[str, Tuple[int, ...], str]] = [("token_embd.weight", (cfg.vocab, h), "mat")]
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        d = cfg.head_dim_of(i)
        order += [
            (p + "attn_norm.weight", (h,), "gain"),
            (p + "attn_q.weight", (cfg.n_heads * d, h), "mat"),
            (p + "attn_k.weight", (cfg.kv_heads(i) * d, h), "mat"),
            (p + "attn_v.weight", (cfg.kv_heads(i) * d, h), "mat"),
            (p + "attn_output.weight", (h, cfg.n_heads * d), "mat"),
            (p + "attn_q_norm.weight", (d,), "qkgain"),
            (p + "attn_k_norm.weight", (d,), "qkgain"),
            (p + "post_attention_norm.weight", (h,), "gain"),
            (p + "ffn_norm.weight", (h,), "gain"),
            (p + "ffn_gate.weight", (f, h), "mat"),
            (p + "ffn_up.weight", (f, h), "mat"),
            (p + "ffn_down.weight", (h, f), "mat"),
            (p + "post_ffw_norm.weight", (h,), "gain"),
        ]
    order.append(("output_norm.weight", (h,), "gain"))
    if len(cfg.head_dims) == 1:
        order.append(("output.weight", (cfg.head_dims[0], h), "mat"))
    else:
        prev = h
        for j, dim in enumerate(cfg.head_dims):
            order.append((f"dense.{j}.weight", (dim, prev), "mat"))
            prev = dim
    if cfg.ple_dim:
        pd = cfg.ple_dim
        order += [("per_layer_model_proj.weight", (cfg.n_layers * pd, h), "mat"),
                  ("per_layer_proj_norm.weight", (pd,), "gain")]
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            order += [(p + "inp_gate.weight", (pd, h), "mat"), (p + "proj.weight", (h, pd), "mat"),
                      (p + "post_norm.weight", (h,), "gain"), (p + "layer_output_scale.weight", (1,), "gain")]
    return order


def _rng(seed: int, index: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence(seed, spawn_key=(index,))))


def generate_tensor(cfg: EncoderConfig, seed: int, index: int, shape, kind: str):
    """Return (ggml_type, raw bytes, logical f32 array or None) for tensor #index."""
    rng = _rng(seed, index)
    if kind in ("gain", "qkgain"):
        g = rng.standard_normal(shape, dtype=np.float32) * np.float32(cfg.gain_std)
        w = (np.float32(1.0) + g).astype(np.float32)
        if kind == "qkgain" and cfg.qk_gain_scale != 1.0:
            w = (w * np.float32(cfg.qk_gain_scale)).astype(np.float32)
        return GGML_F32, w.tobytes(), w
    w = rng.standard_normal(shape, dtype=np.float32) * np.float32(cfg.weight_std)
    if cfg.weight_type == "q8_0":
        blocks = quantize_q8_0(w)
        return GGML_Q8_0, blocks.tobytes(), None
    if cfg.weight_type == "bf16":
        return GGML_BF16, to_bf16_bits(w).tobytes(), None
    raise ValueError(cfg.weight_type)


def metadata(cfg: EncoderConfig, tokenizer: Optional[Tuple[Sequence[str], Sequence[str]]] = None) -> List[bytes]:
    """GGUF key/values; ``tokenizer`` = (tokens, merges) stores a real BPE vocabulary (padded
    with filler tokens to ``cfg.vocab``) instead of the filler-only token table."""
    a = "gemma-embedding2."
    tokens = [f"<t{i}>" for i in range(cfg.vocab)]
    if tokenizer is not None:
        if len(tokenizer[0]) > cfg.vocab:
            raise ValueError("tokenizer vocabulary larger than the model's")
        tokens = list(tokenizer[0]) + tokens[len(tokenizer[0]):]
    kvs = [
        _kv("general.architecture", _STR, "gemma-embedding2"),
        _kv("general.name", _STR, "glypr-b200 synthetic encoder"),
        _kv("general.alignment", _U32, ALIGNMENT),
        _kv(a + "block_count", _U32, cfg.n_layers),
        _kv(a + "embedding_length", _U32, cfg.hidden),
        _kv(a + "feed_forward_length", _U32, cfg.ffn),
        _kv(a + "attention.head_count", _U32, cfg.n_heads),
        _kv(a + "attention.head_count_kv", _ARR, (_U32, [cfg.kv_heads(i) for i in range(cfg.n_layers)])),
        _kv(a + "attention.key_length_swa", _U32, cfg.head_dim),
        _kv(a + "attention.key_length", _U32, cfg.global_head_dim or cfg.head_dim),
        _kv(a + "embedding_length_out", _U32, cfg.embedding_out),
        _kv(a + "context_length", _U32, cfg.context_length),
        _kv(a + "attention.layer_norm_rms_epsilon", _F32, cfg.eps),
        _kv(a + "rope.freq_base_swa", _F32, cfg.rope_theta_swa),
        _kv(a + "rope.freq_base", _F32, cfg.rope_theta_full),
        _kv(a + "attention.sliding_window_pattern", _ARR,
            (_BOOL, [cfg.layer_is_sliding(i) for i in range(cfg.n_layers)])),
        _kv("tokenizer.ggml.model", _STR, "synthetic"),
        _kv("tokenizer.ggml.tokens", _ARR, (_STR, tokens)),
        _kv("tokenizer.ggml.padding_token_id", _U32, 0),
        _kv("tokenizer.ggml.bos_token_id", _U32, 2),
        _kv("tokenizer.ggml.eos_token_id", _U32, 1),
    ]
    if tokenizer is not None:
        kvs.append(_kv("tokenizer.ggml.merges", _ARR, (_STR, list(tokenizer[1]))))
    if cfg.ple_dim:
        kvs.append(_kv(a + "embedding_length_per_layer_input", _U32, cfg.ple_dim))
    return kvs


def _nbytes(shape, ggml_type) -> int:
    n = int(np.prod(shape))
    if ggml_type == GGML_F32:
        return 4 * n
    if ggml_type in (GGML_F16, GGML_BF16):
        return 2 * n
    if ggml_type == GGML_Q8_0:
        return n // Q8_0_BLOCK * Q8_0_BYTES
    raise ValueError(ggml_type)


def write_gguf(path: str, cfg: EncoderConfig = BASELINE, seed: int = MASTER_SEED,
               drop: Iterable[str] = (), extra_f32: Sequence[Tuple[str, Tuple[int, ...]]] = (),
               f32_mats: Iterable[str] = (),
               tokenizer: Optional[Tuple[Sequence[str], Sequence[str]]] = None,
               extra_kv: Sequence[bytes] = (), f32_scalars: Iterable[str] = ()) -> str:
    """Write the synthetic encoder to ``path`` (returns ``path``).

    ``drop`` omits metadata keys or tensors by name, ``extra_f32`` appends zero F32 tensors
    and ``f32_mats`` stores the named matrices as F32 instead of Q8_0/BF16 -- used by the
    host-side fault-injection tests to build malformed files; ``extra_kv`` appends encoded
    key/values (``gguf_kv``; with ``drop`` of the same key it replaces one) and
    ``f32_scalars`` stores the named one-element tensors with two elements (a malformed layer
    scalar); ``tokenizer`` = (tokens, merges) writes a BPE vocabulary into the tokenizer keys."""
    drop = set(drop)
    f32_mats = set(f32_mats)
    f32_scalars = set(f32_scalars)
    order = [(n, (2,) if n in f32_scalars else sh, k) for n, sh, k in _tensor_order(cfg) if n not in drop]
    order_idx = {n: i for i, (n, _, _) in enumerate(_tensor_order(cfg))}
    mat_type = GGML_Q8_0 if cfg.weight_type == "q8_0" else GGML_BF16
    infos = []
    offset = 0
    for name, shape, kind in order:
        t = GGML_F32 if kind in ("gain", "qkgain") or name in f32_mats else mat_type
        infos.append((name, shape, t, offset))
        offset += _nbytes(shape, t)
        offset = (offset + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    for name, shape in extra_f32:
        infos.append((name, shape, GGML_F32, offset))
        order.append((name, shape, "zero"))
        offset += _nbytes(shape, GGML_F32)
        offset = (offset + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    kvs = [kv for kv in metadata(cfg, tokenizer) if _kv_key(kv) not in drop] + list(extra_kv)
    header = struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(infos), len(kvs)) + b"".join(kvs)
    tinfo = b""
    for name, shape, t, off in infos:
        dims = tuple(reversed(shape))  # ne[0] is the innermost (contiguous) dimension
        tinfo += _gstr(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        tinfo += struct.pack("<IQ", t, off)
    head = header + tinfo
    pad = (-len(head)) % ALIGNMENT
    tmp = path + ".tmp"
    with open(tmp, "wb") as fh:
        fh.write(head + b"\0" * pad)
        pos = 0
        for (name, shape, kind), (_, _, t, off) in zip(order, infos):
            if pos < off:
                fh.write(b"\0" * (off - pos))
                pos = off
            if kind == "zero":
                raw = np.zeros(shape, dtype=np.float32).tobytes()
            elif name in f32_mats:
                rng = _rng(seed, order_idx[name])
                raw = (rng.standard_normal(shape, dtype=np.float32) * np.float32(cfg.weight_std)).tobytes()
            else:
                gt, raw, _ = generate_tensor(cfg, seed, order_idx[name], shape, kind)
                assert gt == t, name
            assert len(raw) == _nbytes(shape, t), name
            fh.write(raw)
            pos += len(raw)
    os.replace(tmp, path)
    return path


def ensure_gguf(path: str, cfg: EncoderConfig = BASELINE, seed: int = MASTER_SEED) -> str:
    """Write the file unless an identical-size file already exists."""
    if not os.path.exists(path):
        write_gguf(path, cfg, seed)
    return path


# ---------------------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------------------

def make_batch(n_seq: int, max_len: int, vocab: int, seed: int = MASTER_SEED,
               lengths: Optional[Sequence[int]] = None,
               len_range: Optional[Tuple[int, int]] = None, stream: int = 1_000_003
               ) -> Tuple[np.ndarray, np.ndarray]:
    """Token ids uniform in [2, vocab), right-padded with id 0 (``tokenizer.rs:182-229``).

    Returns ``ids`` int32 [n_seq, max_len] and ``lengths`` int32 [n_seq].  Lengths are all
    ``max_len`` unless ``lengths`` is given or ``len_range=(lo, hi)`` draws them uniformly
    from ``[lo, hi]``.
    """
    rng = _rng(seed, stream)
    if lengths is None:
        if len_range is None:
            lengths = np.full(n_seq, max_len, dtype=np.int32)
        else:
            lengths = rng.integers(len_range[0], len_range[1] + 1, size=n_seq).astype(np.int32)
    lengths = np.asarray(lengths, dtype=np.int32)
    ids = rng.integers(2, vocab, size=(n_seq, max_len)).astype(np.int32)
    col = np.arange(max_len)[None, :]
    ids[col >= lengths[:, None]] = 0
    return ids, lengths
