"""Texts to embeddings through the library (glp_embed_texts, glp_engine_embed_text).

The small conditioned model is written with a real BPE vocabulary in its tokenizer keys
(the golden ``trained`` vocabulary).  Each text entry point must give exactly the embedding
of the ids the oracle tokeniser produces for the reference's formatting of that text, fed
through glp_embed_tokens (the token path is checked against the model oracle elsewhere), and
over-long texts must fail with the reference's message for that path.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from glypr_b200 import api, synth
from glypr_b200.api import GlyprEmbedder, GlyprError, InferenceEngine, Tokenizer
from oracle import tokenizer_ref as R

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
TRAINED = next(s for s in json.load(open(os.path.join(HERE, "golden", "tokenizer_golden.json"),
                                         encoding="utf-8"))["sets"] if s["name"] == "trained")
TEXTS = [c["text"] for c in TRAINED["cases"] if len(c["ids"]) < 600][:48]


@pytest.fixture(scope="module")
def text_model(gguf_dir):
    cfg = synth.small_config(qk_gain_scale=0.25)
    path = os.path.join(str(gguf_dir), "small_cond_tok.gguf")
    if not os.path.exists(path):
        synth.write_gguf(path, cfg, tokenizer=(TRAINED["tokens"], TRAINED["merges"]))
    tokens = TRAINED["tokens"] + [f"<t{i}>" for i in range(len(TRAINED["tokens"]), cfg.vocab)]
    return path, R.BpeTokenizer(tokens, TRAINED["merges"])


def _by_ids(emb, id_rows, out_dim=None):
    return np.stack([emb.embed_tokens(np.asarray(r, np.int32)[None, :], np.array([len(r)], np.int32), out_dim)[0]
                     for r in id_rows])


def test_embed_texts_equal_token_path(text_model):
    path, ref = text_model
    with GlyprEmbedder.load_gguf(path, [0]) as emb, Tokenizer.from_gguf(path) as tok:
        for form in (api.GLP_TOKENS_SINGLE, api.GLP_TOKENS_SEQUENCE):
            got = emb.embed_texts(tok, TEXTS, form)
            want = _by_ids(emb, [ref.encode(t, form) for t in TEXTS])
            np.testing.assert_array_equal(got, want)
        got = emb.embed_texts(tok, TEXTS[:5], api.GLP_TOKENS_SEQUENCE, truncate_dim=128)
        np.testing.assert_array_equal(got, _by_ids(emb, [ref.encode(t, 2) for t in TEXTS[:5]], 128))


def test_query_and_document_helpers(text_model):
    path, ref = text_model
    with GlyprEmbedder.load_gguf(path, [0]) as emb, Tokenizer.from_gguf(path) as tok:
        q = emb.embed_query(tok, "the station and the quing", "question_answering")
        want = _by_ids(emb, [ref.encode(R.format_query("the station and the quing", "question_answering"))])[0]
        np.testing.assert_array_equal(q, want)
        d = emb.embed_document(tok, "ka lo mi ne", "Σ title")
        np.testing.assert_array_equal(d, _by_ids(emb, [ref.encode(R.format_document("ka lo mi ne", "Σ title"))])[0])
        t = emb.embed_text(tok, "ru sta tion", "clustering")
        np.testing.assert_array_equal(t, _by_ids(emb, [ref.encode(R.task_format("clustering", None, "ru sta tion"))])[0])
        qs = emb.embed_batch_queries(tok, TEXTS[:6], "sts")
        np.testing.assert_array_equal(qs, _by_ids(emb, [ref.encode(R.format_query(x, "sts"), 2) for x in TEXTS[:6]]))


def test_text_length_limits(text_model):
    path, ref = text_model
    long_text = "the station " * 40
    n = len(ref.encode(long_text, R.FORM_SEQUENCE))
    with GlyprEmbedder.load_gguf(path, [0]) as emb, Tokenizer.from_gguf(path) as tok:
        cases = [
            (api.GLP_TOKENS_SINGLE, [long_text], f"Text sequence length ({n} tokens) exceeds maximum context limit (50 tokens)"),
            (api.GLP_TOKENS_SINGLE, ["x", long_text],
             f"Batch item 1 sequence length ({n} tokens) exceeds maximum context limit (50 tokens)"),
            (api.GLP_TOKENS_SEQUENCE, ["x", long_text], f"Batch item 1 sequence length ({n}) exceeds maximum context limit (50)"),
            (api.GLP_TOKENS_SEQUENCE, [long_text],
             f"Interleaved multimodal sequence length ({n} tokens) exceeds maximum context limit (50 tokens). "
             "Preflight check failed before neural encoding (parts: 1)."),
        ]
        for form, texts, msg in cases:
            with pytest.raises(GlyprError) as e:
                emb.embed_texts(tok, texts, form, max_seq_len=50)
            assert e.value.code == api.GLP_ERR_CONTEXT_LIMIT and e.value.message == msg


def test_engine_text_requests(text_model):
    path, ref = text_model
    with GlyprEmbedder.load_gguf(path, [0]) as emb, Tokenizer.from_gguf(path) as tok:
        with InferenceEngine(emb, max_batch_size=8) as eng:
            got = [eng.embed_text(tok, t, "search_query") for t in TEXTS[:12]]
            got.append(eng.embed_text(tok, "ka lo", "document", "Doc A", truncate_dim=256))
        want = _by_ids(emb, [ref.encode(R.task_format("search_query", None, t), R.FORM_SEQUENCE) for t in TEXTS[:12]])
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g, w)
        full = _by_ids(emb, [ref.encode(R.task_format("document", "Doc A", "ka lo"), R.FORM_SEQUENCE)])[0]
        np.testing.assert_allclose(got[-1], api.truncate_mrl(full, 256), atol=1e-6)


def _long_texts(n, words):
    rng = np.random.default_rng(11)
    base = [c["text"] for c in TRAINED["cases"] if 20 < len(c["text"]) < 400]
    return [" ".join(base[j] for j in rng.integers(0, len(base), size=words)) for _ in range(n)]


def test_embed_texts_in_parts_equal_one_batch(text_model):
    """A batch of ~0.6 MB of text is tokenised in parts, each overlapping the previous part's
    embedding; the result equals one token batch of the same ids."""
    path, _ = text_model
    texts = _long_texts(64, 60)
    assert sum(len(t.encode()) for t in texts) > 3 * 3 * 65536  # three parts or more
    with GlyprEmbedder.load_gguf(path, [0]) as emb, Tokenizer.from_gguf(path) as tok:
        got = emb.embed_texts(tok, texts, api.GLP_TOKENS_SEQUENCE)
        rows = tok.encode_batch(texts, api.GLP_TOKENS_SEQUENCE)
        width = max(len(r) for r in rows)
        ids = np.zeros((len(rows), width), np.int32)
        for i, r in enumerate(rows):
            ids[i, :len(r)] = r
        want = emb.embed_tokens(ids, np.array([len(r) for r in rows], np.int32))
        np.testing.assert_array_equal(got, want)
        got128 = emb.embed_texts(tok, texts[:40], api.GLP_TOKENS_SINGLE, truncate_dim=128)
        np.testing.assert_allclose(got128, np.stack([api.truncate_mrl(w, 128) for w in
                                                     emb.embed_texts(tok, texts[:40], api.GLP_TOKENS_SINGLE)]),
                                   atol=2e-6)


def test_embed_texts_in_parts_first_error(text_model):
    """Errors of a split batch are the unsplit ones: the first over-limit item in batch order,
    and a later part's preflight error before an earlier part's max-position failure."""
    path, _ = text_model
    texts = _long_texts(64, 60)
    with GlyprEmbedder.load_gguf(path, [0]) as emb, Tokenizer.from_gguf(path) as tok:
        n = [len(r) for r in tok.encode_batch(texts, api.GLP_TOKENS_SEQUENCE)]
        lim = sorted(n)[-3] - 1  # exactly three items exceed it
        first = min(i for i in range(64) if n[i] > lim)
        with pytest.raises(GlyprError) as e:
            emb.embed_texts(tok, texts, api.GLP_TOKENS_SEQUENCE, max_seq_len=lim)
        assert e.value.code == api.GLP_ERR_CONTEXT_LIMIT
        assert e.value.message == f"Batch item {first} sequence length ({n[first]}) exceeds maximum context limit ({lim})"
        # item 2 is longer than the model's 8192 positions but within the default limit 8320;
        # item 50 is beyond the limit: the reference's preflight reports item 50
        unit = "the station "
        per = len(tok.encode(unit * 101, api.GLP_TOKENS_BARE)) - len(tok.encode(unit * 100, api.GLP_TOKENS_BARE))
        k = (8240 - 2) // per
        mid = unit * k
        m = len(tok.encode(mid, api.GLP_TOKENS_SEQUENCE))
        assert emb.info.max_position < m <= 8320, m
        bad = list(texts)
        bad[2] = mid
        bad[50] = unit * (9000 // per)
        nb = len(tok.encode(bad[50], api.GLP_TOKENS_SEQUENCE))
        with pytest.raises(GlyprError) as e:
            emb.embed_texts(tok, bad, api.GLP_TOKENS_SEQUENCE)
        assert e.value.message == f"Batch item 50 sequence length ({nb}) exceeds maximum context limit (8320)"
        # no partial output: parts 0 and 1 embed before part 2's item 50 fails its preflight,
        # and the caller's buffer stays untouched
        import ctypes
        bad2 = list(texts)
        bad2[50] = unit * (9000 // per)
        enc = [t.encode() for t in bad2]
        out = np.full((64, 768), 7.0, np.float32)
        rc = api.load_library().glp_embed_texts(
            emb._h, tok._h, ctypes.cast((ctypes.c_char_p * 64)(*enc), ctypes.c_void_p),
            ctypes.cast((ctypes.c_size_t * 64)(*[len(b) for b in enc]), ctypes.c_void_p), 64,
            api.GLP_TOKENS_SEQUENCE, 0, 768, out.ctypes.data_as(ctypes.c_void_p))
        assert rc == api.GLP_ERR_CONTEXT_LIMIT and (out == 7.0).all()
        bad[50] = texts[50]
        with pytest.raises(GlyprError) as e:
            emb.embed_texts(tok, bad, api.GLP_TOKENS_SEQUENCE)
        assert e.value.code == api.GLP_ERR_CONTEXT_LIMIT and "max_position_embeddings" in e.value.message
