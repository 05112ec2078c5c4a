"""The dynamic-batching engine over the real model (glp_engine_create): requests from many
client threads, batched by the worker into glp_embed_tokens, return exactly what a direct
single-sequence call returns (the path is batch-invariant), Matryoshka-truncated rows match
the reference's host truncation, and a request the model rejects fails with the model's
message while later requests still succeed.
"""
from __future__ import annotations

import threading

import numpy as np
import pytest

from glypr_b200 import api, synth
from glypr_b200.api import GlyprEmbedder, GlyprError, InferenceEngine

pytestmark = pytest.mark.gpu


def test_engine_matches_direct_calls(small_cond_gguf):
    with GlyprEmbedder.load_gguf(small_cond_gguf, [0]) as emb:
        n = 40
        ids, lens = synth.make_batch(n, 600, emb.info.vocab, seed=3, len_range=(1, 600))
        seqs = [ids[i, : lens[i]].copy() for i in range(n)]
        direct = [emb.embed_tokens(s[None, :], np.array([len(s)], np.int32))[0] for s in seqs]
        got, errors = {}, []
        with InferenceEngine(emb, max_batch_size=8) as eng:
            def client(c):
                try:
                    for i in range(c, n, 8):
                        got[i] = eng.embed(seqs[i])
                        got[(i, 256)] = eng.embed(seqs[i], truncate_dim=256)
                except Exception as e:  # pragma: no cover
                    errors.append(e)

            threads = [threading.Thread(target=client, args=(c,)) for c in range(8)]
            for t in threads:
                t.start()
            for t in threads:
                t.join(timeout=300)
            st = eng.stats()
        assert not errors, errors
        for i in range(n):
            np.testing.assert_array_equal(got[i], direct[i])
            np.testing.assert_allclose(got[(i, 256)], api.truncate_mrl(direct[i], 256), atol=1e-6)
        assert st["requests"] == 2 * n and st["largest_batch"] <= 8


def test_engine_reports_model_errors(small_cond_gguf):
    with GlyprEmbedder.load_gguf(small_cond_gguf, [0]) as emb, InferenceEngine(emb, max_batch_size=4) as eng:
        with pytest.raises(GlyprError) as e:
            eng.embed(np.full(emb.info.max_position + 1, 5, np.int32))
        assert "Batch inference error" in e.value.message
        assert "exceeds model max_position_embeddings" in e.value.message
        ok = eng.embed(np.array([5, 6, 7], np.int32))
        np.testing.assert_array_equal(ok, emb.embed_tokens(np.array([[5, 6, 7]], np.int32), np.array([3], np.int32))[0])
