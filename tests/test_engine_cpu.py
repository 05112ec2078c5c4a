"""Dynamic-batching engine (glp_engine_*, the reference server's inference engine,
glypr-server/src/engine.rs:157-325) driven through a Python batch executor on the CPU: many
client threads, results routed back to the right caller, batches bounded by max_batch and
formed under concurrency, Matryoshka truncation on the host, a failed batch failing each of
its requests, and shutdown answering or rejecting every caller without hanging.
"""
from __future__ import annotations

import threading
import time

import numpy as np
import pytest

from glypr_b200 import api

DIM = 64


def fake_row(ids: np.ndarray) -> np.ndarray:
    """A deterministic unit vector per sequence (independent of the batch it runs in)."""
    seed = int(np.sum(ids.astype(np.int64) * (np.arange(ids.size) + 1)) % (2 ** 31)) + ids.size
    v = np.random.default_rng(seed).standard_normal(DIM).astype(np.float32)
    return v / np.linalg.norm(v)


def make_executor(delay=0.0, poison=None, seen=None):
    def fn(ids, lengths, out_dim):
        assert out_dim == DIM
        if seen is not None:
            seen.append(len(lengths))
        if delay:
            time.sleep(delay)
        rows = []
        for i, L in enumerate(lengths):
            row = ids[i, :L]
            if poison is not None and poison in row:
                raise ValueError("poisoned batch")
            rows.append(fake_row(row))
        return np.stack(rows)
    return fn


def seq(i):
    rng = np.random.default_rng(1000 + i)
    return rng.integers(2, 50000, size=int(rng.integers(0, 40)), dtype=np.int32)


@pytest.fixture(autouse=True)
def _lib():
    api.load_library()


def test_concurrent_clients_get_their_own_rows():
    seen = []
    with api.InferenceEngine.with_executor(make_executor(delay=0.004, seen=seen), DIM, max_batch_size=8) as eng:
        results = {}
        errors = []

        def client(c):
            try:
                for k in range(12):
                    i = c * 100 + k
                    results[i] = eng.embed(seq(i))
            except Exception as e:  # pragma: no cover - reported below
                errors.append(e)

        threads = [threading.Thread(target=client, args=(c,)) for c in range(16)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=120)
        assert not errors, errors
        assert len(results) == 16 * 12
        for i, v in results.items():
            np.testing.assert_array_equal(v, fake_row(seq(i)))
        st = eng.stats()
    assert st["requests"] == 16 * 12
    assert 1 < st["largest_batch"] <= 8          # batches formed under concurrency, bounded
    assert st["batches"] < st["requests"]
    assert max(seen) <= 8


def test_truncation_and_empty_sequence():
    with api.InferenceEngine.with_executor(make_executor(), DIM, max_batch_size=4) as eng:
        ids = seq(7)
        full = eng.embed(ids)
        for d in (1, 16, 63):
            got = eng.embed(ids, truncate_dim=d)
            assert got.shape == (d,)
            np.testing.assert_allclose(got, api.truncate_mrl(full, d), atol=1e-6)
        np.testing.assert_array_equal(eng.embed(ids, truncate_dim=DIM), full)  # >= width: full
        np.testing.assert_array_equal(eng.embed(np.zeros(0, np.int32)), fake_row(np.zeros(0, np.int32)))


def test_failed_batch_fails_each_request_then_recovers():
    with api.InferenceEngine.with_executor(make_executor(poison=7), DIM, max_batch_size=4) as eng:
        with pytest.raises(api.GlyprError) as e:
            eng.embed(np.array([5, 7, 9], np.int32))
        assert "Batch inference error" in e.value.message
        np.testing.assert_array_equal(eng.embed(np.array([5, 8], np.int32)), fake_row(np.array([5, 8], np.int32)))


def test_shutdown_answers_or_rejects_every_caller():
    eng = api.InferenceEngine.with_executor(make_executor(delay=0.01), DIM, max_batch_size=2, queue_capacity=4)
    outcomes = []
    lock = threading.Lock()

    def client(i):
        try:
            v = eng.embed(seq(i))
            ok = np.array_equal(v, fake_row(seq(i)))
            with lock:
                outcomes.append("ok" if ok else "wrong")
        except api.GlyprError as e:
            with lock:
                outcomes.append("rejected" if "not running" in e.message else "other")

    threads = [threading.Thread(target=client, args=(i,)) for i in range(24)]
    for t in threads:
        t.start()
    time.sleep(0.02)
    eng.close()  # answers the calls in flight, rejects later ones, stops the worker
    for t in threads:
        t.join(timeout=60)
    assert all(not t.is_alive() for t in threads)
    assert len(outcomes) == 24
    assert "wrong" not in outcomes and "other" not in outcomes
    assert outcomes.count("ok") >= 1
