"""The multi-device coordinator of glp_embed_tokens, driven on the CPU through
glp_embed_tokens_sharded with Python executors standing in for devices (host-side fault
injection: an executor that fails, as a device whose kernel or copy failed would).

The reference's server answers a failed batch with an error for each of its requests and no
partial result (glypr-server/src/engine.rs:308-325); glp_embed_tokens keeps that contract across
devices: the caller's buffer is written only when every shard has succeeded."""
from __future__ import annotations

import threading

import numpy as np
import pytest

from glypr_b200 import api


def _fake_embed(ids, lengths, out_dim):
    """A deterministic stand-in model: row i = (len, sum of ids, first id, ...) normalised."""
    n = ids.shape[0]
    out = np.zeros((n, out_dim), np.float32)
    for i in range(n):
        L = int(lengths[i])
        v = np.arange(1, out_dim + 1, dtype=np.float64) * (L + 1) + ids[i, :L].sum()
        out[i] = (v / np.linalg.norm(v)).astype(np.float32)
    return out


def _batch(n=37, max_len=50, seed=3):
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, max_len + 1, size=n).astype(np.int32)
    ids = np.zeros((n, max_len), np.int32)
    for i, L in enumerate(lens):
        ids[i, :L] = rng.integers(2, 1000, size=L)
    return ids, lens


@pytest.mark.parametrize("n_exec", [1, 2, 3, 8])
def test_sharded_equals_single_executor(n_exec):
    ids, lens = _batch()
    calls = []
    lock = threading.Lock()

    def make(k):
        def fn(a, l, d):
            with lock:
                calls.append((k, a.shape[0], int(l.sum())))
            return _fake_embed(a, l, d)
        return fn

    got = api.embed_tokens_sharded([make(k) for k in range(n_exec)], 16, ids, lens)
    want = _fake_embed(ids, lens, 16)
    np.testing.assert_array_equal(got, want)
    assert sum(c[1] for c in calls) == len(lens)
    if n_exec > 1:  # shards balanced by token count: none above its share by more than one sequence
        total = int(lens.sum())
        for _, _, toks in calls:
            assert toks <= total / n_exec + lens.max()


@pytest.mark.parametrize("bad", [0, 1, 2])
def test_failing_executor_leaves_no_partial_output(bad):
    ids, lens = _batch(n=30)
    ran = []

    def make(k):
        def fn(a, l, d):
            ran.append(k)
            if k == bad:
                raise RuntimeError("device lost")
            return _fake_embed(a, l, d)
        return fn

    out = np.full((30, 8), np.nan, np.float32)
    with pytest.raises(api.GlyprError) as e:
        api.embed_tokens_sharded([make(k) for k in range(3)], 8, ids, lens, out=out)
    assert e.value.message.startswith(f"executor {bad}: ")
    assert sorted(ran) == [0, 1, 2]          # the other shards ran (they were not cancelled) ...
    assert np.isnan(out).all()               # ... yet nothing reached the caller's buffer


def test_sharded_argument_checks():
    ids, lens = _batch(n=4)
    with pytest.raises(api.GlyprError) as e:
        api.embed_tokens_sharded([_fake_embed], 8, ids, lens, out_dim=9)
    assert e.value.code == api.GLP_ERR_INVALID_ARG
    bad = lens.copy()
    bad[2] = ids.shape[1] + 1
    with pytest.raises(api.GlyprError):
        api.embed_tokens_sharded([_fake_embed], 8, ids, bad)
    empty = api.embed_tokens_sharded([_fake_embed, _fake_embed], 8, ids[:0], lens[:0])
    assert empty.shape == (0, 8)
