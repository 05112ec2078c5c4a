"""Shared fixtures.  ``-m gpu`` tests need a B200 and the built ``libglypr_cuda.so``; every
other test runs on the CPU (oracle against golden vectors, host logic, library loading)."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from glypr_b200 import synth  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running (full 24-layer model on the CPU oracle)")


@pytest.fixture(scope="session")
def gguf_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("gguf")


def _model(gguf_dir, name, cfg):
    path = os.path.join(str(gguf_dir), name)
    synth.ensure_gguf(path, cfg)
    return path


@pytest.fixture(scope="session")
def small_gguf(gguf_dir):
    """2 layers, vocab 4096, BASELINE per-layer shapes and init."""
    return _model(gguf_dir, "small.gguf", synth.small_config())


@pytest.fixture(scope="session")
def small_cond_gguf(gguf_dir):
    """Well-conditioned 2-layer variant (q/k gains x0.25: attention logits / 16)."""
    return _model(gguf_dir, "small_cond.gguf", synth.small_config(qk_gain_scale=0.25))


@pytest.fixture(scope="session")
def deep_cond_gguf(gguf_dir):
    """24 layers (BASELINE depth, incl. 4 global layers), vocab 4096, well-conditioned."""
    return _model(gguf_dir, "deep_cond.gguf", synth.EncoderConfig(vocab=4096, qk_gain_scale=0.25))


@pytest.fixture(scope="session")
def deep_gguf(gguf_dir):
    """24 layers, vocab 4096, BASELINE init.  With unit q/k gains and attention scale 1 the
    logits have std ~16 and the 24-layer model amplifies rounding differences (two correct
    implementations that round differently disagree): tests on it check properties, not values."""
    return _model(gguf_dir, "deep.gguf", synth.EncoderConfig(vocab=4096))


@pytest.fixture(scope="session")
def bf16_gguf(gguf_dir):
    """2 layers with BF16 linears and token table (BASELINE config 4's weight format)."""
    return _model(gguf_dir, "small_bf16.gguf", synth.small_config(weight_type="bf16", qk_gain_scale=0.25))


def cosine_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    na = np.linalg.norm(a, axis=1)
    nb = np.linalg.norm(b, axis=1)
    return (a * b).sum(1) / np.maximum(na * nb, 1e-30)
