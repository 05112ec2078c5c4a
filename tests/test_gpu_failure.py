"""Failure detection on the GPU without a GPU fault (the forms this pool allows).

* A kernel waits, with the pipelines' bounded wait, on a barrier nobody arrives at; the wait
  runs out after about a millisecond, the kernel records status 6 and returns, the host reads
  GLP_ERR_DEVICE through glp_kernel_status, the word is cleared by that read, and the device
  keeps working (a GEMM right after is correct).
* The kernel-level entry points' status words read 0 after correct calls.
* glp_options.device_memory_limit_mib: a limit below the model's plan fails before any
  allocation (free device memory unchanged); the plan the library states equals what a
  successful open holds; a limit that the host-API staging would cross fails that call with
  GLP_ERR_OOM and leaves the context usable.
* Two devices in one context (glp_open with [0, 1]): bit-identical to one device.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from glypr_b200 import api, synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    api.load_library()
    yield


def _gemm_ok():
    rng = np.random.default_rng(5)
    n, k, m = 256, 512, 64
    blocks = synth.quantize_q8_0((rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)))
    d_w = torch.from_numpy(blocks.view(np.uint8).reshape(-1).copy()).cuda()
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(torch.bfloat16).cuda()
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    api.q8_0_gemm(d_w.data_ptr(), n, k, x.data_ptr(), m, y.data_ptr(), True)
    torch.cuda.synchronize()
    exact = x.float().cpu().numpy().astype(np.float64) @ synth.dequantize_q8_0(blocks).astype(np.float64).T
    got = y.cpu().numpy().astype(np.float64)
    assert np.abs(got - exact).max() <= 1e-2 * np.abs(exact).max()


def test_bounded_wait_runs_out_and_is_reported():
    assert api.kernel_status(0) == 0
    t0 = time.perf_counter()
    api.selftest_wait_timeout(0, 1000)  # 1 ms limit on a barrier nobody arrives at
    dt = time.perf_counter() - t0
    assert dt < 5.0
    with pytest.raises(api.GlyprError) as e:
        api.kernel_status(0)
    assert e.value.code == api.GLP_ERR_DEVICE
    assert "device status 6" in e.value.message and "self-test" in e.value.message
    assert api.kernel_status(0) == 0          # the read cleared the word
    _gemm_ok()                                 # the context is still usable
    assert api.kernel_status(0) == 0


def test_kernel_status_after_the_noalloc_entry_point():
    rng = np.random.default_rng(9)
    n, k, m = 768, 768, 100
    blocks = synth.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
    d_w = torch.from_numpy(blocks.view(np.uint8).reshape(-1).copy()).cuda()
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(torch.bfloat16).cuda()
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    api.q8_0_gemm_noalloc(d_w.data_ptr(), n, k, x.data_ptr(), m, y.data_ptr(), True)
    assert api.kernel_status(0) == 0


def test_selftest_argument_checks():
    with pytest.raises(api.GlyprError) as e:
        api.selftest_wait_timeout(0, 0)
    assert e.value.code == api.GLP_ERR_INVALID_ARG
    with pytest.raises(api.GlyprError):
        api.selftest_wait_timeout(0, 3_000_000)
    with pytest.raises(api.GlyprError):
        api.kernel_status(torch.cuda.device_count())


def test_device_memory_limit(small_cond_gguf):
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    with pytest.raises(api.GlyprError) as e:
        api.GlyprEmbedder.load_gguf(small_cond_gguf, [0], max_batch_tokens=8192, device_memory_limit_mib=8)
    assert e.value.code == api.GLP_ERR_OOM
    assert torch.cuda.mem_get_info()[0] == free0  # nothing was allocated (or everything released)
    need = int(e.value.message.split("the model needs ")[1].split(" MiB")[0])
    with api.GlyprEmbedder.load_gguf(small_cond_gguf, [0], max_batch_tokens=8192, device_memory_limit_mib=need) as emb:
        plan = emb.info.device_bytes
        assert 0 < plan <= need << 20
        ids, lens = synth.make_batch(4, 64, emb.info.vocab, lengths=[64, 10, 1, 33])
        emb.embed_tokens(ids, lens)
        # the host-API staging grew by a few KB inside the limit
        info = api.GlpModelInfo()
        api.check(api.load_library().glp_model_info(emb._h, api.ctypes.byref(info)))
        assert info.device_bytes > plan
    # the headroom left after the open (the load staging's share): a batch whose staged ids do
    # not fit fails with GLP_ERR_OOM, smaller batches still run
    with api.GlyprEmbedder.load_gguf(small_cond_gguf, [0], max_batch_tokens=8192, device_memory_limit_mib=need) as emb:
        room = (need << 20) - emb.info.device_bytes
        n = room // (4 * 64) + 64  # more staged ids than the headroom holds
        ids, lens = synth.make_batch(int(n), 64, emb.info.vocab)
        with pytest.raises(api.GlyprError) as e2:
            emb.embed_tokens(ids, lens)
        assert e2.value.code == api.GLP_ERR_OOM
        out = emb.embed_tokens(ids[:4], lens[:4])  # smaller batches still run
        assert np.isfinite(out).all()


def test_two_devices_in_one_context(small_cond_gguf):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ids, lens = synth.make_batch(9, 200, 4096, len_range=(1, 200), seed=77)
    with api.GlyprEmbedder.load_gguf(small_cond_gguf, [0]) as one:
        want = one.embed_tokens(ids, lens)
    timing = api.GlpTiming()
    with api.GlyprEmbedder.load_gguf(small_cond_gguf, [0, 1]) as two:
        got = two.embed_tokens(ids, lens, timing=timing)
        assert two.device_status(0) == 0 and two.device_status(1) == 0
    assert timing.n_devices == 2 and timing.device_ms[0] > 0 and timing.device_ms[1] > 0
    np.testing.assert_array_equal(got, want)
