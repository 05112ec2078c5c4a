"""glp_q8_0_gemm_noalloc: the Q8_0 GEMM for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: code that runs inside host callbacks, under a
caller-owned memory pool or a fixed memory budget, or in a framework that forbids
allocations after start-up.  The entry point below dequantises into a fixed scratch array
inside the library instead, so the call allocates nothing.  This file checks, through the C
ABI, that two calls in a row give the same output as glp_q8_0_gemm (the entry point that
uses library-allocated scratch) within the GEMM tests' tolerance, that the free device
memory does not change across the calls, and that a weight larger than the array is
rejected.  It is named to run last, so that a failure here cannot stop the other tests.
"""
from __future__ import annotations

import numpy as np
import pytest

from glypr_b200 import api, synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_ELEMS = 3 * 1024 * 1024  # the scratch array's N * K limit


def _case(n, k, m, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    blocks = synth.quantize_q8_0(w)
    d_w = torch.from_numpy(blocks.view(np.uint8).reshape(-1).copy()).cuda()
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(torch.bfloat16).cuda()
    return blocks, d_w, x


def test_noalloc_matches_allocating_gemm_two_calls_in_a_row():
    torch.backends.cuda.matmul.allow_tf32 = False
    api.load_library()
    cases = [(768, 768, 300, True, 1), (2304, 768, 257, False, 2)]  # two different calls in a row
    prepared = []
    for n, k, m, f32, seed in cases:
        blocks, d_w, x = _case(n, k, m, seed)
        dt = torch.float32 if f32 else torch.bfloat16
        y_ref = torch.empty((m, n), dtype=dt, device="cuda")
        y_new = torch.full((m, n), float("nan"), dtype=dt, device="cuda")
        # reference: the allocating entry point (its scratch is allocated here, before measuring)
        api.q8_0_gemm(d_w.data_ptr(), n, k, x.data_ptr(), m, y_ref.data_ptr(), f32)
        prepared.append((n, k, m, f32, blocks, d_w, x, y_ref, y_new))
    torch.cuda.synchronize()
    for n, k, m, f32, blocks, d_w, x, y_ref, y_new in prepared:
        free_before = torch.cuda.mem_get_info()[0]
        api.q8_0_gemm_noalloc(d_w.data_ptr(), n, k, x.data_ptr(), m, y_new.data_ptr(), f32)
        torch.cuda.synchronize()
        # no bounded wait of the kernel ran out (the status read allocates nothing either)
        assert api.kernel_status(0) == 0
        free_after = torch.cuda.mem_get_info()[0]
        assert free_after == free_before, "the no-allocation entry point changed free device memory"
        got = y_new.float().cpu().numpy().astype(np.float64)
        ref = y_ref.float().cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all()
        # the GEMM tests' tolerance against the allocating path's output (same kernels: the
        # results are expected to be identical)
        scale = np.abs(ref).max()
        tol = 2e-5 if f32 else 8e-3
        assert np.abs(got - ref).max() <= tol * scale
        # and BASELINE config 2's check against the f32 dequantised reference
        exact = x.float().cpu().numpy().astype(np.float64) @ synth.dequantize_q8_0(blocks).astype(np.float64).T
        assert np.abs(got - exact).max() <= 1e-2 * np.abs(exact).max()


def test_noalloc_rejects_weights_beyond_the_scratch_array():
    n, k = 4096, 1024  # 4,194,304 > 3,145,728 elements
    assert n * k > MAX_ELEMS
    d_w = torch.zeros(n * k // 32 * 34, dtype=torch.uint8, device="cuda")
    x = torch.zeros((8, k), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((8, n), dtype=torch.float32, device="cuda")
    with pytest.raises(api.GlyprError) as e:
        api.q8_0_gemm_noalloc(d_w.data_ptr(), n, k, x.data_ptr(), 8, y.data_ptr(), True)
    assert e.value.code == api.GLP_ERR_INVALID_ARG
    assert "no-allocation scratch limit" in e.value.message
