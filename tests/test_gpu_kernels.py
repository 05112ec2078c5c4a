"""Kernel-level parity on the GPU, through the C ABI (libglypr_cuda.so).

* Q8_0 dequantisation: bit-exact against the oracle (and numpy).
* Q8_0 GEMM: within 1e-2 relative of the f32 dequantised reference (BASELINE config 2's
  check), within 1e-5 relative of an f32 GEMM on the same bf16-rounded operands (the
  kernel's own arithmetic), and the reference's own Q8_0 GEMM recipe
  (metal_kernels/mod.rs:1924-1979: out 128 x in 256, w = sin(i*0.031)*1.5,
  x = cos(i*0.059)*3, M in {1, 19, 64}, within 1e-2 of candle QMatMul = oracle M1, relative
  to the output range).
* Flash attention: against the oracle's f32 attention on the same f16 inputs.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from glypr_b200 import api, synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _no_tf32():
    torch.backends.cuda.matmul.allow_tf32 = False
    api.load_library()
    yield


def _q8_blocks(n, k, seed, std=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(std)).astype(np.float32)
    return synth.quantize_q8_0(w)


def _dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("n_blocks", [1, 7, 24 * 768, 262144 * 24 // 16 + 3])
def test_q8_0_dequant_bit_exact(n_blocks):
    rng = np.random.default_rng(n_blocks)
    raw = rng.integers(0, 256, size=n_blocks * 34, dtype=np.uint8)
    # scales: random finite fp16 values incl. subnormals, zero and negative
    d = rng.standard_normal(n_blocks).astype(np.float16)
    d[::5] = np.float16(0.0)
    d[1::7] = np.float16(6e-6)  # subnormal
    raw.reshape(n_blocks, 34)[:, :2] = d.view(np.uint8).reshape(n_blocks, 2)
    want = oracle.q8_0_dequant(raw)
    blocks = raw.view(synth.Q8_0_DTYPE)
    np.testing.assert_array_equal(want.view(np.uint32),
                                  synth.dequantize_q8_0(blocks.reshape(1, -1)).reshape(-1).view(np.uint32))
    d_in = _dev(raw)
    d_out = torch.empty(n_blocks * 32, dtype=torch.float32, device="cuda")
    api.q8_0_dequant(d_in.data_ptr(), n_blocks, d_out.data_ptr())
    torch.cuda.synchronize()
    got = d_out.cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


SHAPES = [(768, 768), (256, 768), (1152, 768), (768, 1152), (1280, 768), (2304, 768), (3072, 768),
          (768, 3072), (128, 256)]


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 19, 130, 512, 4096])
@pytest.mark.parametrize("f32_out", [True, False])
def test_q8_0_gemm(n, k, m, f32_out):
    blocks = _q8_blocks(n, k, seed=n * 7 + k)
    w_exact = synth.dequantize_q8_0(blocks)  # f32(d) * q
    rng = np.random.default_rng(m + n)
    x = rng.standard_normal((m, k), dtype=np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16).cuda()
    d_w = _dev(blocks.view(np.uint8).reshape(-1))
    y = torch.empty((m, n), dtype=torch.float32 if f32_out else torch.bfloat16, device="cuda")
    api.q8_0_gemm(d_w.data_ptr(), n, k, xb.data_ptr(), m, y.data_ptr(), f32_out)
    torch.cuda.synchronize()
    got = y.float().cpu().numpy().astype(np.float64)
    xf = xb.float().cpu().numpy().astype(np.float64)
    ref_exact = xf @ w_exact.astype(np.float64).T
    scale = np.abs(ref_exact).max()
    # within 1e-2 relative of the f32 dequantised reference
    assert np.abs(got - ref_exact).max() <= 1e-2 * scale
    # the kernel's own arithmetic: bf16(q*d) operands, f32 accumulation
    w_bf16 = torch.from_numpy(w_exact).to(torch.bfloat16).float().numpy().astype(np.float64)
    ref_bf = xf @ w_bf16.T
    tol = 2e-5 if f32_out else 8e-3
    assert np.abs(got - ref_bf).max() <= tol * scale


def _gemm_check(blocks, n, k, m, d_w_ptr, f32_out, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16).cuda()
    y = torch.full((m, n), float("nan"), dtype=torch.float32 if f32_out else torch.bfloat16, device="cuda")
    api.q8_0_gemm(d_w_ptr, n, k, xb.data_ptr(), m, y.data_ptr(), f32_out)
    assert api.kernel_status(0) == 0
    got = y.float().cpu().numpy().astype(np.float64)
    xf = xb.float().cpu().numpy().astype(np.float64)
    w_bf16 = torch.from_numpy(synth.dequantize_q8_0(blocks)).to(torch.bfloat16).float().numpy().astype(np.float64)
    ref = xf @ w_bf16.T
    tol = 2e-5 if f32_out else 8e-3
    assert np.abs(got - ref).max() <= tol * np.abs(ref).max()


@pytest.mark.parametrize("n,k", [(768, 768), (1152, 768), (768, 1152), (256, 64), (384, 768)])
@pytest.mark.parametrize("m", [8192, 8193])
def test_q8_0_gemm_both_routes(n, k, m):
    """M = 8192 runs the kernel that streams raw Q8_0 rows and dequantises in shared memory
    (every group-row view: K = 768 and 1152 take 1 and 2 rows per TMA row, K = 64 four), M =
    8193 the dequantise-then-GEMM route; both against bf16(q d) operands with f32 accumulation.
    N = 1152 and 384 (odd multiples of 128) run the second route's CTA-pair GEMM with a last
    256-wide tile half past N: every output is written (NaN-filled beforehand) and nothing
    spills into the next row."""
    blocks = _q8_blocks(n, k, seed=n + k + m)
    d_w = _dev(blocks.view(np.uint8).reshape(-1))
    _gemm_check(blocks, n, k, m, d_w.data_ptr(), True, seed=m)
    _gemm_check(blocks, n, k, m, d_w.data_ptr(), False, seed=m + 1)


def test_q8_0_gemm_unaligned_weight():
    """A weight that starts off a 16-byte boundary (a row slice of a fused weight, as the
    reference's try_concat views are) takes the dequantise-then-GEMM route at any M."""
    n, k = 256, 1152
    blocks = _q8_blocks(n, k, seed=3)
    raw = blocks.view(np.uint8).reshape(-1)
    buf = torch.zeros(raw.size + 16, dtype=torch.uint8, device="cuda")
    buf[2:2 + raw.size] = _dev(raw)
    _gemm_check(blocks, n, k, 300, buf.data_ptr() + 2, True, seed=4)


def test_q8_0_gemm_reference_recipe():
    """metal_kernels/mod.rs:1924-1979 restated: 128 x 256, sin/cos inputs, 1e-2 (relative to
    the output range) vs the candle-faithful QMatMul (oracle M1)."""
    n, k = 128, 256
    i = np.arange(n * k, dtype=np.float32)
    w = (np.sin(i * np.float32(0.031)) * np.float32(1.5)).astype(np.float32).reshape(n, k)
    blocks = synth.quantize_q8_0(w)
    d_w = _dev(blocks.view(np.uint8).reshape(-1))
    for m in (1, 19, 64):
        j = np.arange(m * k, dtype=np.float32)
        x = (np.cos(j * np.float32(0.059)) * np.float32(3.0)).astype(np.float32).reshape(m, k)
        xb = torch.from_numpy(x).to(torch.bfloat16)
        ref = oracle.q8_0_matmul(blocks, n, k, xb.float().numpy(), oracle.M1_CANDLE)
        ref = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()  # reference casts to bf16
        y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        api.q8_0_gemm(d_w.data_ptr(), n, k, xb.cuda().data_ptr(), m, y.data_ptr(), False)
        torch.cuda.synchronize()
        got = y.float().cpu().numpy()
        # 1e-2 relative to the output range: outputs reach ~44, where one bf16 ulp is 0.25
        assert np.abs(got - ref).max() <= 1e-2 * np.abs(ref).max()


def test_gemm_rejects_bad_shapes():
    x = torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(128 * 100 // 32 * 34, dtype=torch.uint8, device="cuda")
    y = torch.zeros((4, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(api.GlyprError) as e:
        api.q8_0_gemm(w.data_ptr(), 128, 100, x.data_ptr(), 4, y.data_ptr(), True)
    assert e.value.code == api.GLP_ERR_INVALID_ARG


def _attn_case(lengths, n_heads, n_kv, window, seed, logit_scale=1.0, d=256):
    rng = np.random.default_rng(seed)
    t = int(sum(lengths))
    width = (n_heads + 2 * n_kv) * d
    qkv = rng.standard_normal((t, width), dtype=np.float32)
    # q/k rows unit-RMS like the QK-normed activations; logit_scale sets the logit spread
    qkv[:, : (n_heads + n_kv) * d] *= np.float32(np.sqrt(logit_scale) / 4.0)
    qkv16 = qkv.astype(np.float16)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    d_qkv = _dev(qkv16)
    d_cu = _dev(cu)
    out = torch.zeros((max(t, 1), n_heads * d), dtype=torch.float16, device="cuda")
    api.flash_attention(d_qkv.data_ptr(), d_cu.data_ptr(), len(lengths), int(max(lengths)), n_heads, n_kv, d,
                        window, out.data_ptr())
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    q32 = qkv16.astype(np.float32)
    for b, L in enumerate(lengths):
        s0 = cu[b]
        sl = slice(s0, s0 + L)
        q = q32[sl, : n_heads * d]
        k = q32[sl, n_heads * d:(n_heads + n_kv) * d]
        v = q32[sl, (n_heads + n_kv) * d:]
        ref = oracle.attention(q, k, v, n_heads, n_kv, d, window if window > 0 else 0, window > 0)
        err = np.abs(got[sl] - ref).max()
        assert err <= 1e-2 * max(1.0, np.abs(ref).max()), (b, L, err)


@pytest.mark.parametrize("lengths", [[1], [7, 64, 100], [128, 129], [512], [300, 512, 1]])
@pytest.mark.parametrize("window", [0, 512])
def test_flash_attention_short(lengths, window):
    _attn_case(lengths, 3, 1, window, seed=sum(lengths) + window)


@pytest.mark.parametrize("window", [0, 512])
def test_flash_attention_long_window(window):
    _attn_case([1300, 700], 3, 1, window, seed=11 + window)


def test_flash_attention_gqa_and_sharp_logits():
    _attn_case([257, 64], 4, 2, 512, seed=5)
    # BASELINE-like logit spread (unit-gain q/k norms, scale 1.0): std ~16
    _attn_case([512], 3, 1, 0, seed=6, logit_scale=16.0)


@pytest.mark.parametrize("lengths", [[1], [7, 64, 100], [300, 512, 33], [700]])
@pytest.mark.parametrize("window", [0, 512])
def test_flash_attention_head_dim_512(lengths, window):
    """512-wide heads (EmbeddingGemma 2's global layers): 4 query heads over 1 and 2 KV heads."""
    _attn_case(lengths, 4, 1, window, seed=sum(lengths) + 3 * window, d=512)
    _attn_case(lengths, 4, 2, window, seed=sum(lengths) + 3 * window + 1, d=512)
