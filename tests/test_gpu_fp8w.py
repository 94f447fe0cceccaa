"""GPU parity of the FP8 weight path: rms_norm_fp8_out codes bit-exact against
the oracle's restatement of rms_norm.bm:62-94 (including scales that clamp to
0x7F / 0xFF and values that flush to 0x00), and gemm_fp8 within bf16 rounding
plus f32 accumulation error of the oracle's fp64 gemm_fp8.bm:31-107 (every
one of the 256 codes in the inputs, including 0x7F = 480, 0x80 = -2^-7 and the
zero-exponent codes the reference decodes as (1 + m/8) 2^-7; ragged M, N, K)."""
import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("rows,hidden,scale", [(1, 64, 1.0), (37, 3584, 40.0), (8, 4096, 600.0),
                                               (5, 100, 0.001)])
def test_rms_norm_fp8_codes_are_bit_exact(dev, rows, hidden, scale):
    from voidweb_b200.kv import rms_norm_fp8_out
    rng = np.random.default_rng(rows + hidden)
    x = oracle.f32_to_io_bits((rng.standard_normal((rows, hidden)) * 2).astype(np.float32), oracle.F16)
    w = oracle.f32_to_io_bits((rng.random(hidden) * 2).astype(np.float32), oracle.F16)
    want = oracle.rms_norm_fp8_out(x, w, scale, 1e-5)
    out = torch.zeros((rows, hidden), dtype=torch.uint8, device=dev)
    rms_norm_fp8_out(torch.from_numpy(x.view(np.int16)).to(dev), torch.from_numpy(w.view(np.int16)).to(dev),
                     out, scale, 1e-5)
    got = out.cpu().numpy()
    assert np.array_equal(got, want), f"{(got != want).sum()} codes differ"
    if scale >= 600:
        assert (got == 0x7F).any() or (got == 0xFF).any()      # clamped values exercised


@pytest.mark.parametrize("M,N,K,with_bias", [(1, 16, 16, False), (37, 48, 80, True),
                                              (128, 128, 128, True), (200, 304, 1024, True),
                                              (512, 1024, 512, False)])
def test_gemm_fp8_matches_the_oracle(dev, M, N, K, with_bias):
    from voidweb_b200.kv import fp8_weight_check, gemm_fp8
    rng = np.random.default_rng(M * 7 + N + K)
    a = rng.integers(0, 256, (M, K), dtype=np.uint8)
    b = rng.integers(0, 256, (K, N), dtype=np.uint8)
    a.flat[:256 if a.size >= 256 else a.size] = np.arange(256, dtype=np.uint8)[:min(256, a.size)]
    bias = oracle.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32)) if with_bias else None
    a_scale, b_scale = 0.01, 0.02
    ref = oracle.gemm_fp8_f64(a, b, bias, a_scale, b_scale)
    out = torch.zeros((M, N), dtype=torch.int16, device=dev)
    gemm_fp8(torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), out,
             None if bias is None else torch.from_numpy(bias.view(np.int16)).to(dev), a_scale, b_scale)
    assert fp8_weight_check() == 0
    got = oracle.bf16_bits_to_f32(out.cpu().numpy().view(np.uint16)).astype(np.float64)
    dec = np.abs(oracle.fp8_decode(np.arange(256, dtype=np.uint8)).astype(np.float64))
    mag = (dec[a] @ dec[b]) * (np.float32(a_scale) * np.float32(b_scale))
    bound = 2.0 ** -8 * np.abs(ref) + 2.0 ** -20 * mag + 1e-30
    bad = np.abs(got - ref) > bound
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance"
