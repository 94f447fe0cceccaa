"""The oracle's FP8 weight path on the CPU: rms_norm_fp8_out
(rms_norm.bm:62-94) against a numpy restatement of the same operation order,
and gemm_fp8 (gemm_fp8.bm:31-107) in fp64 against numpy over the reference
decoder's table."""
import numpy as np

import oracle


def test_rms_norm_fp8_matches_a_numpy_restatement():
    rng = np.random.default_rng(0)
    x = oracle.f32_to_io_bits((rng.standard_normal((5, 96)) * 3).astype(np.float32), oracle.F16)
    w = oracle.f32_to_io_bits((rng.random(96) + 0.5).astype(np.float32), oracle.F16)
    got = oracle.rms_norm_fp8_out(x, w, 40.0, 1e-5)
    xf = oracle.io_bits_to_f32(x, oracle.F16).astype(np.float32)
    wf = oracle.io_bits_to_f32(w, oracle.F16).astype(np.float32)
    for r in range(5):
        part = np.array([np.float32(0)] * 32, dtype=np.float32)
        for lane in range(32):
            acc = np.float32(0)
            for d in range(lane, 96, 32):
                acc = np.float32(acc + np.float32(xf[r, d] * xf[r, d]))
            part[lane] = acc
        for off in (16, 8, 4, 2, 1):
            part = np.array([np.float32(part[l] + part[l ^ off]) for l in range(32)], dtype=np.float32)
        inv = np.float32(1.0) / np.sqrt(np.float32(part[0] / np.float32(96) + np.float32(1e-5)))
        normed = ((xf[r] * inv) * wf) * np.float32(40.0)
        assert np.array_equal(got[r], oracle.fp8_encode(normed.astype(np.float32)))


def test_gemm_fp8_oracle_matches_numpy():
    rng = np.random.default_rng(1)
    a = rng.integers(0, 256, (7, 48), dtype=np.uint8)
    b = rng.integers(0, 256, (48, 32), dtype=np.uint8)
    bias = oracle.f32_to_bf16_bits(rng.standard_normal(32).astype(np.float32))
    got = oracle.gemm_fp8_f64(a, b, bias, 0.5, 0.125)
    dec = np.array([oracle.fp8_decode(np.array([c], np.uint8))[0] for c in range(256)], np.float64)
    want = (dec[a] @ dec[b]) * np.float64(np.float32(0.5) * np.float32(0.125)) + \
        oracle.bf16_bits_to_f32(bias).astype(np.float64)
    assert np.allclose(got, want, rtol=1e-12, atol=1e-9)
