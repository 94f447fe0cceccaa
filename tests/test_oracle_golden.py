"""The C++ oracle against the golden fixtures of the independent Python
transliteration (tests/golden/make_golden.py).  CPU only."""
import math
import struct

import numpy as np
import pytest

import oracle


def bits(f):
    return struct.unpack("<I", struct.pack("<f", f))[0]


def from_bits(u):
    return struct.unpack("<f", struct.pack("<I", u))[0]


def test_fp8_decode_all_256_codes(golden):
    L = oracle.lib()
    got = [bits(L.vwo_fp8_decode_ref(c)) for c in range(256)]
    assert got == golden["fp8_decode_all"]
    # spot values of the reference decoder (gemm_fp8.bm:110-116)
    assert L.vwo_fp8_decode_ref(0x7F) == 480.0
    assert L.vwo_fp8_decode_ref(0x80) == -(2.0 ** -7)
    assert L.vwo_fp8_decode_ref(0x38) == 1.0


def test_fp8_encode_probes(golden):
    L = oracle.lib()
    got = [L.vwo_fp8_encode_ref(from_bits(u)) for u in golden["fp8_encode_in"]]
    assert got == golden["fp8_encode_out"]
    # reference quirks (rms_norm.bm:98-113): 448 saturates to 0x7F, tiny -> +0
    assert L.vwo_fp8_encode_ref(448.0) == 0x7F
    assert L.vwo_fp8_encode_ref(-448.0) == 0xFF
    assert L.vwo_fp8_encode_ref(-(2.0 ** -8)) == 0x00
    assert L.vwo_fp8_encode_ref(1.1875) == 0x39       # truncation, not rounding


def test_fp8_encode_exhaustive_representables():
    """Every value the reference decoder produces for codes with exponent
    field 1..14 re-encodes to its own code (truncation is exact on grid)."""
    L = oracle.lib()
    for c in range(256):
        e = (c >> 3) & 0xF
        if 1 <= e <= 14:
            assert L.vwo_fp8_encode_ref(L.vwo_fp8_decode_ref(c)) == c


def test_fp8_ocp_mode_roundtrip():
    L = oracle.lib()
    for c in range(256):
        if c in (0x7F, 0xFF):
            continue
        v = L.vwo_fp8_decode_ocp(c)
        enc = L.vwo_fp8_encode_ocp(v)
        if c == 0x80:
            assert enc in (0x80, 0x00)
        else:
            assert enc == c, hex(c)
    assert L.vwo_fp8_encode_ocp(1000.0) == 0x7E
    assert L.vwo_fp8_encode_ocp(1.0625) == 0x38        # tie -> even mantissa (1.0)
    assert L.vwo_fp8_encode_ocp(1.1875) == 0x3A        # tie -> even (1.25)


def test_bf16_rne(golden):
    L = oracle.lib()
    got = [L.vwo_f32_to_bf16(from_bits(u)) for u in golden["bf16_in"]]
    assert got == golden["bf16_out"]
    np_got = oracle.f32_to_bf16_bits(
        np.array(golden["bf16_in"], dtype=np.uint32).view(np.float32))
    assert np_got.tolist() == golden["bf16_out"]


def test_f16_conversion_matches_numpy():
    L = oracle.lib()
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 500),
                           rng.normal(0, 3e4, 200), [65519.9, 65520.0, 6e-8, 3e-8]])
    vals = vals.astype(np.float32)
    got = np.array([L.vwo_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    assert (got == vals.astype(np.float16).view(np.uint16)).all()
    for h in range(0, 65536, 7):
        f = np.uint16(h).view(np.float16)
        if np.isnan(f):
            continue
        assert L.vwo_f16_to_f32(h) == np.float32(f)


def test_fp8_quant_rows(golden):
    for row in golden["fp8_quant_rows"]:
        x = np.array(row["x_bits"], dtype=np.uint32).view(np.float32)
        codes, scale = oracle.fp8_quant_row(x)
        assert codes.tolist() == row["codes"]
        assert bits(scale) == row["scale_bits"]


def test_rolling_hash(golden):
    for case in golden["rolling_hash"]:
        assert oracle.rolling_hash(int(case["prev"]), case["tokens"]) == int(case["hash"])


def test_small_decode_matches_transliteration(golden):
    c = golden["decode_small"]
    D, NB, seq_len = c["D"], c["NB"], c["seq_len"]
    g = oracle.geom(1, 1, D, NB, oracle.BF16, oracle.BF16)
    data = np.array(c["kv_bf16"], dtype=np.uint16).reshape(1, NB, 1, 2, 16, D)
    q = np.array(c["q_bf16"], dtype=np.uint16).reshape(1, 2, D)
    bt = np.array([c["table"] + [0]], dtype=np.uint32)
    sl = np.array([seq_len], dtype=np.uint32)
    scale = np.float32(1.0 / math.sqrt(D))
    out = oracle.paged_decode_f32(g, data, None, 0, q, 2, bt, sl, float(scale))
    ref = np.array(c["out_f32_bits"], dtype=np.uint32).view(np.float32)
    got = oracle.bf16_bits_to_f32(out[0])
    # transliteration rounds exp through Python's libm; outputs agree to bf16
    assert np.allclose(got, oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(ref)), atol=1e-2)
    out64 = oracle.paged_decode_f64(g, data, None, 0, q, 2, bt, sl, float(scale))
    assert np.allclose(out64[0], ref, atol=1e-5)


def test_block_manager_trace(golden):
    bm = oracle.BlockManager(16, 12)
    for step in golden["block_manager_trace"]:
        op, args = step["op"], step["args"]
        if op == "alloc_seq":
            try:
                r = bm.alloc_seq(*args)
            except MemoryError:
                r = "OOM"
        else:
            r = getattr(bm, op)(*args)
        assert r == step["ret"], step
        assert bm.free_list() == step["free"], step
        refs = {str(k): bm.ref_count(k) for k in range(12) if bm.ref_count(k) > 0}
        assert refs == step["refs"], step


def test_radix_trace(golden):
    rx = oracle.RadixCache(16, 20)
    for step in golden["radix_trace"]:
        op = step["op"]
        if op == "lookup":
            ml, blocks = rx.lookup(step["tokens"])
            assert [ml, blocks] == step["ret"], step
        elif op == "insert":
            assert rx.insert(step["tokens"], step["blocks"]) == step["ret"], step
            assert rx.total_blocks() == step["total"]
        elif op == "evict_lru":
            assert rx.evict_lru(step["target"]) == step["ret"], step
            assert rx.total_blocks() == step["total"]
        elif op == "lock":
            rx.lock(step["tokens"])
        elif op == "unlock":
            rx.unlock(step["tokens"])


def test_append_and_gather_roundtrip():
    rng = np.random.default_rng(5)
    L_, H, D, NB = 2, 2, 64, 8
    g = oracle.geom(L_, H, D, NB, oracle.F16, oracle.F16)
    data = np.zeros(oracle.pool_shape(g), dtype=np.uint16)
    n = 20
    k = rng.normal(0, 1, (n, H, D)).astype(np.float16).view(np.uint16)
    v = rng.normal(0, 1, (n, H, D)).astype(np.float16).view(np.uint16)
    table = np.array([5, 2], dtype=np.uint32)
    slots = np.array([table[p // 16] * 16 + p % 16 for p in range(n)], dtype=np.int64)
    oracle.kv_append(g, data, None, 1, k, v, slots)
    ok, ov, _, _ = oracle.kv_gather(g, data, None, 1, table, n)
    assert (ok.transpose(1, 0, 2) == k).all() and (ov.transpose(1, 0, 2) == v).all()
    assert (data[0] == 0).all()


def test_block_copy_snapshot_semantics():
    rng = np.random.default_rng(6)
    g = oracle.geom(2, 1, 64, 6, oracle.FP8, oracle.BF16)
    data = rng.integers(0, 255, oracle.pool_shape(g), dtype=np.uint8)
    scales = rng.random((2, 6, 1, 2, 16)).astype(np.float32)
    before, sbefore = data.copy(), scales.copy()
    oracle.block_copy(g, data, scales, np.array([[1, 2], [2, 4]]))   # 2 read before written
    assert (data[:, 2] == before[:, 1]).all() and (data[:, 4] == before[:, 2]).all()
    assert (scales[:, 4] == sbefore[:, 2]).all()
    assert (data[:, [0, 1, 3, 5]] == before[:, [0, 1, 3, 5]]).all()


@pytest.mark.parametrize("io", [oracle.BF16, oracle.F16])
def test_rope_matches_numpy_restatement(io):
    """kernels/rope/rope.bm:22-52 in the oracle against an independent numpy
    restatement with the same f32 steps (freq = 1 / theta^(2d/D), angle =
    freq * pos, rotate, round to the io type): the two sides use different pow
    / sin / cos implementations, so they may differ by two last places of the
    f32 angle (large at large positions) plus one rounding to the io type.
    Position 0 is exact."""
    rng = np.random.default_rng(11)
    n, H, D, theta = 37, 3, 128, 10000.0
    x = oracle.f32_to_io_bits(rng.standard_normal((n, H, D)).astype(np.float32), io)
    pos = rng.integers(0, 32768, n)
    pos[0] = 0
    got = oracle.rope_apply(x, pos, theta, io)
    f32 = np.float32
    xf = oracle.io_bits_to_f32(x, io)
    d = np.arange(D // 2, dtype=np.float32)
    freq = f32(1.0) / np.power(f32(theta), (f32(2.0) * d) / f32(D)).astype(np.float32)
    ang = (freq[None, :] * pos[:, None].astype(np.float32)).astype(np.float32)
    c = np.cos(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    s = np.sin(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    xr, xi = xf[..., : D // 2], xf[..., D // 2:]
    want = np.concatenate([xr * c - xi * s, xr * s + xi * c], axis=-1).astype(np.float32)
    want_bits = oracle.f32_to_io_bits(want, io)
    assert np.array_equal(got[0], x[0])
    g = oracle.io_bits_to_f32(got, io)
    rel = 2.0 ** -7 if io == oracle.BF16 else 2.0 ** -10
    # a last-place difference of freq plus one of the product: two ulps of the
    # angle, each moving the rotated pair by at most ulp * (|x_r| + |x_i|)
    amp = (np.abs(xr) + np.abs(xi)) * 2.0 * np.spacing(ang)[:, None, :]
    bound = np.concatenate([amp, amp], axis=-1) + rel * np.abs(want) + 1e-6
    assert (np.abs(g - want) <= bound).all()
    assert np.mean(got == want_bits) > 0.97


def test_benchmark_config_inputs_follow_their_definition():
    """The C1 and C2 configurations as tests/baseline_configs.py builds them:
    context ranges, pool sizes, distinct pages dealt from one permutation, and
    the oracle's reference-order f32 decode within the attention tolerance of
    its fp64 decode on them."""
    from tests import baseline_configs
    for name, (lo, hi) in (("C1", (1, 512)), ("C2", (512, 4096))):
        c = baseline_configs.build(name)
        assert c.ctx.min() >= lo and c.ctx.max() <= hi
        if name == "C1":
            assert c.NB == 512
        pages = (c.seq_lens.astype(np.int64) + 15) // 16
        dealt = np.concatenate([c.block_tables[b, :pages[b]] for b in range(c.B)])
        assert len(set(dealt.tolist())) == dealt.size and dealt.max() < c.NB
        again = baseline_configs.build(name)
        assert np.array_equal(again.q, c.q) and np.array_equal(again.block_tables, c.block_tables)
        sub = slice(0, 4) if name == "C2" else slice(None)
        f64 = oracle.paged_decode_f64(c.geom, c.data, None, 0, c.q[0][sub], c.Hq,
                                      c.block_tables[sub], c.seq_lens[sub], 1.0 / np.sqrt(c.D))
        f32 = oracle.paged_decode_f32(c.geom, c.data, None, 0, c.q[0][sub], c.Hq,
                                      c.block_tables[sub], c.seq_lens[sub],
                                      float(np.float32(1.0) / np.sqrt(np.float32(c.D))))
        got = oracle.io_bits_to_f32(f32, c.io).astype(np.float64)
        assert (np.abs(got - f64) <= 2e-3 + 1e-2 * np.abs(f64)).all()
