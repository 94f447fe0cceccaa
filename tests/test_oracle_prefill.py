"""The oracle's prefill attention (flash_attention.bm:31-106 over the pool)
checked on the CPU: the f32 restatement against the fp64 two-pass reference,
the fp64 reference against a direct numpy computation over the gathered K/V,
and the causal prefill of a chunk's last token against the decode oracle,
which computes the same function by another route."""
import numpy as np

import oracle
from tests import kvgen
from tests.kvgen import BF16, F16


def chunked(seed, io, D, Hq, Hkv, chunks):
    """A pool whose sequences hold ctx_start + n tokens; chunks: [(ctx_start, n)]."""
    ctx = [cs + n for cs, n in chunks]
    c = kvgen.make_case(seed, 1, Hkv, D, Hq, len(chunks), 1, 1, BF16 if io == BF16 else F16, io,
                        ctx=ctx)
    rng = np.random.Generator(np.random.PCG64(seed + 99))
    cu = np.zeros(len(chunks) + 1, dtype=np.int32)
    cu[1:] = np.cumsum([n for _, n in chunks])
    cs = np.array([s for s, _ in chunks], dtype=np.int32)
    q = kvgen.io_bits(rng, (int(cu[-1]), Hq, D), io)
    return c, q, cu, cs


def numpy_prefill(c, q, cu, cs, causal, scale):
    G = c.Hq // c.Hkv
    out = np.zeros(q.shape, dtype=np.float64)
    for b in range(cu.size - 1):
        n = int(cu[b + 1] - cu[b])
        total = int(cs[b]) + n
        ok, ov, _, _ = oracle.kv_gather(c.geom, c.data, c.scales, 0, c.block_tables[b], total)
        K = oracle.io_bits_to_f32(ok, c.io).astype(np.float64)
        V = oracle.io_bits_to_f32(ov, c.io).astype(np.float64)
        for i in range(n):
            p = int(cs[b]) + i
            kend = p + 1 if causal else total
            for hq in range(c.Hq):
                h = hq // G
                qv = oracle.io_bits_to_f32(q[cu[b] + i, hq], c.io).astype(np.float64)
                s = K[h, :kend] @ qv * scale
                w = np.exp(s - s.max())
                out[cu[b] + i, hq] = (w @ V[h, :kend]) / w.sum()
    return out


def test_prefill_oracle_f32_f64_numpy_agree():
    c, q, cu, cs = chunked(5, BF16, 64, 8, 2, [(0, 5), (20, 17), (63, 2), (0, 1)])
    scale = 1.0 / np.sqrt(c.D)
    for causal in (True, False):
        ref = oracle.paged_prefill_f64(c.geom, c.data, c.scales, 0, q, c.Hq, c.block_tables, cu, cs,
                                       causal, scale)
        direct = numpy_prefill(c, q, cu, cs, causal, scale)
        assert np.allclose(ref, direct, rtol=1e-12, atol=1e-12)
        f32 = oracle.paged_prefill_f32(c.geom, c.data, c.scales, 0, q, c.Hq, c.block_tables, cu, cs,
                                       causal, scale)
        got = oracle.io_bits_to_f32(f32, c.io).astype(np.float64)
        assert (np.abs(got - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all()


def test_causal_prefill_last_token_is_the_decode():
    # the chunk's last token at position ctx_start + n - 1 sees exactly the
    # decode's seq_len = ctx_start + n keys, causal or not
    c, q, cu, cs = chunked(6, F16, 128, 8, 4, [(30, 3), (100, 1), (0, 40)])
    scale = 1.0 / np.sqrt(c.D)
    last = cu[1:] - 1
    dec = oracle.paged_decode_f64(c.geom, c.data, c.scales, 0, q[last], c.Hq, c.block_tables,
                                  (cs + np.diff(cu)).astype(np.uint32), scale)
    for causal in (True, False):
        ref = oracle.paged_prefill_f64(c.geom, c.data, c.scales, 0, q, c.Hq, c.block_tables, cu, cs,
                                       causal, scale)
        assert np.allclose(ref[last], dec, rtol=1e-12, atol=1e-12)


def test_prefill_slots_follow_the_paging_rule():
    bt = np.array([[7, 3, 9], [1, 2, 0]], dtype=np.uint32)
    slots = oracle.prefill_slots(bt, [0, 3, 5], [14, 31])
    # seq 0: positions 14, 15, 16; seq 1: positions 31, 32
    assert slots.tolist() == [7 * 16 + 14, 7 * 16 + 15, 3 * 16 + 0, 2 * 16 + 15, 0 * 16 + 0]
