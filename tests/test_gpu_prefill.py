"""GPU parity of the chunked prefill (vw_paged_prefill): the chunk append is
bit-exact against the oracle's append at the paging rule's slots, and the
attention is within |gpu - ref| <= 2e-3 + 1e-2 * |ref| of the oracle's fp64
restatement of flash_attention.bm:31-106 over the pool, causal and not.
Cases: ragged chunks (1, 16, 63, 64, 65, 129, 300 tokens), cached prefixes
(ctx_start 0 to 30,000), an empty chunk, the largest batch (1024 sequences),
GQA groups 1 to 7, head_dim 64 and 128,
f16 and bf16 pages, FP8 E4M3 pages with per-token-per-head scales (codes and
scales of the append bit-exact, the attention against the fp64 oracle over the
same dequantised codes), NaN garbage past every sequence's end, RoPE, the error
paths, and prefill descriptors through voidweb_forward_pass."""
import numpy as np
import pytest

import oracle
from tests import kvgen
from tests.kvgen import BF16, F16, FP8
from tests.test_gpu_kv import check_close, download_pool, make_pool, t16, tu32, upload_pool

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def chunk_case(seed, io, D, Hq, Hkv, chunks, L=2, kv=None):
    """Sequences that hold ctx_start + n tokens once their chunk [(ctx_start, n)]
    is appended; q, k_new, v_new rows of the chunks, packed."""
    ctx = [cs + n for cs, n in chunks]
    c = kvgen.make_case(seed, L, Hkv, D, Hq, len(chunks), 1, 1, io if kv is None else kv, io, ctx=ctx)
    rng = np.random.Generator(np.random.PCG64(seed + 7))
    cu = np.zeros(len(chunks) + 1, dtype=np.int32)
    cu[1:] = np.cumsum([n for _, n in chunks])
    cs = np.array([s for s, _ in chunks], dtype=np.int32)
    T = int(cu[-1])
    q = kvgen.io_bits(rng, (T, Hq, D), io)
    k = kvgen.io_bits(rng, (T, Hkv, D), io)
    v = kvgen.io_bits(rng, (T, Hkv, D), io)
    return c, q, k, v, cu, cs


def run_prefill(pool, c, layer, q, k, v, cu, cs, dev, causal=True, rope_theta=0.0):
    qt = t16(q, dev)
    out = torch.zeros_like(qt)
    pool.paged_prefill(layer, qt, tu32(cu, dev), tu32(cs, dev), tu32(c.block_tables, dev), out,
                       k_new=None if k is None else t16(k, dev),
                       v_new=None if v is None else t16(v, dev), causal=causal,
                       rope_theta=rope_theta)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)


CASES = [
    # (kv, io, head_dim, Hq, Hkv, chunks)
    (BF16, BF16, 128, 28, 4, [(0, 64), (37, 100), (500, 7), (0, 1), (1000, 300)]),
    (F16, F16, 64, 14, 2, [(0, 1), (16, 16), (5, 200), (0, 129)]),
    (BF16, BF16, 128, 8, 8, [(123, 65), (0, 63)]),
    (F16, F16, 128, 32, 8, [(0, 200), (300, 0), (7, 63)]),
    (FP8, BF16, 128, 28, 4, [(0, 64), (37, 100), (500, 7), (0, 1), (1000, 300)]),
    (FP8, F16, 128, 32, 8, [(0, 200), (300, 0), (7, 63), (16, 16)]),
    (FP8, BF16, 128, 8, 1, [(123, 65), (0, 129)]),
]


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("kv,io,D,Hq,Hkv,chunks", CASES)
def test_prefill_append_and_attention(dev, kv, io, D, Hq, Hkv, chunks, causal):
    c, q, k, v, cu, cs = chunk_case(40 + len(chunks) + D, io, D, Hq, Hkv, chunks, kv=kv)
    pool = make_pool(c, dev)
    layer = 1
    got = run_prefill(pool, c, layer, q, k, v, cu, cs, dev, causal=causal)
    assert pool.check() == 0
    # the append, bit for bit, at block_tables[b][p/16]*16 + p%16 (FP8: the
    # codes and the scales)
    slots = oracle.prefill_slots(c.block_tables, cu, cs)
    oracle.kv_append(c.geom, c.data, c.scales, layer, k, v, slots)
    gdata, gscales = download_pool(pool, c)
    assert np.array_equal(gdata, c.data)
    if kv == FP8:
        assert np.array_equal(gscales, c.scales, equal_nan=True)
    ref = oracle.paged_prefill_f64(c.geom, c.data, c.scales, layer, q, Hq, c.block_tables, cu, cs,
                                   causal, 1.0 / np.sqrt(D))
    check_close(got, ref, io, f"prefill causal={causal}")
    pool.close()


@pytest.mark.parametrize("kv", [BF16, FP8])
def test_prefill_long_context(dev, kv):
    # chunks after 30,000 and 12,345 cached tokens: hundreds of rounds through
    # the K and V rings and dozens of block-id windows per query tile
    c, q, k, v, cu, cs = chunk_case(23 + kv, BF16, 128, 8, 2, [(30000, 64), (12345, 130)], L=1, kv=kv)
    pool = make_pool(c, dev)
    got = run_prefill(pool, c, 0, q, k, v, cu, cs, dev)
    assert pool.check() == 0
    oracle.kv_append(c.geom, c.data, c.scales, 0, k, v, oracle.prefill_slots(c.block_tables, cu, cs))
    ref = oracle.paged_prefill_f64(c.geom, c.data, c.scales, 0, q, c.Hq, c.block_tables, cu, cs, True,
                                   1.0 / np.sqrt(128))
    check_close(got, ref, BF16, f"long-context prefill kv={kv}")
    pool.close()


@pytest.mark.parametrize("kv", [BF16, FP8])
def test_prefill_max_batch(dev, kv):
    # 1024 sequences (the most one launch takes), each a chunk of 0 to 3 tokens
    # after 0 to 40 cached tokens: the per-sequence query-tile prefix the kernel
    # builds in shared memory at its full size
    rng = np.random.default_rng(17 + kv)
    chunks = [(int(rng.integers(0, 41)), int(rng.integers(0, 4))) for _ in range(1024)]
    chunks[0] = (0, 1)
    c, q, k, v, cu, cs = chunk_case(19 + kv, BF16, 128, 8, 2, chunks, L=1, kv=kv)
    pool = make_pool(c, dev)
    got = run_prefill(pool, c, 0, q, k, v, cu, cs, dev)
    assert pool.check() == 0
    oracle.kv_append(c.geom, c.data, c.scales, 0, k, v, oracle.prefill_slots(c.block_tables, cu, cs))
    gdata, _ = download_pool(pool, c)
    assert np.array_equal(gdata, c.data)
    ref = oracle.paged_prefill_f64(c.geom, c.data, c.scales, 0, q, c.Hq, c.block_tables, cu, cs, True,
                                   1.0 / np.sqrt(128))
    check_close(got, ref, BF16, f"max batch prefill kv={kv}")
    pool.close()


def test_prefill_over_cached_pages_without_append(dev):
    # k_new = None: the pages already hold the chunk's rows (e.g. a re-run)
    c, q, _, _, cu, cs = chunk_case(77, BF16, 128, 16, 4, [(50, 80), (0, 3)])
    pool = make_pool(c, dev)
    got = run_prefill(pool, c, 0, q, None, None, cu, cs, dev)
    assert pool.check() == 0
    ref = oracle.paged_prefill_f64(c.geom, c.data, c.scales, 0, q, c.Hq, c.block_tables, cu, cs,
                                   True, 1.0 / np.sqrt(c.D))
    check_close(got, ref, BF16, "prefill over cached pages")
    gdata, _ = download_pool(pool, c)
    assert np.array_equal(gdata, c.data)      # nothing written
    pool.close()


@pytest.mark.parametrize("kv,io,D", [(BF16, BF16, 128), (F16, F16, 64), (FP8, BF16, 128)])
def test_prefill_rope(dev, kv, io, D):
    # q and the appended K rows are rotated at their positions (RoPE,
    # kernels/rope/rope.bm:22-52) as separate passes would leave them; the
    # device's sin/cos may round an angle differently from the oracle's, so the
    # rotated K rows are checked to a few units of the io type (most bit-exact;
    # FP8: most K codes equal, V codes and scales exact)
    theta = 10000.0
    c, q, k, v, cu, cs = chunk_case(91, io, D, 8, 2, [(40, 50), (0, 33), (700, 5)], kv=kv)
    pool = make_pool(c, dev)
    got = run_prefill(pool, c, 0, q, k, v, cu, cs, dev, rope_theta=theta)
    assert pool.check() == 0
    pos = np.concatenate([cs[b] + np.arange(cu[b + 1] - cu[b]) for b in range(cs.size)])
    k_rot = oracle.rope_apply(k, pos, theta, io)
    q_rot = oracle.rope_apply(q, pos, theta, io)
    slots = oracle.prefill_slots(c.block_tables, cu, cs)
    gdata, gscales = download_pool(pool, c)
    blk, t = slots // 16, slots % 16
    if kv == FP8:
        want, wsc = c.data.copy(), c.scales.copy()
        oracle.kv_append(c.geom, want, wsc, 0, k_rot, v, slots)
        assert np.array_equal(gdata[0, blk, :, 1, t], want[0, blk, :, 1, t]), "V codes"
        assert np.array_equal(gscales[0, blk, :, 1, t], wsc[0, blk, :, 1, t]), "V scales"
        assert np.mean(gdata[0, blk, :, 0, t] == want[0, blk, :, 0, t]) >= 0.9, "K codes"
        ref = oracle.paged_prefill_f64(c.geom, gdata, gscales, 0, q_rot, c.Hq, c.block_tables, cu, cs,
                                       True, 1.0 / np.sqrt(D))
        check_close(got, ref, io, "prefill rope fp8")
        pool.close()
        return
    want = c.data.copy()
    oracle.kv_append(c.geom, want, None, 0, k_rot, v, slots)
    g_k = oracle.io_bits_to_f32(gdata[0, blk, :, 0, t], io)
    w_k = oracle.io_bits_to_f32(want[0, blk, :, 0, t], io)
    rel = 2.0 ** -7 if io == BF16 else 2.0 ** -10
    assert (np.abs(g_k - w_k) <= 8e-3 + rel * np.abs(w_k)).all(), "rotated K rows"
    assert np.mean(gdata[0, blk, :, 0, t] == want[0, blk, :, 0, t]) >= 0.9
    assert np.array_equal(gdata[0, blk, :, 1, t], want[0, blk, :, 1, t]), "V rows"
    # attention against the pool as the device wrote it, with the oracle's q rotation
    ref = oracle.paged_prefill_f64(c.geom, gdata, None, 0, q_rot, c.Hq, c.block_tables, cu, cs,
                                   True, 1.0 / np.sqrt(D))
    check_close(got, ref, io, "prefill rope")
    pool.close()


@pytest.mark.parametrize("kv", [BF16, FP8])
def test_prefill_scheduler_chunk(dev, kv):
    # one 2048-token chunk (scheduler/scheduler.bm:255, the largest it cuts)
    # after a 512-token cached prefix, Qwen2.5-7B heads
    c, q, k, v, cu, cs = chunk_case(5, BF16, 128, 28, 4, [(512, 2048)], L=1, kv=kv)
    pool = make_pool(c, dev)
    got = run_prefill(pool, c, 0, q, k, v, cu, cs, dev)
    assert pool.check() == 0
    oracle.kv_append(c.geom, c.data, c.scales, 0, k, v, oracle.prefill_slots(c.block_tables, cu, cs))
    # every 8th query token against the fp64 oracle (the full check is slow on
    # the CPU): token r of the chunk, causal, is a one-token chunk at 512 + r
    rows = np.arange(0, 2048, 8)
    ref = np.zeros((rows.size, c.Hq, c.D))
    one = np.array([0, 1], dtype=np.int32)
    for r_i, r in enumerate(rows):
        at = np.array([512 + r], dtype=np.int32)
        ref[r_i] = oracle.paged_prefill_f64(c.geom, c.data, c.scales, 0, q[r:r + 1], c.Hq,
                                            c.block_tables, one, at, True, 1.0 / np.sqrt(c.D))[0]
    check_close(got[rows], ref, BF16, "2048-token chunk")
    pool.close()


@pytest.mark.parametrize("kv", [BF16, FP8])
def test_prefill_errors(dev, kv):
    from voidweb_b200 import _lib as C
    c, q, k, v, cu, cs = chunk_case(3, BF16, 128, 8, 2, [(0, 20)], kv=kv)
    # a chunk past its block-table row: flagged on the device, nothing written
    pool = make_pool(c, dev)
    bad_cs = np.array([c.stride * 16], dtype=np.int32)
    run_prefill(pool, c, 0, q, k, v, cu, bad_cs, dev)
    assert pool.check() & C.VW_DEV_ERR_SEQ_LEN
    gdata, _ = download_pool(pool, c)
    assert np.array_equal(gdata, c.data)
    # a block id outside the pool: flagged, its rows zero-filled for the attention
    c.block_tables[0, 0] = c.NB + 5
    run_prefill(pool, c, 0, q, k, v, cu, cs, dev)
    assert pool.check() & C.VW_DEV_ERR_BLOCK_ID
    pool.close()


def test_forward_pass_with_prefill_and_decode_descriptors(dev):
    from voidweb_b200 import KernelLib
    from voidweb_b200 import _lib as C
    theta = 10000.0
    L, Hkv, D, Hq = 2, 2, 128, 8
    # sequence 2000: a 37-token chunk after 16 cached tokens; 2001: a decode at 100
    c = kvgen.make_case(8, L, Hkv, D, Hq, 2, 1, 1, BF16, BF16, ctx=[16 + 37, 101])
    rng = np.random.Generator(np.random.PCG64(8))
    T = 37 + 1
    q = kvgen.io_bits(rng, (L, T, Hq, D), BF16)
    k = kvgen.io_bits(rng, (L, T, Hkv, D), BF16)
    v = kvgen.io_bits(rng, (L, T, Hkv, D), BF16)
    pool = make_pool(c, dev)
    # the device path: per layer, prefill of the chunk, then the decode step
    want = np.zeros_like(q)
    bt_a = c.block_tables[0:1, :]
    bt_b = c.block_tables[1:2, :]
    for layer in range(L):
        qa = t16(q[layer, :37], dev)
        oa = torch.zeros_like(qa)
        pool.paged_prefill(layer, qa, tu32(np.array([0, 37]), dev), tu32(np.array([16]), dev),
                           tu32(bt_a, dev), oa, k_new=t16(k[layer, :37], dev),
                           v_new=t16(v[layer, :37], dev), rope_theta=theta)
        qb = t16(q[layer, 37:], dev)
        ob = torch.zeros_like(qb)
        pool.paged_decode(layer, qb, tu32(bt_b, dev), tu32(np.array([101]), dev), ob,
                          k_new=t16(k[layer, 37:], dev), v_new=t16(v[layer, 37:], dev),
                          rope_theta=theta)
        torch.cuda.synchronize()
        want[layer, :37] = oa.cpu().numpy().view(np.uint16)
        want[layer, 37:] = ob.cpu().numpy().view(np.uint16)
    assert pool.check() == 0
    after_device, _ = download_pool(pool, c)
    # the engine-facing symbol over the same inputs: prefill chunk first
    upload_pool(pool, c)
    got = np.zeros_like(q)
    lib = C.lib()
    lib.vw_forward_bind(pool.handle, q.ctypes.data, k.ctypes.data, v.ctypes.data, got.ctypes.data)
    lib.vw_forward_set_seq_len(2000, 16)
    lib.vw_forward_set_seq_len(2001, 100)
    kl = KernelLib.open(C.LIB_PATH)
    n_a = (16 + 37 + 15) // 16
    kl.forward_pass(dict(num_heads=Hq, num_kv_heads=Hkv, num_layers=L, head_dim=D, rope_theta=theta),
                    [(2001, 5, c.block_tables[1, :7])],
                    prefill_seqs=[(2000, np.arange(37), c.block_tables[0, :n_a])])
    assert np.array_equal(got, want)
    after_shim, _ = download_pool(pool, c)
    assert np.array_equal(after_shim, after_device)
    lib.vw_forward_release(2000)
    lib.vw_forward_release(2001)
    lib.vw_forward_bind(None, None, None, None, None)
    pool.close()
