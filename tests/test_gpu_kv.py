"""GPU parity tests: every CUDA path of libvoidweb_kv.so against the oracle.

Bars: bit-exact for append, gather, block copy and FP8 codes/scales;
attention outputs within |gpu - ref| <= 2e-3 + 1e-2 * |ref| of the fp64
oracle (the fp32-reference tolerance of bf16 attention, applied to f16 and to
FP8 pages too, where ref is computed from the same dequantised codes).
"""
import zlib

import numpy as np
import pytest

import oracle
from tests import kvgen
from tests.kvgen import BF16, F16, FP8

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def make_pool(c, dev):
    from voidweb_b200.kv import KvPool, PoolSpec
    pool = KvPool(PoolSpec(**kvgen.pool_spec_kwargs(c)), device=dev.index or 0)
    upload_pool(pool, c)
    return pool


def upload_pool(pool, c):
    pool.pages_u8().copy_(torch.from_numpy(np.ascontiguousarray(c.data).view(np.uint8).ravel()))
    if c.kv == FP8:
        pool.scales_f32().copy_(torch.from_numpy(c.scales.ravel()))
    torch.cuda.synchronize()


def download_pool(pool, c):
    raw = pool.pages_u8().cpu().numpy()
    data = raw.view(np.uint8 if c.kv == FP8 else np.uint16).reshape(oracle.pool_shape(c.geom))
    scales = pool.scales_f32().cpu().numpy().reshape(oracle.pool_shape(c.geom)[:-1]) \
        if c.kv == FP8 else None
    return data, scales


def t16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)


def tu32(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).astype(np.int32)).to(dev)


def check_close(got_bits, ref64, io, what=""):
    got = oracle.io_bits_to_f32(got_bits, io).astype(np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref64)
    bound = ATOL + RTOL * np.abs(ref64)
    bad = err > bound
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance, "
                           f"max err {err.max():.3g} (worst ratio {(err / bound).max():.3g})")


def run_decode(pool, c, layer, dev, fused=False, rope_theta=0.0):
    q = t16(c.q[layer], dev)
    out = torch.zeros_like(q)
    bt, sl = tu32(c.block_tables, dev), tu32(c.seq_lens, dev)
    kn = t16(c.k_new[layer], dev) if fused else None
    vn = t16(c.v_new[layer], dev) if fused else None
    pool.paged_decode(layer, q, bt, sl, out, k_new=kn, v_new=vn, rope_theta=rope_theta)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)


DECODE_CASES = [
    # (name, L, Hkv, D, Hq, B, ctx_lo, ctx_hi, kv, io)
    ("plumbing_f16_d64_g7", 1, 2, 64, 14, 8, 1, 512, F16, F16),
    ("qwen_bf16_d128_g7", 1, 4, 128, 28, 6, 300, 1500, BF16, BF16),
    ("llama70b_bf16_g8", 1, 2, 128, 16, 5, 100, 900, BF16, BF16),
    ("g16_two_ntiles", 1, 1, 128, 16, 4, 20, 700, BF16, BF16),
    # two query-head tiles, the second one partly padded (group 12), and the
    # two-tile variants of the other page types
    ("g12_bf16_padded_tile", 1, 2, 128, 24, 5, 1, 900, BF16, BF16),
    ("g16_f16", 1, 2, 128, 32, 4, 20, 700, F16, F16),
    ("g16_fp8", 1, 1, 128, 16, 4, 20, 900, FP8, BF16),
    ("g12_fp8_f16io", 1, 2, 128, 24, 3, 1, 600, FP8, F16),
    ("bf16_d64", 1, 3, 64, 12, 7, 1, 300, BF16, BF16),
    ("f16_d128_g4", 1, 2, 128, 8, 6, 1, 800, F16, F16),
    ("fp8_llama8b_g4", 1, 2, 128, 8, 5, 50, 900, FP8, BF16),
    ("fp8_f16io_g8", 1, 1, 128, 8, 4, 1, 400, FP8, F16),
    # long contexts (the Llama-3-8B FP8 configuration reaches 32K tokens)
    ("long_bf16_32k", 1, 2, 128, 8, 3, 16000, 32768, BF16, BF16),
    ("long_fp8_32k", 1, 2, 128, 8, 3, 16000, 32768, FP8, BF16),
]


@pytest.mark.parametrize("case", DECODE_CASES, ids=[c[0] for c in DECODE_CASES])
def test_decode_matches_fp64(dev, case):
    name, L, Hkv, D, Hq, B, lo, hi, kv, io = case
    c = kvgen.make_case(zlib.crc32(name.encode()) % 1000, L, Hkv, D, Hq, B, lo, hi, kv, io)
    pool = make_pool(c, dev)
    got = run_decode(pool, c, 0, dev)
    assert pool.check() == 0
    ref = oracle.paged_decode_f64(c.geom, c.data, c.scales, 0, c.q[0], Hq, c.block_tables,
                                  c.seq_lens, 1.0 / np.sqrt(D))
    check_close(got, ref, io, name)
    # the reference's own f32 order agrees with the fp64 reference too
    f32 = oracle.paged_decode_f32(c.geom, c.data, c.scales, 0, c.q[0], Hq, c.block_tables,
                                  c.seq_lens, float(np.float32(1.0) / np.sqrt(np.float32(D))))
    check_close(f32, ref, io, name + " (oracle f32 order)")
    pool.close()


@pytest.mark.parametrize("kv,io,mode", [(F16, F16, 0), (BF16, BF16, 0), (FP8, BF16, 0),
                                        (FP8, BF16, 1), (FP8, F16, 0)])
def test_fused_append_decode(dev, kv, io, mode):
    D = 128 if kv != F16 else 64
    c = kvgen.make_case(7 + kv * 3 + mode, 2, 2, D, 8, 6, 1, 600, kv, io, fp8_mode=mode)
    pool = make_pool(c, dev)
    got = [run_decode(pool, c, layer, dev, fused=True) for layer in range(c.L)]
    assert pool.check() == 0
    data, scales = c.data.copy(), None if c.scales is None else c.scales.copy()
    slots = kvgen.new_token_slots(c)
    for layer in range(c.L):
        oracle.kv_append(c.geom, data, scales, layer, c.k_new[layer], c.v_new[layer], slots)
    gdata, gscales = download_pool(pool, c)
    assert np.array_equal(gdata, data), "pages after fused append differ from the oracle"
    if kv == FP8:
        assert np.array_equal(gscales.view(np.uint32), scales.view(np.uint32))
    for layer in range(c.L):
        ref = oracle.paged_decode_f64(c.geom, data, scales, layer, c.q[layer], c.Hq,
                                      c.block_tables, c.seq_lens, 1.0 / np.sqrt(D))
        check_close(got[layer], ref, io, f"layer {layer}")
    pool.close()


@pytest.mark.parametrize("kv,io,D", [(BF16, BF16, 128), (FP8, BF16, 128), (F16, F16, 64)])
def test_max_batch_fused_append_decode(dev, kv, io, D):
    # the largest batch one launch takes (1024 sequences: the prefix tables the
    # decode keeps in shared memory at their full size), short ragged contexts
    c = kvgen.make_case(31 + kv, 1, 2, D, 8, 1024, 1, 40, kv, io)
    pool = make_pool(c, dev)
    got = run_decode(pool, c, 0, dev, fused=True)
    assert pool.check() == 0
    data, scales = c.data.copy(), None if c.scales is None else c.scales.copy()
    oracle.kv_append(c.geom, data, scales, 0, c.k_new[0], c.v_new[0], kvgen.new_token_slots(c))
    gdata, _ = download_pool(pool, c)
    assert np.array_equal(gdata, data), "pages after the fused append differ from the oracle"
    ref = oracle.paged_decode_f64(c.geom, data, scales, 0, c.q[0], c.Hq, c.block_tables, c.seq_lens,
                                  1.0 / np.sqrt(D))
    check_close(got, ref, io, f"max batch kv={kv}")
    pool.close()


@pytest.mark.parametrize("kv,io,mode", [(F16, F16, 0), (BF16, BF16, 0), (FP8, BF16, 0),
                                        (FP8, BF16, 1), (FP8, F16, 1)])
def test_append_bit_exact(dev, kv, io, mode):
    D = 128
    c = kvgen.make_case(21 + kv + mode, 3, 2, D, 4, 5, 10, 200, kv, io, fp8_mode=mode)
    pool = make_pool(c, dev)
    rng = np.random.default_rng(5)
    n = 70
    slots = rng.choice(c.NB * 16, n, replace=False).astype(np.int64)
    slots[[3, 17, 40]] = -1                               # padding tokens are skipped
    k = kvgen.io_bits(rng, (n, c.Hkv, D), io, 3.0, True)
    v = kvgen.io_bits(rng, (n, c.Hkv, D), io, 3.0, True)
    k[0, 0, :] = 0                                        # amax == 0 -> scale 1
    pool.append(1, t16(k, dev), t16(v, dev), torch.from_numpy(slots).to(dev))
    assert pool.check() == 0
    data, scales = c.data.copy(), None if c.scales is None else c.scales.copy()
    oracle.kv_append(c.geom, data, scales, 1, k, v, slots)
    gdata, gscales = download_pool(pool, c)
    assert np.array_equal(gdata, data)
    if kv == FP8:
        assert np.array_equal(gscales.view(np.uint32), scales.view(np.uint32))
    pool.close()


@pytest.mark.parametrize("kv", [BF16, FP8])
def test_gather_and_block_copy_bit_exact(dev, kv):
    io = BF16
    c = kvgen.make_case(33 + kv, 2, 2, 128, 4, 4, 17, 300, kv, io)
    pool = make_pool(c, dev)
    b = 2
    n = int(c.seq_lens[b])
    ok, ov, ks, vs = pool.gather(1, tu32(c.block_tables[b], dev), n)
    rk, rv, rks, rvs = oracle.kv_gather(c.geom, c.data, c.scales, 1, c.block_tables[b], n)
    dt = np.uint8 if kv == FP8 else np.uint16
    assert np.array_equal(ok.cpu().numpy().view(dt), rk)
    assert np.array_equal(ov.cpu().numpy().view(dt), rv)
    if kv == FP8:
        assert np.array_equal(ks.cpu().numpy(), rks) and np.array_equal(vs.cpu().numpy(), rvs)
    # copy-on-write / compaction copies (distinct destinations, not sources)
    used = set(c.block_tables[:, :].ravel().tolist())
    free = [i for i in range(c.NB) if i not in used] or [c.NB - 1]
    srcs = [int(c.block_tables[0, 0]), int(c.block_tables[1, 1])]
    dsts = free[:2] if len(free) >= 2 else [free[0], int(c.block_tables[3, 0])]
    pairs = np.array(list(zip(srcs, dsts)), dtype=np.uint32)
    pool.block_copy(torch.from_numpy(pairs.astype(np.int32)).to(dev))
    assert pool.check() == 0
    data, scales = c.data.copy(), None if c.scales is None else c.scales.copy()
    oracle.block_copy(c.geom, data, scales, pairs)
    gdata, gscales = download_pool(pool, c)
    assert np.array_equal(gdata, data)
    if kv == FP8:
        assert np.array_equal(gscales.view(np.uint32), scales.view(np.uint32))
    pool.close()


def test_split_k_extremes(dev):
    """Very long and very short sequences in one batch: segments cut across many
    CTAs and CTAs spanning many segments, merged by the combine grid; repeated
    launches alternate the two partial sets and must give identical results."""
    ctx = [1, 2, 15, 16, 17, 31, 32, 33, 9000, 3, 1, 4097, 64, 5, 12000]
    c = kvgen.make_case(99, 1, 2, 128, 14, len(ctx), 0, 0, BF16, BF16, ctx=ctx)
    pool = make_pool(c, dev)
    first = run_decode(pool, c, 0, dev)
    for _ in range(3):
        again = run_decode(pool, c, 0, dev)
        assert np.array_equal(first, again), "repeated launch changed the result"
    assert pool.check() == 0
    ref = oracle.paged_decode_f64(c.geom, c.data, None, 0, c.q[0], c.Hq, c.block_tables,
                                  c.seq_lens, 1.0 / np.sqrt(128), nthreads=0)
    check_close(first, ref, BF16, "split-K extremes")
    pool.close()


def test_single_sequence_ctx1(dev):
    c = kvgen.make_case(5, 1, 1, 128, 1, 1, 1, 1, BF16, BF16)
    pool = make_pool(c, dev)
    got = run_decode(pool, c, 0, dev)
    # one token: softmax weight 1, output is exactly V row 0
    blk = int(c.block_tables[0, 0])
    assert np.array_equal(got[0, 0], c.data[0, blk, 0, 1, 0])
    pool.close()


def test_bad_block_id_and_seq_len_are_flagged(dev):
    from voidweb_b200 import _lib as C
    c = kvgen.make_case(8, 1, 2, 128, 4, 3, 20, 60, BF16, BF16)
    pool = make_pool(c, dev)
    bt = c.block_tables.copy()
    bt[1, 0] = c.NB + 7                        # outside the pool
    q = t16(c.q[0], dev)
    out = torch.zeros_like(q)
    pool.paged_decode(0, q, tu32(bt, dev), tu32(c.seq_lens, dev), out,
                      k_new=t16(c.k_new[0], dev), v_new=t16(c.v_new[0], dev))
    err = pool.check()
    assert err & C.DEV_ERR_BLOCK_ID
    assert not (err & C.DEV_ERR_TIMEOUT)
    sl = c.seq_lens.copy()
    sl[2] = 0
    pool.paged_decode(0, q, tu32(c.block_tables, dev), tu32(sl, dev), out)
    assert pool.check() & C.DEV_ERR_SEQ_LEN
    # untouched data outside the pool: the bad id was skipped, not written
    pool.close()


def test_seq_len_beyond_table_appends_nothing(dev):
    """A seq_len longer than its block-table row is flagged; the kernel reads
    the row's pages as full and must not append into a neighbouring row."""
    from voidweb_b200 import _lib as C
    c = kvgen.make_case(12, 1, 2, 128, 4, 3, 20, 60, BF16, BF16)
    pool = make_pool(c, dev)
    sl = c.seq_lens.copy()
    sl[0] = c.block_tables.shape[1] * 16 + 5
    q = t16(c.q[0], dev)
    out = torch.zeros_like(q)
    pool.paged_decode(0, q, tu32(c.block_tables, dev), tu32(sl, dev), out,
                      k_new=t16(c.k_new[0], dev), v_new=t16(c.v_new[0], dev))
    assert pool.check() & C.DEV_ERR_SEQ_LEN
    data = c.data.copy()
    slots = kvgen.new_token_slots(c)
    slots[0] = -1                              # nothing written for sequence 0
    oracle.kv_append(c.geom, data, None, 0, c.k_new[0], c.v_new[0], slots)
    gdata, _ = download_pool(pool, c)
    assert np.array_equal(gdata, data)
    pool.close()


def test_host_step_and_forward_pass_match_device_path(dev):
    from voidweb_b200 import KernelLib
    from voidweb_b200 import _lib as C
    c = kvgen.make_case(12, 3, 2, 128, 8, 4, 5, 200, BF16, BF16)
    pool = make_pool(c, dev)
    # the engine passes its model's rope_theta (ForwardArgs); the shim applies it
    theta = 10000.0
    dev_out = [run_decode(pool, c, layer, dev, fused=True, rope_theta=theta)
               for layer in range(c.L)]
    upload_pool(pool, c)
    out = np.zeros_like(c.q)
    pool.decode_step_host(torch.from_numpy(c.q.view(np.int16)),
                          torch.from_numpy(c.k_new.view(np.int16)),
                          torch.from_numpy(c.v_new.view(np.int16)),
                          torch.from_numpy(c.block_tables.astype(np.int32)),
                          torch.from_numpy(c.seq_lens.astype(np.int32)),
                          torch.from_numpy(out.view(np.int16)), rope_theta=theta)
    for layer in range(c.L):
        assert np.array_equal(out[layer], dev_out[layer])
    # repeated calls: pinned buffers are recorded as a CUDA graph on the second
    # call with the same arguments and replayed on the third; pageable buffers
    # stay on the direct path.  Every call gives the device path's outputs.
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    pinned = (pin(c.q.view(np.int16)), pin(c.k_new.view(np.int16)), pin(c.v_new.view(np.int16)),
              pin(c.block_tables.astype(np.int32)), pin(c.seq_lens.astype(np.int32)),
              torch.zeros(c.q.shape, dtype=torch.int16).pin_memory())
    pageable = (torch.from_numpy(c.q.view(np.int16)), torch.from_numpy(c.k_new.view(np.int16)),
                torch.from_numpy(c.v_new.view(np.int16)), torch.from_numpy(c.block_tables.astype(np.int32)),
                torch.from_numpy(c.seq_lens.astype(np.int32)), torch.from_numpy(out.view(np.int16)))
    for name, bufs in (("pinned", pinned), ("pageable", pageable), ("pinned", pinned)):
        for call in range(3):
            upload_pool(pool, c)
            bufs[5].zero_()
            pool.decode_step_host(*bufs, rope_theta=theta)
            got = bufs[5].numpy().view(np.uint16)
            for layer in range(c.L):
                assert np.array_equal(got[layer], dev_out[layer]), f"{name} call {call} layer {layer}"
    assert pool.check() == 0
    # the engine-facing symbol: same step through voidweb_forward_pass
    upload_pool(pool, c)
    out2 = np.zeros_like(c.q)
    L = C.lib()
    L.vw_forward_bind(pool.handle, c.q.ctypes.data, c.k_new.ctypes.data, c.v_new.ctypes.data,
                      out2.ctypes.data)
    for b in range(c.B):
        L.vw_forward_set_seq_len(1000 + b, int(c.seq_lens[b]) - 1)
    kl = KernelLib.open(C.LIB_PATH)
    seqs = [(1000 + b, 7, c.block_tables[b, : (int(c.seq_lens[b]) + 15) // 16])
            for b in range(c.B)]
    kl.forward_pass(dict(num_heads=c.Hq, num_kv_heads=c.Hkv, num_layers=c.L, head_dim=c.D,
                         rope_theta=theta), seqs)
    for layer in range(c.L):
        assert np.array_equal(out2[layer], dev_out[layer])
    for b in range(c.B):
        L.vw_forward_release(1000 + b)
    L.vw_forward_bind(None, None, None, None, None)
    pool.close()


def test_full_size_qwen_layer_sampled(dev):
    """Qwen2.5-7B decode shapes at full size (B 16, ctx U[512,4096], 28/4 heads,
    D 128, bf16), one layer: fused append + decode, checked on every sequence
    against the fp64 oracle."""
    c = kvgen.make_case(1, 1, 4, 128, 28, 16, 512, 4096, BF16, BF16)
    pool = make_pool(c, dev)
    got = run_decode(pool, c, 0, dev, fused=True)
    assert pool.check() == 0
    data = c.data.copy()
    oracle.kv_append(c.geom, data, None, 0, c.k_new[0], c.v_new[0], kvgen.new_token_slots(c))
    ref = oracle.paged_decode_f64(c.geom, data, None, 0, c.q[0], c.Hq, c.block_tables,
                                  c.seq_lens, 1.0 / np.sqrt(128))
    check_close(got, ref, BF16, "qwen full-size layer")
    pool.close()


@pytest.mark.parametrize("graph,planned", [(False, False), (True, False), (False, True),
                                           (True, True)])
def test_pdl_layer_chain(dev, graph, planned):
    """Consecutive layers launched as programmatic dependents with early page
    streaming (the flags a decode step uses), eagerly and inside a CUDA graph,
    with and without a decode plan made at the start of the step: every layer's
    pages and outputs must match the oracle."""
    from voidweb_b200 import _lib as C
    c = kvgen.make_case(41, 6, 2, 128, 14, 9, 20, 2500, BF16, BF16)
    pool = make_pool(c, dev)
    bt, sl = tu32(c.block_tables, dev), tu32(c.seq_lens, dev)
    qs = [t16(c.q[l], dev) for l in range(c.L)]
    ks = [t16(c.k_new[l], dev) for l in range(c.L)]
    vs = [t16(c.v_new[l], dev) for l in range(c.L)]
    outs = [torch.zeros_like(qs[0]) for _ in range(c.L)]
    chain = C.VW_DECODE_PDL | C.VW_DECODE_EARLY_PAGES
    s = torch.cuda.Stream(device=dev)

    def step(stream):
        if planned:
            pool.plan(bt, sl, c.Hq, stream=stream)
        for l in range(c.L):
            # the layer right after the plan launch waits for it in stream order
            flags = (C.VW_DECODE_PLANNED | (chain if l > 0 else 0)) if planned else chain
            pool.paged_decode(l, qs[l], bt, sl, outs[l], k_new=ks[l], v_new=vs[l],
                              stream=stream, flags=flags)

    if graph:
        with torch.cuda.stream(s):
            step(s)                     # attribute set-up outside the capture
        s.synchronize()
        upload_pool(pool, c)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step(torch.cuda.current_stream())
        for _ in range(3):              # replays re-append the same rows: idempotent
            g.replay()
        torch.cuda.synchronize()
        del g
    else:
        with torch.cuda.stream(s):
            step(s)
        s.synchronize()
    assert pool.check() == 0
    data = c.data.copy()
    slots = kvgen.new_token_slots(c)
    for l in range(c.L):
        oracle.kv_append(c.geom, data, None, l, c.k_new[l], c.v_new[l], slots)
    gdata, _ = download_pool(pool, c)
    assert np.array_equal(gdata, data)
    for l in range(c.L):
        ref = oracle.paged_decode_f64(c.geom, data, None, l, c.q[l], c.Hq, c.block_tables,
                                      c.seq_lens, 1.0 / np.sqrt(128))
        check_close(outs[l].cpu().numpy().view(np.uint16), ref, BF16, f"layer {l}")
    pool.close()


def test_planned_decode_is_bit_identical(dev):
    """A planned launch uses the same page split and arithmetic as a plain one:
    on the split-K extremes batch the outputs match bit for bit."""
    from voidweb_b200 import _lib as C
    ctx = [1, 2, 15, 16, 17, 31, 32, 33, 9000, 3, 1, 4097, 64, 5, 12000]
    c = kvgen.make_case(98, 1, 2, 128, 14, len(ctx), 0, 0, BF16, BF16, ctx=ctx)
    pool = make_pool(c, dev)
    q, bt, sl = t16(c.q[0], dev), tu32(c.block_tables, dev), tu32(c.seq_lens, dev)
    plain, planned = torch.zeros_like(q), torch.zeros_like(q)
    pool.paged_decode(0, q, bt, sl, plain)
    pool.plan(bt, sl, c.Hq)
    pool.paged_decode(0, q, bt, sl, planned, flags=C.VW_DECODE_PLANNED)
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert torch.equal(plain, planned)
    # a plan of other tables is refused, not used
    other = bt.clone()
    with pytest.raises(C.VoidwebError):
        pool.paged_decode(0, q, other, sl, planned, flags=C.VW_DECODE_PLANNED)
    pool.close()


@pytest.mark.parametrize("kv,io,D", [(BF16, BF16, 128), (F16, F16, 64), (FP8, BF16, 128)])
def test_fused_rope_append_decode(dev, kv, io, D):
    """RoPE fused into the decode (kernels/rope/rope.bm:22-52): q and the new K
    row are rotated to position seq_len-1.  The appended K rows match the
    oracle's rotation within one unit in the last place of the io type (f32
    sin/cos may round differently); V rows and, for FP8, their codes are exact;
    outputs are within the attention tolerance of the fp64 oracle run on the
    rotated q and the device's own pages."""
    theta = 1000000.0 if D == 128 else 10000.0
    c = kvgen.make_case(60 + kv + D, 1, 2, D, 8, 6, 1, 3000, kv, io)
    pool = make_pool(c, dev)
    got = run_decode(pool, c, 0, dev, fused=True, rope_theta=theta)
    assert pool.check() == 0
    pos = c.seq_lens.astype(np.int64) - 1
    q_rot = oracle.rope_apply(c.q[0], pos, theta, io)
    k_rot = oracle.rope_apply(c.k_new[0], pos, theta, io)
    gdata, gscales = download_pool(pool, c)
    slots = kvgen.new_token_slots(c)
    if kv != FP8:
        want = c.data.copy()
        oracle.kv_append(c.geom, want, None, 0, k_rot, c.v_new[0], slots)
        rel = 2.0 ** -7 if io == BF16 else 2.0 ** -10
        exact = 0
        for s in slots:
            blk, t = int(s) // 16, int(s) % 16
            # V rows are untouched by the rotation: bit for bit
            assert np.array_equal(gdata[0, blk, :, 1, t], want[0, blk, :, 1, t])
            # rotated K rows: two last places of an f32 angle below 2^12 rad
            # (< 2.5e-4 rad each) times |x_r| + |x_i| < 8, plus one io rounding
            g = oracle.io_bits_to_f32(gdata[0, blk, :, 0, t], io)
            w = oracle.io_bits_to_f32(want[0, blk, :, 0, t], io)
            assert (np.abs(g - w) <= 8e-3 + rel * np.abs(w)).all(), "rotated K row"
            exact += np.sum(gdata[0, blk, :, 0, t] == want[0, blk, :, 0, t])
        assert exact >= 0.9 * len(slots) * c.Hkv * D
        # and nothing else in the pool moved
        mask = np.ones(gdata.shape, dtype=bool)
        for s in slots:
            mask[0, int(s) // 16, :, :, int(s) % 16] = False
        assert np.array_equal(gdata[mask], want[mask])
    ref = oracle.paged_decode_f64(c.geom, gdata, gscales, 0, q_rot, c.Hq, c.block_tables,
                                  c.seq_lens, 1.0 / np.sqrt(D))
    check_close(got, ref, io, f"rope {kv}/{io}/D{D}")
    pool.close()
