"""vw_paged_decode_static (split-K scratch in a fixed array compiled into the
library, no allocation) against vw_paged_decode (scratch owned by the pool),
both called through the C ABI on the same inputs, twice in a row.

Tolerance: |static - pool| <= 2e-3 + 1e-2 * |pool| elementwise on the f32
values of the outputs, and both within the same bound of the fp64 oracle.
"""
import ctypes

import numpy as np
import pytest

import oracle
from tests import kvgen
from tests.kvgen import BF16, FP8

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _t16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)


def _tu32(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).astype(np.int32)).to(dev)


def _call(entry, pool, layer, q, bt, sl, out, kn, vn, flags=0, stream=None):
    from voidweb_b200 import _lib as C
    a = C.DecodeArgs(layer, q.shape[0], q.shape[1], bt.shape[1], q.data_ptr(), bt.data_ptr(),
                     sl.data_ptr(), out.data_ptr(),
                     kn.data_ptr() if kn is not None else None,
                     vn.data_ptr() if vn is not None else None, 0.0, flags)
    s = stream if stream is not None else torch.cuda.current_stream()
    C.check(getattr(C.lib(), entry)(pool._h, ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)))


def _allocs():
    from voidweb_b200 import _lib as C
    return C.lib().vw_debug_alloc_count()


def _close(got_bits, ref_f64, io, what):
    got = oracle.io_bits_to_f32(got_bits, io).astype(np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref_f64)
    bound = ATOL + RTOL * np.abs(ref_f64)
    assert (err <= bound).all(), f"{what}: {(err > bound).sum()} outside, max err {err.max():.3g}"


CASES = [
    # name, seed, Hkv, Hq, B, ctx_lo, ctx_hi, kv, fused append
    ("qwen_bf16_split", 21, 4, 28, 12, 300, 3000, BF16, False),
    ("fp8_fused_append", 22, 2, 8, 9, 40, 2000, FP8, True),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_static_scratch_decode_matches_pool_scratch(case):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voidweb_b200.kv import KvPool, PoolSpec
    _, seed, Hkv, Hq, B, lo, hi, kv, fused = case
    dev = torch.device("cuda", 0)
    c = kvgen.make_case(seed, 1, Hkv, 128, Hq, B, lo, hi, kv, BF16)
    pool = KvPool(PoolSpec(**kvgen.pool_spec_kwargs(c)), device=0)
    pool.pages_u8().copy_(torch.from_numpy(np.ascontiguousarray(c.data).view(np.uint8).ravel()))
    if kv == FP8:
        pool.scales_f32().copy_(torch.from_numpy(c.scales.ravel()))
    q, bt, sl = _t16(c.q[0], dev), _tu32(c.block_tables, dev), _tu32(c.seq_lens, dev)
    kn = _t16(c.k_new[0], dev) if fused else None
    vn = _t16(c.v_new[0], dev) if fused else None
    ref_out = torch.zeros_like(q)
    outs = [torch.zeros_like(q) for _ in range(3)]
    torch.cuda.synchronize()

    _call("vw_paged_decode", pool, 0, q, bt, sl, ref_out, kn, vn)
    _call("vw_paged_decode_static", pool, 0, q, bt, sl, outs[0], kn, vn)   # first call: setup
    torch.cuda.synchronize()
    # the library's own allocation count must not move; the device's free
    # memory is only a loose second check (the GPU may be shared)
    allocs = _allocs()
    free_before = torch.cuda.mem_get_info(dev)[0]
    _call("vw_paged_decode_static", pool, 0, q, bt, sl, outs[1], kn, vn)
    _call("vw_paged_decode_static", pool, 0, q, bt, sl, outs[2], kn, vn)
    torch.cuda.synchronize()
    assert _allocs() == allocs, "a static-scratch call allocated"
    assert torch.cuda.mem_get_info(dev)[0] >= free_before - (64 << 20)
    assert pool.check() == 0

    # the pages the oracle reads: the upload, plus the fused append's rows
    data = c.data.copy()
    scales = c.scales.copy() if kv == FP8 else None
    if fused:
        oracle.kv_append(c.geom, data, scales, 0, c.k_new[0], c.v_new[0], kvgen.new_token_slots(c))
    ref64 = oracle.paged_decode_f64(c.geom, data, scales, 0, c.q[0], Hq, c.block_tables,
                                    c.seq_lens, 1.0 / np.sqrt(128))
    pool_bits = ref_out.cpu().numpy().view(np.uint16)
    _close(pool_bits, ref64, BF16, "vw_paged_decode vs oracle")
    pool_f64 = oracle.io_bits_to_f32(pool_bits, BF16).astype(np.float64)
    for i, o in enumerate(outs):
        bits = o.cpu().numpy().view(np.uint16)
        _close(bits, pool_f64, BF16, f"static call {i} vs vw_paged_decode")
        _close(bits, ref64, BF16, f"static call {i} vs oracle")
    pool.close()


def test_static_scratch_layer_chain_with_pdl_and_plan():
    """Consecutive layers through vw_paged_decode_static on one stream as
    programmatic dependents with early page streaming (one partial set shared
    by overlapping launches: a launch writes partials only after the one
    before it has completed), on a batch whose segments are split across
    decode CTAs; then the same chain with VW_DECODE_PLANNED.  Every layer's
    pages and outputs against the oracle; the planned chain bit-identical."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voidweb_b200 import _lib as C
    from voidweb_b200.kv import KvPool, PoolSpec
    dev = torch.device("cuda", 0)
    ctx = [5, 9000, 17, 3000, 1, 4100, 33, 12000, 700]
    c = kvgen.make_case(23, 5, 2, 128, 14, len(ctx), 0, 0, BF16, BF16, ctx=ctx)
    pool = KvPool(PoolSpec(**kvgen.pool_spec_kwargs(c)), device=0)
    pool.pages_u8().copy_(torch.from_numpy(np.ascontiguousarray(c.data).view(np.uint8).ravel()))
    bt, sl = _tu32(c.block_tables, dev), _tu32(c.seq_lens, dev)
    qs = [_t16(c.q[l], dev) for l in range(c.L)]
    ks = [_t16(c.k_new[l], dev) for l in range(c.L)]
    vs = [_t16(c.v_new[l], dev) for l in range(c.L)]
    chain = C.VW_DECODE_PDL | C.VW_DECODE_EARLY_PAGES
    s = torch.cuda.Stream(device=dev)
    results = []
    for planned in (False, True):
        outs = [torch.zeros_like(qs[0]) for _ in range(c.L)]
        torch.cuda.synchronize()
        allocs = _allocs()
        with torch.cuda.stream(s):
            if planned:
                pool.plan(bt, sl, c.Hq, stream=s)
            for l in range(c.L):
                f = (chain if l > 0 else 0) | (C.VW_DECODE_PLANNED if planned else 0)
                _call("vw_paged_decode_static", pool, l, qs[l], bt, sl, outs[l], ks[l], vs[l],
                      flags=f, stream=s)
        s.synchronize()
        # (the plan lives in pool memory made at creation: nothing new either way)
        assert _allocs() == allocs, "a static-scratch call allocated"
        assert pool.check() == 0
        results.append([o.cpu().numpy().view(np.uint16) for o in outs])
    data = c.data.copy()
    slots = kvgen.new_token_slots(c)
    for l in range(c.L):
        oracle.kv_append(c.geom, data, None, l, c.k_new[l], c.v_new[l], slots)
    gdata = pool.pages_u8().cpu().numpy().view(np.uint16).reshape(data.shape)
    assert np.array_equal(gdata, data)
    for l in range(c.L):
        ref = oracle.paged_decode_f64(c.geom, data, None, l, c.q[l], c.Hq, c.block_tables,
                                      c.seq_lens, 1.0 / np.sqrt(128), nthreads=0)
        _close(results[0][l], ref, BF16, f"static chain layer {l}")
        assert np.array_equal(results[1][l], results[0][l]), f"planned layer {l}"
    pool.close()
