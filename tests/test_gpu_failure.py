"""Failure detection on the GPU without a fault: the bounded waits of the
decode and prefill kernels.

Every wait (for a page copy, a query tile, a free stage, a tensor-core result)
gives up after a deadline; the launch then records VW_DEV_ERR_TIMEOUT, waits
for the copies and MMAs it has in flight, frees its tensor memory, and
returns, leaving the context usable.  The test hook vw_debug_set_wait_limit
shortens the deadline to one SM cycle and withholds the copies the first waits
need (query tiles for the decode, K/V tiles for the prefill), so those waits
run out; nothing else is changed (no trap, no bad address, no endless loop).
The pool must then report the timeout, and after vw_pool_check the next normal
launch must give the oracle's results."""
import numpy as np
import pytest

import oracle
from tests import kvgen
from tests.kvgen import BF16, FP8
from tests.test_gpu_kv import check_close, download_pool, make_pool, run_decode, t16, tu32, upload_pool

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("kv", [BF16, FP8])
@pytest.mark.parametrize("chained", [False, True], ids=["plain", "pdl_early_pages"])
def test_decode_wait_timeout_unwinds_and_pool_recovers(dev, kv, chained):
    from voidweb_b200 import _lib as C
    # enough pages per decode CTA that copies are in flight when the waits give up
    c = kvgen.make_case(71 + kv, 1, 2, 128, 8, 6, 2000, 6000, kv, BF16)
    pool = make_pool(c, dev)
    q, bt, sl = t16(c.q[0], dev), tu32(c.block_tables, dev), tu32(c.seq_lens, dev)
    kn, vn = t16(c.k_new[0], dev), t16(c.v_new[0], dev)
    out = torch.zeros_like(q)
    flags = (C.VW_DECODE_PDL | C.VW_DECODE_EARLY_PAGES) if chained else 0
    pool.set_wait_limit(1)
    for _ in range(2):
        pool.paged_decode(0, q, bt, sl, out, k_new=kn, v_new=vn, flags=flags)
    err = pool.check()
    assert err & C.DEV_ERR_TIMEOUT, f"device word 0x{err:x}"
    # nothing but the timeout: no block id or length was misread on the way out
    assert err == C.DEV_ERR_TIMEOUT, f"device word 0x{err:x}"
    # the context is intact: a normal launch on the same pool matches the oracle
    pool.set_wait_limit(0)
    upload_pool(pool, c)
    got = run_decode(pool, c, 0, dev, fused=True)
    assert pool.check() == 0
    data = c.data.copy()
    scales = c.scales.copy() if kv == FP8 else None
    oracle.kv_append(c.geom, data, scales, 0, c.k_new[0], c.v_new[0], kvgen.new_token_slots(c))
    gdata, _ = download_pool(pool, c)
    assert np.array_equal(gdata, data)
    ref = oracle.paged_decode_f64(c.geom, data, scales, 0, c.q[0], c.Hq, c.block_tables,
                                  c.seq_lens, 1.0 / np.sqrt(128))
    check_close(got, ref, BF16, f"after timeout kv={kv}")
    pool.close()


@pytest.mark.parametrize("kv", [BF16, FP8])
def test_prefill_wait_timeout_unwinds_and_pool_recovers(dev, kv):
    from voidweb_b200 import _lib as C
    from tests.test_gpu_prefill import chunk_case, run_prefill
    c, q, k, v, cu, cs = chunk_case(91 + kv, BF16, 128, 8, 2, [(700, 130), (0, 64)], L=1, kv=kv)
    pool = make_pool(c, dev)
    pool.set_wait_limit(1)
    run_prefill(pool, c, 0, q, k, v, cu, cs, dev)
    err = pool.check()
    assert err == C.DEV_ERR_TIMEOUT, f"device word 0x{err:x}"
    pool.set_wait_limit(0)
    upload_pool(pool, c)
    got = run_prefill(pool, c, 0, q, k, v, cu, cs, dev)
    assert pool.check() == 0
    oracle.kv_append(c.geom, c.data, c.scales, 0, k, v, oracle.prefill_slots(c.block_tables, cu, cs))
    ref = oracle.paged_prefill_f64(c.geom, c.data, c.scales, 0, q, c.Hq, c.block_tables, cu, cs, True,
                                   1.0 / np.sqrt(128))
    check_close(got, ref, BF16, f"prefill after timeout kv={kv}")
    pool.close()
