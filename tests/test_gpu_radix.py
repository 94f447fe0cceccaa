"""Shared-prefix workload on the GPU (the copy-on-write decision of
engine/kv_cache.bm:94-113, the LRU eviction of radix_cache/radix_cache.bm:231-285
and compaction moves around a decode): the device pool must equal the oracle's
mirror bit for bit after every phase, and the decode outputs must stay within
|gpu - ref| <= 2e-3 + 1e-2 * |ref| of the fp64 oracle over the mirror."""
import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _close(got_bits, ref, what):
    got = oracle.bf16_bits_to_f32(got_bits).astype(np.float64)
    err = np.abs(got - ref)
    bad = err > ATOL + RTOL * np.abs(ref)
    assert np.isfinite(got).all() and not bad.any(), f"{what}: {bad.sum()} outside, max {err.max():.3g}"


@pytest.mark.parametrize("layers", [2, 28])
def test_shared_prefix_cow_evict_compact_decode(layers):
    """Seed 2, Qwen2.5-7B KV shapes (4 KV heads, head_dim 128, bf16), 64 requests
    sharing a 128-token prefix, suffixes U[32, 1024]; at 2 layers and at the
    model's full 28 layers, every layer's decode compared."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.radix_workload import DeviceSide, Workload
    wl = Workload(seed=2, L=layers)
    dev = DeviceSide(wl, torch)
    pairs = wl.build(dev)
    assert len(pairs) == wl.n_fork
    assert np.array_equal(dev.pages(wl), wl.mirror), "pool after prefix/suffix appends and COW"
    # every request and fork shares the 8 prefix pages
    prefix_ids = [int(b) for b in wl.seqs[0]["table"][:8]]
    assert all(wl.bm.ref_count(b) == 1 + len(wl.seqs) for b in prefix_ids)

    outs, refs = wl.decode_step(dev, wl.seqs)
    for layer, (o, r) in enumerate(zip(outs, refs)):
        _close(o, r, f"decode before eviction, layer {layer}")
    assert np.array_equal(dev.pages(wl), wl.mirror), "pool after fused append"

    evicted, moves = wl.finish_and_evict(dev, n_finish=32)
    assert len(evicted) > 0 and len(moves) > 0
    assert np.array_equal(dev.pages(wl), wl.mirror), "pool after compaction moves"
    used = [b for b in range(wl.NB) if wl.bm.ref_count(b) > 0]
    assert used == list(range(len(used))), "compaction leaves used ids dense from 0"

    outs, refs = wl.decode_step(dev, wl.seqs)
    for layer, (o, r) in enumerate(zip(outs, refs)):
        _close(o, r, f"decode after eviction and compaction, layer {layer}")
    assert np.array_equal(dev.pages(wl), wl.mirror), "pool after the second step"
    assert dev.pool.check() == 0
    dev.pool.close()
