"""Host bookkeeping (C++ BlockManager / RadixCacheManager in libvoidweb_kv.so)
against the oracle restatement of engine/kv_cache.bm and radix_cache.bm:
golden traces plus randomized differential runs.  CPU only."""
import numpy as np
import pytest

import oracle
from voidweb_b200 import BlockManager, RadixCacheManager, rolling_hash


def test_rolling_hash_golden(golden):
    for case in golden["rolling_hash"]:
        assert rolling_hash(int(case["prev"]), case["tokens"]) == int(case["hash"])


def test_block_manager_golden_trace(golden):
    bm = BlockManager(1, 1, 64, 16, 12)
    for step in golden["block_manager_trace"]:
        op, args = step["op"], step["args"]
        if op == "alloc_seq":
            try:
                r = bm.alloc_seq(*args)
            except MemoryError as e:
                assert "KV cache OOM" in str(e)
                r = "OOM"
        else:
            r = getattr(bm, op)(*args)
        assert r == step["ret"], step
        assert bm.free_list() == step["free"], step
        refs = {str(k): bm.ref_count(k) for k in range(12) if bm.ref_count(k) > 0}
        assert refs == step["refs"], step


@pytest.mark.parametrize("seed", range(6))
def test_block_manager_differential(seed):
    rng = np.random.default_rng(seed)
    nb = 64
    a, b = BlockManager(1, 1, 64, 16, nb), oracle.BlockManager(16, nb)
    live = []
    hashes = []
    for _ in range(600):
        op = rng.integers(0, 9)
        if op == 0:
            assert a.alloc() == b.alloc()
        elif op == 1:
            n = int(rng.integers(0, 6))
            try:
                ra = a.alloc_seq(n)
            except MemoryError:
                ra = None
            try:
                rb = b.alloc_seq(n)
            except MemoryError:
                rb = None
            assert ra == rb
            if ra:
                live.extend(ra)
        elif op in (2, 3):
            i = int(rng.integers(0, nb + 3))
            (a.incref if op == 2 else a.decref)(i)
            (b.incref if op == 2 else b.decref)(i)
        elif op == 4 and live:
            t = [live[int(k)] for k in rng.integers(0, len(live), int(rng.integers(1, 5)))]
            a.free_seq(t)
            b.free_seq(t)
        elif op == 5:
            toks = [int(x) for x in rng.integers(0, 50, int(rng.integers(1, 40)))]
            h = oracle.rolling_hash(0, toks[:16])
            i = int(rng.integers(0, nb))
            a.register_prefix_block(i, h)
            b.register_prefix_block(i, h)
            hashes.append(toks)
        elif op == 6 and hashes:
            t = hashes[int(rng.integers(0, len(hashes)))]
            assert a.prefix_lookup(t) == b.prefix_lookup(t)
        assert a.free_count() == b.free_count()
        assert a.capacity() == b.capacity()
    assert a.free_list() == b.free_list()
    for i in range(nb):
        assert a.ref_count(i) == b.ref_count(i)


def test_radix_golden_trace(golden):
    rx = RadixCacheManager(16, 20)
    for step in golden["radix_trace"]:
        op = step["op"]
        if op == "lookup":
            assert list(rx.lookup(step["tokens"])) == step["ret"], step
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


@pytest.mark.parametrize("seed", range(8))
def test_radix_differential(seed):
    rng = np.random.default_rng(100 + seed)
    a, b = RadixCacheManager(16, 60), oracle.RadixCache(16, 60)
    prefixes = [[int(x) for x in rng.integers(0, 30, int(rng.integers(1, 48)))] for _ in range(4)]
    seqs = []
    nxt = 0
    for _ in range(120):
        op = rng.integers(0, 6)
        if op <= 1:
            pre = prefixes[int(rng.integers(0, 4))]
            suf = [int(x) for x in rng.integers(0, 30, int(rng.integers(0, 40)))]
            s = pre + suf
            if not s:
                continue
            nbk = (len(s) + 15) // 16
            blocks = list(range(nxt, nxt + nbk))
            nxt += nbk
            assert a.insert(s, blocks) == b.insert(s, blocks)
            seqs.append(s)
        elif op == 2 and seqs:
            s = seqs[int(rng.integers(0, len(seqs)))][: int(rng.integers(1, 80))]
            assert a.lookup(s) == b.lookup(s)
        elif op == 3:
            t = int(rng.integers(1, 6))
            assert a.evict_lru(t) == b.evict_lru(t)
        elif op == 4 and seqs:
            s = seqs[int(rng.integers(0, len(seqs)))]
            a.lock(s)
            b.lock(s)
        elif op == 5 and seqs:
            s = seqs[int(rng.integers(0, len(seqs)))]
            a.unlock(s)
            b.unlock(s)
        assert a.total_blocks() == b.total_blocks()
    assert a.evict_lru(10 ** 6) == b.evict_lru(10 ** 6)


def test_cow_and_compact():
    bm = BlockManager(1, 1, 64, 16, 16)
    t = np.array(bm.alloc_seq(3), dtype=np.uint32)          # [15, 14, 13]
    assert t.tolist() == [15, 14, 13]
    assert bm.cow(t, 2) is None                              # not shared
    bm.incref(13)                                            # a second owner
    pair = bm.cow(t, 2)
    assert pair == (13, 12) and t.tolist() == [15, 14, 12]
    assert bm.ref_count(13) == 1 and bm.ref_count(12) == 1
    bm.decref(14)
    # used: 15, 13, 12 -> compact to ids 0..2
    pairs = bm.compact()
    assert sorted(pairs[:, 0].tolist()) == [12, 13, 15]
    assert sorted(pairs[:, 1].tolist()) == [0, 1, 2]
    assert [bm.ref_count(i) for i in range(4)] == [1, 1, 1, 0]
    assert bm.alloc() == 3                                  # lowest free id next
    rx = RadixCacheManager(16, 100)
    rx.insert(list(range(20)), [12, 15])
    rx.remap(pairs)
    m = dict(zip(pairs[:, 0].tolist(), pairs[:, 1].tolist()))
    assert rx.lookup(list(range(20)))[1] == [m[12], m[15]]
