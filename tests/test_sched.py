"""The continuous-batching scheduler wired to the block manager (vw_sched_*):
the batching rules of scheduler/scheduler.bm:241-326 (token budget, chunks of
at most max_chunk prompt tokens, prefill descriptors before decodes, commit /
drain) and the KV bookkeeping around them (block tables, prefix reuse of full
pages, LRU release of cached pages, preemption, chunk continuation).  Every
step is checked against the invariants: a scheduled sequence's table covers
the positions it writes, the pages it writes are its own (ref_count 1), and
the block manager's references are the tables' entries plus one per page the
prefix index keeps."""
import numpy as np
import pytest

from voidweb_b200 import BlockManager
from voidweb_b200.sched import Scheduler


def check_step(bm, s, batch, max_batch_tokens=None, max_chunk=None):
    st = s.stats()
    refs = sum(bm.ref_count(b) for b in range(bm.capacity()))
    assert refs == st["table_refs"] + st["cached_pages"]
    assert st["free_blocks"] + sum(1 for b in range(bm.capacity()) if bm.ref_count(b) > 0) == bm.capacity()
    seen_prefill_done = False
    prefill_tokens = 0
    for q in batch.seqs:
        n = len(q.tokens)
        assert len(q.table) == (q.ctx_start + n + 15) // 16
        assert len(set(q.table.tolist())) == len(q.table)
        for p in range(q.ctx_start // 16, len(q.table)):
            assert bm.ref_count(int(q.table[p])) == 1, "a written page is shared"
        if q.is_prefill:
            assert not seen_prefill_done, "prefill descriptors come first"
            prefill_tokens += n
            if max_chunk:
                assert n <= max_chunk
        else:
            seen_prefill_done = True
            assert n == 1 and q.samples
    if max_batch_tokens:
        assert prefill_tokens <= max_batch_tokens


def run(bm, s, steps, sampler, **kw):
    """Drive schedule/commit; sampler(seq_id, step) -> token.  Returns the
    batches and the finished (id, tokens) pairs."""
    batches, finished = [], []
    for step in range(steps):
        b = s.schedule()
        check_step(bm, s, b, **kw)
        batches.append(b)
        s.commit({q.seq_id: sampler(q.seq_id, step) for q in b.seqs if q.samples})
        finished += s.take_finished()
        if not b.seqs and s.stats()["waiting"] == 0 and s.stats()["running"] == 0:
            break
    return batches, finished


def test_chunks_continue_and_only_the_last_chunk_samples():
    bm = BlockManager(1, 1, 128, 16, 1024)
    s = Scheduler(bm, max_batch_tokens=8192, max_chunk=2048)
    rid = s.add_request(np.arange(5000) % 3000, 3)
    batches, finished = run(bm, s, 10, lambda i, k: 7, max_chunk=2048)
    pf = [q for b in batches for q in b.seqs if q.is_prefill]
    assert [(q.ctx_start, len(q.tokens), q.samples) for q in pf] == \
        [(0, 2048, False), (2048, 2048, False), (4096, 904, True)]
    dc = [q.ctx_start for b in batches for q in b.seqs if not q.is_prefill]
    assert dc == [5000, 5001]
    assert finished == [(rid, finished[0][1])] and finished[0][1].tolist() == [7, 7, 7]


def test_token_budget_is_shared_across_admissions():
    bm = BlockManager(1, 1, 128, 16, 4096)
    s = Scheduler(bm, max_batch_tokens=4096, max_chunk=2048)
    rng = np.random.default_rng(0)
    for _ in range(6):
        s.add_request(rng.integers(0, 30000, 3000), 4)
    batches, finished = run(bm, s, 60, lambda i, k: 5, max_batch_tokens=4096, max_chunk=2048)
    assert len(finished) == 6 and all(len(t) == 4 for _, t in finished)


def test_prefix_reuse_shares_full_pages():
    bm = BlockManager(1, 1, 128, 16, 256)
    s = Scheduler(bm)
    prompt = np.arange(100) + 1000
    a = s.add_request(prompt, 2)
    batches, _ = run(bm, s, 10, lambda i, k: 1)
    a_table = [q.table for b in batches for q in b.seqs if q.seq_id == a][-1]
    assert s.stats()["cached_pages"] == 6                # floor(101 cached tokens / 16)
    b = s.add_request(np.concatenate([prompt, np.arange(20)]), 2)
    first = s.schedule()
    check_step(bm, s, first)
    q = first.seqs[0]
    assert q.seq_id == b and q.ctx_start == 96            # 6 pages reused, prefill from 96
    assert q.table[:6].tolist() == a_table[:6].tolist()
    assert q.tokens.tolist() == list(range(1096, 1100)) + list(range(20))
    # the identical prompt again: at least its last token is computed
    s.commit({q.seq_id: 3 for q in first.seqs if q.samples})
    c = s.add_request(prompt[:32], 1)
    nxt = s.schedule()
    qc = [q for q in nxt.seqs if q.seq_id == c][0]
    assert qc.ctx_start == 16 and len(qc.tokens) == 16
    s.close()


def test_cached_pages_are_released_under_pressure():
    bm = BlockManager(1, 1, 128, 16, 24)
    s = Scheduler(bm)
    rng = np.random.default_rng(1)
    done = 0
    for r in range(12):                                   # each keeps 4 full pages cached
        s.add_request(rng.integers(0, 30000, 64), 1)
        _, fin = run(bm, s, 10, lambda i, k: 9)
        done += len(fin)
        assert s.stats()["cached_pages"] <= 24
    assert done == 12
    assert s.stats()["free_blocks"] + s.stats()["cached_pages"] == 24


def test_preemption_when_decodes_outgrow_the_pool():
    bm = BlockManager(1, 1, 128, 16, 16)
    s = Scheduler(bm, prefix_cache=False)
    rng = np.random.default_rng(2)
    ids = [s.add_request(rng.integers(0, 30000, 30), 40) for _ in range(4)]
    batches, finished = run(bm, s, 2000, lambda i, k: (i * 7 + k) % 1000)
    assert s.stats()["preemptions"] > 0
    assert sorted(i for i, _ in finished) == sorted(ids)
    assert all(len(t) == 40 for _, t in finished)
    # a preempted request re-prefills its prompt and its sampled tokens but the last
    re = [q for b in batches for q in b.seqs if q.is_prefill and not q.samples and q.ctx_start == 0
          and len(q.tokens) > 30]
    assert re, "no recompute prefill after a preemption"
    assert s.stats()["free_blocks"] == 16


def test_stop_token_and_errors():
    bm = BlockManager(1, 1, 128, 16, 64)
    s = Scheduler(bm, max_seq_len=100)
    rid = s.add_request([1, 2, 3], 10, stop_token=42)
    b = s.schedule()
    s.commit({rid: 5})
    b = s.schedule()
    s.commit({rid: 42})
    fin = s.take_finished()
    assert fin[0][0] == rid and fin[0][1].tolist() == [5, 42]
    with pytest.raises(Exception):
        s.add_request(np.arange(95), 10)                   # longer than max_seq_len
    with pytest.raises(Exception):
        s.commit({12345: 1})                               # not a sampling sequence
