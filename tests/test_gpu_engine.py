"""The scheduler and the kernels together, end to end on the GPU: requests with
shared prefixes are scheduled (chunked prefill, decodes, prefix reuse of full
pages, LRU release of cached pages and preemption in a small pool), and every
step runs the block copies, one vw_paged_prefill per layer for the prefill
chunks and one fused append + vw_paged_decode per layer for the decodes.  The
K/V/q rows of a token are a deterministic function of its position and of the
whole prefix up to it (as a model's would be), so reused pages and recomputed
sequences must hold exactly the rows a fresh computation gives; every
attention output is checked against an fp64 attention over the sequence's rows
computed from scratch (|gpu - ref| <= 2e-3 + 1e-2 |ref|)."""
import numpy as np
import pytest

import oracle
from tests.test_gpu_kv import check_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

L, HKV, D, HQ = 2, 2, 128, 8
P = 0x9E3779B97F4A7C15
MASK = (1 << 64) - 1


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


class Rows:
    """K, V, q rows (bf16 bits) of every position of a token sequence."""

    def __init__(self):
        self.cache = {}

    def of(self, tokens):
        h, out_k, out_v, out_q = 0, [], [], []
        for p, t in enumerate(tokens):
            h = (h * P + int(t) + 1) & MASK
            key = (h, p)
            if key not in self.cache:
                rng = np.random.Generator(np.random.PCG64([h & 0xFFFFFFFF, h >> 32, p]))
                x = rng.standard_normal((2 * L * HKV + L * HQ, D), dtype=np.float32)
                b = oracle.f32_to_bf16_bits(x)
                self.cache[key] = (b[:L * HKV].reshape(L, HKV, D), b[L * HKV:2 * L * HKV].reshape(L, HKV, D),
                                   b[2 * L * HKV:].reshape(L, HQ, D))
            k, v, q = self.cache[key]
            out_k.append(k); out_v.append(v); out_q.append(q)
        return np.stack(out_k, 1), np.stack(out_v, 1), np.stack(out_q, 1)   # [L][n][H][D]


def attention_ref(k, v, q_row, pos):
    """fp64 causal attention of one query row at position pos: [HQ][D]."""
    kf = oracle.bf16_bits_to_f32(k[:pos + 1]).astype(np.float64)      # [pos+1][HKV][D]
    vf = oracle.bf16_bits_to_f32(v[:pos + 1]).astype(np.float64)
    qf = oracle.bf16_bits_to_f32(q_row).astype(np.float64)            # [HQ][D]
    out = np.zeros((HQ, D))
    g = HQ // HKV
    for j in range(HQ):
        s = kf[:, j // g] @ qf[j] / np.sqrt(D)
        w = np.exp(s - s.max())
        out[j] = (w @ vf[:, j // g]) / w.sum()
    return out


def test_scheduler_drives_prefill_and_decode(dev):
    from voidweb_b200 import BlockManager
    from voidweb_b200.kv import KvPool, PoolSpec
    from voidweb_b200.sched import Scheduler
    NB = 40
    bm = BlockManager(L, HKV, D, 16, NB)
    s = Scheduler(bm, max_batch_tokens=64, max_chunk=32, max_running_seqs=4)
    pool = KvPool(PoolSpec(L, HKV, D, NB, "bf16", "bf16", max_batch=8), device=0)
    pool.pages_u8().zero_()
    rows = Rows()
    rng = np.random.default_rng(4)
    shared = rng.integers(100, 5000, 50)
    seqs = {}
    for r in range(6):
        tail = rng.integers(100, 5000, int(rng.integers(5, 40)))
        prompt = np.concatenate([shared, tail]) if r % 2 == 0 else rng.integers(100, 5000, 60)
        rid = s.add_request(prompt, int(rng.integers(4, 10)))
        seqs[rid] = list(int(t) for t in prompt)
    t16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)
    ti32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)
    checked = reused = 0
    finished, started = [], set()
    for step in range(400):
        b = s.schedule()
        if not b.seqs:
            if s.stats()["running"] == 0 and s.stats()["waiting"] == 0:
                break
            continue
        if len(b.copies):
            pool.block_copy(ti32(b.copies))
        pf = [q for q in b.seqs if q.is_prefill]
        dc = [q for q in b.seqs if not q.is_prefill]
        for q in pf:                                       # a request's first chunk
            if q.seq_id not in started:
                started.add(q.seq_id)
                reused += q.ctx_start > 0
        stride = max(len(q.table) for q in b.seqs)
        want = {}
        # inputs: the rows of the tokens this step appends, from the sequence so far
        if pf:
            cu = np.zeros(len(pf) + 1, np.int32)
            cu[1:] = np.cumsum([len(q.tokens) for q in pf])
            T = int(cu[-1])
            qk = np.zeros((L, T, HKV, D), np.uint16); qv = np.zeros_like(qk)
            qq = np.zeros((L, T, HQ, D), np.uint16)
            bt = np.zeros((len(pf), stride), np.int32)
            for i, q in enumerate(pf):
                toks = seqs[q.seq_id][:q.ctx_start + len(q.tokens)]
                assert toks[q.ctx_start:] == q.tokens.tolist()
                k, v, qr = rows.of(toks)
                qk[:, cu[i]:cu[i + 1]] = k[:, q.ctx_start:]
                qv[:, cu[i]:cu[i + 1]] = v[:, q.ctx_start:]
                qq[:, cu[i]:cu[i + 1]] = qr[:, q.ctx_start:]
                bt[i, :len(q.table)] = q.table
                want[q.seq_id] = (k, v, qr, q.ctx_start, len(q.tokens), cu[i])
            cs = np.array([q.ctx_start for q in pf], np.int32)
            for layer in range(L):
                out = torch.zeros((T, HQ, D), dtype=torch.int16, device=dev)
                pool.paged_prefill(layer, t16(qq[layer]), ti32(cu), ti32(cs), ti32(bt), out,
                                   k_new=t16(qk[layer]), v_new=t16(qv[layer]))
                got = out.cpu().numpy().view(np.uint16)
                for i, q in enumerate(pf):
                    k, v, qr, c0, n, off = want[q.seq_id]
                    for t in range(n):
                        ref = attention_ref(k[layer], v[layer], qr[layer, c0 + t], c0 + t)
                        check_close(got[off + t], ref, oracle.BF16, f"prefill seq {q.seq_id} pos {c0 + t}")
                        checked += 1
        if dc:
            B = len(dc)
            bt = np.zeros((B, stride), np.int32)
            dk = np.zeros((L, B, HKV, D), np.uint16); dv = np.zeros_like(dk)
            dq = np.zeros((L, B, HQ, D), np.uint16)
            refs = []
            for i, q in enumerate(dc):
                toks = seqs[q.seq_id][:q.ctx_start + 1]
                assert toks[-1] == int(q.tokens[0])
                k, v, qr = rows.of(toks)
                dk[:, i] = k[:, -1]; dv[:, i] = v[:, -1]; dq[:, i] = qr[:, -1]
                bt[i, :len(q.table)] = q.table
                refs.append((k, v, qr))
            sl = np.array([q.ctx_start + 1 for q in dc], np.int32)
            for layer in range(L):
                out = torch.zeros((B, HQ, D), dtype=torch.int16, device=dev)
                pool.paged_decode(layer, t16(dq[layer]), ti32(bt), ti32(sl), out,
                                  k_new=t16(dk[layer]), v_new=t16(dv[layer]))
                got = out.cpu().numpy().view(np.uint16)
                for i, q in enumerate(dc):
                    k, v, qr = refs[i]
                    ref = attention_ref(k[layer], v[layer], qr[layer, -1], q.ctx_start)
                    check_close(got[i], ref, oracle.BF16, f"decode seq {q.seq_id} pos {q.ctx_start}")
                    checked += 1
        torch.cuda.synchronize()
        assert pool.check() == 0
        sampled = {q.seq_id: int(100 + (q.seq_id * 131 + step) % 4000) for q in b.seqs if q.samples}
        s.commit(sampled)
        for rid, tok in sampled.items():
            seqs[rid].append(tok)
        finished += s.take_finished()
    assert len(finished) == 6
    assert reused > 0, "no prefix reuse happened"
    assert checked > 500
    s.close()
    pool.close()
