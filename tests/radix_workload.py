"""Shared-prefix workload (Qwen2.5-7B KV shapes): requests that share one
128-token prefix through the radix tree, forks of sequences whose last page is
partial (copy-on-write on divergence), an LRU eviction of a quarter of the
tree's unreferenced blocks, compaction, and decode steps in between.

The host decisions come from the library's own bookkeeping (BlockManager,
RadixCacheManager); every device operation is mirrored on a numpy copy of the
pool with the oracle (append, block copy), so the device pool can be compared
with the mirror bit for bit after each phase and the decode outputs with the
oracle's decode over the mirror.

Reference-count protocol (the engine's, which the reference leaves implicit):
a block holds one reference per request table that lists it and one for the
radix tree when the tree keeps it.
"""
from __future__ import annotations

import numpy as np

import oracle

PREFIX_TOKENS = 128


class Workload:
    def __init__(self, seed, L=2, Hkv=4, D=128, Hq=28, n_req=64, suffix=(32, 1024), n_fork=8,
                 num_blocks=2600):
        from voidweb_b200 import BlockManager, RadixCacheManager
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.L, self.Hkv, self.D, self.Hq = L, Hkv, D, Hq
        self.NB = num_blocks
        self.geom = oracle.geom(L, Hkv, D, num_blocks, oracle.BF16, oracle.BF16)
        self.mirror = np.zeros(oracle.pool_shape(self.geom), dtype=np.uint16)
        self.bm = BlockManager(L, Hkv, D, 16, num_blocks)
        self.rx = RadixCacheManager(16, num_blocks)
        self.n_req, self.suffix, self.n_fork = n_req, suffix, n_fork
        self.seqs = []          # dicts: tokens (list), table (np.uint32), len (int)

    # -- token / row generation ------------------------------------------------
    def rows(self, n):
        """n new K and V rows [n][Hkv][D] (bf16 bits)."""
        k = oracle.f32_to_bf16_bits(self.rng.standard_normal((n, self.Hkv, self.D), dtype=np.float32))
        v = oracle.f32_to_bf16_bits(self.rng.standard_normal((n, self.Hkv, self.D), dtype=np.float32))
        return k, v

    @staticmethod
    def slots(table, start, n):
        pos = np.arange(start, start + n)
        return (table[pos // 16].astype(np.int64) * 16 + pos % 16).astype(np.int64)

    # -- phases (dev is a DeviceSide below) ---------------------------------------
    def build(self, dev):
        """Prefix + n_req requests + n_fork forks (copy-on-write on the partial page)."""
        prefix = self.rng.integers(1000, 30000, PREFIX_TOKENS).tolist()
        ptable = np.array(self.bm.alloc_seq(PREFIX_TOKENS // 16), dtype=np.uint32)
        for layer in range(self.L):
            k, v = self.rows(PREFIX_TOKENS)
            dev.append(self, layer, k, v, self.slots(ptable, 0, PREFIX_TOKENS))
        self.rx.insert(prefix, ptable.tolist())
        for b in ptable:                        # the tree's reference
            self.bm.incref(int(b))
        self.bm.free_seq(ptable)                # the builder's own reference
        first_tokens = self.rng.permutation(np.arange(40000, 40000 + self.n_req))
        for i in range(self.n_req):
            n_sfx = int(self.rng.integers(self.suffix[0], self.suffix[1] + 1))
            sfx = [int(first_tokens[i])] + self.rng.integers(1000, 30000, n_sfx - 1).tolist()
            tokens = prefix + sfx
            matched, reuse = self.rx.lookup(tokens)
            assert matched == PREFIX_TOKENS and len(reuse) == PREFIX_TOKENS // 16
            for b in reuse:
                self.bm.incref(b)
            own = self.bm.alloc_seq(-(-n_sfx // 16))
            table = np.array(reuse + own, dtype=np.uint32)
            for layer in range(self.L):
                k, v = self.rows(n_sfx)
                dev.append(self, layer, k, v, self.slots(table, PREFIX_TOKENS, n_sfx))
            self.seqs.append({"tokens": tokens, "table": table, "len": len(tokens)})
        # forks of sequences whose last page is partial: they share every page,
        # and the first token each side writes into that page needs a private copy
        parents = [s for s in self.seqs if s["len"] % 16][: self.n_fork]
        pairs = []
        for par in parents:
            child = {"tokens": list(par["tokens"]), "table": par["table"].copy(), "len": par["len"]}
            for b in child["table"]:
                self.bm.incref(int(b))
            pair = self.bm.cow(child["table"], child["len"] // 16)
            assert pair is not None
            pairs.append(pair)
            self.seqs.append(child)
        dev.block_copy(self, np.array(pairs, dtype=np.uint32).reshape(-1, 2))
        return pairs

    def decode_step(self, dev, live):
        """One token per live sequence on every layer: fused append + decode.
        Returns per-layer outputs (device) and the oracle's."""
        outs, refs = [], []
        B = len(live)
        stride = max(-(-(s["len"] + 1) // 16) for s in live)
        bt = np.zeros((B, stride), dtype=np.uint32)
        for i, s in enumerate(live):
            need = -(-(s["len"] + 1) // 16)
            if need > len(s["table"]):                        # the new token opens a page
                s["table"] = np.concatenate([s["table"], np.array(self.bm.alloc_seq(1), dtype=np.uint32)])
            bt[i, :len(s["table"])] = s["table"]
        seq_lens = np.array([s["len"] + 1 for s in live], dtype=np.uint32)
        new_slots = np.array([int(bt[i, (s["len"]) // 16]) * 16 + s["len"] % 16
                              for i, s in enumerate(live)], dtype=np.int64)
        for layer in range(self.L):
            q = oracle.f32_to_bf16_bits(self.rng.standard_normal((B, self.Hq, self.D), dtype=np.float32))
            k, v = self.rows(B)
            outs.append(dev.decode(self, layer, q, k, v, bt, seq_lens))
            oracle.kv_append(self.geom, self.mirror, None, layer, k, v, new_slots)
            refs.append(oracle.paged_decode_f64(self.geom, self.mirror, None, layer, q, self.Hq, bt,
                                                seq_lens, 1.0 / np.sqrt(self.D)))
        for s in live:
            s["len"] += 1
            s["tokens"].append(int(self.rng.integers(1000, 30000)))
        return outs, refs

    def finish_and_evict(self, dev, n_finish, evict_frac=0.25):
        """Finish n_finish requests into the tree, evict evict_frac of the tree's
        unreferenced blocks (LRU), then compact the pool."""
        done, live = self.seqs[:n_finish], self.seqs[n_finish:]
        for s in done:
            before = self.rx.total_blocks()
            freed = self.rx.insert(s["tokens"][: s["len"]], s["table"].tolist())
            taken = s["table"][PREFIX_TOKENS // 16:]
            assert self.rx.total_blocks() - before + len(freed) == len(taken)
            for b in taken:                    # the tree keeps the suffix pages
                self.bm.incref(int(b))
            for b in freed:
                self.bm.decref(b)
            self.bm.free_seq(s["table"])       # the request's references
        # unreferenced = pages the tree keeps that no live table lists
        live_ids = {int(b) for s in live for b in s["table"]}
        tree_only = [int(b) for s in done for b in s["table"][PREFIX_TOKENS // 16:]
                     if int(b) not in live_ids]
        assert all(self.bm.ref_count(b) == 1 for b in tree_only)
        target = max(1, int(len(tree_only) * evict_frac))
        evicted = self.rx.evict_lru(target)
        for b in evicted:
            self.bm.decref(b)
        pairs = self.bm.compact()
        dev.block_copy(self, pairs)
        m = dict(zip(pairs[:, 0].tolist(), pairs[:, 1].tolist()))
        for s in live:
            s["table"] = np.array([m.get(int(b), int(b)) for b in s["table"]], dtype=np.uint32)
        self.rx.remap(pairs)
        self.seqs = live
        return evicted, pairs


class DeviceSide:
    """The device pool behind a Workload: every operation also updates the mirror."""

    def __init__(self, wl, torch, device=0):
        from voidweb_b200.kv import KvPool, PoolSpec
        self.torch = torch
        self.dev = torch.device("cuda", device)
        self.pool = KvPool(PoolSpec(wl.L, wl.Hkv, wl.D, wl.NB, "bf16", "bf16", max_batch=256),
                           device=device)
        self.pool.pages_u8().zero_()
        torch.cuda.synchronize()

    def _t(self, a, dtype):
        return self.torch.from_numpy(np.ascontiguousarray(a).view(dtype)).to(self.dev)

    def append(self, wl, layer, k, v, slots):
        t = self.torch
        self.pool.append(layer, self._t(k, np.int16), self._t(v, np.int16),
                         t.from_numpy(np.ascontiguousarray(slots)).to(self.dev))
        oracle.kv_append(wl.geom, wl.mirror, None, layer, k, v, slots)

    def block_copy(self, wl, pairs):
        if len(pairs) == 0:
            return
        pairs = np.ascontiguousarray(pairs, dtype=np.uint32).reshape(-1, 2)
        self.pool.block_copy(self._t(pairs.astype(np.int32), np.int32))
        oracle.block_copy(wl.geom, wl.mirror, None, pairs)

    def decode(self, wl, layer, q, k, v, bt, seq_lens):
        qd = self._t(q, np.int16)
        out = self.torch.zeros_like(qd)
        self.pool.paged_decode(layer, qd, self._t(bt.astype(np.int32), np.int32),
                               self._t(seq_lens.astype(np.int32), np.int32), out,
                               k_new=self._t(k, np.int16), v_new=self._t(v, np.int16))
        self.torch.cuda.synchronize()
        return out.cpu().numpy().view(np.uint16)

    def pages(self, wl):
        raw = self.pool.pages_u8().cpu().numpy()
        return raw.view(np.uint16).reshape(oracle.pool_shape(wl.geom))
