"""Generate the golden fixtures under tests/golden/.

The reference (VOIDWEB) is written in the BlackMagic language, which cannot be
compiled here, and it ships no tests or golden vectors.  This script is a
second restatement of the reference functions, written in plain Python
independently of the C++ oracle (oracle/vw_oracle.cpp), so that the two can be
checked against each other.  Each function cites the reference file:line it
transliterates.  Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def bits_f32(u: int) -> float:
    return struct.unpack("<f", struct.pack("<I", u & 0xFFFFFFFF))[0]


def f32(x: float) -> float:
    """Round a Python float to binary32."""
    return struct.unpack("<f", struct.pack("<f", x))[0]


# kernels/norm/rms_norm.bm:98-113
def fp8_encode_ref(x: float) -> int:
    clamped = min(max(f32(x), -448.0), 448.0)
    bits = f32_bits(clamped)
    sign = bits >> 31
    exp = ((bits >> 23) & 0xFF) - 127 + 7
    mant = (bits >> 20) & 0x7
    if exp <= 0:
        return 0
    if exp >= 15:
        return (sign << 7) | (0xF << 3) | 0x7
    return (sign << 7) | (exp << 3) | mant


# kernels/gemm/gemm_fp8.bm:110-116
def fp8_decode_ref(x: int) -> float:
    if x == 0:
        return 0.0
    sign = -1.0 if (x >> 7) != 0 else 1.0
    exp = ((x >> 3) & 0xF) - 7
    mant = 1.0 + (x & 0x7) / 8.0
    return f32(sign * mant * (2.0 ** exp))


# utils/simd.bm:153-158
def f32_to_bf16(x: float) -> int:
    bits = f32_bits(x)
    rnd = (bits >> 16) & 1
    return ((bits + 0x7FFF + rnd) >> 16) & 0xFFFF


# engine/kv_cache.bm:157-164
def rolling_hash(prev: int, tokens) -> int:
    P = 0x9E3779B97F4A7C15
    M = (1 << 64) - 1
    h = (prev + len(tokens) * P) & M
    for t in tokens:
        h = (h * P + t) & M
    return h


def quant_row(x, mode_ref=True):
    """amax / 448 as one binary32 division; amax == 0 -> 1; code = enc(x/scale)."""
    amax = 0.0
    for v in x:
        amax = max(amax, abs(v))
    scale = 1.0 if amax == 0.0 else f32(amax / 448.0)
    return [fp8_encode_ref(f32(v / scale)) for v in x], scale


# kernels/attention/flash_attention.bm:113-162 for one query head in binary32,
# token by token (the k/v rows are given already gathered in page order).
def decode_one_head_f32(q, ks, vs, scale):
    D = len(q)
    acc = [0.0] * D
    m = -math.inf
    l = 0.0
    for k, v in zip(ks, vs):
        dot = 0.0
        for dd in range(D):
            dot = f32(dot + f32(q[dd] * k[dd]))
        s = f32(dot * scale)
        m_new = max(m, s)
        exp_s = f32(math.exp(f32(s - m_new)))
        alpha = f32(math.exp(f32(m - m_new))) if m != -math.inf else 0.0
        acc = [f32(f32(alpha * acc[d]) + f32(exp_s * v[d])) for d in range(D)]
        l = f32(f32(alpha * l) + exp_s)
        m = m_new
    return [f32(a / l) for a in acc]


# engine/kv_cache.bm:29-151
class PyBlockManager:
    def __init__(self, block_size, max_blocks):
        self.block_size = block_size
        self.free_blocks = list(range(max_blocks))
        self.used = {}
        self.prefix = {}

    def alloc(self):
        if not self.free_blocks:
            return None
        i = self.free_blocks.pop()
        self.used[i] = {"ref": 1, "hash": 0}
        return i

    def alloc_seq(self, n):
        if len(self.free_blocks) < n:
            return "OOM"
        return [self.alloc() for _ in range(n)]

    def incref(self, i):
        if i in self.used:
            self.used[i]["ref"] += 1

    def decref(self, i):
        if i in self.used:
            self.used[i]["ref"] = max(0, self.used[i]["ref"] - 1)
            if self.used[i]["ref"] == 0:
                del self.used[i]
                self.free_blocks.append(i)

    def free_seq(self, t):
        for i in t:
            self.decref(i)

    def prefix_lookup(self, toks):
        out, h = [], 0
        for off in range(0, len(toks), self.block_size):
            h = rolling_hash(h, toks[off:off + self.block_size])
            if h not in self.prefix:
                break
            out.extend(self.prefix[h])
        return out

    def register_prefix_block(self, i, h):
        if i in self.used:
            self.used[i]["hash"] = h
        self.prefix.setdefault(h, []).append(i)
        self.incref(i)


# radix_cache/radix_cache.bm:27-285 with this build's documented fixes
# (logical clock, edge-walk eviction that removes the emptied leaf,
# lock/unlock of matched paths).
class Node:
    def __init__(self, edge, blocks, clock):
        self.edge, self.blocks, self.children = list(edge), list(blocks), {}
        self.last = clock
        self.ref = 0


class PyRadix:
    def __init__(self, bs, max_blocks):
        self.bs, self.max_blocks, self.clock = bs, max_blocks, 0
        self.root = Node([], [], self._tick())

    def _tick(self):
        self.clock += 1
        return self.clock

    def touch(self, n):
        n.last = self._tick()

    def lookup(self, toks):
        node, pos, matched, out = self.root, 0, 0, []
        while True:
            self.touch(node)
            if pos >= len(toks):
                break
            c = node.children.get(toks[pos])
            if c is None:
                break
            ml = 0
            while ml < len(c.edge) and pos + ml < len(toks) and c.edge[ml] == toks[pos + ml]:
                ml += 1
            if ml == 0:
                break
            matched += ml
            out.extend(c.blocks)
            self.touch(c)
            if ml < len(c.edge):
                break
            pos += ml
            node = c
        return matched, out

    def total(self, n=None):
        n = n or self.root
        return len(n.blocks) + sum(self.total(c) for c in n.children.values())

    def insert(self, toks, blocks):
        node, pos, blk, bs = self.root, 0, 0, self.bs
        while pos < len(toks) and blk < len(blocks):
            first = toks[pos]
            c = node.children.get(first)
            if c is not None:
                edge = list(c.edge)
                ml = 0
                while ml < len(edge) and pos + ml < len(toks) and edge[ml] == toks[pos + ml]:
                    ml += 1
                if ml == len(edge):
                    self.touch(c)
                    pos += ml
                    blk += (ml + bs - 1) // bs
                    node = c
                    continue
                suf = Node(edge[ml:], c.blocks, c.last)
                suf.children, suf.ref = c.children, c.ref
                take = (ml + bs - 1) // bs
                c.edge, c.blocks = edge[:ml], blocks[blk:blk + take]
                c.children = {suf.edge[0]: suf}
                self.touch(c)
                pos += ml
                blk += take
                node = c
                continue
            chunk = min(bs, len(toks) - pos)
            leaf = Node(toks[pos:pos + chunk], blocks[blk:blk + 1], self._tick())
            node.children[first] = leaf
            pos += chunk
            blk += 1
            node = leaf
        freed = []
        if self.total() > self.max_blocks:
            self._evict_one(freed)
        return freed

    def _find(self, node, path, best):
        if not node.children and node.blocks and node.ref == 0:
            if node.last < best[0]:
                best[0], best[1] = node.last, list(path)
            return
        for k in sorted(node.children):
            c = node.children[k]
            self._find(c, path + c.edge, best)

    def _evict_one(self, freed):
        best = [float("inf"), []]
        self._find(self.root, [], best)
        if not best[1]:
            return 0
        parent, node, pos = None, self.root, 0
        path = best[1]
        while pos < len(path):
            parent, node = node, node.children[path[pos]]
            pos += len(node.edge)
        n = len(node.blocks)
        freed.extend(node.blocks)
        node.blocks = []
        if parent is not None and not node.children:
            del parent.children[node.edge[0]]
        return n

    def evict_lru(self, target):
        freed, total = [], 0
        while total < target:
            e = self._evict_one(freed)
            if e == 0:
                break
            total += e
        return freed

    def _lock(self, toks, delta):
        node, pos = self.root, 0
        while pos < len(toks):
            c = node.children.get(toks[pos])
            if c is None:
                break
            ml = 0
            while ml < len(c.edge) and pos + ml < len(toks) and c.edge[ml] == toks[pos + ml]:
                ml += 1
            if ml == 0:
                break
            c.ref = c.ref + 1 if delta > 0 else max(0, c.ref - 1)
            if ml < len(c.edge):
                break
            pos += ml
            node = c

    def lock(self, t):
        self._lock(t, 1)

    def unlock(self, t):
        self._lock(t, -1)


def main():
    rng = np.random.Generator(np.random.PCG64(1234))
    gold = {}

    # FP8: every code through the decoder; encoder at boundaries and randoms.
    gold["fp8_decode_all"] = [f32_bits(fp8_decode_ref(c)) for c in range(256)]
    probes = [0.0, -0.0, 1.0, -1.0, 448.0, -448.0, 449.0, 1e9, -1e9, 256.0, 255.9, 240.0,
              2.0 ** -6, 2.0 ** -7, 2.0 ** -6 * 1.9, -(2.0 ** -6), 0.015625, 0.0146, 3.14159,
              -2.71828, 1.0625, 1.125, 1.1875, 17.5, 100.0, 447.9, 0.5, 0.75, 1e-30]
    probes += [float(v) for v in rng.normal(0, 50, 200)]
    probes += [float(v) for v in rng.normal(0, 0.02, 50)]
    probes = [f32(v) for v in probes]
    gold["fp8_encode_in"] = [f32_bits(v) for v in probes]
    gold["fp8_encode_out"] = [fp8_encode_ref(v) for v in probes]

    # bf16 RNE
    vals = [f32(v) for v in rng.normal(0, 3, 300)] + [1.0, 1.00390625, 1.005859375, 65504.0]
    gold["bf16_in"] = [f32_bits(v) for v in vals]
    gold["bf16_out"] = [f32_to_bf16(v) for v in vals]

    # per-row quantisation (N(0,1)*3 with outliers, as the FP8 workload)
    rows = []
    for _ in range(8):
        x = rng.normal(0, 3, 128)
        x[rng.random(128) < 0.02] *= 20
        xb = [bits_f32(f32_to_bf16(f32(v)) << 16) for v in x]
        codes, scale = quant_row(xb)
        rows.append({"x_bits": [f32_bits(v) for v in xb], "codes": codes,
                     "scale_bits": f32_bits(scale)})
    rows.append({"x_bits": [0] * 128, "codes": [0] * 128, "scale_bits": f32_bits(1.0)})
    gold["fp8_quant_rows"] = rows

    # rolling hash
    hashes = []
    for n in (0, 1, 5, 16, 17, 64):
        toks = [int(t) for t in rng.integers(0, 152064, n)]
        prev = int(rng.integers(0, 2 ** 63))
        hashes.append({"prev": str(prev), "tokens": toks, "hash": str(rolling_hash(prev, toks))})
    gold["rolling_hash"] = hashes

    # one small paged decode: 1 layer, Hkv 1, Hq 2, D 8, 3 blocks, seq_len 21
    D, NB, seq_len = 8, 4, 21
    kv = rng.normal(0, 1, (NB, 2, 16, D)).astype(np.float32)
    kvb = np.array([[[[f32_to_bf16(float(v)) for v in row] for row in page] for page in kvp]
                    for kvp in kv], dtype=np.uint16)
    q = rng.normal(0, 1, (2, D)).astype(np.float32)
    qb = np.array([[f32_to_bf16(float(v)) for v in row] for row in q], dtype=np.uint16)
    table = [3, 0, 2]
    scale = f32(1.0 / math.sqrt(D))
    outs = []
    for hq in range(2):
        qf = [bits_f32(int(v) << 16) for v in qb[hq]]
        ks, vs = [], []
        for p in range(seq_len):
            blk = table[p // 16]
            ks.append([bits_f32(int(v) << 16) for v in kvb[blk, 0, p % 16]])
            vs.append([bits_f32(int(v) << 16) for v in kvb[blk, 1, p % 16]])
        outs.append([f32_bits(v) for v in decode_one_head_f32(qf, ks, vs, scale)])
    gold["decode_small"] = {"D": D, "NB": NB, "seq_len": seq_len, "table": table,
                            "kv_bf16": kvb.ravel().tolist(), "q_bf16": qb.ravel().tolist(),
                            "out_f32_bits": outs}

    # BlockManager trace
    bm = PyBlockManager(16, 12)
    trace = []

    def rec(op, *a):
        fn = getattr(bm, op)
        r = fn(*a)
        trace.append({"op": op, "args": list(a), "ret": r,
                      "free": list(bm.free_blocks),
                      "refs": {str(k): v["ref"] for k, v in sorted(bm.used.items())}})

    rec("alloc")
    rec("alloc_seq", 3)
    rec("incref", 10)
    rec("decref", 10)
    rec("decref", 10)
    rec("decref", 99)
    rec("alloc")
    toks = [int(t) for t in rng.integers(0, 1000, 40)]
    h1 = rolling_hash(0, toks[:16])
    h2 = rolling_hash(h1, toks[16:32])
    rec("register_prefix_block", 8, h1)
    rec("register_prefix_block", 7, h2)
    rec("register_prefix_block", 8, h1)
    rec("prefix_lookup", toks)
    rec("prefix_lookup", toks[:20])
    rec("free_seq", [8, 7, 9])
    rec("alloc_seq", 20)
    rec("alloc_seq", 5)
    gold["block_manager_trace"] = trace

    # Radix trace (fixed semantics)
    rx = PyRadix(16, 20)
    rtrace = []
    prefix = [int(t) for t in rng.integers(0, 500, 32)]
    seqs = []
    for i in range(5):
        suf = [int(t) for t in rng.integers(0, 500, int(rng.integers(3, 40)))]
        seqs.append(prefix + suf)
    next_block = [0]

    def blocks_for(n):
        out = list(range(next_block[0], next_block[0] + (n + 15) // 16))
        next_block[0] += len(out)
        return out

    for s in seqs:
        rtrace.append({"op": "lookup", "tokens": s, "ret": list(rx.lookup(s))})
        b = blocks_for(len(s))
        rtrace.append({"op": "insert", "tokens": s, "blocks": b, "ret": rx.insert(s, b),
                       "total": rx.total()})
    rx.lock(seqs[1])
    rtrace.append({"op": "lock", "tokens": seqs[1]})
    rtrace.append({"op": "evict_lru", "target": 3, "ret": rx.evict_lru(3), "total": rx.total()})
    rx.unlock(seqs[1])
    rtrace.append({"op": "unlock", "tokens": seqs[1]})
    rtrace.append({"op": "lookup", "tokens": seqs[0], "ret": list(rx.lookup(seqs[0]))})
    rtrace.append({"op": "evict_lru", "target": 100, "ret": rx.evict_lru(100),
                   "total": rx.total()})
    gold["radix_trace"] = rtrace

    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(gold, f, separators=(",", ":"))
    print("wrote", os.path.join(HERE, "golden.json"))


if __name__ == "__main__":
    main()
