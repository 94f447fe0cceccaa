"""The benchmark configurations of the paged-KV path, built at their stated
sizes and seeds for the parity tests (one layer of each model, the whole
batch).

    C1  plumbing: 1 layer, 14 query / 2 KV heads, head_dim 64, f16 pages,
        a pool of 512 blocks, 8 sequences, context U[1, 512], seed 0
    C2  Qwen2.5-7B: 28 / 4 heads, head_dim 128, bf16, 16 sequences,
        context U[512, 4096], seed 1
    C4  Llama-3-8B FP8: 32 / 8 heads, head_dim 128, E4M3 pages with one f32
        scale per token per head, 64 sequences, context log-U[1k, 32k],
        K/V N(0,1) x 3 with 0.1 % of the elements x 20, seed 3
    C5  Llama-3-70B, one GPU's shard: one KV head of the 64 / 8 model with its
        8 query heads, bf16, 256 sequences, context U[2k, 8k], seed 4

Draw order from numpy Generator(PCG64(seed)): the B context lengths
(integers uniform inclusive, or exp(U[ln lo, ln hi]) rounded); a permutation
of the pool's block ids dealt to the sequences in order (C1: the 512-block
pool; the others: the pages the batch needs plus 16 spare blocks); q
[B][Hq][D]; the step's new K rows and new V rows [B][Hkv][D].  The cached K/V
rows come from child generators PCG64(SeedSequence(seed, spawn_key=...)) so
that they can be drawn in parallel: 16-bit pools N(0,1) over the whole pool,
chunk i of 2^20 elements from spawn_key (1, i); FP8 pools per sequence b
(spawn_key (2, b)), its K rows then its V rows for positions 0 .. ctx-1, each
row quantised by the codec on the way in.  Values are drawn in f32 and rounded
to the io dtype (f16, or bf16 round-to-nearest-even).  The step appends one
token per sequence at position ctx and decodes over ctx + 1 tokens.
"""
from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

import oracle
from tests.kvgen import BF16, F16, FP8, Case, io_bits

CONFIGS = {
    "C1": dict(seed=0, Hq=14, Hkv=2, D=64, B=8, ctx=("uniform", 1, 512), kv=F16, io=F16, pool=512),
    "C2": dict(seed=1, Hq=28, Hkv=4, D=128, B=16, ctx=("uniform", 512, 4096), kv=BF16, io=BF16),
    "C4": dict(seed=3, Hq=32, Hkv=8, D=128, B=64, ctx=("loguniform", 1024, 32768), kv=FP8, io=BF16,
               kv_scale=3.0, outliers=True),
    "C5": dict(seed=4, Hq=8, Hkv=1, D=128, B=256, ctx=("uniform", 2048, 8192), kv=BF16, io=BF16),
}

_CHUNK = 1 << 20


def draw_ctx(rng, rule, B):
    kind, lo, hi = rule
    if kind == "uniform":
        return rng.integers(lo, hi + 1, B).astype(np.int64)
    return np.rint(np.exp(rng.uniform(math.log(lo), math.log(hi), B))).astype(np.int64)


def build(name: str) -> Case:
    cfg = CONFIGS[name]
    rng = np.random.Generator(np.random.PCG64(cfg["seed"]))
    c = Case()
    c.name = name
    c.L, c.Hq, c.Hkv, c.D, c.B = 1, cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["B"]
    c.kv, c.io, c.fp8_mode = cfg["kv"], cfg["io"], 0
    ctx = draw_ctx(rng, cfg["ctx"], c.B)
    c.ctx = ctx
    c.seq_lens = (ctx + 1).astype(np.uint32)
    pages = (ctx + 1 + 15) // 16
    c.NB = cfg.get("pool") or int(pages.sum()) + 16
    assert pages.sum() <= c.NB
    c.stride = int(pages.max())
    perm = rng.permutation(c.NB).astype(np.uint32)
    c.block_tables = np.zeros((c.B, c.stride), dtype=np.uint32)
    off = 0
    for b in range(c.B):
        c.block_tables[b, :pages[b]] = perm[off:off + pages[b]]
        off += int(pages[b])
    c.geom = oracle.geom(1, c.Hkv, c.D, c.NB, c.kv, c.io, 0)
    shape = oracle.pool_shape(c.geom)
    kv_scale = cfg.get("kv_scale", 1.0)
    outl = cfg.get("outliers", False)
    c.q = io_bits(rng, (c.B, c.Hq, c.D), c.io)[None]
    c.k_new = io_bits(rng, (c.B, c.Hkv, c.D), c.io, kv_scale, outl)[None]
    c.v_new = io_bits(rng, (c.B, c.Hkv, c.D), c.io, kv_scale, outl)[None]

    def child(*key):
        return np.random.Generator(np.random.PCG64(np.random.SeedSequence(cfg["seed"], spawn_key=key)))

    if c.kv == FP8:
        c.data = np.zeros(shape, dtype=np.uint8)
        c.scales = np.zeros(shape[:-1], dtype=np.float32)

        def fill(b):       # sequence b's slots only: the sequences run in parallel
            g = child(2, b)
            n = int(ctx[b])
            pos = np.arange(n)
            slots = c.block_tables[b, pos // 16].astype(np.int64) * 16 + pos % 16
            k = io_bits(g, (n, c.Hkv, c.D), c.io, kv_scale, outl)
            v = io_bits(g, (n, c.Hkv, c.D), c.io, kv_scale, outl)
            oracle.kv_append(c.geom, c.data, c.scales, 0, k, v, slots)
        jobs = range(c.B)
    else:
        flat = np.empty(int(np.prod(shape)), dtype=np.uint16)
        c.data = flat.reshape(shape)
        c.scales = None

        def fill(i):
            o = i * _CHUNK
            n = min(_CHUNK, flat.size - o)
            flat[o:o + n] = io_bits(child(1, i), (n,), c.io)
        jobs = range((flat.size + _CHUNK - 1) // _CHUNK)
    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, jobs))
    return c


def algorithmic_bytes(c: Case) -> int:
    """Bytes one layer's append + decode moves (pages read once per KV head)."""
    e = 1 if c.kv == FP8 else 2
    s = 4 if c.kv == FP8 else 0
    sl = c.seq_lens.astype(np.int64)
    per = (sl * 2 * c.Hkv * (c.D * e + s) + 2 * c.Hkv * (c.D * e + s) + 2 * c.Hkv * c.D * 2 +
           2 * c.Hq * c.D * 2 + ((sl + 15) // 16) * 4 * c.Hkv)
    return int(per.sum())
