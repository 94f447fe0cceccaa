"""Seeded synthetic paged-KV cases for the parity tests.

Inputs follow the workload definitions: Q/K/V drawn N(0,1) in f32 and rounded
to the io dtype (f16 or bf16 round-to-nearest-even), FP8 cases N(0,1)*3 with
0.1% outliers *20; block tables deal a random permutation of the pool's block
ids to the sequences.  Slots past each sequence's length hold garbage (NaN
patterns for 16-bit pools) so masking is exercised.
"""
from __future__ import annotations

import numpy as np

import oracle

F16, BF16, FP8 = oracle.F16, oracle.BF16, oracle.FP8


def io_bits(rng, shape, io, scale=1.0, outliers=False):
    x = rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
    if outliers:
        m = rng.random(shape) < 0.001
        x[m] *= np.float32(20.0)
    return oracle.f32_to_io_bits(x, io)


class Case:
    pass


def make_case(seed, L, Hkv, D, Hq, B, ctx_lo, ctx_hi, kv=BF16, io=BF16, fp8_mode=0,
              extra_blocks=4, ctx=None, stride_extra=1):
    rng = np.random.Generator(np.random.PCG64(seed))
    c = Case()
    c.L, c.Hkv, c.D, c.Hq, c.B, c.kv, c.io, c.fp8_mode = L, Hkv, D, Hq, B, kv, io, fp8_mode
    if ctx is None:
        ctx = rng.integers(ctx_lo, ctx_hi + 1, B)
    c.seq_lens = np.asarray(ctx, dtype=np.uint32)
    pages = (c.seq_lens.astype(np.int64) + 15) // 16
    c.stride = int(pages.max()) + stride_extra
    c.NB = int(pages.sum()) + extra_blocks
    perm = rng.permutation(c.NB).astype(np.uint32)
    c.block_tables = np.zeros((B, c.stride), dtype=np.uint32)
    off = 0
    for b in range(B):
        n = int(pages[b])
        c.block_tables[b, :n] = perm[off:off + n]
        off += n
    c.geom = oracle.geom(L, Hkv, D, c.NB, kv, io, fp8_mode)
    shape = oracle.pool_shape(c.geom)
    if kv == FP8:
        c.data = rng.integers(0, 256, shape, dtype=np.uint8)
        c.scales = np.full(shape[:-1], np.nan, dtype=np.float32)
        # every valid token of every layer is written through the oracle append
        for layer in range(L):
            slots = []
            for b in range(B):
                for p in range(int(c.seq_lens[b])):
                    slots.append(int(c.block_tables[b, p // 16]) * 16 + p % 16)
            n = len(slots)
            k = io_bits(rng, (n, Hkv, D), io, 3.0, True)
            v = io_bits(rng, (n, Hkv, D), io, 3.0, True)
            oracle.kv_append(c.geom, c.data, c.scales, layer, k, v, np.array(slots))
    else:
        c.data = io_bits(rng, shape, io)
        c.scales = None
        # garbage (quiet NaN) in the slots past each sequence's end
        for b in range(B):
            n = int(c.seq_lens[b])
            if n % 16:
                blk = int(c.block_tables[b, n // 16])
                c.data[:, blk, :, :, n % 16:, :] = 0x7FC0 if io == BF16 else 0x7E00
    c.q = np.stack([io_bits(rng, (B, Hq, D), io) for _ in range(L)])
    sc = 3.0 if kv == FP8 else 1.0
    c.k_new = np.stack([io_bits(rng, (B, Hkv, D), io, sc, kv == FP8) for _ in range(L)])
    c.v_new = np.stack([io_bits(rng, (B, Hkv, D), io, sc, kv == FP8) for _ in range(L)])
    return c


def new_token_slots(c):
    """Slot of position seq_len-1 of every sequence."""
    pos = c.seq_lens.astype(np.int64) - 1
    return np.array([int(c.block_tables[b, pos[b] // 16]) * 16 + int(pos[b] % 16)
                     for b in range(c.B)], dtype=np.int64)


def pool_spec_kwargs(c):
    names = {F16: "f16", BF16: "bf16", FP8: "fp8"}
    return dict(num_layers=c.L, num_kv_heads=c.Hkv, head_dim=c.D, num_blocks=c.NB,
                kv_dtype=names[c.kv], io_dtype=names[c.io],
                fp8_mode="ocp" if c.fp8_mode else "reference", max_batch=max(c.B, 1))
