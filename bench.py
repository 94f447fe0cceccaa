#!/usr/bin/env python
"""Paged-KV decode benchmark: KV GB/s (fraction of HBM peak) and tok/s.

One step = append one token per sequence + paged decode attention over every
layer (the fused vw_paged_decode launch, one per layer), on the
Qwen2.5-7B-shaped batch by default: 28 layers, 28 query / 4 KV heads,
head_dim 128, bf16 KV, 16 sequences with context lengths uniform in
[512, 4096] (seed 1), random non-contiguous block tables, 16-token pages.
Synthetic inputs (no dataset); K/V/Q drawn N(0,1).

N GPUs (torchrun, one process per GPU): every rank holds its own 16 sequences
with the 1-GPU run's length draw (weak scaling; with --scaling strong the one
16-sequence batch of the 1-GPU run is split across the GPUs; with --placement
kv_heads every rank holds the same sequences and its own KV heads, the
Llama-3-70B placement), and the per-shard attention outputs of each step are
all-gathered over NCCL.

--impl reference times the reference's CPU implementation of this path (the
oracle's restatement of paged_attention_decode + append, f32, all host
threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: layers, q heads, kv heads, head_dim, seqs per GPU, ctx rule, kv / io dtype, seed
    "qwen2.5-7b-decode-b16": dict(L=28, Hq=28, Hkv=4, D=128, B=16, ctx=("uniform", 512, 4096),
                                  kv="bf16", io="bf16", seed=1),
    # the Qwen batch's pages with 16 query heads per KV head (the two-tile
    # decode variant): same KV bytes, twice the query heads per page
    "g16-bf16-b16": dict(L=28, Hq=64, Hkv=4, D=128, B=16, ctx=("uniform", 512, 4096),
                         kv="bf16", io="bf16", seed=1),
    "plumbing-l1-b8": dict(L=1, Hq=14, Hkv=2, D=64, B=8, ctx=("uniform", 1, 512),
                           kv="f16", io="f16", seed=0),
    "llama3-8b-fp8-b64": dict(L=32, Hq=32, Hkv=8, D=128, B=64, ctx=("loguniform", 1024, 32768),
                              kv="fp8", io="bf16", seed=3),
    # the FP8 batch with bf16 pages: the same page walk with 8 KB page-heads
    "llama3-8b-bf16-b64": dict(L=32, Hq=32, Hkv=8, D=128, B=64, ctx=("loguniform", 1024, 32768),
                               kv="bf16", io="bf16", seed=3),
    "llama3-70b-1kvhead-b256": dict(L=80, Hq=8, Hkv=1, D=128, B=256, ctx=("uniform", 2048, 8192),
                                    kv="bf16", io="bf16", seed=4),
    # chunked prefill (vw_paged_prefill): B sequences, each a `chunk`-token chunk
    # (the scheduler's largest, scheduler/scheduler.bm:255) after a cached prefix
    "qwen2.5-7b-prefill-4x2048": dict(kind="prefill", L=28, Hq=28, Hkv=4, D=128, B=4, chunk=2048,
                                      ctx=("uniform", 0, 2048), kv="bf16", io="bf16", seed=11),
    "llama3-8b-fp8-prefill-4x2048": dict(kind="prefill", L=32, Hq=32, Hkv=8, D=128, B=4, chunk=2048,
                                         ctx=("uniform", 0, 2048), kv="fp8", io="bf16", seed=13),
    # the FP8 weight path's GEMM (gemm_fp8.bm:31-107): E4M3 A [M][K] x B [K][N] -> bf16
    "fp8-gemm-8192": dict(kind="gemm", M=8192, N=8192, K=8192, seed=12),
    # shared-prefix radix workload at Qwen2.5-7B KV shapes: 64 requests sharing a
    # 128-token prefix (8 ref-counted pages), suffixes U[32, 1024], 8 forks of
    # requests with a partial last page (copy-on-write), then 32 requests finish
    # into the radix tree, 25 % of its unreferenced blocks are LRU-evicted and the
    # pool is compacted; decode steps before and after
    # the standalone page kernels at Qwen2.5-7B KV shapes: append of a 2048-token
    # chunk's rows into one layer, gather of a 4096-token sequence from one layer,
    # and 64 whole-block copies (all 28 layers each)
    "qwen2.5-7b-kvops": dict(kind="kvops", L=28, Hkv=4, D=128, append_tokens=2048, gather_tokens=4096,
                             copy_pairs=64, kv="bf16", io="bf16", seed=5),
    "qwen2.5-7b-radix-64": dict(kind="radix", L=28, Hq=28, Hkv=4, D=128, n_req=64, prefix=128,
                                suffix=(32, 1024), n_fork=8, finish=32, evict_frac=0.25,
                                kv="bf16", io="bf16", seed=2),
}
DEFAULT = "qwen2.5-7b-decode-b16"
L2_BYTES = 126 * 1024 * 1024


def ctx_lengths(w, rank=0):
    """Context lengths of one GPU's batch before the step's token: rank 0 draws
    them from numpy PCG64(seed) (the workload's seed), other ranks of a
    sequence-sharded run from PCG64(seed * 1000 + rank)."""
    rng = np.random.Generator(np.random.PCG64(w["seed"] if rank == 0 else w["seed"] * 1000 + rank))
    kind, lo, hi = w["ctx"]
    if kind == "uniform":
        return rng.integers(lo, hi + 1, w["B"]).astype(np.int64)
    return np.rint(np.exp(rng.uniform(math.log(lo), math.log(hi), w["B"]))).astype(np.int64)


def verify_layer(pool, w, layer, q, kn, vn, out, bt, seq_lens, threads=0):
    """One layer of the benchmarked step against the oracle, outside the timed
    region: the pages of that layer after the step (appends are idempotent, so
    the oracle's append of the step's rows must leave them unchanged: the
    fused append was bit-exact, codes and scales included) and the step's
    attention outputs against the oracle's fp64 paged decode over those pages
    (|gpu - ref| <= 2e-3 + 1e-2 * |ref|)."""
    import torch
    import oracle
    kvk = {"f16": oracle.F16, "bf16": oracle.BF16, "fp8": oracle.FP8}
    fp8 = w["kv"] == "fp8"
    NB, Hkv, D, Hq = pool.spec.num_blocks, w["Hkv"], w["D"], w["Hq"]
    g = oracle.geom(1, Hkv, D, NB, kvk[w["kv"]], kvk[w["io"]])
    shape = oracle.pool_shape(g)
    n = int(np.prod(shape))
    eb = 1 if fp8 else 2
    raw = pool.pages_u8()[layer * n * eb:(layer + 1) * n * eb].cpu().numpy()
    data = raw.view(np.uint8 if fp8 else np.uint16).reshape(shape)
    scales = None
    if fp8:
        ns = n // D
        scales = pool.scales_f32()[layer * ns:(layer + 1) * ns].cpu().numpy().reshape(shape[:-1])
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    sl = np.asarray(seq_lens, dtype=np.int64)
    btn = np.asarray(bt, dtype=np.uint32)
    slots = np.array([int(btn[b, (sl[b] - 1) // 16]) * 16 + int((sl[b] - 1) % 16) for b in range(len(sl))],
                     dtype=np.int64)
    want = data.copy()
    wscales = scales.copy() if fp8 else None
    oracle.kv_append(g, want, wscales, 0, bits(kn), bits(vn), slots)
    append_ok = bool(np.array_equal(want, data)) and (
        not fp8 or bool(np.array_equal(wscales.view(np.uint32), scales.view(np.uint32))))
    ref = oracle.paged_decode_f64(g, data, scales, 0, bits(q), Hq, btn, sl.astype(np.uint32),
                                  1.0 / math.sqrt(D), nthreads=threads)
    got = oracle.io_bits_to_f32(bits(out), kvk[w["io"]]).astype(np.float64)
    err = np.abs(got - ref)
    ratio = float((err / (2e-3 + 1e-2 * np.abs(ref))).max())
    return {"layer": layer, "append_bit_exact": append_ok, "max_abs_err": float(err.max()),
            "worst_tolerance_ratio": round(ratio, 4), "ok": append_ok and ratio <= 1.0 and
            bool(np.isfinite(got).all())}


def choose_gather(w, world):
    """How a multi-GPU decode run all-gathers each step's outputs.  Measured on
    B200s: an overlapped gather keeps its NCCL CTAs resident while the next
    step runs, and a decode CTA that cannot start beside them holds back its
    layer: cheap while the gather is short (Qwen step, 3.2 MB received per rank
    on 2 GPUs: 8940 GB/s against 8304 serial), costly when it is long (22 MB on
    8 GPUs: 26480 against 30995; Llama-3-70B one KV head, 42 MB on 2 GPUs:
    11308 against 12065, 126 MB on 4: 20948 against 24249).  Serial from 8 MB
    received per rank and step."""
    out_bytes = w["L"] * w["B"] * w["Hq"] * w["D"] * 2 if "B" in w and "Hq" in w else 0
    return "serial" if (world - 1) * out_bytes >= 8 << 20 else "overlap"


def algorithmic_bytes_per_launch(w, seq_lens):
    """Bytes one layer's append + decode must move, counting each page once per
    KV head (a GQA group shares it), as the paging walk of
    kernels/attention/flash_attention.bm:132-140 generalised to KV heads reads them:
    KV read ctx*2*Hkv*(D*e+s), append write 2*Hkv*(D*e+s) + new rows read
    2*Hkv*D*2, q read and o write Hq*D*2 each, block table ceil(ctx/16)*4*Hkv."""
    e = 1 if w["kv"] == "fp8" else 2
    s = 4 if w["kv"] == "fp8" else 0
    H, D, Hq = w["Hkv"], w["D"], w["Hq"]
    ctx = np.asarray(seq_lens, dtype=np.int64)
    per = (ctx * 2 * H * (D * e + s) + 2 * H * (D * e + s) + 2 * H * D * 2 + 2 * Hq * D * 2 +
           ((ctx + 15) // 16) * 4 * H)
    return int(per.sum())


# dram__bytes_read.sum + dram__bytes_write.sum of one decode_kernel launch (one
# layer) of the named decode workloads, from one ncu --set full capture of that
# launch; ncu cannot run inside the timed bench, so the figure is carried here.
NCU_TRAFFIC_PER_LAUNCH = {"qwen2.5-7b-decode-b16": 79_991_808,
                          "llama3-8b-fp8-b64": 1_180_007_936,
                          # one prefill_kernel launch (one layer), read + write
                          "qwen2.5-7b-prefill-4x2048": 111_355_904,
                          "llama3-8b-fp8-prefill-4x2048": 123_923_456}


def tensor_peak():
    """Measured bf16 dense TFLOP/s: (burst, sustained, kind)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 1590.0, 1400.0, "fallback"


def prefill_flops(w, prefix):
    """Attention FLOPs of one layer of the prefill workload: each query token at
    position p attends to p + 1 keys (causal), 2*D FLOPs per key for Q K^T and
    2*D for P V, for every query head."""
    keys = 0
    for cs in prefix:
        keys += int(w["chunk"]) * int(cs) + w["chunk"] * (w["chunk"] + 1) // 2
    return 4 * w["D"] * w["Hq"] * keys


def run_prefill_bench(args, w):
    """Chunked prefill of every layer (append of the chunk rows + causal prefill
    attention over the pool), timed with CUDA events over K steps."""
    import torch
    from voidweb_b200.kv import KvPool, PoolSpec
    import oracle
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        print(json.dumps({"metric": "prefill attention TFLOP/s", "error": "single GPU only"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    L, Hq, Hkv, D, B, n = w["L"], w["Hq"], w["Hkv"], w["D"], w["B"], w["chunk"]
    prefix = ctx_lengths(w, 0)
    pages = (prefix + n + 15) // 16
    NB = int(pages.sum()) + 64
    rng = np.random.Generator(np.random.PCG64(w["seed"] * 7919))
    perm = rng.permutation(NB)
    stride = int(pages.max())
    bt = np.zeros((B, stride), dtype=np.int32)
    off = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[off:off + pages[b]]
        off += pages[b]
    T = B * n
    pool = KvPool(PoolSpec(L, Hkv, D, NB, w["kv"], w["io"], max_batch=B), device=0)
    fp8 = w["kv"] == "fp8"
    if fp8:     # random codes of the cached prefixes, row scales amax / 448 of N(0, 1) rows
        pool.pages_u8().random_(0, 256)
        pool.scales_f32().uniform_(0.005, 0.01)
    else:
        pool.pages_u8().view(torch.bfloat16).normal_()
    q = torch.randn((L, T, Hq, D), device=dev).bfloat16()
    kn = torch.randn((L, T, Hkv, D), device=dev).bfloat16()
    vn = torch.randn((L, T, Hkv, D), device=dev).bfloat16()
    out = torch.empty_like(q)
    cu = torch.arange(0, T + 1, n, dtype=torch.int32, device=dev)
    cs = torch.from_numpy(prefix.astype(np.int32)).to(dev)
    btd = torch.from_numpy(bt).to(dev)

    def step():
        for layer in range(L):
            pool.paged_prefill(layer, q[layer], cu, cs, btd, out[layer], k_new=kn[layer],
                               v_new=vn[layer], causal=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert pool.check() == 0
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    assert pool.check() == 0
    ms = e0.elapsed_time(e1) / args.steps
    flops = prefill_flops(w, prefix) * L
    tflops = flops / (ms * 1e-3) / 1e12
    burst, sustained, kind = tensor_peak()
    # CPU: the oracle's f32 restatement on a bounded sample (one layer, the
    # first 16 query tokens of each chunk), with all host threads
    cpu = None
    if not args.no_cpu_baseline:
        thr = cpu_threads()
        g = oracle.geom(1, Hkv, D, NB, oracle.FP8 if fp8 else oracle.BF16, oracle.BF16)
        rows = NB * Hkv * 2 * 16
        if fp8:
            data = pool.pages_u8()[: rows * D].cpu().numpy()
            scales = pool.scales_f32()[:rows].cpu().numpy().reshape(oracle.pool_shape(g)[:-1])
        else:
            data = pool.pages_u8().view(torch.int16)[: rows * D].cpu().numpy().view(np.uint16)
            scales = None
        data = data.reshape(oracle.pool_shape(g))
        m = 16
        qs = q[0].view(torch.int16).cpu().numpy().view(np.uint16).reshape(B, n, Hq, D)[:, :m].reshape(B * m, Hq, D)
        cus = np.arange(0, B * m + 1, m, dtype=np.int32)
        t0 = time.perf_counter()
        oracle.paged_prefill_f32(g, data, scales, 0, qs, Hq, bt, cus, prefix.astype(np.int32), True,
                                 1.0 / math.sqrt(D), nthreads=thr)
        dt = time.perf_counter() - t0
        sample_flops = sum(4 * D * Hq * (m * int(c0) + m * (m + 1) // 2) for c0 in prefix)
        cpu = {"value": round(sample_flops / dt / 1e12, 6), "unit": "TFLOP/s", "cores": thr,
               "kind": "port",
               "sample": f"1 layer, the first {m} query tokens of each of the {B} chunks"}
    print(json.dumps({
        "metric": "prefill attention TFLOP/s", "value": round(tflops, 2), "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 pages, f16 MMA" if fp8 else "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "layers": L, "q_heads": Hq, "kv_heads": Hkv,
                   "head_dim": D, "seqs": B, "chunk_tokens": n,
                   "cached_prefix": [int(x) for x in prefix], "block_size": 16, "kv_dtype": w["kv"],
                   "causal": True, "parallelism": "single",
                   "l2": f"inputs larger than L2 ({NB * Hkv * 2 * 16 * (D * (1 if fp8 else 2) + (4 if fp8 else 0)) * L / 1e9:.2f} GB of pages)"},
        "tok_per_s": round(T / (ms * 1e-3), 1),
        "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": sustained,
                     "unit": "TFLOP/s", "frac": round(tflops / sustained, 4),
                     "traffic": NCU_TRAFFIC_PER_LAUNCH.get(args.workload),
                     "peak_kind": f"{kind} sustained (burst {burst})",
                     "flops_per_step": flops},
        "cpu_baseline": cpu, "e2e": None, "clocks": clk, "gpu_launches": args.steps * L * 2,
    }))


def run_gemm_bench(args, w):
    """vw_gemm_fp8 on E4M3 codes, timed with CUDA events over K launches."""
    import torch
    from voidweb_b200.kv import fp8_weight_check, gemm_fp8
    import oracle
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        print(json.dumps({"metric": "fp8 gemm TFLOP/s", "error": "single GPU only"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    M, N, K = w["M"], w["N"], w["K"]
    g = torch.Generator(device=dev).manual_seed(w["seed"])
    # codes of N(0,1)-like magnitudes: exponent field 4..9, any sign and mantissa
    def codes(shape):
        e = torch.randint(4, 10, shape, device=dev, generator=g, dtype=torch.int32)
        m = torch.randint(0, 16, shape, device=dev, generator=g, dtype=torch.int32)
        return ((e << 3) | (m & 7) | ((m >> 3) << 7)).to(torch.uint8)
    a, b = codes((M, K)), codes((K, N))
    bias = torch.randn(N, device=dev).bfloat16()
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    for _ in range(args.warmup):
        gemm_fp8(a, b, out, bias, 0.01, 0.01)
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(args.steps):
        gemm_fp8(a, b, out, bias, 0.01, 0.01)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    assert fp8_weight_check() == 0
    ms = e0.elapsed_time(e1) / args.steps
    tflops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    burst, sustained, kind = tensor_peak()
    cpu = None
    if not args.no_cpu_baseline:
        thr = cpu_threads()
        m = 16
        an, bn = a[:m].cpu().numpy(), b.cpu().numpy()
        t0 = time.perf_counter()
        oracle.gemm_fp8_f64(an, bn, None, 0.01, 0.01, nthreads=thr)
        dt = time.perf_counter() - t0
        cpu = {"value": round(2.0 * m * N * K / dt / 1e12, 6), "unit": "TFLOP/s", "cores": thr,
               "kind": "port", "sample": f"{m} rows of A against all of B (fp64 oracle)"}
    print(json.dumps({
        "metric": "fp8 gemm TFLOP/s", "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 in, f16 mma, bf16 out",
        "data": "synthetic",
        "config": {"workload": args.workload, "M": M, "N": N, "K": K, "parallelism": "single",
                   "l2": f"inputs larger than L2 ({(M * K + K * N) / 1e6:.0f} MB of codes)"},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": burst, "unit": "TFLOP/s",
                     "frac": round(tflops / burst, 4), "traffic": None,
                     "peak_kind": f"{kind} bf16 burst (the MMAs run in f16)"},
        "cpu_baseline": cpu, "e2e": None, "clocks": clk, "gpu_launches": args.steps,
    }))


def run_radix_bench(args, w):
    """The shared-prefix workload on one GPU: host decisions from this library's
    block manager and radix tree (engine/kv_cache.bm:94-113 copy-on-write,
    radix_cache/radix_cache.bm:231-285 LRU eviction, then compaction), device
    copies and decodes through the C ABI.  Timed: the copy-on-write block
    copies, the compaction moves (GB/s of bytes read + written), and the decode
    step of every layer before and after the eviction (KV GB/s, logical bytes:
    a shared page counts once per sequence that reads it)."""
    import torch
    from voidweb_b200 import _lib as C
    from voidweb_b200.blocks import BlockManager, RadixCacheManager
    from voidweb_b200.kv import KvPool, PoolSpec
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        print(json.dumps({"metric": "paged decode KV GB/s", "error": "single GPU only"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    L, Hq, Hkv, D = w["L"], w["Hq"], w["Hkv"], w["D"]
    rng = np.random.Generator(np.random.PCG64(w["seed"]))
    P = w["prefix"] // 16
    sfx = rng.integers(w["suffix"][0], w["suffix"][1] + 1, w["n_req"])
    NB = P + int(((sfx + 1 + 15) // 16).sum()) + 4 * w["n_fork"] + 64
    bm = BlockManager(L, Hkv, D, 16, NB)
    rx = RadixCacheManager(16, NB)
    pool = KvPool(PoolSpec(L, Hkv, D, NB, "bf16", "bf16", max_batch=256), device=0)
    pool.pages_u8().view(torch.bfloat16).normal_()
    block_bytes = L * Hkv * 2 * 16 * D * 2
    t_host = {}
    # -- build: the prefix in the tree, requests sharing its pages
    th = time.perf_counter()
    prefix = rng.integers(1000, 30000, w["prefix"]).tolist()
    ptable = bm.alloc_seq(P)
    rx.insert(prefix, ptable)
    for b in ptable:
        bm.incref(b)                       # the tree's reference
    bm.free_seq(ptable)                    # the builder's own
    seqs = []
    first = rng.permutation(np.arange(40000, 40000 + w["n_req"]))
    for i in range(w["n_req"]):
        toks = prefix + [int(first[i])] + rng.integers(1000, 30000, int(sfx[i]) - 1).tolist()
        matched, reuse = rx.lookup(toks)
        assert matched == w["prefix"] and len(reuse) == P
        for b in reuse:
            bm.incref(b)
        table = np.array(reuse + bm.alloc_seq(-(-int(sfx[i]) // 16)), dtype=np.uint32)
        seqs.append({"tokens": toks, "table": table, "len": len(toks)})
    parents = [s for s in seqs if s["len"] % 16][: w["n_fork"]]
    cow = []
    for par in parents:
        child = {"tokens": list(par["tokens"]), "table": par["table"].copy(), "len": par["len"]}
        for b in child["table"]:
            bm.incref(int(b))
        cow.append(bm.cow(child["table"], child["len"] // 16))
        seqs.append(child)
    t_host["build_ms"] = round((time.perf_counter() - th) * 1e3, 3)
    cow = np.array(cow, dtype=np.uint32).reshape(-1, 2)

    def time_copies(pairs, reps):
        pt = torch.from_numpy(pairs.astype(np.int32)).to(dev)
        pool.block_copy(pt)                      # idempotent: the same copy again
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(reps):
            pool.block_copy(pt)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        # the copies must equal their sources on every layer
        pg = pool.pages_u8().view(L, NB, block_bytes // L)
        src = torch.from_numpy(pairs[:, 0].astype(np.int64)).to(dev)
        dst = torch.from_numpy(pairs[:, 1].astype(np.int64)).to(dev)
        assert torch.equal(pg[:, src], pg[:, dst]), "block copy differs from its source"
        return {"pairs": int(len(pairs)), "us": round(us, 3),
                "GB/s": round(2 * len(pairs) * block_bytes / (us * 1e-6) / 1e9, 2)}

    def decode_phase(live):
        B = len(live)
        stride = max(-(-(s["len"] + 1) // 16) for s in live)
        bt = np.zeros((B, stride), dtype=np.int32)
        for i, s in enumerate(live):
            if -(-(s["len"] + 1) // 16) > len(s["table"]):
                s["table"] = np.concatenate([s["table"], np.array(bm.alloc_seq(1), dtype=np.uint32)])
            bt[i, :len(s["table"])] = s["table"]
        seq_lens = np.array([s["len"] + 1 for s in live], dtype=np.int64)
        q = torch.randn((L, B, Hq, D), device=dev).bfloat16()
        kn = torch.randn((L, B, Hkv, D), device=dev).bfloat16()
        vn = torch.randn((L, B, Hkv, D), device=dev).bfloat16()
        out = torch.zeros_like(q)
        btd = torch.from_numpy(bt).to(dev)
        sld = torch.from_numpy(seq_lens.astype(np.int32)).to(dev)
        st = torch.cuda.Stream(device=dev)
        flags = C.VW_DECODE_PDL | C.VW_DECODE_EARLY_PAGES

        def step(sx):
            for l in range(L):
                pool.paged_decode(l, q[l], btd, sld, out[l], k_new=kn[l], v_new=vn[l], stream=sx,
                                  flags=flags if l else 0)
        with torch.cuda.stream(st):
            step(st)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            step(torch.cuda.current_stream())
        for _ in range(max(3, args.warmup)):
            g.replay()
        torch.cuda.synchronize()
        wl = dict(w, B=B)
        chk = verify_layer(pool, wl, L // 2, q[L // 2], kn[L // 2], vn[L // 2], out[L // 2], bt, seq_lens)
        assert chk["ok"], f"radix decode differs from the oracle: {chk}"
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        logical = algorithmic_bytes_per_launch(wl, seq_lens) * L
        pages = {int(b) for s in live for b in s["table"][: -(-(s["len"] + 1) // 16)]}
        del g
        return {"seqs": B, "ms_per_step": round(ms, 4), "GB/s": round(logical / (ms * 1e-3) / 1e9, 2),
                "logical_bytes_per_step": int(logical),
                "physical_page_bytes": int(len(pages) * block_bytes), "oracle_check": chk}, logical, ms

    assert pool.check() == 0
    clocks = ClockSampler(0)
    clocks.start()
    res = {"cow_copy": time_copies(cow, 200)}
    dec1, logical1, ms1 = decode_phase(seqs)
    for s in seqs:
        s["len"] += 1
        s["tokens"].append(int(rng.integers(1000, 30000)))
    # -- finish, evict, compact
    th = time.perf_counter()
    done, live = seqs[: w["finish"]], seqs[w["finish"]:]
    for s in done:
        freed = rx.insert(s["tokens"][: s["len"]], s["table"].tolist())
        for b in s["table"][P:]:
            bm.incref(int(b))              # the tree keeps the suffix pages
        for b in freed:
            bm.decref(b)
        bm.free_seq(s["table"])
    live_ids = {int(b) for s in live for b in s["table"]}
    tree_only = [int(b) for s in done for b in s["table"][P:] if int(b) not in live_ids]
    evicted = rx.evict_lru(max(1, int(len(tree_only) * w["evict_frac"])))
    for b in evicted:
        bm.decref(b)
    moves = bm.compact()
    m = dict(zip(moves[:, 0].tolist(), moves[:, 1].tolist()))
    for s in live:
        s["table"] = np.array([m.get(int(b), int(b)) for b in s["table"]], dtype=np.uint32)
    rx.remap(moves)
    t_host["finish_evict_compact_ms"] = round((time.perf_counter() - th) * 1e3, 3)
    res["compaction_moves"] = time_copies(np.asarray(moves, dtype=np.uint32).reshape(-1, 2), 50)
    res["evicted_blocks"] = len(evicted)
    dec2, _, _ = decode_phase(live)
    clk = clocks.stop()
    assert pool.check() == 0
    peak, peak_kind = hbm_peak()
    cpu = None
    if not args.no_cpu_baseline:
        import oracle
        cpu = {"value": None, "unit": "ns/op", "cores": 1, "kind": "port", "cpu_model": cpu_model(),
               "sample": "block bookkeeping ns/op, one thread: the oracle's restatement of the reference "
                         "(kv_cache.bm / radix_cache.bm) beside this library's own",
               "block_ops_ns_per_op_1_thread": oracle.bench_block_ops(200000),
               "block_ops_ns_per_op_product_1_thread": product_block_ops(200000)}
    print(json.dumps({
        "metric": "paged decode KV GB/s", "value": dec1["GB/s"], "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dec1["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": args.workload, "layers": L, "q_heads": Hq, "kv_heads": Hkv, "head_dim": D,
                   "requests": w["n_req"], "forks": w["n_fork"], "prefix_tokens": w["prefix"],
                   "suffix": list(w["suffix"]), "pool_blocks": NB, "parallelism": "single",
                   "l2": f"inputs larger than L2 ({logical1 / 1e9:.2f} GB logical per step)"},
        "tok_per_s": round(dec1["seqs"] / (ms1 * 1e-3), 1),
        "decode_before_eviction": dec1, "decode_after_compaction": dec2, **res, "host_ms": t_host,
        "roofline": {"bound": "hbm", "achieved": dec1["GB/s"], "peak": peak, "unit": "GB/s",
                     "frac": round(dec1["GB/s"] / peak, 4), "traffic": None, "peak_kind": peak_kind},
        "cpu_baseline": cpu, "e2e": None, "clocks": clk,
        "gpu_launches": args.steps * L * 2 * 2 + 250,
    }), flush=True)
    pool.close()


def run_kvops_bench(args, w):
    """vw_kv_append, vw_kv_gather and vw_block_copy alone, each timed with CUDA
    events over K launches on inputs larger than L2 in total; GB/s of the bytes
    each launch must read and write."""
    import torch
    from voidweb_b200.kv import KvPool, PoolSpec
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        print(json.dumps({"metric": "page kernels GB/s", "error": "single GPU only"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    L, Hkv, D = w["L"], w["Hkv"], w["D"]
    T, G, NP = w["append_tokens"], w["gather_tokens"], w["copy_pairs"]
    NB = 2 * NP + (T + G) // 16 * 8 + 64
    rng = np.random.Generator(np.random.PCG64(w["seed"]))
    pool = KvPool(PoolSpec(L, Hkv, D, NB, "bf16", "bf16", max_batch=1), device=0)
    pool.pages_u8().view(torch.bfloat16).normal_()
    row = Hkv * D * 2
    perm = rng.permutation(NB)
    # append: T rows into distinct random slots of one layer (rotating layers)
    slots = torch.from_numpy((perm[: T // 16 * 2].repeat(16)[:T] * 16 +
                              np.tile(np.arange(16), T // 16)).astype(np.int64)).to(dev)
    kn = torch.randn((T, Hkv, D), device=dev).bfloat16()
    vn = torch.randn((T, Hkv, D), device=dev).bfloat16()
    gtable = torch.from_numpy(perm[-(G // 16):].astype(np.int32)).to(dev)
    pairs_np = np.stack([perm[T // 8: T // 8 + NP], perm[T // 8 + NP: T // 8 + 2 * NP]], 1)
    pairs = torch.from_numpy(pairs_np.astype(np.int32)).to(dev)
    block_bytes = L * Hkv * 2 * 16 * D * 2
    gk = torch.empty((Hkv, G, D), dtype=torch.int16, device=dev)
    gv = torch.empty_like(gk)
    from voidweb_b200 import _lib as C
    from voidweb_b200.kv import _ptr
    lib = C.lib()
    st = torch.cuda.Stream(device=dev)
    sp = st.cuda_stream
    ops = {
        "kv_append_kernel": (lambda i: C.check(lib.vw_kv_append(pool.handle, i % L, _ptr(kn), _ptr(vn),
                                                                 _ptr(slots), T, sp)), 2 * T * row * 2),
        "kv_gather_kernel": (lambda i: C.check(lib.vw_kv_gather(pool.handle, i % L, _ptr(gtable), G, _ptr(gk),
                                                                 _ptr(gv), None, None, sp)), 2 * G * row * 2),
        "block_copy_kernel": (lambda i: C.check(lib.vw_block_copy(pool.handle, _ptr(pairs), NP, sp)),
                              2 * NP * block_bytes),
    }
    res = {}
    clocks = ClockSampler(0)
    clocks.start()
    for name, (fn, nbytes) in ops.items():
        # the launches are recorded as one CUDA graph and replayed, so that the
        # timing is the kernels' and not the host's issue rate
        with torch.cuda.stream(st):
            for i in range(args.warmup):
                fn(i)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(args.steps):
                fn(i)
        with torch.cuda.stream(st):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        with torch.cuda.stream(st):       # replay and events on the same stream
            e0.record(st)
            g.replay()
            e1.record(st)
        torch.cuda.synchronize()
        del g
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        res[name] = {"bytes_per_launch": nbytes, "us_per_launch": round(us, 3),
                     "GB/s": round(nbytes / (us * 1e-6) / 1e9, 2)}
    clk = clocks.stop()
    assert pool.check() == 0
    peak, peak_kind = hbm_peak()
    for v in res.values():
        v["frac_of_peak"] = round(v["GB/s"] / peak, 4)
    top = res["block_copy_kernel"]
    print(json.dumps({
        "metric": "page kernels GB/s", "value": top["GB/s"], "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(top["us_per_launch"] / 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": args.workload, "layers": L, "kv_heads": Hkv, "head_dim": D,
                   "append_tokens": T, "gather_tokens": G, "copy_pairs": NP, "parallelism": "single"},
        "kernels": res,
        "roofline": {"bound": "hbm", "achieved": top["GB/s"], "peak": peak, "unit": "GB/s",
                     "frac": top["frac_of_peak"], "traffic": None, "peak_kind": peak_kind},
        "cpu_baseline": None, "e2e": None, "clocks": clk, "gpu_launches": 3 * (args.steps + args.warmup),
    }), flush=True)
    pool.close()


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def product_block_ops(iters):
    """ns/op of this library's own block manager and radix tree (vw_bm_*,
    vw_radix_*), one thread, from the vw_bench_ops tool built beside it."""
    exe = os.path.join(ROOT, "voidweb_b200", "vw_bench_ops")
    try:
        out = subprocess.run([exe, str(iters)], capture_output=True, text=True, timeout=120, check=True)
        return json.loads(out.stdout)
    except Exception as e:          # reported, not fatal: the GPU figures stand alone
        return {"error": str(e)[:200]}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class CpuSample:
    """The oracle (the reference's paged_attention_decode restated in C++: f32,
    per-token online softmax in reference order, OpenMP over (seq, head)) plus
    the append, on one layer of the workload's sequences."""

    def __init__(self, w, seq_lens, threads):
        import oracle
        self.o, self.w, self.threads = oracle, w, threads
        kvk = {"f16": oracle.F16, "bf16": oracle.BF16, "fp8": oracle.FP8}
        rng = np.random.Generator(np.random.PCG64(w["seed"]))
        self.seq_lens = np.asarray(seq_lens, dtype=np.int64)
        pages = (self.seq_lens + 15) // 16
        NB = int(pages.sum()) + 1
        self.g = oracle.geom(1, w["Hkv"], w["D"], NB, kvk[w["kv"]], kvk[w["io"]])
        shape = oracle.pool_shape(self.g)
        if w["kv"] == "fp8":
            self.data = rng.integers(0, 255, shape, dtype=np.uint8)
            self.scales = np.full(shape[:-1], 0.01, dtype=np.float32)
        else:
            self.data = oracle.f32_to_io_bits(rng.standard_normal(shape, dtype=np.float32),
                                              kvk[w["io"]])
            self.scales = None
        perm = rng.permutation(NB)
        self.bt = np.zeros((w["B"], int(pages.max())), dtype=np.uint32)
        off = 0
        for b in range(w["B"]):
            self.bt[b, :pages[b]] = perm[off:off + pages[b]]
            off += pages[b]
        io = kvk[w["io"]]
        self.q = oracle.f32_to_io_bits(rng.standard_normal((w["B"], w["Hq"], w["D"]),
                                                           dtype=np.float32), io)
        self.kn = oracle.f32_to_io_bits(rng.standard_normal((w["B"], w["Hkv"], w["D"]),
                                                            dtype=np.float32), io)
        pos = self.seq_lens - 1
        self.slots = np.array([int(self.bt[b, pos[b] // 16]) * 16 + int(pos[b] % 16)
                               for b in range(w["B"])], dtype=np.int64)
        self.scale = float(np.float32(1.0) / np.sqrt(np.float32(w["D"])))

    def launch(self, seqs):
        """Append + decode of one layer over the sequence indices `seqs`;
        returns the algorithmic bytes moved."""
        o, w = self.o, self.w
        o.kv_append(self.g, self.data, self.scales, 0, self.kn[seqs], self.kn[seqs],
                    self.slots[seqs])
        o.paged_decode_f32(self.g, self.data, self.scales, 0, self.q[seqs], w["Hq"],
                           self.bt[seqs], self.seq_lens[seqs].astype(np.uint32), self.scale,
                           nthreads=self.threads)
        return algorithmic_bytes_per_launch(w, self.seq_lens[seqs])


def cpu_decode_sample(w, seq_lens, launches, threads):
    cs = CpuSample(w, seq_lens, threads)
    allseq = np.arange(w["B"])
    cs.launch(allseq)
    t0 = time.perf_counter()
    moved = sum(cs.launch(allseq) for _ in range(launches))
    dt = time.perf_counter() - t0
    gbs = moved / dt / 1e9
    tok_s = w["B"] / (dt / launches * w["L"])
    return gbs, tok_s, dt, launches


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = cpu_threads()
    seq_lens = ctx_lengths(w, 0) + 1         # the step's token at position ctx
    cs = CpuSample(w, seq_lens, threads)
    allseq = np.arange(w["B"])
    t0 = time.perf_counter()
    cs.launch(allseq)
    t_full = time.perf_counter() - t0
    # bounded sample: each step is one layer over a rotating window of
    # sequences, sized so warm-up + K steps take about a minute at most
    budget = 60.0
    per = max(1, min(w["B"], int(w["B"] * budget / ((args.steps + args.warmup) * t_full))))
    windows = [np.arange(i, i + per) % w["B"] for i in range(0, w["B"] * 64, per)]
    for i in range(args.warmup):
        cs.launch(windows[i % len(windows)])
    moved = 0
    t0 = time.perf_counter()
    for i in range(args.steps):
        moved += cs.launch(windows[(i + args.warmup) % len(windows)])
    dt = time.perf_counter() - t0
    gbs = moved / dt / 1e9
    # tok/s of a full step (all layers, all sequences) at the sampled speed
    full_step_s = algorithmic_bytes_per_launch(w, seq_lens) * w["L"] / (moved / dt)
    tok_s = w["B"] / full_step_s
    sample = (f"{args.steps} steps, each 1 of {w['L']} layers over {per} of {w['B']} sequences "
              f"(rotating); ctx {int(seq_lens.min())}-{int(seq_lens.max())}; oracle f32 "
              f"reference-order decode + append, {threads} OpenMP threads")
    line = {
        "impl": "reference", "metric": "paged decode KV GB/s", "value": round(gbs, 4),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": w["kv"], "data": "synthetic",
        "config": {"workload": args.workload, "layers": w["L"], "q_heads": w["Hq"],
                   "kv_heads": w["Hkv"], "head_dim": w["D"], "seqs_per_gpu": w["B"],
                   "ctx": list(w["ctx"]), "block_size": 16, "parallelism": "cpu"},
        "tok_per_s": round(tok_s, 3),
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample, "cpu_model": cpu_model()},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=DEFAULT, choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: every GPU brings the workload's batch; strong: one batch split across the GPUs")
    ap.add_argument("--gather", default="auto", choices=["auto", "overlap", "serial"],
                    help="N>1: all-gather each step's outputs on a side stream while the next step "
                         "runs (few NCCL channels), or inside the step's graph after its last layer "
                         "(NCCL's own channel count); auto: serial from 8 MB received per rank "
                         "and step")
    ap.add_argument("--placement", default="sequences", choices=["sequences", "kv_heads", "kv_heads_seqs"],
                    help="N GPUs: sequences = each GPU its own sequences (every KV head); kv_heads = "
                         "every GPU the same sequences and block tables with its own KV heads "
                         "(the workload's kv_heads per GPU: Llama-3-70B one KV head per GPU)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--plan", action="store_true",
                    help="compute the decode plan (vw_decode_plan) once per step and launch every "
                         "layer with VW_DECODE_PLANNED")
    ap.add_argument("--layers", type=int, default=0,
                    help="run only this many layers of the workload (a small case for ncu "
                         "captures; the JSON line's config.layers says so)")
    args = ap.parse_args()
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gather == "auto":
        args.gather = choose_gather(WORKLOADS[args.workload], world_env)
    if world_env > 1:
        # set before torch loads NCCL.  The per-step output all-gather overlaps
        # the next step's decode on a side stream; every NCCL channel is a CTA
        # that can take an SM slot a decode CTA needs (2 B200s: 8909 GB/s with one
        # channel, 8371 with two), while the bytes each rank receives per step
        # grow with the ranks (N - 1 times 3.2 MB on the Qwen step): one channel
        # up to 2 GPUs, then one per two GPUs.  (NCCL's set-up lines -- ranks,
        # NVLink / NVLS paths -- come with NCCL_DEBUG=INFO and an NCCL_DEBUG_FILE
        # set by the caller; without a file they would go to stdout, which keeps
        # the JSON line alone.)
        if args.gather == "overlap":
            os.environ.setdefault("NCCL_MAX_NCHANNELS", str(max(1, world_env // 2)))
            # the gather's NCCL CTA displaces a decode CTA while the next step
            # runs; the split with the smaller segment-boundary cost leaves the
            # CTAs the slack to absorb it (2 B200s, Qwen step: 8981 GB/s at 12
            # against 7869 at the library's 18, which is best on a GPU that only
            # decodes: 4687 against 4531 at 12)
            os.environ.setdefault("VOIDWEB_KV_SEGMENT_COST", "12")
    w = dict(WORKLOADS[args.workload])
    if args.layers > 0:
        w["L"] = min(args.layers, w["L"])
    if w.get("kind") == "gemm":
        if args.warmup < 3:
            args.warmup = 3
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the decode "
                              "workloads; the gemm line's cpu_baseline is the oracle sample"}))
            return
        return run_gemm_bench(args, w)
    if w.get("kind") == "kvops":
        if args.warmup < 3:
            args.warmup = 3
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the decode "
                              "workloads"}))
            return
        return run_kvops_bench(args, w)
    if w.get("kind") == "radix":
        if args.warmup < 3:
            args.warmup = 3
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the decode "
                              "workloads; the radix line's cpu_baseline holds the block-op figures"}))
            return
        return run_radix_bench(args, w)
    if w.get("kind") == "prefill":
        if args.warmup < 3:
            args.warmup = 3
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the decode "
                              "workloads; the prefill line's cpu_baseline is the oracle sample"}))
            return
        return run_prefill_bench(args, w)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args, w)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from voidweb_b200.kv import KvPool, PoolSpec

    L, Hq, Hkv, D, B = w["L"], w["Hq"], w["Hkv"], w["D"], w["B"]
    heads_split = args.placement == "kv_heads"
    if heads_split and args.scaling == "strong":
        raise SystemExit("--placement kv_heads is a weak-scaling placement (one KV head per GPU)")
    seq_slice = rank            # which sequence slice (and block-table draw) this rank holds
    head_groups = 1
    if args.placement == "kv_heads_seqs":
        # the one batch of the 1-GPU run cut into KV-head groups x sequence slices
        # (Qwen2.5-7B on 8 GPUs: one KV head and 8 sequences per GPU)
        if args.scaling != "strong":
            raise SystemExit("--placement kv_heads_seqs splits the 1-GPU batch: use --scaling strong")
        from voidweb_b200.shard import ShardPlan
        plan = ShardPlan("kv_heads_seqs", world, rank, B, Hq, Hkv)
        s0, s1 = plan.seqs()
        h0, h1 = plan.kv_heads()
        g0, g1 = plan.q_heads()
        ctx = ctx_lengths(w, 0)[s0:s1]
        B, Hkv, Hq = s1 - s0, h1 - h0, g1 - g0
        w = dict(w, B=B, Hkv=Hkv, Hq=Hq)
        seq_slice, head_groups = rank % plan.seq_groups, plan.head_groups
    elif args.scaling == "strong":
        # one fixed batch (the 1-GPU workload's seeded contexts) split across the ranks
        if B % world:
            raise SystemExit(f"--scaling strong needs the batch ({B}) divisible by the GPUs ({world})")
        from voidweb_b200.shard import shard_range
        s0, s1 = shard_range(B, world, rank)
        ctx = ctx_lengths(w, 0)[s0:s1]
        B = s1 - s0
    else:
        # kv_heads: every rank the same sequences (its own KV heads); sequences:
        # each rank its own sequences with the same length draw, so that the
        # per-GPU work is the 1-GPU workload exactly (weak scaling); the page
        # contents and block tables differ by rank
        ctx = ctx_lengths(w, 0)
    # the step appends the token at position ctx and decodes over ctx + 1 tokens
    seq_lens = ctx + 1
    pages = (seq_lens + 15) // 16
    NB = int(pages.sum()) + 64
    # kv_heads: the same block ids on every rank (the bookkeeping is replicated)
    rng = np.random.Generator(np.random.PCG64(w["seed"] * 7919 + (0 if heads_split else seq_slice)))
    perm = rng.permutation(NB)
    stride = int(pages.max())
    bt = np.zeros((B, stride), dtype=np.int32)
    off = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[off:off + pages[b]]
        off += pages[b]

    spec = PoolSpec(num_layers=L, num_kv_heads=Hkv, head_dim=D, num_blocks=NB, kv_dtype=w["kv"],
                    io_dtype=w["io"], max_batch=B)
    pool = KvPool(spec, device=local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(w["seed"] * 31 + rank)
    iod = torch.bfloat16 if w["io"] == "bf16" else torch.float16
    pages_t = pool.pages_u8()
    if w["kv"] == "fp8":
        chunk = 1 << 28
        for o in range(0, pages_t.numel(), chunk):
            n = min(chunk, pages_t.numel() - o)
            pages_t[o:o + n].copy_(torch.randint(0, 120, (n,), device=dev, generator=gen,
                                                 dtype=torch.uint8))
        pool.scales_f32().fill_(0.01)
    else:
        view = pages_t.view(iod)
        chunk = 1 << 27
        for o in range(0, view.numel(), chunk):
            n = min(chunk, view.numel() - o)
            view[o:o + n].copy_(torch.randn(n, device=dev, generator=gen, dtype=torch.float32))
    q = torch.randn((L, B, Hq, D), device=dev, generator=gen, dtype=torch.float32).to(iod)
    kn = torch.randn((L, B, Hkv, D), device=dev, generator=gen, dtype=torch.float32).to(iod)
    vn = torch.randn((L, B, Hkv, D), device=dev, generator=gen, dtype=torch.float32).to(iod)
    # two output buffers: with N GPUs the all-gather of one step's outputs runs on
    # a side stream while the next step writes the other buffer
    outs = [torch.zeros((L, B, Hq, D), device=dev, dtype=iod) for _ in range(2)]
    out = outs[0]
    bt_d = torch.from_numpy(bt).to(dev)
    sl_d = torch.from_numpy(seq_lens.astype(np.int32)).to(dev)
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device=dev)

    from voidweb_b200 import _lib as C
    # consecutive layers: each launch may start while the previous one drains and
    # stream its pages early (the previous launch writes only its own layer)
    flags = C.VW_DECODE_PDL | C.VW_DECODE_EARLY_PAGES

    def step(s, o):
        if args.plan:
            pool.plan(bt_d, sl_d, Hq, stream=s)
        for layer in range(L):
            f = flags
            if args.plan:      # the layer right after the plan waits for it in stream order
                f = C.VW_DECODE_PLANNED | (flags if layer > 0 else 0)
            pool.paged_decode(layer, q[layer], bt_d, sl_d, o[layer], k_new=kn[layer],
                              v_new=vn[layer], stream=s, flags=f)

    # first launches outside capture (per-device kernel attribute set-up)
    with torch.cuda.stream(stream):
        step(stream, outs[0])
    stream.synchronize()
    assert pool.check() == 0, "device bounds check tripped"
    gathered = [torch.empty((world, L, B, Hq, D), device=dev, dtype=iod) for _ in range(2)] \
        if world > 1 else None
    serial = world > 1 and args.gather == "serial"
    if serial:
        # one eager collective first: the communicator exists before the capture
        with torch.cuda.stream(stream):
            dist.all_gather_into_tensor(gathered[0], outs[0])
        stream.synchronize()
    graphs = []
    for i, o in enumerate(outs):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(torch.cuda.current_stream(), o)
            if serial:
                # the step's all-gather, recorded in the step's graph after its last layer
                dist.all_gather_into_tensor(gathered[i], o)
        graphs.append(g)
    del g       # the graphs hold NCCL work when serial: only `graphs` keeps them, and it is
                # released before the process group is destroyed
    gather_stream = torch.cuda.Stream(device=dev) if world > 1 else None
    gather_done = [torch.cuda.Event(), torch.cuda.Event()]
    pending = [False, False]
    step_no = [0]

    def run_step():
        i = step_no[0] % 2
        step_no[0] += 1
        if pending[i]:
            stream.wait_event(gather_done[i])    # the gather reading outs[i] has finished
        graphs[i].replay()
        if world > 1 and not serial:
            ready = torch.cuda.Event()
            ready.record(stream)
            gather_stream.wait_event(ready)
            with torch.cuda.stream(gather_stream):
                dist.all_gather_into_tensor(gathered[i], outs[i])
            gather_done[i].record(gather_stream)
            pending[i] = True

    def join_gathers():
        for i in range(2):
            if pending[i]:
                stream.wait_event(gather_done[i])

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            run_step()
        join_gathers()
    stream.synchronize()
    # one layer of the step (the middle one) against the oracle, untimed
    vl = L // 2
    verified = verify_layer(pool, w, vl, q[vl], kn[vl], vn[vl], outs[(args.warmup - 1) % 2][vl], bt,
                            seq_lens, threads=max(1, cpu_threads() // max(world, 1)))
    if not verified["ok"]:
        raise SystemExit(f"rank {rank}: the benchmarked step differs from the oracle: {verified}")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(args.steps):
            run_step()
        join_gathers()                  # every step's gather ends inside the timed region
        t1.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    assert pool.check() == 0, "device bounds check tripped"

    bytes_launch = algorithmic_bytes_per_launch(w, seq_lens)
    if world > 1:
        t = torch.tensor([bytes_launch], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        total_launch_bytes = float(t.item())
        tb = torch.tensor([float(B)], device=dev, dtype=torch.float64)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
        # kv_heads: the ranks advance the same sequences (each its own heads);
        # kv_heads_seqs: each head group advances the whole batch
        total_seqs = float(B) if heads_split else float(tb.item()) / head_groups
    else:
        total_launch_bytes, total_seqs = float(bytes_launch), float(B)
    step_bytes_all = total_launch_bytes * L
    value = step_bytes_all / (ms * 1e-3) / 1e9
    tok_s = total_seqs / (ms * 1e-3)
    peak, peak_kind = hbm_peak()
    launch_us = ms * 1e3 / L
    achieved = bytes_launch / (launch_us * 1e-6) / 1e9

    # per-launch kernel durations with events around each launch (ungraphed pass)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(L)]
    kdur = []
    with torch.cuda.stream(stream):
        for _ in range(5):
            for layer in range(L):
                evs[layer][0].record(stream)
                pool.paged_decode(layer, q[layer], bt_d, sl_d, out[layer], k_new=kn[layer],
                                  v_new=vn[layer], stream=stream)
                evs[layer][1].record(stream)
            stream.synchronize()
            kdur += [a.elapsed_time(b) for a, b in evs]
    kernel_us = statistics.median(kdur) * 1e3

    # end to end through the public host-buffer API (pinned host memory)
    e2e = None
    if args.e2e_steps > 0:
        hq = q.cpu().pin_memory()
        hk = kn.cpu().pin_memory()
        hv = vn.cpu().pin_memory()
        hbt = torch.from_numpy(bt).pin_memory()
        hsl = torch.from_numpy(seq_lens.astype(np.int32)).pin_memory()
        ho = torch.empty_like(out, device="cpu").pin_memory()
        for _ in range(3):
            pool.decode_step_host(hq, hk, hv, hbt, hsl, ho, stream=stream)
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            pool.decode_step_host(hq, hk, hv, hbt, hsl, ho, stream=stream)
        e1.record(stream)
        e1.synchronize()
        ems = e0.elapsed_time(e1) / args.e2e_steps
        if world > 1:
            m = torch.tensor([ems], device=dev, dtype=torch.float64)
            dist.all_reduce(m, op=dist.ReduceOp.MAX)
            ems = float(m.item())
        h2d = (hq.numel() + hk.numel() + hv.numel()) * 2 + hbt.numel() * 4 + hsl.numel() * 4
        e2e = {"value": round(step_bytes_all / (ems * 1e-3) / 1e9, 3), "unit": "GB/s",
               "ms_per_step": round(ems, 4), "tok_per_s": round(total_seqs / (ems * 1e-3), 1),
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(ho.numel() * 2),
               "path": "vw_decode_step_host (pinned host buffers; from the second call with "
                       "the same buffers the step replays as one recorded CUDA graph)"}
        if world > 1:
            # no device-side gather here: the step's result is each rank's shard of
            # the outputs in that rank's host memory
            e2e["outputs"] = "each rank's shard, read back to its own host"
        # the same step through the symbol the engine dlopens: voidweb_forward_pass
        # with the packed descriptors KernelLib.forward_pass builds (engine/ffi.bm:86-121);
        # the bound q / new K / new V / output buffers are the pinned ones above
        import ctypes
        from voidweb_b200 import KernelLib
        Lb = C.lib()
        kl = KernelLib.open(C.LIB_PATH)
        Lb.vw_forward_bind(pool.handle, hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), ho.data_ptr())
        # the engine builds its descriptors natively; here they are built once and
        # the bound symbol is called directly, so that Python adds little per step
        toks = np.full(B, 7, dtype=np.uint32)
        tables = [np.ascontiguousarray(bt[b, :pages[b]], dtype=np.uint32) for b in range(B)]
        descs = (C.SeqDescriptor * B)()
        for b in range(B):
            descs[b] = C.SeqDescriptor(1000 + b, toks.ctypes.data + 4 * b, 1, tables[b].ctypes.data,
                                       tables[b].size, 0)
        fargs = C.ForwardArgs(ctypes.cast(descs, ctypes.c_void_p), B, 0, Hq, Hkv, L, 1, D, 0.0, 0, None)
        set_len, fwd = Lb.vw_forward_set_seq_len, kl._forward
        ids = [1000 + b for b in range(B)]
        lens = [int(x) for x in ctx]

        def fwd_step():
            for i, n in zip(ids, lens):   # every step decodes the same position (fixed workload)
                set_len(i, n)
            rc = fwd(ctypes.byref(fargs))
            if rc != 0:
                raise RuntimeError(f"GPU forward pass failed with code {rc}: {Lb.vw_last_error()}")

        for _ in range(3):
            fwd_step()
        if world > 1:
            dist.barrier()
        ds = torch.cuda.default_stream(dev)
        e0.record(ds)
        for _ in range(args.e2e_steps):
            fwd_step()
        e1.record(ds)
        e1.synchronize()
        fms = e0.elapsed_time(e1) / args.e2e_steps
        if world > 1:
            m = torch.tensor([fms], device=dev, dtype=torch.float64)
            dist.all_reduce(m, op=dist.ReduceOp.MAX)
            fms = float(m.item())
        Lb.vw_forward_bind(None, None, None, None, None)
        for b in range(B):
            Lb.vw_forward_release(1000 + b)
        e2e["forward_pass"] = {
            "value": round(step_bytes_all / (fms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "ms_per_step": round(fms, 4), "tok_per_s": round(total_seqs / (fms * 1e-3), 1),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(ho.numel() * 2),
            "path": "voidweb_forward_pass as KernelLib::forward_pass calls it (packed SeqDescriptor / "
                    "ForwardArgs with host block lists, pinned bound buffers; rope_theta 0)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        threads = cpu_threads()
        cs_probe = CpuSample(w, seq_lens, threads)
        tp = time.perf_counter()
        cs_probe.launch(np.arange(B))
        n_launch = max(1, min(200, int(10.0 / max(time.perf_counter() - tp, 1e-3))))
        del cs_probe
        gbs, ctok, dt, launches = cpu_decode_sample(w, seq_lens, n_launch, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "cpu_model": cpu_model(),
               "tok_per_s": round(ctok, 2),
               "sample": f"{launches} layer launches (1 of {w['L']} layers, same {B} sequences), "
                         f"{dt:.1f} s; oracle f32 reference-order decode + append, OpenMP",
               "block_ops_ns_per_op_1_thread": oracle.bench_block_ops(200000),
               "block_ops_ns_per_op_product_1_thread": product_block_ops(200000)}

    if rank == 0:
        line = {
            "metric": "paged decode KV GB/s", "value": round(value, 3), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": w["kv"], "data": "synthetic",
            "config": {"workload": args.workload, "layers": L, "q_heads": Hq, "kv_heads": Hkv,
                       "head_dim": D, "seqs_per_gpu": B, "seqs_total": int(total_seqs), "ctx": list(w["ctx"]),
                       "block_size": 16, "kv_dtype": w["kv"],
                       "parallelism": ({"sequences": "sequence", "kv_heads": "kv-head",
                                        "kv_heads_seqs": "kv-head x sequence"}[args.placement] +
                                       f"-shard x{world}" if world > 1 else "single"),
                       "placement": args.placement,
                       "l2": f"inputs larger than L2 ({bytes_launch * L / 1e9:.2f} GB of KV "
                             f"per step per GPU vs {L2_BYTES / 1e6:.0f} MB L2)",
                       "graph": "one CUDA graph per step: one fused append+decode launch per layer, "
                                "programmatic dependent launches with early page streaming" +
                                (", decode plan made once per step" if args.plan else ""),
                       "gather": (None if world == 1 else
                                  "NCCL all-gather of each step's outputs in the step's CUDA graph after "
                                  "its last layer" if args.gather == "serial" else
                                  "NCCL all-gather of each step's outputs on a side stream, overlapping "
                                  "the next step (double-buffered outputs)")},
            "tok_per_s": round(tok_s, 1),
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": NCU_TRAFFIC_PER_LAUNCH.get(args.workload),
                         "peak_kind": peak_kind, "launch_us_in_region": round(launch_us, 3),
                         "kernel_us_event_median": round(kernel_us, 3),
                         "kernel_only_frac": round(bytes_launch / (kernel_us * 1e-6) / 1e9 / peak, 4),
                         "algorithmic_bytes_per_launch": bytes_launch},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks,
            "oracle_check": verified,
            # per layer: the fused append+decode grid and its split-K combine grid
            "gpu_launches": args.steps * (L * 2 + (1 if args.plan else 0)),
        }
        print(json.dumps(line), flush=True)
    del graphs
    pool.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
