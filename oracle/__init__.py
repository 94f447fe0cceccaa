"""CPU oracle for the paged KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the cpu_baseline / reference arm
of ``bench.py`` may import this package.  It is the checker, never the thing
measured as the product, and the product package (``voidweb_b200``) never
imports it.

PARITY UNPINNED: the reference is written in the BlackMagic language, which
cannot be compiled here, and it ships no tests or golden vectors.  The oracle
(``vw_oracle.cpp``) restates the reference source function by function and is
cross-checked against the independent pure-Python transliteration in
``tests/golden/make_golden.py`` (fixtures committed under ``tests/golden/``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libvw_oracle.so")

F16, BF16, FP8 = 0, 1, 2
FP8_REFERENCE, FP8_OCP = 0, 1


def build() -> str:
    """Compile the oracle with its Makefile (only when the .so is stale)."""
    src = os.path.join(_HERE, "vw_oracle.cpp")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        u8, u16, u32, u64, i32, i64 = (ctypes.c_uint8, ctypes.c_uint16, ctypes.c_uint32,
                                       ctypes.c_uint64, ctypes.c_int32, ctypes.c_int64)
        f32, f64, vp = ctypes.c_float, ctypes.c_double, ctypes.c_void_p
        sig = {
            "vwo_bf16_to_f32": (f32, [u16]), "vwo_f32_to_bf16": (u16, [f32]),
            "vwo_f16_to_f32": (f32, [u16]), "vwo_f32_to_f16": (u16, [f32]),
            "vwo_fp8_encode_ref": (u8, [f32]), "vwo_fp8_decode_ref": (f32, [u8]),
            "vwo_fp8_encode_ocp": (u8, [f32]), "vwo_fp8_decode_ocp": (f32, [u8]),
            "vwo_fp8_quant_row": (None, [vp, ctypes.c_int, ctypes.c_int, vp, vp]),
            "vwo_kv_append": (None, [vp, vp, vp, u32, vp, vp, vp, u32]),
            "vwo_block_copy": (None, [vp, vp, vp, vp, u32]),
            "vwo_kv_gather": (None, [vp, vp, vp, u32, vp, u32, vp, vp, vp, vp]),
            "vwo_paged_decode_f32": (i32, [vp, vp, vp, u32, vp, u32, vp, u32, vp, u32, f32, vp,
                                           ctypes.c_int]),
            "vwo_paged_decode_f64": (i32, [vp, vp, vp, u32, vp, u32, vp, u32, vp, u32, f64, vp,
                                           ctypes.c_int]),
            "vwo_paged_prefill_f32": (i32, [vp, vp, vp, u32, vp, u32, vp, vp, vp, u32, u32,
                                            ctypes.c_int, f32, vp, ctypes.c_int]),
            "vwo_paged_prefill_f64": (i32, [vp, vp, vp, u32, vp, u32, vp, vp, vp, u32, u32,
                                            ctypes.c_int, f64, vp, ctypes.c_int]),
            "vwo_rope_apply": (None, [vp, u32, u32, u32, vp, f32, u32]),
            "vwo_rms_norm_fp8_out": (None, [vp, vp, u32, u32, f32, f32, vp]),
            "vwo_gemm_fp8_f64": (None, [vp, vp, vp, u32, u32, u32, f32, f32, vp, ctypes.c_int]),
            "vwo_rolling_hash": (u64, [u64, vp, u32]),
            "vwo_bm_new": (vp, [u32, u32]), "vwo_bm_delete": (None, [vp]),
            "vwo_bm_capacity": (u32, [vp]), "vwo_bm_free_count": (u32, [vp]),
            "vwo_bm_alloc": (i64, [vp]), "vwo_bm_alloc_seq": (i32, [vp, u32, vp]),
            "vwo_bm_incref": (None, [vp, u32]), "vwo_bm_decref": (None, [vp, u32]),
            "vwo_bm_free_seq": (None, [vp, vp, u32]), "vwo_bm_ref_count": (u32, [vp, u32]),
            "vwo_bm_prefix_lookup": (u32, [vp, vp, u32, vp, u32]),
            "vwo_bm_register_prefix_block": (None, [vp, u32, u64]),
            "vwo_bm_free_list": (u32, [vp, vp, u32]),
            "vwo_radix_new": (vp, [u32, u32]), "vwo_radix_delete": (None, [vp]),
            "vwo_radix_lookup": (u32, [vp, vp, u32, vp, vp, u32]),
            "vwo_radix_total_blocks": (u32, [vp]),
            "vwo_radix_insert": (u32, [vp, vp, u32, vp, u32, vp, u32]),
            "vwo_radix_evict_lru": (u32, [vp, u32, vp, u32]),
            "vwo_radix_lock": (None, [vp, vp, u32]), "vwo_radix_unlock": (None, [vp, vp, u32]),
            "vwo_bench_block_ops": (None, [u32, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


class Geom(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_uint32), ("num_kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("num_blocks", ctypes.c_uint32),
                ("kv_dtype", ctypes.c_uint32), ("io_dtype", ctypes.c_uint32),
                ("fp8_mode", ctypes.c_uint32)]


def geom(L, Hkv, D, NB, kv_dtype, io_dtype, fp8_mode=FP8_REFERENCE) -> Geom:
    return Geom(L, Hkv, D, NB, kv_dtype, io_dtype, fp8_mode)


# ---- codecs (numpy, vectorised through the scalar C functions) -------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """utils/simd.bm:153-158 round-to-nearest-even on the raw bits."""
    # u32 arithmetic wrapping like the reference's (bits + 0x7FFF + round) >> 16
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (b >> np.uint32(16)) & np.uint32(1)
    r += b
    r += np.uint32(0x7FFF)
    r >>= np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def io_bits_to_f32(h: np.ndarray, io_dtype: int) -> np.ndarray:
    if io_dtype == BF16:
        return bf16_bits_to_f32(h)
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_io_bits(x: np.ndarray, io_dtype: int) -> np.ndarray:
    if io_dtype == BF16:
        return f32_to_bf16_bits(x)
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def fp8_encode(x: np.ndarray, mode: int = FP8_REFERENCE) -> np.ndarray:
    f = lib().vwo_fp8_encode_ref if mode == FP8_REFERENCE else lib().vwo_fp8_encode_ocp
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.array([f(float(v)) for v in flat], dtype=np.uint8).reshape(np.shape(x))


def fp8_decode(c: np.ndarray, mode: int = FP8_REFERENCE) -> np.ndarray:
    f = lib().vwo_fp8_decode_ref if mode == FP8_REFERENCE else lib().vwo_fp8_decode_ocp
    table = np.array([f(i) for i in range(256)], dtype=np.float32)
    return table[np.asarray(c, dtype=np.uint8)]


def fp8_quant_row(x: np.ndarray, mode: int = FP8_REFERENCE):
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(x.shape, dtype=np.uint8)
    scale = np.zeros(1, dtype=np.float32)
    lib().vwo_fp8_quant_row(_p(x), x.size, mode, _p(codes), _p(scale))
    return codes, float(scale[0])


# ---- pool-level ops ----------------------------------------------------------

def pool_shape(g: Geom):
    """[L][NB][Hkv][2][16][D]: per head, a page is K rows then V rows."""
    return (g.num_layers, g.num_blocks, g.num_kv_heads, 2, 16, g.head_dim)


def rope_apply(x: np.ndarray, pos, theta: float, io_dtype: int) -> np.ndarray:
    """kernels/rope/rope.bm:22-52 on a copy of x [n][H][D] (io dtype bits),
    token i at position pos[i]."""
    y = np.array(x, dtype=np.uint16, copy=True, order="C")
    n, H, D = y.shape
    p = np.ascontiguousarray(pos, dtype=np.uint32)
    lib().vwo_rope_apply(_p(y), n, H, D, _p(p), theta, io_dtype)
    return y


def kv_append(g: Geom, data: np.ndarray, scales, layer: int, k_new: np.ndarray,
              v_new: np.ndarray, slots: np.ndarray) -> None:
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    lib().vwo_kv_append(ctypes.byref(g), _p(data), _p(scales), layer,
                        _p(np.ascontiguousarray(k_new)), _p(np.ascontiguousarray(v_new)),
                        _p(slots), slots.size)


def block_copy(g: Geom, data: np.ndarray, scales, pairs: np.ndarray) -> None:
    pairs = np.ascontiguousarray(pairs, dtype=np.uint32).reshape(-1, 2)
    lib().vwo_block_copy(ctypes.byref(g), _p(data), _p(scales), _p(pairs), pairs.shape[0])


def kv_gather(g: Geom, data, scales, layer, block_table, seq_len):
    eb_dtype = np.uint8 if g.kv_dtype == FP8 else np.uint16
    H, D = g.num_kv_heads, g.head_dim
    ok = np.zeros((H, seq_len, D), dtype=eb_dtype)
    ov = np.zeros((H, seq_len, D), dtype=eb_dtype)
    oks = np.zeros((H, seq_len), dtype=np.float32)
    ovs = np.zeros((H, seq_len), dtype=np.float32)
    bt = np.ascontiguousarray(block_table, dtype=np.uint32)
    lib().vwo_kv_gather(ctypes.byref(g), _p(data), _p(scales), layer, _p(bt), seq_len,
                        _p(ok), _p(ov), _p(oks), _p(ovs))
    return ok, ov, oks, ovs


def paged_decode_f32(g: Geom, data, scales, layer, q, Hq, block_tables, seq_lens, scale,
                     nthreads=0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint16)
    bt = np.ascontiguousarray(block_tables, dtype=np.uint32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.uint32)
    B = sl.size
    out = np.zeros((B, Hq, g.head_dim), dtype=np.uint16)
    rc = lib().vwo_paged_decode_f32(ctypes.byref(g), _p(data), _p(scales), layer, _p(q), Hq,
                                    _p(bt), bt.shape[1], _p(sl), B, scale, _p(out), nthreads)
    if rc != 0:
        raise ValueError("oracle: seq_len 0")
    return out


def paged_decode_f64(g: Geom, data, scales, layer, q, Hq, block_tables, seq_lens, scale,
                     nthreads=0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint16)
    bt = np.ascontiguousarray(block_tables, dtype=np.uint32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.uint32)
    B = sl.size
    out = np.zeros((B, Hq, g.head_dim), dtype=np.float64)
    rc = lib().vwo_paged_decode_f64(ctypes.byref(g), _p(data), _p(scales), layer, _p(q), Hq,
                                    _p(bt), bt.shape[1], _p(sl), B, scale, _p(out), nthreads)
    if rc != 0:
        raise ValueError("oracle: seq_len 0")
    return out


def prefill_slots(block_tables, cu_q, ctx_start) -> np.ndarray:
    """Slot of every chunk token: token i of sequence b at position
    p = ctx_start[b] + i - cu_q[b] lives at block_tables[b][p // 16] * 16 + p % 16
    (the paging rule of flash_attention.bm:132-140)."""
    bt = np.asarray(block_tables, dtype=np.int64)
    cu = np.asarray(cu_q, dtype=np.int64)
    cs = np.asarray(ctx_start, dtype=np.int64)
    out = np.empty(int(cu[-1]), dtype=np.int64)
    for b in range(cu.size - 1):
        p = cs[b] + np.arange(cu[b + 1] - cu[b])
        out[cu[b]:cu[b + 1]] = bt[b, p // 16] * 16 + p % 16
    return out


def _prefill(fn, g: Geom, data, scales, layer, q, Hq, block_tables, cu_q, ctx_start, causal,
             scale, out, nthreads):
    q = np.ascontiguousarray(q, dtype=np.uint16)
    bt = np.ascontiguousarray(block_tables, dtype=np.uint32)
    cu = np.ascontiguousarray(cu_q, dtype=np.int32)
    cs = np.ascontiguousarray(ctx_start, dtype=np.int32)
    rc = fn(ctypes.byref(g), _p(data), _p(scales), layer, _p(q), Hq, _p(cu), _p(cs), _p(bt),
            bt.shape[1], cs.size, 1 if causal else 0, scale, _p(out), nthreads)
    if rc != 0:
        raise ValueError("oracle: chunk outside its block table")
    return out


def paged_prefill_f32(g: Geom, data, scales, layer, q, Hq, block_tables, cu_q, ctx_start, causal,
                      scale, nthreads=0) -> np.ndarray:
    """flash_attention.bm:31-106 over the pool (f32, the reference's tile order);
    q [T][Hq][D] io bits -> out [T][Hq][D] io bits."""
    out = np.zeros((int(np.asarray(cu_q)[-1]), Hq, g.head_dim), dtype=np.uint16)
    return _prefill(lib().vwo_paged_prefill_f32, g, data, scales, layer, q, Hq, block_tables, cu_q,
                    ctx_start, causal, scale, out, nthreads)


def paged_prefill_f64(g: Geom, data, scales, layer, q, Hq, block_tables, cu_q, ctx_start, causal,
                      scale, nthreads=0) -> np.ndarray:
    """The same attention in fp64 with a two-pass softmax -> out [T][Hq][D] f64."""
    out = np.zeros((int(np.asarray(cu_q)[-1]), Hq, g.head_dim), dtype=np.float64)
    return _prefill(lib().vwo_paged_prefill_f64, g, data, scales, layer, q, Hq, block_tables, cu_q,
                    ctx_start, causal, scale, out, nthreads)


def rms_norm_fp8_out(x_f16: np.ndarray, weight_f16: np.ndarray, scale: float, eps: float) -> np.ndarray:
    """rms_norm.bm:62-94: rows of f16 bits -> E4M3 codes (reference encoder)."""
    x = np.ascontiguousarray(x_f16, dtype=np.uint16)
    w = np.ascontiguousarray(weight_f16, dtype=np.uint16)
    rows, hidden = x.shape
    out = np.zeros((rows, hidden), dtype=np.uint8)
    lib().vwo_rms_norm_fp8_out(_p(x), _p(w), rows, hidden, scale, eps, _p(out))
    return out


def gemm_fp8_f64(a: np.ndarray, b: np.ndarray, bias_bf16, a_scale: float, b_scale: float,
                 nthreads: int = 0) -> np.ndarray:
    """gemm_fp8.bm:31-107 in f64: A [M][K], B [K][N] E4M3 codes -> C [M][N]."""
    a = np.ascontiguousarray(a, dtype=np.uint8)
    b = np.ascontiguousarray(b, dtype=np.uint8)
    M, K = a.shape
    N = b.shape[1]
    bias = None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, dtype=np.uint16)
    c = np.zeros((M, N), dtype=np.float64)
    lib().vwo_gemm_fp8_f64(_p(a), _p(b), _p(bias), M, N, K, a_scale, b_scale, _p(c), nthreads)
    return c


def rolling_hash(prev: int, tokens) -> int:
    t = np.ascontiguousarray(tokens, dtype=np.uint32)
    return int(lib().vwo_rolling_hash(prev, _p(t), t.size))


class BlockManager:
    """engine/kv_cache.bm:29-151 restated (see vw_oracle.cpp)."""

    def __init__(self, block_size: int, max_blocks: int):
        self._h = lib().vwo_bm_new(block_size, max_blocks)
        self.max_blocks = max_blocks

    def __del__(self):
        if getattr(self, "_h", None):
            lib().vwo_bm_delete(self._h)
            self._h = None

    def capacity(self): return lib().vwo_bm_capacity(self._h)
    def free_count(self): return lib().vwo_bm_free_count(self._h)

    def alloc(self):
        r = lib().vwo_bm_alloc(self._h)
        return None if r < 0 else int(r)

    def alloc_seq(self, n):
        out = np.zeros(max(n, 1), dtype=np.uint32)
        if lib().vwo_bm_alloc_seq(self._h, n, _p(out)) != 0:
            raise MemoryError("KV cache OOM")
        return [int(x) for x in out[:n]]

    def incref(self, i): lib().vwo_bm_incref(self._h, i)
    def decref(self, i): lib().vwo_bm_decref(self._h, i)
    def ref_count(self, i): return lib().vwo_bm_ref_count(self._h, i)

    def free_seq(self, table):
        t = np.ascontiguousarray(table, dtype=np.uint32)
        lib().vwo_bm_free_seq(self._h, _p(t), t.size)

    def prefix_lookup(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        cap = 4096
        out = np.zeros(cap, dtype=np.uint32)
        n = lib().vwo_bm_prefix_lookup(self._h, _p(t), t.size, _p(out), cap)
        return [int(x) for x in out[:min(n, cap)]]

    def register_prefix_block(self, i, h): lib().vwo_bm_register_prefix_block(self._h, i, h)

    def free_list(self):
        out = np.zeros(self.max_blocks + 1, dtype=np.uint32)
        n = lib().vwo_bm_free_list(self._h, _p(out), out.size)
        return [int(x) for x in out[:n]]


class RadixCache:
    """radix_cache/radix_cache.bm:199-285 restated with the documented fixes."""

    def __init__(self, block_size: int, max_blocks: int):
        self._h = lib().vwo_radix_new(block_size, max_blocks)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().vwo_radix_delete(self._h)
            self._h = None

    def lookup(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        cap = 1 << 16
        out = np.zeros(cap, dtype=np.uint32)
        ml = ctypes.c_uint32(0)
        n = lib().vwo_radix_lookup(self._h, _p(t), t.size, ctypes.byref(ml), _p(out), cap)
        return int(ml.value), [int(x) for x in out[:n]]

    def insert(self, tokens, blocks):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        b = np.ascontiguousarray(blocks, dtype=np.uint32)
        out = np.zeros(4096, dtype=np.uint32)
        n = lib().vwo_radix_insert(self._h, _p(t), t.size, _p(b), b.size, _p(out), out.size)
        return [int(x) for x in out[:n]]

    def evict_lru(self, target):
        out = np.zeros(1 << 16, dtype=np.uint32)
        n = lib().vwo_radix_evict_lru(self._h, target, _p(out), out.size)
        return [int(x) for x in out[:n]]

    def total_blocks(self): return lib().vwo_radix_total_blocks(self._h)

    def lock(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        lib().vwo_radix_lock(self._h, _p(t), t.size)

    def unlock(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        lib().vwo_radix_unlock(self._h, _p(t), t.size)


BLOCK_OP_NAMES = ["alloc", "alloc_seq_16", "free_seq_16", "prefix_lookup_16", "radix_insert_256",
                  "radix_lookup_hit", "radix_lookup_miss", "radix_evict_lru_1", "rolling_hash_16"]


def bench_block_ops(iters: int = 200000) -> dict:
    """ns/op of the reference's block bookkeeping restated in C++ (one thread)."""
    out = np.zeros(len(BLOCK_OP_NAMES), dtype=np.float64)
    lib().vwo_bench_block_ops(iters, _p(out))
    return {k: round(float(v), 1) for k, v in zip(BLOCK_OP_NAMES, out)}
