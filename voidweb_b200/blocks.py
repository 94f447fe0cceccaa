"""Host block bookkeeping: Python mirror of engine/kv_cache.bm (BlockManager)
and radix_cache/radix_cache.bm (RadixCacheManager), backed by the C++
implementation in libvoidweb_kv.so.  Method names, argument meaning and error
behaviour follow the reference: ``alloc`` returns None when the pool is empty
(kv_cache.bm:69-78), ``alloc_seq`` fails with "KV cache OOM" (kv_cache.bm:81-91),
incref/decref of unknown ids are no-ops (kv_cache.bm:94-113).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as C


def _arr(x, dtype=np.uint32):
    a = np.ascontiguousarray(x, dtype=dtype)
    return a, ctypes.c_void_p(a.ctypes.data)


def rolling_hash(prev: int, tokens) -> int:
    """kv_cache.bm:157-164."""
    a, p = _arr(tokens)
    return int(C.lib().vw_rolling_hash(prev, p, a.size))


class BlockManager:
    """engine/kv_cache.bm:29-151.  block_size is 16 in the engine (engine.bm:102)."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, block_size: int,
                 max_blocks: int):
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.block_size, self.max_blocks = block_size, max_blocks
        h = ctypes.c_void_p()
        C.check(C.lib().vw_bm_create(block_size, max_blocks, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            C.lib().vw_bm_destroy(self._h)
            self._h = None

    def capacity(self) -> int:
        return C.lib().vw_bm_capacity(self._h)

    def free_count(self) -> int:
        return C.lib().vw_bm_free_count(self._h)

    def alloc(self):
        out = ctypes.c_uint32()
        return int(out.value) if C.lib().vw_bm_alloc(self._h, ctypes.byref(out)) == C.VW_OK else None

    def alloc_seq(self, n: int):
        a = np.zeros(max(n, 1), dtype=np.uint32)
        if C.lib().vw_bm_alloc_seq(self._h, n, ctypes.c_void_p(a.ctypes.data)) != C.VW_OK:
            raise MemoryError(f"KV cache OOM: need {n} blocks, only {self.free_count()} free")
        return [int(x) for x in a[:n]]

    def incref(self, block_id: int) -> None:
        C.lib().vw_bm_incref(self._h, block_id)

    def decref(self, block_id: int) -> None:
        C.lib().vw_bm_decref(self._h, block_id)

    def ref_count(self, block_id: int) -> int:
        return C.lib().vw_bm_ref_count(self._h, block_id)

    def free_seq(self, block_table) -> None:
        a, p = _arr(block_table)
        C.lib().vw_bm_free_seq(self._h, p, a.size)

    def prefix_lookup(self, token_ids):
        a, p = _arr(token_ids)
        cap = max(16, self.max_blocks * 4)
        out = np.zeros(cap, dtype=np.uint32)
        n = C.lib().vw_bm_prefix_lookup(self._h, p, a.size, ctypes.c_void_p(out.ctypes.data), cap)
        return [int(x) for x in out[:min(n, cap)]]

    def register_prefix_block(self, block_id: int, token_hash: int) -> None:
        C.lib().vw_bm_register_prefix_block(self._h, block_id, token_hash)

    def free_list(self):
        out = np.zeros(self.max_blocks + 1, dtype=np.uint32)
        n = C.lib().vw_bm_free_list(self._h, ctypes.c_void_p(out.ctypes.data), out.size)
        return [int(x) for x in out[:n]]

    # -- extensions the reference lacks (copy-on-write, compaction) -----------
    def cow(self, block_table: np.ndarray, index: int):
        """Before appending into block_table[index]: if that block is shared
        (ref_count > 1), swap in a fresh block and return the (src, dst) pair
        that must be copied on the device; else None.  Mutates block_table."""
        assert block_table.dtype == np.uint32 and block_table.flags.c_contiguous
        pair = np.zeros(2, dtype=np.uint32)
        copied = ctypes.c_uint32(0)
        rc = C.lib().vw_bm_cow(self._h, ctypes.c_void_p(block_table.ctypes.data), index,
                               ctypes.c_void_p(pair.ctypes.data), ctypes.byref(copied))
        if rc == C.VW_ERR_OOM:
            raise MemoryError("KV cache OOM: no free block for copy-on-write")
        C.check(rc)
        return (int(pair[0]), int(pair[1])) if copied.value else None

    def compact(self):
        """Move used blocks to the lowest ids; returns the (src, dst) pairs to
        copy on the device and to remap block tables / the radix tree with."""
        out = np.zeros((self.max_blocks, 2), dtype=np.uint32)
        n = C.lib().vw_bm_compact(self._h, ctypes.c_void_p(out.ctypes.data), self.max_blocks)
        return out[:n].copy()


class RadixCacheManager:
    """radix_cache/radix_cache.bm:199-285 (RadixAttention prefix cache)."""

    def __init__(self, block_size: int, max_blocks: int):
        self.block_size, self.max_blocks = block_size, max_blocks
        h = ctypes.c_void_p()
        C.check(C.lib().vw_radix_create(block_size, max_blocks, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            C.lib().vw_radix_destroy(self._h)
            self._h = None

    def lookup(self, tokens):
        """Returns (matched_len, reuse_blocks) (radix_cache.bm:53-57)."""
        a, p = _arr(tokens)
        cap = max(64, self.max_blocks * 2)
        out = np.zeros(cap, dtype=np.uint32)
        ml = ctypes.c_uint32(0)
        n = C.lib().vw_radix_lookup(self._h, p, a.size, ctypes.byref(ml),
                                    ctypes.c_void_p(out.ctypes.data), cap)
        return int(ml.value), [int(x) for x in out[:min(n, cap)]]

    def insert(self, tokens, blocks):
        """Insert a finished sequence; returns ids freed by the over-budget eviction."""
        a, p = _arr(tokens)
        b, q = _arr(blocks)
        out = np.zeros(max(16, b.size + 16), dtype=np.uint32)
        n = C.lib().vw_radix_insert(self._h, p, a.size, q, b.size,
                                    ctypes.c_void_p(out.ctypes.data), out.size)
        return [int(x) for x in out[:min(n, out.size)]]

    def evict_lru(self, target_free: int):
        """Evict LRU leaves until target_free ids are freed; returns the ids."""
        cap = max(64, self.max_blocks * 2)
        out = np.zeros(cap, dtype=np.uint32)
        n = C.lib().vw_radix_evict_lru(self._h, target_free, ctypes.c_void_p(out.ctypes.data), cap)
        return [int(x) for x in out[:min(n, cap)]]

    def total_blocks(self) -> int:
        return C.lib().vw_radix_total_blocks(self._h)

    def lock(self, tokens) -> None:
        a, p = _arr(tokens)
        C.lib().vw_radix_lock(self._h, p, a.size)

    def unlock(self, tokens) -> None:
        a, p = _arr(tokens)
        C.lib().vw_radix_unlock(self._h, p, a.size)

    def remap(self, pairs) -> None:
        a, p = _arr(np.asarray(pairs).reshape(-1, 2))
        C.lib().vw_radix_remap(self._h, p, a.shape[0])
