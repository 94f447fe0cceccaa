"""voidweb_b200 -- B200-native paged KV-cache hot path for the VOIDWEB engine.

The product is libvoidweb_kv.so (C ABI: include/voidweb_kv.h): hand-written
sm_100a CUDA kernels for KV append, GQA split-K paged decode (optionally fused
with the append), copy-on-write / compaction block copies, the block-table
gather and FP8 E4M3 KV pages; plus the C++ block manager and radix prefix tree.
This package is its Python host mirror (ctypes); it has no fallback path.
"""
from ._lib import build, lib, VoidwebError  # noqa: F401
from .blocks import BlockManager, RadixCacheManager, rolling_hash  # noqa: F401
from .ffi import KernelLib  # noqa: F401


def __getattr__(name):
    # torch-backed pieces load lazily so the host bookkeeping works without torch
    if name in ("KvPool", "PoolSpec", "launch_paged_attn_decode", "default_scale"):
        from . import kv
        return getattr(kv, name)
    raise AttributeError(name)
