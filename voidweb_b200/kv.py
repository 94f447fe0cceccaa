"""Device side of the paged KV cache: the pool and its operations.

Python mirror of the library-side operator surface behind engine/ffi.bm.  The
reference exposes one decode launcher,
``launch_paged_attn_decode(q, kv_cache, block_table, seq_lens, o)``
(kernels/attention/flash_attention.bm:180-189); this module keeps that name and
argument meaning and adds the operations the reference leaves undefined
(append, copy-on-write block copy, gather, FP8 pools).  Every call goes
through libvoidweb_kv.so; tensors are torch CUDA tensors and work is enqueued
on torch's current stream.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib as C

_IO = {torch.float16: C.VW_F16, torch.bfloat16: C.VW_BF16}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


@dataclass
class PoolSpec:
    num_layers: int
    num_kv_heads: int
    head_dim: int
    num_blocks: int
    kv_dtype: str = "bf16"      # "f16" | "bf16" | "fp8"
    io_dtype: str = "bf16"      # "f16" | "bf16"
    fp8_mode: str = "reference"  # "reference" (reference encoder) | "ocp"
    max_batch: int = 256

    @property
    def block_bytes(self) -> int:
        """Bytes one block id addresses across all layers (engine/engine.bm:170-182)."""
        eb = 1 if self.kv_dtype == "fp8" else 2
        s = 4 if self.kv_dtype == "fp8" else 0
        return self.num_layers * 2 * self.num_kv_heads * 16 * (self.head_dim * eb + s)


_DT = {"f16": C.VW_F16, "bf16": C.VW_BF16, "fp8": C.VW_FP8_E4M3}


class KvPool:
    """A paged KV pool on one GPU: pages [L][NB][Hkv][2][16][D] (+ FP8 scales)."""

    def __init__(self, spec: PoolSpec, device: int | torch.device = 0,
                 data: torch.Tensor | None = None, scales: torch.Tensor | None = None):
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.spec = spec
        self.device = dev
        cfg = C.PoolConfig(spec.num_layers, spec.num_kv_heads, spec.head_dim, spec.num_blocks,
                           _DT[spec.kv_dtype], _DT[spec.io_dtype],
                           C.VW_FP8_OCP if spec.fp8_mode == "ocp" else C.VW_FP8_REFERENCE,
                           spec.max_batch, dev.index or 0, 0,
                           _ptr(data) if data is not None else None,
                           _ptr(scales) if scales is not None else None)
        h = ctypes.c_void_p()
        C.check(C.lib().vw_pool_create(ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h
        self._keep = (data, scales)
        dptr, sptr = ctypes.c_void_p(), ctypes.c_void_p()
        db, sb = ctypes.c_uint64(), ctypes.c_uint64()
        C.check(C.lib().vw_pool_info(h, ctypes.byref(dptr), ctypes.byref(sptr), ctypes.byref(db),
                                     ctypes.byref(sb)))
        self.data_ptr, self.scales_ptr = dptr.value, sptr.value
        self.data_bytes, self.scale_bytes = db.value, sb.value

    def close(self):
        if getattr(self, "_h", None):
            C.lib().vw_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    @property
    def page_shape(self):
        s = self.spec
        return (s.num_layers, s.num_blocks, s.num_kv_heads, 2, 16, s.head_dim)

    # -- views of the library-owned pages (for tests and inspection) ----------
    def pages_u8(self) -> torch.Tensor:
        """The page buffer as a flat uint8 tensor aliasing device memory."""
        return _alias_u8(self.data_ptr, self.data_bytes, self.device)

    def scales_f32(self) -> torch.Tensor | None:
        if not self.scale_bytes:
            return None
        return _alias_u8(self.scales_ptr, self.scale_bytes, self.device).view(torch.float32)

    def check(self) -> int:
        """Synchronise and return (and clear) the device error word; raise if set."""
        w = ctypes.c_uint32(0)
        rc = C.lib().vw_pool_check(self._h, ctypes.byref(w))
        if rc not in (C.VW_OK, C.VW_ERR_DEVICE_CHECK):
            C.check(rc)
        return int(w.value)

    def set_wait_limit(self, cycles: int) -> None:
        """Test hook: bound this pool's decode waits to `cycles` SM cycles (0:
        the default, about 2 s); see vw_debug_set_wait_limit."""
        C.check(C.lib().vw_debug_set_wait_limit(self._h, cycles))

    # -- operations -------------------------------------------------------------
    def append(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor,
               slot_mapping: torch.Tensor, stream=None) -> None:
        """Reshape-and-cache: k_new/v_new [n][Hkv][D]; slot = block*16 + offset."""
        n = k_new.shape[0]
        C.check(C.lib().vw_kv_append(self._h, layer, _ptr(k_new), _ptr(v_new),
                                     _ptr(slot_mapping), n, _stream(stream)))

    def paged_decode(self, layer: int, q: torch.Tensor, block_tables: torch.Tensor,
                     seq_lens: torch.Tensor, out: torch.Tensor, k_new=None, v_new=None,
                     scale: float = 0.0, stream=None, flags: int = 0,
                     rope_theta: float = 0.0) -> torch.Tensor:
        """o = softmax(q K^T * scale) V over each sequence's pages (GQA, split-K).

        With k_new/v_new given, the new token's rows are first written at
        position seq_len-1 (fused append).  q/out: [B][Hq][D]; block_tables:
        [B][stride] int32 ids; seq_lens: [B] int32 (including the new token).
        flags: VW_DECODE_PDL / VW_DECODE_EARLY_PAGES / VW_DECODE_PLANNED (see
        include/voidweb_kv.h).  rope_theta > 0 rotates q and the new K row at
        position seq_len-1 first (VW_DECODE_ROPE).
        """
        B, Hq, _ = q.shape
        if rope_theta > 0.0:
            flags |= C.VW_DECODE_ROPE
        a = C.DecodeArgs(layer, B, Hq, block_tables.shape[1], _ptr(q), _ptr(block_tables),
                         _ptr(seq_lens), _ptr(out), _ptr(k_new), _ptr(v_new), scale, flags,
                         rope_theta, 0)
        C.check(C.lib().vw_paged_decode(self._h, ctypes.byref(a), _stream(stream)))
        return out

    def paged_prefill(self, layer: int, q: torch.Tensor, cu_seqlens: torch.Tensor,
                      ctx_start: torch.Tensor, block_tables: torch.Tensor, out: torch.Tensor,
                      k_new=None, v_new=None, causal: bool = True, scale: float = 0.0,
                      rope_theta: float = 0.0, stream=None, flags: int = 0) -> torch.Tensor:
        """Chunked prefill of one layer (launch_flash_attn_prefill,
        flash_attention.bm:167-177, over the pool's pages).

        Sequence b's chunk is rows cu_seqlens[b] .. cu_seqlens[b+1]-1 of q
        [T][Hq][D] at positions ctx_start[b] + i; with k_new / v_new [T][Hkv][D]
        its rows are appended first.  causal: token i attends to keys 0 .. its
        position, else to the whole ctx_start[b] + n_b context.  rope_theta > 0
        rotates q and the appended K rows at their positions (VW_PREFILL_ROPE).
        cu_seqlens, ctx_start: int32; block_tables: [B][stride] int32.
        """
        T, Hq, _ = q.shape
        if causal:
            flags |= C.VW_PREFILL_CAUSAL
        if rope_theta > 0.0:
            flags |= C.VW_PREFILL_ROPE
        a = C.PrefillArgs(layer, ctx_start.shape[0], T, Hq, block_tables.shape[1], flags, _ptr(q),
                          _ptr(k_new), _ptr(v_new), _ptr(cu_seqlens), _ptr(ctx_start),
                          _ptr(block_tables), _ptr(out), scale, rope_theta)
        C.check(C.lib().vw_paged_prefill(self._h, ctypes.byref(a), _stream(stream)))
        return out

    def plan(self, block_tables: torch.Tensor, seq_lens: torch.Tensor, num_q_heads: int,
             stream=None) -> None:
        """Page assignment of a decode batch for every layer's paged_decode with
        VW_DECODE_PLANNED (same block_tables / seq_lens tensors, unchanged until
        the next plan)."""
        C.check(C.lib().vw_decode_plan(self._h, _ptr(block_tables), _ptr(seq_lens),
                                       block_tables.shape[0], block_tables.shape[1], num_q_heads,
                                       _stream(stream)))

    def block_copy(self, pairs: torch.Tensor, stream=None) -> None:
        """Copy-on-write / compaction copy of whole blocks: pairs [n][2] (src, dst)."""
        C.check(C.lib().vw_block_copy(self._h, _ptr(pairs), pairs.shape[0], _stream(stream)))

    def gather(self, layer: int, block_table: torch.Tensor, seq_len: int, stream=None):
        """Raw K/V rows of one sequence, [Hkv][seq_len][D] (+ FP8 scales)."""
        s = self.spec
        dt = torch.uint8 if s.kv_dtype == "fp8" else torch.int16
        ok = torch.empty((s.num_kv_heads, seq_len, s.head_dim), dtype=dt, device=self.device)
        ov = torch.empty_like(ok)
        ks = vs = None
        if s.kv_dtype == "fp8":
            ks = torch.empty((s.num_kv_heads, seq_len), dtype=torch.float32, device=self.device)
            vs = torch.empty_like(ks)
        C.check(C.lib().vw_kv_gather(self._h, layer, _ptr(block_table), seq_len, _ptr(ok),
                                     _ptr(ov), _ptr(ks), _ptr(vs), _stream(stream)))
        return ok, ov, ks, vs

    def decode_step_host(self, q, k_new, v_new, block_tables, seq_lens, out,
                         scale: float = 0.0, stream=None, rope_theta: float = 0.0) -> None:
        """One step over all layers with host (CPU, ideally pinned) tensors."""
        B, Hq = q.shape[1], q.shape[2]
        a = C.StepHostArgs(B, Hq, block_tables.shape[1], 0, _ptr(q), _ptr(k_new), _ptr(v_new),
                           _ptr(block_tables), _ptr(seq_lens), _ptr(out), scale, rope_theta)
        C.check(C.lib().vw_decode_step_host(self._h, ctypes.byref(a), _stream(stream)))


def _alias_u8(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    """A uint8 CUDA tensor over library-owned memory (no copy, no ownership)."""
    class _Cai:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                    "version": 3, "strides": None}
    with torch.cuda.device(device):
        return torch.as_tensor(_Cai(), device=device)


def launch_paged_attn_decode(pool: KvPool, layer: int, q, block_table, seq_lens, o,
                             scale: float | None = None):
    """Name and argument order of the reference launcher
    (kernels/attention/flash_attention.bm:180-189); scale defaults to
    1/sqrt(head_dim) as there (:187)."""
    return pool.paged_decode(layer, q, block_table, seq_lens, o,
                             scale=0.0 if scale is None else scale)


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


# ---- FP8 weight path (kernels/norm/rms_norm.bm:62-94, kernels/gemm/gemm_fp8.bm:31-107) ----

def rms_norm_fp8_out(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, scale: float,
                     eps: float = 1e-5, stream=None) -> torch.Tensor:
    """E4M3 codes of RMSNorm(x) * weight * scale: x f16 [rows][hidden], weight f16
    [hidden], out uint8 [rows][hidden] (the reference encoder; bit-exact)."""
    rows, hidden = x.shape
    C.check(C.lib().vw_rms_norm_fp8_out(_ptr(x), _ptr(weight), _ptr(out), rows, hidden, scale, eps,
                                        _stream(stream)))
    return out


def gemm_fp8(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, bias=None, a_scale: float = 1.0,
             b_scale: float = 1.0, stream=None) -> torch.Tensor:
    """C = (a_scale * b_scale) * (A . B) + bias: A uint8 [M][K], B uint8 [K][N] E4M3
    codes (the reference decoder), bias bf16 [N] or None, out bf16 [M][N]."""
    M, K = a.shape
    N = b.shape[1]
    C.check(C.lib().vw_gemm_fp8(_ptr(a), _ptr(b), _ptr(out), _ptr(bias), M, N, K, a_scale, b_scale,
                                _stream(stream)))
    return out


def fp8_weight_check() -> int:
    """Synchronise; return (and clear) the device error word of the two calls above."""
    w = ctypes.c_uint32(0)
    rc = C.lib().vw_fp8_weight_check(ctypes.byref(w))
    if rc not in (C.VW_OK, C.VW_ERR_DEVICE_CHECK):
        C.check(rc)
    return int(w.value)
