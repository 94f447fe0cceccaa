"""ctypes binding of libvoidweb_kv.so (the C ABI in include/voidweb_kv.h).

The shared library is the product: every operation of this package runs its
CUDA kernels or its C++ host code.  There is no Python or CPU fallback; if
the library is missing or fails to load, importing an operation raises.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
# VOIDWEB_KV_LIB selects another build of the same library (e.g. one compiled
# with different tile parameters); by default the in-tree build is used.
LIB_PATH = os.environ.get("VOIDWEB_KV_LIB") or os.path.join(_HERE, "libvoidweb_kv.so")
CSRC = os.path.join(_HERE, "csrc")

VW_OK = 0
VW_ERR_INVALID_ARG = 1
VW_ERR_UNSUPPORTED = 2
VW_ERR_CUDA = 3
VW_ERR_OOM = 4
VW_ERR_DEVICE_CHECK = 5
# device error word bits (vw_pool_check)
VW_DEV_ERR_BLOCK_ID, VW_DEV_ERR_SEQ_LEN, VW_DEV_ERR_TIMEOUT, VW_DEV_ERR_SLOT = 0x1, 0x2, 0x4, 0x8
VW_DEV_ERR_LAUNCH = 0x10

VW_F16, VW_BF16, VW_FP8_E4M3 = 0, 1, 2
VW_FP8_REFERENCE, VW_FP8_OCP = 0, 1
VW_DECODE_PDL, VW_DECODE_EARLY_PAGES, VW_DECODE_PLANNED, VW_DECODE_ROPE = 0x1, 0x2, 0x4, 0x8
VW_PREFILL_CAUSAL, VW_PREFILL_ROPE, VW_PREFILL_PDL = 0x1, 0x2, 0x4
VW_FAULT_OOM, VW_FAULT_INVALID_ARG, VW_FAULT_CUDA = 1, 2, 3

DEV_ERR_BLOCK_ID, DEV_ERR_SEQ_LEN, DEV_ERR_TIMEOUT, DEV_ERR_SLOT = 1, 2, 4, 8

u8, u32, u64, i32, i64, f32 = (ctypes.c_uint8, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32,
                               ctypes.c_int64, ctypes.c_float)
vp = ctypes.c_void_p


class PoolConfig(ctypes.Structure):
    _fields_ = [("num_layers", u32), ("num_kv_heads", u32), ("head_dim", u32),
                ("num_blocks", u32), ("kv_dtype", u32), ("io_dtype", u32), ("fp8_mode", u32),
                ("max_batch", u32), ("device", i32), ("reserved", u32), ("kv_data", vp),
                ("kv_scales", vp)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [("layer", u32), ("num_seqs", u32), ("num_q_heads", u32),
                ("block_table_stride", u32), ("q", vp), ("block_tables", vp), ("seq_lens", vp),
                ("out", vp), ("k_new", vp), ("v_new", vp), ("scale", f32), ("flags", u32),
                ("rope_theta", f32), ("reserved", u32)]


class StepHostArgs(ctypes.Structure):
    _fields_ = [("num_seqs", u32), ("num_q_heads", u32), ("block_table_stride", u32),
                ("reserved", u32), ("q", vp), ("k_new", vp), ("v_new", vp),
                ("block_tables", vp), ("seq_lens", vp), ("out", vp), ("scale", f32),
                ("rope_theta", f32)]


class PrefillArgs(ctypes.Structure):
    _fields_ = [("layer", u32), ("num_seqs", u32), ("num_tokens", u32), ("num_q_heads", u32),
                ("block_table_stride", u32), ("flags", u32), ("q", vp), ("k_new", vp),
                ("v_new", vp), ("cu_seqlens", vp), ("ctx_start", vp), ("block_tables", vp),
                ("out", vp), ("scale", f32), ("rope_theta", f32)]


class SchedConfig(ctypes.Structure):
    _fields_ = [("max_batch_tokens", u32), ("max_running_seqs", u32), ("max_chunk", u32),
                ("max_seq_len", u32), ("prefix_cache", u32), ("reserved", u32)]


class SchedSeq(ctypes.Structure):
    _fields_ = [("seq_id", u64), ("is_prefill", u32), ("num_tokens", u32), ("ctx_start", u32),
                ("samples", u32), ("token_offset", u32), ("reserved", u32)]


class SchedBatch(ctypes.Structure):
    _fields_ = [("num_seqs", u32), ("table_stride", u32), ("seqs", ctypes.POINTER(SchedSeq)),
                ("tokens", ctypes.POINTER(u32)), ("block_tables", ctypes.POINTER(u32)),
                ("num_copies", u32), ("reserved", u32), ("copies", ctypes.POINTER(u32))]


class SchedStat(ctypes.Structure):
    _fields_ = [("waiting", u32), ("running", u32), ("finished", u32), ("cached_pages", u32),
                ("table_refs", u32), ("free_blocks", u32), ("preemptions", u32), ("reserved", u32)]


class SeqDescriptor(ctypes.Structure):
    """engine/ffi.bm:15-24 (#[repr(C)] #[packed], 33 bytes)."""
    _pack_ = 1
    _fields_ = [("seq_id", u64), ("token_ptr", u64), ("num_tokens", u32), ("block_ptr", u64),
                ("num_blocks", u32), ("is_prefill", u8)]


class ForwardArgs(ctypes.Structure):
    """engine/ffi.bm:26-40 (#[repr(C)] #[packed], 52 bytes)."""
    _pack_ = 1
    _fields_ = [("seqs", vp), ("num_seqs", u32), ("hidden_size", u32), ("num_heads", u32),
                ("num_kv_heads", u32), ("num_layers", u32), ("vocab_size", u32),
                ("head_dim", u32), ("rope_theta", f32), ("quant_type", u32),
                ("logits_out", vp)]


# name -> (restype, argtypes); mirrors include/voidweb_kv.h line by line
SIGNATURES = {
    "vw_pool_create": (i32, [ctypes.POINTER(PoolConfig), ctypes.POINTER(vp)]),
    "vw_pool_destroy": (i32, [vp]),
    "vw_pool_info": (i32, [vp, ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(u64),
                           ctypes.POINTER(u64)]),
    "vw_pool_check": (i32, [vp, ctypes.POINTER(u32)]),
    "vw_kv_append": (i32, [vp, u32, vp, vp, vp, u32, vp]),
    "vw_paged_decode": (i32, [vp, ctypes.POINTER(DecodeArgs), vp]),
    "vw_paged_prefill": (i32, [vp, ctypes.POINTER(PrefillArgs), vp]),
    "vw_rms_norm_fp8_out": (i32, [vp, vp, vp, u32, u32, f32, f32, vp]),
    "vw_gemm_fp8": (i32, [vp, vp, vp, vp, u32, u32, u32, f32, f32, vp]),
    "vw_fp8_weight_check": (i32, [ctypes.POINTER(u32)]),
    "vw_sched_create": (i32, [ctypes.POINTER(SchedConfig), vp, ctypes.POINTER(vp)]),
    "vw_sched_destroy": (i32, [vp]),
    "vw_sched_add_request": (i32, [vp, vp, u32, u32, ctypes.c_int64, ctypes.POINTER(u64)]),
    "vw_sched_schedule": (i32, [vp, ctypes.POINTER(SchedBatch)]),
    "vw_sched_commit": (i32, [vp, vp, vp, u32]),
    "vw_sched_take_finished": (i32, [vp, ctypes.POINTER(u64), vp, u32, ctypes.POINTER(u32)]),
    "vw_sched_stats": (i32, [vp, ctypes.POINTER(SchedStat)]),
    "vw_decode_plan": (i32, [vp, vp, vp, u32, u32, u32, vp]),
    "vw_paged_decode_static": (i32, [vp, ctypes.POINTER(DecodeArgs), vp]),
    "vw_block_copy": (i32, [vp, vp, u32, vp]),
    "vw_kv_gather": (i32, [vp, u32, vp, u32, vp, vp, vp, vp, vp]),
    "vw_decode_step_host": (i32, [vp, ctypes.POINTER(StepHostArgs), vp]),
    "vw_bm_create": (i32, [u32, u32, ctypes.POINTER(vp)]),
    "vw_bm_destroy": (i32, [vp]),
    "vw_bm_capacity": (u32, [vp]),
    "vw_bm_free_count": (u32, [vp]),
    "vw_bm_alloc": (i32, [vp, ctypes.POINTER(u32)]),
    "vw_bm_alloc_seq": (i32, [vp, u32, vp]),
    "vw_bm_incref": (None, [vp, u32]),
    "vw_bm_decref": (None, [vp, u32]),
    "vw_bm_free_seq": (None, [vp, vp, u32]),
    "vw_bm_ref_count": (u32, [vp, u32]),
    "vw_bm_prefix_lookup": (u32, [vp, vp, u32, vp, u32]),
    "vw_bm_register_prefix_block": (None, [vp, u32, u64]),
    "vw_rolling_hash": (u64, [u64, vp, u32]),
    "vw_bm_free_list": (u32, [vp, vp, u32]),
    "vw_bm_cow": (i32, [vp, vp, u32, vp, vp]),
    "vw_bm_compact": (u32, [vp, vp, u32]),
    "vw_radix_create": (i32, [u32, u32, ctypes.POINTER(vp)]),
    "vw_radix_destroy": (i32, [vp]),
    "vw_radix_lookup": (u32, [vp, vp, u32, ctypes.POINTER(u32), vp, u32]),
    "vw_radix_insert": (u32, [vp, vp, u32, vp, u32, vp, u32]),
    "vw_radix_evict_lru": (u32, [vp, u32, vp, u32]),
    "vw_radix_total_blocks": (u32, [vp]),
    "vw_radix_lock": (None, [vp, vp, u32]),
    "vw_radix_unlock": (None, [vp, vp, u32]),
    "vw_radix_remap": (None, [vp, vp, u32]),
    "vw_last_error": (ctypes.c_char_p, []),
    "vw_forward_bind": (i32, [vp, vp, vp, vp, vp]),
    "vw_forward_set_seq_len": (i32, [u64, u32]),
    "vw_forward_release": (i32, [u64]),
    "voidweb_forward_pass": (i32, [ctypes.POINTER(ForwardArgs)]),
    "vw_fault_inject": (i32, [u32, u32]),
    "vw_fault_pending": (u32, [u32]),
    "vw_debug_set_wait_limit": (i32, [vp, u64]),
    "vw_debug_alloc_count": (u64, []),
}


def build(force: bool = False) -> str:
    """Compile libvoidweb_kv.so for sm_100a with nvcc (csrc/Makefile)."""
    if force or not os.path.exists(LIB_PATH) or _stale():
        subprocess.check_call(["make", "-s", "-C", CSRC])
    return LIB_PATH


def _stale() -> bool:
    t = os.path.getmtime(LIB_PATH)
    for f in os.listdir(CSRC):
        if os.path.getmtime(os.path.join(CSRC, f)) > t:
            return True
    hdr = os.path.join(os.path.dirname(_HERE), "include", "voidweb_kv.h")
    return os.path.exists(hdr) and os.path.getmtime(hdr) > t


_lib = None


def lib() -> ctypes.CDLL:
    """Load the library (building it if the sources are newer); raise if absent."""
    global _lib
    if _lib is None:
        if not os.environ.get("VOIDWEB_KV_LIB") and (not os.path.exists(LIB_PATH) or _stale()):
            try:
                build()
            except Exception as e:  # no silent fallback: the product path needs the .so
                raise ImportError(f"libvoidweb_kv.so missing and could not be built: {e}") from e
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class VoidwebError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != VW_OK:
        msg = lib().vw_last_error().decode(errors="replace")
        if rc == VW_ERR_OOM:
            raise MemoryError(msg)
        raise VoidwebError(rc, msg)
