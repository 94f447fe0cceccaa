"""Python mirror of the engine's kernel-library bridge (engine/ffi.bm).

``KernelLib.open(path)`` dlopens the library with RTLD_NOW and binds
``voidweb_forward_pass`` exactly as engine/ffi.bm:61-77 does; a missing
library or symbol is an error at open time (ffi.bm:64-73).  ``forward_pass``
packs the descriptors (ffi.bm:15-40, scheduler/scheduler.bm:134-170) and turns
a nonzero return code into an error (ffi.bm:112-118).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _lib as C

RTLD_NOW = 2


class KernelLib:
    def __init__(self, handle: ctypes.CDLL, fn):
        self._handle = handle
        self._forward = fn

    @classmethod
    def open(cls, path: str | None = None) -> "KernelLib":
        path = path or C.build()
        if not os.path.exists(path):
            raise OSError(f"dlopen failed for {path}")
        h = ctypes.CDLL(path, mode=RTLD_NOW)
        try:
            fn = h.voidweb_forward_pass
        except AttributeError as e:
            raise OSError(f"voidweb_forward_pass not found in {path}") from e
        fn.restype = ctypes.c_int32
        fn.argtypes = [ctypes.POINTER(C.ForwardArgs)]
        return cls(h, fn)

    def close(self) -> None:
        self._handle = None
        self._forward = None

    def forward_pass(self, cfg: dict, decode_seqs, vocab_size: int = 1,
                     prefill_seqs=()) -> np.ndarray:
        """decode_seqs: list of (seq_id, last_token, block_table) like DecodeSeq
        (scheduler/scheduler.bm:112-116); prefill_seqs: list of (seq_id,
        chunk_tokens, block_table) like PrefillSeq (:106-110).  Descriptors are
        built as build_seq_descriptors does (:134-170): prefill chunks first
        (is_prefill 1, num_tokens = chunk length), then decodes (num_tokens 1).
        cfg: num_heads, num_kv_heads, num_layers, head_dim, hidden_size,
        rope_theta, quant_type.  Returns the logits buffer [num_seqs *
        vocab_size] (ffi.bm:94); this library fills the bound attention outputs,
        not logits."""
        entries = [(sid, np.ascontiguousarray(toks, dtype=np.uint32), bt, 1)
                   for (sid, toks, bt) in prefill_seqs]
        entries += [(sid, np.array([t], dtype=np.uint32), bt, 0) for (sid, t, bt) in decode_seqs]
        n = len(entries)
        tok_storage = [e[1] for e in entries]
        blk_storage = [np.ascontiguousarray(e[2], dtype=np.uint32) for e in entries]
        descs = (C.SeqDescriptor * max(n, 1))()
        for i, (sid, toks, _, is_pf) in enumerate(entries):
            descs[i] = C.SeqDescriptor(sid, tok_storage[i].ctypes.data, toks.size,
                                       blk_storage[i].ctypes.data, blk_storage[i].size, is_pf)
        logits = np.zeros(n * vocab_size, dtype=np.float32)
        args = C.ForwardArgs(ctypes.cast(descs, ctypes.c_void_p), n, cfg.get("hidden_size", 0),
                             cfg["num_heads"], cfg["num_kv_heads"], cfg["num_layers"], vocab_size,
                             cfg["head_dim"], cfg.get("rope_theta", 10000.0),
                             cfg.get("quant_type", 0), logits.ctypes.data)
        rc = self._forward(ctypes.byref(args))
        if rc != 0:
            raise RuntimeError(f"GPU forward pass failed with code {rc}: "
                               f"{C.lib().vw_last_error().decode(errors='replace')}")
        return logits
