"""Continuous-batching scheduler wired to the KV block bookkeeping: the Python
face of vw_sched_* (scheduler/scheduler.bm:186-326, engine/engine.bm:127-146).

``schedule()`` returns the step's sequences in descriptor order (prefill chunks
first, scheduler.bm:134-170) with their input tokens, the first token's
position (``ctx_start``, the tokens already cached), block tables covering the
positions written, and the (src, dst) block copies to run before the step;
``commit()`` takes the tokens sampled for the sequences with ``samples``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib as C


@dataclass
class StepSeq:
    seq_id: int
    is_prefill: bool
    ctx_start: int
    tokens: np.ndarray          # uint32 [num_tokens]
    table: np.ndarray           # uint32 [pages covering ctx_start + num_tokens]
    samples: bool


@dataclass
class StepBatch:
    seqs: list
    copies: np.ndarray          # uint32 [n][2]
    table_stride: int


class Scheduler:
    def __init__(self, block_manager, max_batch_tokens: int = 8192, max_running_seqs: int = 256,
                 max_chunk: int = 2048, max_seq_len: int = 1 << 20, prefix_cache: bool = True):
        self.bm = block_manager                  # kept alive: the scheduler calls into it
        cfg = C.SchedConfig(max_batch_tokens, max_running_seqs, max_chunk, max_seq_len,
                            1 if prefix_cache else 0, 0)
        h = ctypes.c_void_p()
        C.check(C.lib().vw_sched_create(ctypes.byref(cfg), block_manager._h, ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            C.lib().vw_sched_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def add_request(self, prompt, max_new_tokens: int, stop_token: int | None = None) -> int:
        a = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = ctypes.c_uint64()
        C.check(C.lib().vw_sched_add_request(self._h, ctypes.c_void_p(a.ctypes.data), a.size,
                                             max_new_tokens, -1 if stop_token is None else stop_token,
                                             ctypes.byref(out)))
        return int(out.value)

    def schedule(self) -> StepBatch:
        b = C.SchedBatch()
        C.check(C.lib().vw_sched_schedule(self._h, ctypes.byref(b)))
        seqs = []
        for k in range(b.num_seqs):
            q = b.seqs[k]
            toks = np.ctypeslib.as_array(b.tokens, shape=(q.token_offset + q.num_tokens,))[
                q.token_offset:].copy() if q.num_tokens else np.zeros(0, np.uint32)
            row = np.ctypeslib.as_array(b.block_tables, shape=((k + 1) * b.table_stride,))[
                k * b.table_stride:(k + 1) * b.table_stride]
            pages = (q.ctx_start + q.num_tokens + 15) // 16
            seqs.append(StepSeq(int(q.seq_id), bool(q.is_prefill), int(q.ctx_start), toks,
                                row[:pages].copy(), bool(q.samples)))
        copies = (np.ctypeslib.as_array(b.copies, shape=(2 * b.num_copies,)).reshape(-1, 2).copy()
                  if b.num_copies else np.zeros((0, 2), np.uint32))
        return StepBatch(seqs, copies, int(b.table_stride))

    def commit(self, sampled: dict) -> None:
        ids = np.array(list(sampled.keys()), dtype=np.uint64)
        toks = np.array(list(sampled.values()), dtype=np.uint32)
        C.check(C.lib().vw_sched_commit(self._h, ctypes.c_void_p(ids.ctypes.data),
                                        ctypes.c_void_p(toks.ctypes.data), ids.size))

    def take_finished(self) -> list:
        out = []
        buf = np.zeros(1 << 16, dtype=np.uint32)
        while True:
            rid, n = ctypes.c_uint64(), ctypes.c_uint32()
            if C.lib().vw_sched_take_finished(self._h, ctypes.byref(rid),
                                              ctypes.c_void_p(buf.ctypes.data), buf.size,
                                              ctypes.byref(n)) != C.VW_OK:
                return out
            out.append((int(rid.value), buf[:n.value].copy()))

    def stats(self) -> dict:
        st = C.SchedStat()
        C.check(C.lib().vw_sched_stats(self._h, ctypes.byref(st)))
        return {k: getattr(st, k) for k, _ in C.SchedStat._fields_ if k != "reserved"}
