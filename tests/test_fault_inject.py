"""Host-side failure injection (vw_fault_inject / VOIDWEB_KV_FAULT): the
engine's error paths -- a nonzero voidweb_forward_pass status becomes a failed
step (engine/ffi.bm:112-118), an exhausted block pool an allocation error
(engine/kv_cache.bm:82-85) -- tested without a GPU and without faulting one.
Every injected failure returns before the call touches the device or the
bookkeeping, so these run on CPU."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

from voidweb_b200 import _lib as C

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def disarm():
    L = C.lib()
    for k in (C.VW_FAULT_OOM, C.VW_FAULT_INVALID_ARG, C.VW_FAULT_CUDA):
        L.vw_fault_inject(k, 0)
    yield
    for k in (C.VW_FAULT_OOM, C.VW_FAULT_INVALID_ARG, C.VW_FAULT_CUDA):
        L.vw_fault_inject(k, 0)


def test_injected_oom_on_pool_create_and_block_manager():
    L = C.lib()
    assert L.vw_fault_inject(C.VW_FAULT_OOM, 1) == C.VW_OK
    cfg = C.PoolConfig(1, 1, 128, 16, C.VW_BF16, C.VW_BF16, 0, 1, 0, 0, None, None)
    h = ctypes.c_void_p()
    assert L.vw_pool_create(ctypes.byref(cfg), ctypes.byref(h)) == C.VW_ERR_OOM
    assert b"injected" in L.vw_last_error()
    assert not h.value and L.vw_fault_pending(C.VW_FAULT_OOM) == 0

    bm = ctypes.c_void_p()
    assert L.vw_bm_create(16, 8, ctypes.byref(bm)) == C.VW_OK
    L.vw_fault_inject(C.VW_FAULT_OOM, 2)
    one = ctypes.c_uint32()
    assert L.vw_bm_alloc(bm, ctypes.byref(one)) == C.VW_ERR_OOM
    ids = (ctypes.c_uint32 * 3)()
    assert L.vw_bm_alloc_seq(bm, 3, ids) == C.VW_ERR_OOM
    # all or nothing, as kv_cache.bm:82-85: nothing was taken
    assert L.vw_bm_free_count(bm) == 8
    assert L.vw_fault_pending(C.VW_FAULT_OOM) == 0
    # disarmed: the LIFO pop of kv_cache.bm:69-78 again
    assert L.vw_bm_alloc_seq(bm, 3, ids) == C.VW_OK and list(ids) == [7, 6, 5]
    # copy-on-write needs a fresh block only for a shared one
    L.vw_bm_incref(bm, 7)
    table = (ctypes.c_uint32 * 3)(7, 6, 5)
    pair = (ctypes.c_uint32 * 2)()
    copied = ctypes.c_uint32()
    L.vw_fault_inject(C.VW_FAULT_OOM, 1)
    assert L.vw_bm_cow(bm, table, 1, pair, ctypes.byref(copied)) == C.VW_OK and copied.value == 0
    assert L.vw_fault_pending(C.VW_FAULT_OOM) == 1
    assert L.vw_bm_cow(bm, table, 0, pair, ctypes.byref(copied)) == C.VW_ERR_OOM
    assert table[0] == 7 and L.vw_bm_ref_count(bm, 7) == 2
    assert L.vw_bm_cow(bm, table, 0, pair, ctypes.byref(copied)) == C.VW_OK and copied.value == 1
    L.vw_bm_destroy(bm)


def test_injected_launch_failures_return_before_any_device_work():
    L = C.lib()
    a = C.DecodeArgs()
    L.vw_fault_inject(C.VW_FAULT_CUDA, 2)
    # a null pool would be rejected as an invalid argument; the armed failure wins
    assert L.vw_paged_decode(None, ctypes.byref(a), None) == C.VW_ERR_CUDA
    assert L.vw_block_copy(None, None, 1, None) == C.VW_ERR_CUDA
    assert L.vw_paged_decode(None, ctypes.byref(a), None) == C.VW_ERR_INVALID_ARG
    L.vw_fault_inject(C.VW_FAULT_INVALID_ARG, 1)
    assert L.vw_kv_append(None, 0, None, None, None, 0, None) == C.VW_ERR_INVALID_ARG
    assert b"injected" in L.vw_last_error()
    # an OOM is not a failure a launch-only call can have: it stays armed
    L.vw_fault_inject(C.VW_FAULT_OOM, 1)
    assert L.vw_kv_gather(None, 0, None, 0, None, None, None, None, None) == C.VW_ERR_INVALID_ARG
    assert L.vw_fault_pending(C.VW_FAULT_OOM) == 1


def test_forward_pass_failure_reaches_the_engine_as_an_error():
    """KernelLib.forward_pass (the engine's bridge) turns the nonzero status
    into an error, as engine/ffi.bm:112-118 does, for each injected kind."""
    from voidweb_b200 import KernelLib
    kl = KernelLib.open(C.LIB_PATH)
    cfg = dict(num_heads=8, num_kv_heads=2, num_layers=1, head_dim=128)
    for kind, rc in ((C.VW_FAULT_OOM, C.VW_ERR_OOM), (C.VW_FAULT_INVALID_ARG, C.VW_ERR_INVALID_ARG),
                     (C.VW_FAULT_CUDA, C.VW_ERR_CUDA)):
        C.lib().vw_fault_inject(kind, 1)
        with pytest.raises(RuntimeError, match=f"failed with code {rc}.*injected"):
            kl.forward_pass(cfg, [(1, 5, np.array([0], dtype=np.uint32))])
        assert C.lib().vw_fault_pending(kind) == 0


def test_environment_arms_faults_at_load():
    code = ("from voidweb_b200 import _lib as C; L = C.lib(); "
            "print(L.vw_fault_pending(1), L.vw_fault_pending(2), L.vw_fault_pending(3))")
    env = dict(os.environ, VOIDWEB_KV_FAULT="oom:2,cuda:5, invalid:1")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True,
                         text=True, check=True).stdout.split()
    assert out == ["2", "1", "5"]
