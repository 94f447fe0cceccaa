"""The C-ABI library loads and exports every symbol include/voidweb_kv.h
declares; the packed engine structs have the reference's sizes.  CPU only:
no kernel is launched."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from voidweb_b200 import _lib as C

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "voidweb_kv.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^VW_API [^(]*?\b(\w+)\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    L = C.lib()
    names = declared_symbols()
    assert "voidweb_forward_pass" in names and "vw_paged_decode" in names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    nm = subprocess.run(["nm", "-D", "--defined-only", C.LIB_PATH], capture_output=True,
                        text=True, check=True).stdout
    exported = set(re.findall(r" T (\w+)$", nm, flags=re.M))
    assert set(names) <= exported
    # the Python binding declares exactly the header's surface
    assert set(C.SIGNATURES) == set(names)


def test_packed_struct_sizes_match_engine():
    # engine/ffi.bm:15-40 (#[repr(C)] #[packed]): 8+8+4+8+4+1 and 8+4*7+4+4+8
    assert ctypes.sizeof(C.SeqDescriptor) == 33
    assert ctypes.sizeof(C.ForwardArgs) == 52
    code = r'''
#include "voidweb_kv.h"
#include <stddef.h>
_Static_assert(sizeof(SeqDescriptor) == 33, "SeqDescriptor");
_Static_assert(sizeof(ForwardArgs) == 52, "ForwardArgs");
_Static_assert(offsetof(ForwardArgs, logits_out) == 44, "logits_out");
_Static_assert(sizeof(vw_decode_args) == 80, "vw_decode_args");
_Static_assert(sizeof(vw_pool_config) == 56, "vw_pool_config");
_Static_assert(sizeof(vw_prefill_args) == 88, "vw_prefill_args");
_Static_assert(offsetof(vw_prefill_args, q) == 24, "vw_prefill_args.q");
int main(void) { return 0; }
'''
    with tempfile.TemporaryDirectory() as d:
        f = os.path.join(d, "t.c")
        open(f, "w").write(code)
        subprocess.run(["gcc", "-std=c11", "-I", os.path.dirname(HEADER), f, "-o",
                        os.path.join(d, "t")], check=True)
    assert ctypes.sizeof(C.DecodeArgs) == 80
    assert ctypes.sizeof(C.PoolConfig) == 56
    assert ctypes.sizeof(C.PrefillArgs) == 88
    assert C.PrefillArgs.q.offset == 24


def test_errors_cross_the_boundary_as_codes():
    L = C.lib()
    # null config -> invalid argument, with a message; no exception, no crash
    assert L.vw_pool_create(None, None) == C.VW_ERR_INVALID_ARG
    assert b"null" in L.vw_last_error()
    cfg = C.PoolConfig(1, 2, 96, 8, C.VW_BF16, C.VW_BF16, 0, 8, 0, 0, None, None)
    h = ctypes.c_void_p()
    assert L.vw_pool_create(ctypes.byref(cfg), ctypes.byref(h)) == C.VW_ERR_UNSUPPORTED
    cfg = C.PoolConfig(1, 2, 128, 8, C.VW_BF16, C.VW_F16, 0, 8, 0, 0, None, None)
    assert L.vw_pool_create(ctypes.byref(cfg), ctypes.byref(h)) == C.VW_ERR_INVALID_ARG
    assert L.vw_paged_decode(None, None, None) == C.VW_ERR_INVALID_ARG
    assert L.vw_paged_prefill(None, None, None) == C.VW_ERR_INVALID_ARG
    # the forward-pass symbol refuses to run without a bound pool
    args = C.ForwardArgs()
    assert L.voidweb_forward_pass(ctypes.byref(args)) != 0


def test_kernel_lib_open_mirrors_engine():
    from voidweb_b200 import KernelLib
    kl = KernelLib.open(C.LIB_PATH)
    kl.close()
    with pytest.raises(OSError):
        KernelLib.open("/nonexistent/libkernels.so")
