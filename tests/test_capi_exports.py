"""The C ABI library loads and exports every entry point include/b2f.h declares.

No kernel is launched here (the host-only size helpers are called).
"""

import ctypes
import os
import re

from conftest import ROOT

from oracle import kv_sym

HEADER = os.path.join(ROOT, "include", "b2f.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b2f_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from b200flash import _capi

    names = declared_functions()
    assert len(names) >= 15
    handle = ctypes.CDLL(_capi.LIB_PATH)
    missing = [n for n in names if not hasattr(handle, n)]
    assert not missing, missing
    assert set(names) == set(_capi.SIGNATURES), set(names) ^ set(_capi.SIGNATURES)


def test_host_helpers():
    from b200flash import _capi

    L = _capi.lib()
    assert b"sm_100a" in L.b2f_version()
    assert L.b2f_status_string(-2) == b"unsupported bits/group_size/dtype/size"
    for D in (1, 7, 64, 100, 128, 200):
        for bits in (2, 4, 8):
            for gs in (3, 32, 64, 256):
                assert L.b2f_kv_packed_len(D, bits, gs) == kv_sym.packed_len(D, bits, gs)
                assert L.b2f_kv_num_groups(D, gs) == kv_sym.num_groups(D, gs)
    assert L.b2f_moe_plan_workspace_bytes(512, 128, 16) > 512 * 4
    assert L.b2f_moe_plan_max_slots(512, 128, 16) >= 128
