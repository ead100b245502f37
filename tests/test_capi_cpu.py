"""CPU-side checks of the C-ABI library: it loads, exports every entry point
that ``include/pkm_b200.h`` declares, and rejects bad arguments before any
launch (no GPU needed for any of this)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from modelos_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"PKM_API\s+[\w\s\*]+?\b(pkm_\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    L = _native.lib()
    decl = declared_symbols()
    assert decl, "no declarations found"
    for name in decl:
        assert hasattr(L, name), name
    assert decl == set(_native.EXPORTED)


def test_version_and_status_strings():
    L = _native.lib()
    assert L.pkm_version() >= 100
    assert L.pkm_status_string(0) == b"ok"
    assert L.pkm_status_string(1) == b"invalid argument"


def test_argument_errors_are_reported_before_launch():
    L = _native.lib()
    # negative sizes -> invalid argument; no pointer is touched
    rc = L.pkm_bag_fwd(None, None, 0, None, 0, -1, 4, 8, 16, None, 0, None, None)
    assert rc == 1 and b"negative" in L.pkm_last_error()
    # rows that are not 16-byte multiples are unsupported
    fake = ctypes.c_void_p(256)  # never dereferenced: the check comes first
    rc = L.pkm_bag_fwd(fake, None, 0, fake, 0, 1, 1, 8, 3, fake, 0, None, None)
    assert rc == 2 and b"multiple of 16" in L.pkm_last_error()
    # knn above 32
    rc = L.pkm_product_topk(None, 0, 4, 64, 33, None, None, None, None, None, None)
    assert rc == 1
    # zero-size work is a no-op that needs no device
    assert L.pkm_bag_fwd(None, None, 0, None, 0, 0, 4, 8, 16, None, 0, None, None) == 0
    assert L.pkm_product_topk(None, 0, 0, 64, 32, None, None, None, None, None, None) == 0


def test_workspace_query():
    n = _native.bag_bwd_workspace(16384, 128, 262144, 1024)
    assert n > 0 and n % 256 == 0
    assert _native.bag_bwd_workspace(0, 128, 16, 16) > 0


def test_cpu_tensors_are_rejected():
    import torch
    idx = torch.zeros(2, 3, dtype=torch.long)
    w = torch.zeros(4, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        _native.bag_fwd(idx, w, None)
