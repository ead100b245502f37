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


def test_new_entry_points_reject_bad_arguments():
    """Argument checks of the batch-norm, SwiGLU, column-sum, fused-update,
    ragged, phased and exchange entry points come before any device work."""
    L = _native.lib()
    fake = ctypes.c_void_p(256)
    c_d = ctypes.c_double
    # batch norm: unsupported dtype, channels not a multiple of 8
    assert L.pkm_batchnorm_fwd(fake, 7, 4, 16, None, None, 0, None, None, 0, 1, c_d(0.1), c_d(1e-6), fake, fake,
                               fake, None, 0, None) == 2
    assert L.pkm_batchnorm_fwd(fake, 0, 4, 12, None, None, 0, None, None, 0, 1, c_d(0.1), c_d(1e-6), fake, fake,
                               fake, None, 0, None) == 2
    assert L.pkm_batchnorm_bwd(fake, fake, 1, 0, 16, fake, fake, None, 0, fake, None, None, None, 0, None) == 1
    # SwiGLU and column sums
    assert L.pkm_swiglu_fwd(fake, fake, 1, 4, 12, fake, None) == 2
    assert L.pkm_colsum(fake, 1, -1, 16, fake, 1, None, 0, None) == 1
    # fused fast-weight update: bad dtype, negative rows
    assert L.pkm_fw_update(fake, fake, 2, 4, 16, None, 0, c_d(1), c_d(0.1), c_d(0), 1, fake, None, fake, None,
                           None) == 2
    assert L.pkm_fw_update(fake, fake, 0, -4, 16, None, 0, c_d(1), c_d(0.1), c_d(0), 1, fake, None, fake, None,
                           None) == 1
    # ragged segment sum: negative sizes
    assert L.pkm_segment_sum(fake, 0, 10, 16, fake, fake, -1, fake, 2, fake, 0, None, 0, None, None) == 1
    # phased backward: row range outside the table
    assert L.pkm_bag_bwd_rows(fake, fake, 0, fake, 0, fake, 4, 2, 10, 16, 5, 11, fake, 0, None, 0, fake, 1 << 20,
                              None, None) == 1
    # exchange: world above one NVLink domain, shard rows not covering the table
    ptrs = (ctypes.c_void_p * 9)(*([fake] * 9))
    assert L.pkm_grad_shard_reduce(fake, 1, 100, 16, 9, 0, 12, ptrs, ctypes.c_float(1.0), 0, None) == 1
    assert L.pkm_grad_shard_reduce(fake, 1, 100, 16, 2, 0, 12, ptrs, ctypes.c_float(1.0), 0, None) == 1
    assert L.pkm_grad_multimem_allreduce(fake, fake, 1, 100, 16, 2, 3, 50, 0, -1, ctypes.c_float(1.0), 0,
                                         None) == 1
    # zero-size work is a no-op without a device
    assert L.pkm_segment_sum(None, 0, 10, 16, None, None, 0, None, 0, None, 0, None, 0, None, None) == 0
    assert L.pkm_fw_update(None, None, 0, 0, 16, None, 0, c_d(1), c_d(0.1), c_d(0), 1, None, None, None, None,
                           None) == 0


def test_score_transform_rejects_bad_arguments():
    """The FwPKM score transform checks width, mode, temperature and dtype
    before any device work."""
    L = _native.lib()
    fake = ctypes.c_void_p(256)
    c_d = ctypes.c_double
    assert L.pkm_score_transform_fwd(fake, 0, 4, 513, c_d(1.0), 0, fake, None) == 2   # wider than 512
    assert L.pkm_score_transform_fwd(fake, 0, 4, 128, c_d(1.0), 3, fake, None) == 1   # unknown mode
    assert L.pkm_score_transform_fwd(fake, 0, 4, 128, c_d(0.0), 0, fake, None) == 1   # temperature 0
    assert L.pkm_score_transform_fwd(fake, 9, 4, 128, c_d(1.0), 0, fake, None) == 1   # dtype
    assert L.pkm_score_transform_bwd(fake, None, fake, 0, 4, 128, c_d(1.0), 0, fake, None) == 1  # softmax needs out
    assert L.pkm_score_transform_fwd(None, 0, 0, 128, c_d(1.0), 0, None, None) == 0   # empty
