"""The allocation-free backward entry point (pkm_bag_bwd_noalloc).

It serves callers that cannot allocate device memory, for example an FFI
binding without a device allocator of its own, or a latency-critical loop in
which a cudaMalloc (which may synchronise the device) is not allowed: its
scratch is a fixed 16 MiB device array inside the library.  This file is
collected last so that a run which stops at the first failure has already
run every other test.  The test calls the entry point through the C ABI twice
in a row (the array keeps the previous call's contents) and compares both
results with the workspace entry point, pkm_bag_bwd.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import cases

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _call_noalloc(L, idx, psw, W, g, gw, gp, counts, err, dt):
    from modelos_b200 import _native
    B, Lb = idx.shape
    K, D = W.shape
    return L.pkm_bag_bwd_noalloc(
        ctypes.c_void_p(idx.data_ptr()), ctypes.c_void_p(psw.data_ptr()), _native.DT[psw.dtype],
        ctypes.c_void_p(W.data_ptr()), _native.DT[W.dtype], ctypes.c_void_p(g.data_ptr()), B, Lb, K, D,
        ctypes.c_void_p(gw.data_ptr()), _native.DT[gw.dtype], ctypes.c_void_p(gp.data_ptr()),
        _native.DT[gp.dtype], ctypes.c_void_p(counts.data_ptr()), ctypes.c_void_p(err.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_noalloc_backward_matches_workspace_backward(dtype, tol):
    from modelos_b200 import _native
    L = _native.lib()
    # benchmark config-0 bag geometry: 256 bags x 128, 16384 x 512 table
    idx, psw, W, g = cases.embbag_case(256, 128, 16384, 512, seed=9, heads=4)
    idx, psw, W, g = idx.to(DEV), psw.to(DEV, dtype), W.to(DEV, dtype), g.to(DEV, dtype)
    idx[0, :64] = 7  # one row with a long segment
    ref_w, ref_p, ref_c = _native.bag_bwd(idx, W, psw, g, want_counts=True)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):
        gw = torch.full_like(W, float("nan"))
        gp = torch.full_like(psw, float("nan"))
        counts = torch.full((W.shape[0],), -1, dtype=torch.int32, device=DEV)
        rc = _call_noalloc(L, idx, psw, W, g, gw, gp, counts, err, dtype)
        assert rc == 0, L.pkm_last_error()
        torch.cuda.synchronize()
        for got, ref in ((gw, ref_w), (gp, ref_p)):
            den = ref.float().abs().max().item()
            assert (got.float() - ref.float()).abs().max().item() <= tol * den
        assert torch.equal(counts, ref_c)
    assert err.item() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from modelos_b200 import _native
    L = _native.lib()
    fake = ctypes.c_void_p(256)  # never dereferenced: the size check comes first
    rc = L.pkm_bag_bwd_noalloc(fake, fake, 0, fake, 1, fake, 16384, 128, 262144, 1024, fake, 1, fake, 1, None,
                               None, None)
    assert rc == 2
    assert b"static scratch" in L.pkm_last_error()
