"""Addressing statistics on the device (``pkm_addr_stats``) against the
reference's ``compute_addr_stats`` (``modeling_qwen3pkm.py:447-471``, golden
fixture ``addr_stats.npz``) and the oracle."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases
from oracle import pkm_oracle as po

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", cases.ADDR_CASES)
def test_matches_reference_and_oracle(name):
    from modelos_b200.fwpkm.addr_stats import compute_addr_stats
    d = np.load(os.path.join(GOLD, "addr_stats.npz"))
    idx, K, loss = cases.addr_case(name)
    np.testing.assert_allclose(cases.checksum(idx), d[name + "_idx_checksum"], rtol=1e-12, atol=1e-9)
    st = compute_addr_stats(idx.to(DEV), K, loss.to(DEV), "me")
    ref = d[name + "_stats"]
    # integer counts over the reference's own denominators: exact
    assert st["collision_ratio"] == ref[0]
    assert st["coverage_ratio"] == ref[1]
    # the reference's KL is fp32 (1e-5 relative); the oracle's fp64 sum runs
    # in another order (1e-12)
    assert abs(st["kld"] - ref[2]) <= 1e-5 * max(1.0, abs(ref[2]))
    o = po.addr_stats(idx.numpy(), K)
    assert abs(st["kld"] - o["kld"]) <= 1e-12 * max(1.0, abs(o["kld"]))
    assert st["collision_ratio"] == o["collision_ratio"] and st["coverage_ratio"] == o["coverage_ratio"]
    # addr_loss.mean() in fp32 on another device: 1e-6 relative
    assert abs(st["addressing_loss/me"] - ref[3]) <= 1e-6 * abs(ref[3])


def test_async_and_deterministic():
    from modelos_b200 import _native
    from modelos_b200.fwpkm.addr_stats import launch_addr_stats
    idx, K, _ = cases.addr_case("c4_chunk")
    idx = idx.to(DEV)
    pend = [launch_addr_stats(idx, K) for _ in range(3)]
    res = [p.result() for p in pend]
    assert all(p.ready() for p in pend)
    assert res[0] == res[1] == res[2]
    assert "addressing_loss/me" not in res[0]
    raw = _native.addr_stats(idx, K).cpu().tolist()
    assert raw[3] == idx.numel()


def test_out_of_range_index_raises():
    from modelos_b200 import _native
    from modelos_b200.fwpkm.addr_stats import compute_addr_stats
    _native.read_device_errors()
    idx = torch.tensor([0, 3, 64, 5], dtype=torch.long, device=DEV)  # 64 is outside [0, 64)
    with pytest.raises(IndexError):
        compute_addr_stats(idx, 64)
    assert _native.read_device_errors() == 0  # the raise consumed the flag
    with pytest.raises(ValueError):
        compute_addr_stats(torch.empty(0, dtype=torch.long, device=DEV), 64)
