"""Routing kernels of the row-sharded bag (pack, segments, combine) against
their torch restatements on the CPU (``tests/fake_native.py``): equal
element for element, including the fp32 sums of the combine (same order)."""
from __future__ import annotations

import pytest
import torch

import fake_native as fk

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(B, L, K, world, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, K, (B, L), generator=g)
    psw = torch.rand(B, L, generator=g).to(dtype) if dtype is not None else None
    shard_rows = -(-K // world)
    return idx, psw, shard_rows


@pytest.mark.parametrize("B,L,K,world", [(512, 128, 4096, 2), (300, 7, 1000, 3), (64, 32, 262144, 8),
                                         (1, 1, 10, 1), (5000, 16, 50, 5), (0, 8, 100, 2)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, None])
def test_pack_and_segments(B, L, K, world, dtype):
    from modelos_b200 import _native
    idx, psw, S = _case(B, L, K, world, dtype, seed=B + L + world)
    got = _native.route_pack(idx.to(DEV), None if psw is None else psw.to(DEV), S, world)
    ref = fk.route_pack(idx, psw, S, world)
    for a, b in zip(got, ref):
        assert torch.equal(a.cpu(), b.to(a.dtype))
    send, order, local_row, bag, weight = got
    # the sending side's segments: groups = owners
    g_seg = _native.route_segments(bag, send, world)
    r_seg = fk.route_segments(bag.cpu(), send.cpu(), world)
    n_seg = int(r_seg[3].sum())
    assert torch.equal(g_seg[3].cpu(), r_seg[3])
    assert torch.equal(g_seg[0].cpu(), r_seg[0])
    assert torch.equal(g_seg[1][:n_seg + 1].cpu(), r_seg[1][:n_seg + 1])
    assert torch.equal(g_seg[2][:n_seg].cpu(), r_seg[2][:n_seg])


@pytest.mark.parametrize("groups", [1, 2, 7])
@pytest.mark.parametrize("dtype,out_dtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                             (torch.bfloat16, torch.float32)])
def test_segments_of_received_entries_and_combine(groups, dtype, out_dtype):
    """Entries as an all-to-all delivers them (grouped by source, bags
    ascending inside a source, some groups empty), their segments, and the
    combine of one partial row per segment."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(groups)
    n_bags, D = 200, 96
    parts, counts = [], []
    for r in range(groups):
        c = 0 if (r == 1 and groups > 2) else int(torch.randint(0, 600, (1,), generator=g))
        parts.append(torch.sort(torch.randint(0, n_bags, (c,), generator=g)).values)
        counts.append(c)
    bag = torch.cat(parts).to(torch.int32)
    gc = torch.tensor(counts, dtype=torch.int64)
    got = _native.route_segments(bag.to(DEV), gc.to(DEV), groups)
    ref = fk.route_segments(bag, gc, groups)
    n_seg = int(ref[3].sum())
    assert torch.equal(got[0].cpu(), ref[0])
    assert torch.equal(got[3].cpu(), ref[3])
    assert torch.equal(got[1][:n_seg + 1].cpu(), ref[1][:n_seg + 1])
    assert torch.equal(got[2][:n_seg].cpu(), ref[2][:n_seg])
    partial = torch.randn(n_seg, D, generator=g).to(dtype)
    out = _native.route_combine(partial.to(DEV), got[2][:n_seg], got[3], groups, n_bags, out_dtype=out_dtype)
    exp = fk.route_combine(partial, ref[2][:n_seg], ref[3], groups, n_bags, out_dtype=out_dtype)
    assert torch.equal(out.cpu(), exp)


def test_out_of_range_indices_are_left_out_and_flagged():
    from modelos_b200 import _native
    idx, psw, S = _case(40, 9, 300, 3, torch.float32, seed=3)
    idx[0, 0] = -2
    idx[7, 4] = 3 * S  # one past the last owner's rows
    _native.read_device_errors()
    send, order, local_row, bag, weight = _native.route_pack(idx.to(DEV), psw.to(DEV), S, 3)
    assert _native.read_device_errors() & _native.DEVERR_INDEX
    ref = fk.route_pack(idx, psw, S, 3)
    assert int(send.sum()) == idx.numel() - 2
    for a, b in zip((send, order, local_row, bag, weight), ref):
        assert torch.equal(a.cpu(), b.to(a.dtype))
