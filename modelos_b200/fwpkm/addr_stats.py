"""Addressing statistics of memory-slot indices, computed on the device.

Counterpart of ``Qwen3PKMDecoderLayer.compute_addr_stats``
(``modeling_qwen3pkm.py:447-471``): the same keys and values
(``collision_ratio``, ``coverage_ratio``, ``kld`` and, with an addressing
loss, ``addressing_loss/<type>``), but the histogram and its reductions run
in one native call (``pkm_addr_stats``) and the numbers reach the host in
one asynchronous copy instead of four ``.item()`` synchronisations.

``launch_addr_stats`` queues the work on the current stream and returns at
once; ``PendingAddrStats.result()`` waits for that stream's copy only, so a
training loop can read the statistics of step ``t`` while step ``t + 1``
runs.  ``compute_addr_stats`` is the blocking form.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from .. import _native


class PendingAddrStats:
    """Statistics in flight: a pinned host copy and the event that ends it."""

    def __init__(self, values: torch.Tensor, numel: int, size: int, loss_key: Optional[str]):
        self._host = torch.empty(values.numel(), dtype=torch.float64, pin_memory=True)
        self._host.copy_(values, non_blocking=True)
        self._event = torch.cuda.Event()
        self._event.record(torch.cuda.current_stream(values.device))
        self._numel, self._size, self._loss_key = numel, size, loss_key
        self._device = values.device
        self._values = values  # kept alive until the copy has ended

    def ready(self) -> bool:
        return self._event.query()

    def result(self) -> Dict[str, float]:
        self._event.synchronize()
        collided, covered, kld, counted = self._host[:4].tolist()
        if int(counted) != self._numel:
            _native.check_device_errors(self._device)
            raise IndexError("an addressing index was outside [0, size)")
        # modeling_qwen3pkm.py:456-462
        stats = {
            "collision_ratio": collided / (self._numel + 1e-6),
            "coverage_ratio": covered / self._size,
            "kld": kld,
        }
        if self._loss_key is not None:
            stats[self._loss_key] = float(self._host[4])
        return stats


def launch_addr_stats(idcs: torch.LongTensor, size: int, addr_loss: Optional[torch.Tensor] = None,
                      addr_loss_type: Optional[str] = "me") -> PendingAddrStats:
    """Queue the statistics of ``idcs`` (any shape, int64 slot indices in
    ``[0, size)``; ``size`` = ``n_subkeys ** 2``) on the current stream."""
    with torch.no_grad():
        vals = torch.empty(5, dtype=torch.float64, device=idcs.device)
        _native.addr_stats(idcs, size, out=vals)
        loss_key = None
        if addr_loss is not None:
            # the reference reports addr_loss.mean() of the loss's own dtype
            vals[4:].copy_(addr_loss.detach().mean().reshape(1))
            loss_key = f"addressing_loss/{addr_loss_type}"
        return PendingAddrStats(vals, idcs.numel(), int(size), loss_key)


def compute_addr_stats(idcs: torch.LongTensor, size: int, addr_loss: Optional[torch.Tensor] = None,
                       addr_loss_type: Optional[str] = "me") -> Dict[str, float]:
    """Blocking form of :func:`launch_addr_stats`."""
    return launch_addr_stats(idcs, size, addr_loss, addr_loss_type).result()
