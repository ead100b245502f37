"""ctypes binding of ``libpkm_b200.so`` and thin tensor-level wrappers.

Every wrapper checks shapes, dtypes and devices the way the reference's
launchers assert them (``pkm/xformer_embeddingbag.py:226-233``), allocates the
outputs and any scratch space with torch's caching allocator, and enqueues
the kernels on the current CUDA stream.  There is no CPU path: the library
must be built (``python -m modelos_b200.csrc.build``) and tensors must live
on a CUDA device, otherwise these functions raise.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libpkm_b200.so")
_lib = None
_lock = threading.Lock()

DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

_SIGS = {
    "pkm_version": ([], _I),
    "pkm_status_string": ([_I], ctypes.c_char_p),
    "pkm_last_error": ([], ctypes.c_char_p),
    "pkm_bag_fwd": ([_P, _P, _I, _P, _I, _I64, _I64, _I64, _I64, _P, _I, _P, _P], _I),
    "pkm_bag_bwd_workspace": ([_I64, _I64, _I64, _I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_bag_bwd": ([_P, _P, _I, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _I, _P, _P,
                     ctypes.c_size_t, _P, _P], _I),
    "pkm_bag_bwd_noalloc": ([_P, _P, _I, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _I, _P, _P, _P], _I),
    "pkm_bag_bwd2": ([_P, _P, _I, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _I, _P, _P], _I),
    "pkm_subkey_scores": ([_P, _P, _I, _I64, _I64, _I64, _I64, _I, _P, _P, _P], _I),
    "pkm_product_topk": ([_P, _I, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P], _I),
    "pkm_score_bwd_prep": ([_P, _P, _P, _I, _I64, _I64, _I64, _I64, _P, _P, _P], _I),
    "pkm_score_grad_dense": ([_P, _P, _P, _I, _I64, _I64, _I64, _P, _P], _I),
    "pkm_score_transform_fwd": ([_P, _I, _I64, _I64, ctypes.c_double, _I, _P, _P], _I),
    "pkm_gemm_workspace": ([_I64, _I64, _I64, _I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_gemm_bf16": ([_P, _I, _I64, _I64, _I64, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                       _I64, _I64, _P, _I, _P, _I, _I64, _I64, _P, ctypes.c_size_t, _P, _P], _I),
    "pkm_debug_set_wait_limit": ([_I64], _I),
    "pkm_debug_gemm_pair": ([_I], _I),
    "pkm_gemm_f32": ([_P, _I, _I64, _I64, _I64, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                      _I64, _I64, _P, _I64, _I64, _P], _I),
    "pkm_gemm_f32_workspace": ([_I64, _I64, _I64, _I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_gemm_f32_ws": ([_P, _I, _I64, _I64, _I64, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                         _I64, _I64, _P, _I64, _I64, _P, ctypes.c_size_t, _P], _I),
    "pkm_gemm_swiglu_fwd": ([_P, _I64, _P, _P, _I, _P, _I64, _I64, _I64, _P, _P, _I64, _P, _P], _I),
    "pkm_gemm_swiglu_bwd": ([_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _P, _P, _I64, _P, _P], _I),
    "pkm_score_transform_bwd": ([_P, _P, _P, _I, _I64, _I64, ctypes.c_double, _I, _P, _P], _I),
    "pkm_bag_bwd_sharded": ([_P, _P, _I, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I, _I, _I64, _I, _P, _I, _P, _P,
                             ctypes.c_size_t, _P, _P], _I),
    "pkm_grad_shard_reduce": ([_P, _I, _I64, _I64, _I, _I, _I64, _P, ctypes.c_float, _I, _P], _I),
    "pkm_grad_shard_sgd": ([_P, _I, _I64, _I64, _I, _I, _I64, _P, ctypes.c_float, ctypes.c_float, ctypes.c_float, _I,
                            _P], _I),
    "pkm_segment_sum_workspace": ([_I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_segment_sum": ([_P, _I, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _I, _P, ctypes.c_size_t, _P, _P], _I),
    "pkm_bag_bwd_ragged": ([_P, _P, _P, _I, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _I, _P, _P,
                            ctypes.c_size_t, _P, _P], _I),
    "pkm_grad_multimem_allreduce": ([_P, _P, _I, _I64, _I64, _I, _I, _I64, _I64, _I64, ctypes.c_float, _I, _P],
                                    _I),
    "pkm_bag_bwd_sort": ([_P, _P, _I, _P, _I, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _P, ctypes.c_size_t, _P, _P],
                         _I),
    "pkm_bag_bwd_rows": ([_P, _P, _I, _P, _I, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I, _P, _I, _P,
                          ctypes.c_size_t, _P, _P], _I),
    "pkm_colsum_workspace": ([_I64, _I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_swiglu_fwd": ([_P, _P, _I, _I64, _I64, _P, _P], _I),
    "pkm_swiglu_bwd": ([_P, _P, _P, _I, _I64, _I64, _P, _P, _P, _I, _P, ctypes.c_size_t, _P], _I),
    "pkm_colsum": ([_P, _I, _I64, _I64, _P, _I, _P, ctypes.c_size_t, _P], _I),
    "pkm_fw_update": ([_P, _P, _I, _I64, _I64, _P, _I64, ctypes.c_double, ctypes.c_double, ctypes.c_double, _I,
                       _P, _P, _P, _P, _P], _I),
    "pkm_fw_update_bwd": ([_P, _P, _P, _P, _I, _I64, _I64, ctypes.c_double, ctypes.c_double, ctypes.c_double, _I,
                           _P, _P, _P], _I),
    "pkm_route_pack_workspace": ([_I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_route_pack": ([_P, _P, _I, _I64, _I64, _I64, _I, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P], _I),
    "pkm_route_segments_workspace": ([_I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_route_segments": ([_P, _I64, _P, _I, _P, _P, _P, _P, _P, ctypes.c_size_t, _P], _I),
    "pkm_route_combine_workspace": ([_I, _I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_route_combine": ([_P, _I, _I64, _I64, _P, _P, _I, _I64, _P, _I, _P, ctypes.c_size_t, _P, _P], _I),
    "pkm_addr_stats_workspace": ([_I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_addr_stats": ([_P, _I64, _I64, _P, _P, ctypes.c_size_t, _P, _P], _I),
    "pkm_batchnorm_workspace": ([_I64, _I64, ctypes.POINTER(ctypes.c_size_t)], _I),
    "pkm_batchnorm_fwd": ([_P, _I, _I64, _I64, _P, _P, _I, _P, _P, _I, _I, ctypes.c_double, ctypes.c_double,
                           _P, _P, _P, _P, ctypes.c_size_t, _P], _I),
    "pkm_batchnorm_bwd": ([_P, _P, _I, _I64, _I64, _P, _P, _P, _I, _P, _P, _P, _P, ctypes.c_size_t, _P], _I),
}

EXPORTED = tuple(_SIGS)


def library_path() -> str:
    return _LIB_PATH


def lib():
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    f"modelos_b200 native library missing at {_LIB_PATH}; "
                    "build it with `python -m modelos_b200.csrc.build`")
            L = ctypes.CDLL(_LIB_PATH)
            for name, (args, res) in _SIGS.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = res
            _lib = L
    return _lib


def _check(rc: int, name: str):
    if rc != 0:
        L = lib()
        detail = L.pkm_last_error().decode(errors="replace")
        status = L.pkm_status_string(rc).decode()
        raise RuntimeError(f"{name} failed ({status}): {detail}")


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("modelos_b200 kernels need CUDA tensors (there is no CPU path)")


# ---------------------------------------------------------------------------
# optional CUDA-event probe around selected entry points (used by bench.py to
# time the dominant kernels on their own stream inside the timed region)
# ---------------------------------------------------------------------------
class EventProbe:
    def __init__(self, names, min_rows: int = 0):
        self.names = set(names)
        self.min_rows = min_rows
        self.events: dict = {n: [] for n in names}

    def start(self, name: str, rows: int):
        if name not in self.names or rows < self.min_rows:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def stop(self, name: str, ev0):
        if ev0 is None:
            return
        ev1 = torch.cuda.Event(enable_timing=True)
        ev1.record()
        self.events[name].append((ev0, ev1))

    def total_ms(self, name: str) -> float:
        return sum(a.elapsed_time(b) for a, b in self.events.get(name, []))

    def mean_ms(self, name: str) -> Optional[float]:
        ev = self.events.get(name, [])
        if not ev:
            return None
        return self.total_ms(name) / len(ev)

    def count(self, name: str) -> int:
        return len(self.events.get(name, []))


_probe: Optional[EventProbe] = None


def set_probe(probe: Optional[EventProbe]):
    global _probe
    _probe = probe


def _pstart(name, rows):
    return _probe.start(name, rows) if _probe is not None else None


def _pstop(name, ev):
    if ev is not None:
        _probe.stop(name, ev)


# ---------------------------------------------------------------------------
# device error word
# ---------------------------------------------------------------------------
_err_words: dict = {}


def err_word(dev: torch.device) -> torch.Tensor:
    """Per-device uint32 word the kernels OR error bits into."""
    key = (dev.type, dev.index if dev.index is not None else torch.cuda.current_device())
    w = _err_words.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=dev)
        _err_words[key] = w
    return w


DEVERR_INDEX = 1
DEVERR_TIMEOUT = 2


def read_device_errors(dev: Optional[torch.device] = None, reset: bool = True) -> int:
    """Synchronising read of the error word (bit 1: an index was out of range,
    bit 2: a bounded wait timed out)."""
    dev = dev or torch.device("cuda", torch.cuda.current_device())
    w = err_word(dev)
    v = int(w.item())
    if reset:
        w.zero_()
    return v


def check_device_errors(dev: Optional[torch.device] = None):
    v = read_device_errors(dev)
    if v & DEVERR_INDEX:
        raise IndexError("modelos_b200: an embedding index was outside [0, num_rows)")
    if v & DEVERR_TIMEOUT:
        raise RuntimeError("modelos_b200: a bounded wait inside a kernel timed out")


# ---------------------------------------------------------------------------
# embedding bag
# ---------------------------------------------------------------------------
def _bag_checks(indices, weight, psw):
    assert indices.dim() == 2 and indices.dtype == torch.long, "indices must be [B, bag] int64"
    assert weight.dim() == 2, "weight must be [K, dim]"
    assert indices.is_contiguous() and weight.is_contiguous()
    if psw is not None:
        assert psw.shape == indices.shape, "per_sample_weights must match indices"
        assert psw.is_contiguous()
    _need_cuda(indices, weight, psw)


def bag_fwd(indices: torch.Tensor, weight: torch.Tensor, psw: Optional[torch.Tensor],
            out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """K3: ``out[b] = sum_j psw[b,j] * weight[indices[b,j]]``."""
    _bag_checks(indices, weight, psw)
    B, L = indices.shape
    K, D = weight.shape
    out_dtype = out_dtype or weight.dtype
    out = torch.empty((B, D), dtype=out_dtype, device=weight.device)
    ev = _pstart("pkm_bag_fwd", K)
    rc = lib().pkm_bag_fwd(_ptr(indices), _ptr(psw), DT[psw.dtype] if psw is not None else 0,
                           _ptr(weight), DT[weight.dtype], B, L, K, D, _ptr(out), DT[out_dtype],
                           _ptr(err_word(weight.device)), _stream(weight.device))
    _pstop("pkm_bag_fwd", ev)
    _check(rc, "pkm_bag_fwd")
    return out


def bag_bwd_workspace(B: int, L: int, K: int, D: int) -> int:
    n = ctypes.c_size_t(0)
    _check(lib().pkm_bag_bwd_workspace(B, L, K, D, ctypes.byref(n)), "pkm_bag_bwd_workspace")
    return int(n.value)


def bag_bwd(indices: torch.Tensor, weight: Optional[torch.Tensor], psw: Optional[torch.Tensor],
            grad_out: torch.Tensor, *, num_rows: Optional[int] = None, need_dpsw: bool = True,
            want_counts: bool = False, grad_weight_dtype: Optional[torch.dtype] = None,
            out: Optional[torch.Tensor] = None):
    """K4: dense weight gradient, per-sample-weight gradient, row counts."""
    assert indices.dim() == 2 and indices.dtype == torch.long and indices.is_contiguous()
    assert grad_out.dim() == 2 and grad_out.shape[0] == indices.shape[0] and grad_out.is_contiguous()
    _need_cuda(indices, grad_out, weight, psw)
    B, L = indices.shape
    D = grad_out.shape[1]
    if weight is not None:
        assert weight.dim() == 2 and weight.is_contiguous() and weight.shape[1] == D
        K = weight.shape[0]
        row_dtype = weight.dtype
    else:
        assert num_rows is not None and not need_dpsw
        K = num_rows
        row_dtype = grad_out.dtype
    assert grad_out.dtype == row_dtype, "grad_out must have the table's dtype"
    if psw is not None:
        assert psw.shape == indices.shape and psw.is_contiguous()
    dev = grad_out.device
    gw_dtype = grad_weight_dtype or row_dtype
    if out is not None:
        assert out.shape == (K, D) and out.dtype == gw_dtype and out.is_contiguous() and out.device == dev
        grad_weight = out
    else:
        grad_weight = torch.empty((K, D), dtype=gw_dtype, device=dev)
    grad_psw = torch.empty_like(psw) if (need_dpsw and psw is not None) else None
    counts = torch.empty((K,), dtype=torch.int32, device=dev) if want_counts else None
    ws_bytes = bag_bwd_workspace(B, L, K, D)
    ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
    ev = _pstart("pkm_bag_bwd", K)
    rc = lib().pkm_bag_bwd(_ptr(indices), _ptr(psw), DT[psw.dtype] if psw is not None else 0,
                           _ptr(weight), DT[row_dtype], _ptr(grad_out), B, L, K, D,
                           _ptr(grad_weight), DT[gw_dtype], _ptr(grad_psw),
                           DT[grad_psw.dtype] if grad_psw is not None else 0, _ptr(counts), _ptr(ws),
                           ws_bytes, _ptr(err_word(dev)), _stream(dev))
    _pstop("pkm_bag_bwd", ev)
    _check(rc, "pkm_bag_bwd")
    return grad_weight, grad_psw, counts


def _ptr_array(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p)) for p in ptrs])


def bag_bwd_sharded(indices: torch.Tensor, weight: torch.Tensor, psw: Optional[torch.Tensor],
                    grad_out: torch.Tensor, recv_bases, rank: int, shard_rows: int, *, need_dpsw: bool = True):
    """K4 with the table gradient stored into the owners' receive buffers
    (``recv_bases[o]``: device address of rank o's [world, shard_rows, D]
    buffer).  Returns the per-sample-weight gradient (or None)."""
    assert indices.dim() == 2 and indices.dtype == torch.long and indices.is_contiguous()
    assert grad_out.dim() == 2 and grad_out.shape[0] == indices.shape[0] and grad_out.is_contiguous()
    assert weight.dim() == 2 and weight.is_contiguous() and weight.shape[1] == grad_out.shape[1]
    assert grad_out.dtype == weight.dtype, "grad_out must have the table's dtype"
    _need_cuda(indices, grad_out, weight, psw)
    B, L = indices.shape
    K, D = weight.shape
    dev = grad_out.device
    grad_psw = torch.empty_like(psw) if (need_dpsw and psw is not None) else None
    ws_bytes = bag_bwd_workspace(B, L, K, D)
    ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
    world = len(recv_bases)
    ev = _pstart("pkm_bag_bwd", K)
    rc = lib().pkm_bag_bwd_sharded(_ptr(indices), _ptr(psw), DT[psw.dtype] if psw is not None else 0, _ptr(weight),
                                   DT[weight.dtype], _ptr(grad_out), B, L, K, D, _ptr_array(recv_bases), world, rank,
                                   shard_rows, DT[weight.dtype], _ptr(grad_psw),
                                   DT[grad_psw.dtype] if grad_psw is not None else 0, None, _ptr(ws), ws_bytes,
                                   _ptr(err_word(dev)), _stream(dev))
    _pstop("pkm_bag_bwd", ev)
    _check(rc, "pkm_bag_bwd_sharded")
    return grad_psw


def grad_shard_reduce(recv: torch.Tensor, num_rows: int, rank: int, shard_rows: int, grad_bases, scale: float = 1.0,
                      max_blocks: int = 0):
    """Sum this rank's received partial shard rows and store them into every
    rank's gradient (``grad_bases``: device addresses, one per rank)."""
    _need_cuda(recv)
    world = len(grad_bases)
    assert recv.is_contiguous() and recv.shape[0] == world and recv.shape[1] == shard_rows
    D = recv.shape[2]
    _check(lib().pkm_grad_shard_reduce(_ptr(recv), DT[recv.dtype], num_rows, D, world, rank, shard_rows,
                                       _ptr_array(grad_bases), float(scale), int(max_blocks), _stream(recv.device)),
           "pkm_grad_shard_reduce")


def grad_shard_sgd(recv: torch.Tensor, num_rows: int, rank: int, shard_rows: int, table_bases, lr: float,
                   weight_decay: float = 0.0, scale: float = 1.0, max_blocks: int = 0):
    """Sum this rank's received shard rows, apply SGD to this rank's rows of
    the table and store them into every rank's table (``table_bases``:
    device addresses, one per rank)."""
    _need_cuda(recv)
    world = len(table_bases)
    assert recv.is_contiguous() and recv.shape[0] == world and recv.shape[1] == shard_rows
    D = recv.shape[2]
    _check(lib().pkm_grad_shard_sgd(_ptr(recv), DT[recv.dtype], num_rows, D, world, rank, shard_rows,
                                    _ptr_array(table_bases), float(lr), float(weight_decay), float(scale),
                                    int(max_blocks), _stream(recv.device)), "pkm_grad_shard_sgd")


def grad_multimem_allreduce(mc_src: int, mc_dst: int, dtype: torch.dtype, num_rows: int, dim: int, world: int,
                            rank: int, shard_rows: int, device: torch.device, scale: float = 1.0, max_blocks: int = 0,
                            row_begin: int = 0, row_end: int = -1):
    """In-switch all-reduce of this rank's shard rows in [row_begin, row_end)."""
    _check(lib().pkm_grad_multimem_allreduce(ctypes.c_void_p(mc_src), ctypes.c_void_p(mc_dst), DT[dtype], num_rows,
                                             dim, world, rank, shard_rows, row_begin, row_end, float(scale),
                                             int(max_blocks), _stream(device)), "pkm_grad_multimem_allreduce")


class BagBwdPhases:
    """``bag_bwd`` split into the sort and row-range segment passes on one
    workspace: ``sort()`` once, then ``rows(r0, r1, out)`` for each range."""

    def __init__(self, indices: torch.Tensor, weight: torch.Tensor, psw: Optional[torch.Tensor],
                 grad_out: torch.Tensor, need_dpsw: bool = True):
        assert indices.dim() == 2 and indices.dtype == torch.long and indices.is_contiguous()
        assert grad_out.dim() == 2 and grad_out.shape[0] == indices.shape[0] and grad_out.is_contiguous()
        assert weight.dim() == 2 and weight.is_contiguous() and grad_out.dtype == weight.dtype
        _need_cuda(indices, grad_out, weight, psw)
        self.indices, self.weight, self.psw, self.grad_out = indices, weight, psw, grad_out
        self.B, self.L = indices.shape
        self.K, self.D = weight.shape
        dev = weight.device
        self.dpsw = torch.empty_like(psw) if (need_dpsw and psw is not None) else None
        self.ws_bytes = bag_bwd_workspace(self.B, self.L, self.K, self.D)
        self.ws = torch.empty((max(self.ws_bytes, 1),), dtype=torch.uint8, device=dev)

    def _common(self):
        p = self.psw
        return (_ptr(self.indices), _ptr(p), DT[p.dtype] if p is not None else 0, _ptr(self.weight),
                DT[self.weight.dtype], _ptr(self.grad_out), self.B, self.L, self.K, self.D)

    def sort(self):
        d = self.dpsw
        ev = _pstart("pkm_bag_bwd_sort", self.K)
        rc = lib().pkm_bag_bwd_sort(*self._common(), _ptr(d), DT[d.dtype] if d is not None else 0, None,
                                    _ptr(self.ws), self.ws_bytes, _ptr(err_word(self.weight.device)),
                                    _stream(self.weight.device))
        _pstop("pkm_bag_bwd_sort", ev)
        _check(rc, "pkm_bag_bwd_sort")

    def rows(self, r0: int, r1: int, out: torch.Tensor):
        assert out.shape == (self.K, self.D) and out.is_contiguous() and out.dtype == self.weight.dtype
        d = self.dpsw
        ev = _pstart("pkm_bag_bwd_rows", self.K)
        rc = lib().pkm_bag_bwd_rows(*self._common(), r0, r1, _ptr(out), DT[out.dtype], _ptr(d),
                                    DT[d.dtype] if d is not None else 0, _ptr(self.ws), self.ws_bytes,
                                    _ptr(err_word(self.weight.device)), _stream(self.weight.device))
        _pstop("pkm_bag_bwd_rows", ev)
        _check(rc, "pkm_bag_bwd_rows")


def bag_bwd2(indices: torch.Tensor, a: Optional[torch.Tensor], gbar: torch.Tensor,
             grad_out: torch.Tensor, *, d_grad_out_dtype: Optional[torch.dtype] = None,
             d_a_dtype: Optional[torch.dtype] = None):
    """K5: ``dG[b] = sum_j a[b,j] gbar[idx]``, ``da[b,j] = <gbar[idx], g[b]>``."""
    _bag_checks(indices, gbar, a)
    assert grad_out.shape == (indices.shape[0], gbar.shape[1]) and grad_out.is_contiguous()
    _need_cuda(grad_out)
    B, L = indices.shape
    K, D = gbar.shape
    g = grad_out if grad_out.dtype == gbar.dtype else grad_out.to(gbar.dtype)
    dgo = torch.empty((B, D), dtype=d_grad_out_dtype or grad_out.dtype, device=gbar.device)
    da = None
    if a is not None:
        da = torch.empty((B, L), dtype=d_a_dtype or a.dtype, device=gbar.device)
    rc = lib().pkm_bag_bwd2(_ptr(indices), _ptr(a), DT[a.dtype] if a is not None else 0,
                            _ptr(gbar), DT[gbar.dtype], _ptr(g), B, L, K, D, _ptr(dgo),
                            DT[dgo.dtype], _ptr(da), DT[da.dtype] if da is not None else 0,
                            _ptr(err_word(gbar.device)), _stream(gbar.device))
    _check(rc, "pkm_bag_bwd2")
    return dgo, da


# ---------------------------------------------------------------------------
# scoring and top-k
# ---------------------------------------------------------------------------
def subkey_scores(query: torch.Tensor, keys: torch.Tensor, heads: int, mode: str = "dot") -> torch.Tensor:
    """K1: ``[N*H, k_dim]`` queries x ``[2*H*n, k_dim/2]`` keys -> ``[N*H, 2, n]``.

    ``mode``: "dot" (bf16 on the tensor cores), "dot_seq" (sequential fp32
    sum), "idw" or "dist" (distance)."""
    assert query.dim() == 2 and keys.dim() == 2 and query.is_contiguous() and keys.is_contiguous()
    assert query.dtype == keys.dtype, "query and keys must share a dtype"
    _need_cuda(query, keys)
    NH, kd = query.shape
    assert NH % heads == 0 and keys.shape[1] * 2 == kd and keys.shape[0] % (2 * heads) == 0
    n = keys.shape[0] // (2 * heads)
    out = torch.empty((NH, 2, n), dtype=query.dtype, device=query.device)
    rc = lib().pkm_subkey_scores(_ptr(query), _ptr(keys), DT[query.dtype], NH // heads, heads, kd, n,
                                 {"dot": 0, "idw": 1, "dist": 2, "dot_seq": 3}[mode], _ptr(out),
                                 _ptr(err_word(query.device)), _stream(query.device))
    _check(rc, "pkm_subkey_scores")
    return out


def product_topk(scores: torch.Tensor, knn: int, want_psw: bool = False, want_sub: bool = False):
    """K2 on ``[R, 2, n]`` scores -> (indices, top_scores, psw|None, sub1|None, sub2|None)."""
    assert scores.dim() == 3 and scores.shape[1] == 2 and scores.is_contiguous()
    _need_cuda(scores)
    R, _, n = scores.shape
    dev = scores.device
    idx = torch.empty((R, knn), dtype=torch.long, device=dev)
    ts = torch.empty((R, knn), dtype=scores.dtype, device=dev)
    psw = torch.empty_like(ts) if want_psw else None
    s1 = torch.empty((R, knn), dtype=torch.long, device=dev) if want_sub else None
    s2 = torch.empty((R, knn), dtype=torch.long, device=dev) if want_sub else None
    rc = lib().pkm_product_topk(_ptr(scores), DT[scores.dtype], R, n, knn, _ptr(idx), _ptr(ts),
                                _ptr(psw), _ptr(s1), _ptr(s2), _stream(dev))
    _check(rc, "pkm_product_topk")
    return idx, ts, psw, s1, s2


def score_bwd_prep(indices: torch.Tensor, psw: Optional[torch.Tensor], dpsw: torch.Tensor,
                   heads: int, n_keys: int):
    """Softmax backward + sub-key bags: returns (sub_idx [2R, knn], sub_w [2R, knn])."""
    assert indices.dim() == 2 and dpsw.shape == indices.shape
    _need_cuda(indices, psw, dpsw)
    R, knn = indices.shape
    dpsw = dpsw.contiguous()
    if psw is not None:
        psw = psw.contiguous().to(dpsw.dtype)
    sub_idx = torch.empty((2 * R, knn), dtype=torch.long, device=dpsw.device)
    sub_w = torch.empty((2 * R, knn), dtype=dpsw.dtype, device=dpsw.device)
    rc = lib().pkm_score_bwd_prep(_ptr(indices), _ptr(psw), _ptr(dpsw), DT[dpsw.dtype], R, knn, heads,
                                  n_keys, _ptr(sub_idx), _ptr(sub_w), _stream(dpsw.device))
    _check(rc, "pkm_score_bwd_prep")
    return sub_idx, sub_w


def score_grad_dense(indices: torch.Tensor, psw: Optional[torch.Tensor], dpsw: torch.Tensor,
                     n_keys: int) -> torch.Tensor:
    """Dense ``[R, 2, n]`` gradient of the sub-key scores (softmax backward
    included when ``psw`` is given)."""
    assert indices.dim() == 2 and dpsw.shape == indices.shape
    _need_cuda(indices, psw, dpsw)
    R, knn = indices.shape
    dpsw = dpsw.contiguous()
    if psw is not None:
        psw = psw.contiguous().to(dpsw.dtype)
    out = torch.empty((R, 2, n_keys), dtype=dpsw.dtype, device=dpsw.device)
    rc = lib().pkm_score_grad_dense(_ptr(indices), _ptr(psw), _ptr(dpsw), DT[dpsw.dtype], R, knn, n_keys,
                                    _ptr(out), _stream(dpsw.device))
    _check(rc, "pkm_score_grad_dense")
    return out


# ---------------------------------------------------------------------------
# dense GEMM on the tensor cores
# ---------------------------------------------------------------------------
def gemm_workspace(batch: int, M: int, N: int, K: int) -> int:
    n = ctypes.c_size_t(0)
    _check(lib().pkm_gemm_workspace(batch, M, N, K, ctypes.byref(n)), "pkm_gemm_workspace")
    return int(n.value)


def _mat(t: torch.Tensor):
    """(rows, cols, row pitch) of a 2-D row-major view (unit column stride)."""
    assert t.dim() == 2 and t.stride(1) == 1 and t.dtype == torch.bfloat16, "GEMM operands: 2-D bf16, unit column stride"
    return t.shape[0], t.shape[1], t.stride(0)


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False, bias=None,
         out: Optional[torch.Tensor] = None, out_dtype=torch.bfloat16, batch: int = 1, M: Optional[int] = None,
         N: Optional[int] = None, K: Optional[int] = None, a_batch=(0, 0), b_batch=(0, 0),
         c_batch_stride: int = 0) -> torch.Tensor:
    """``C[m, n] = sum_k A[m, k] B[n, k] (+ bias[n])`` on the tensor cores.

    ``a`` is read K-major (``a[m, k]``) or, with ``a_mn``, MN-major
    (``a[k, m]``); ``b`` likewise (``b[n, k]`` or ``b[k, n]``).  So
    ``x @ w.T`` is ``gemm(x, w)``, ``dy @ w`` is ``gemm(dy, w, b_mn=True)``
    and ``dy.T @ x`` is ``gemm(dy, x, a_mn=True, b_mn=True)``.  For a batch
    of GEMMs, ``a_batch`` / ``b_batch`` are the (column, row) shifts of one
    batch's operand region and ``c_batch_stride`` its output offset; ``out``
    must then be given, as must M, N, K."""
    ar, ac, lda = _mat(a)
    br, bc, ldb = _mat(b)
    _need_cuda(a, b, bias, out)
    if M is None:
        M = ac if a_mn else ar
    if K is None:
        K = ar if a_mn else ac
    if N is None:
        N = bc if b_mn else br
    if out is None:
        assert batch == 1
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    assert out.stride(-1) == 1
    ldc = out.stride(-2) if out.dim() >= 2 else N
    ws_bytes = gemm_workspace(batch, M, N, K)
    ws = torch.empty((max(ws_bytes, 16) // 4,), dtype=torch.float32, device=a.device) if ws_bytes else None
    rc = lib().pkm_gemm_bf16(_ptr(a), int(a_mn), ar, ac, lda, _ptr(b), int(b_mn), br, bc, ldb, batch, M, N, K,
                             a_batch[0], a_batch[1], b_batch[0], b_batch[1], _ptr(bias),
                             DT[bias.dtype] if bias is not None else 0, _ptr(out), DT[out.dtype], ldc,
                             c_batch_stride, _ptr(ws), ws_bytes, _ptr(err_word(a.device)), _stream(a.device))
    _check(rc, "pkm_gemm_bf16")
    return out


def gemm_f32(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False,
             out: Optional[torch.Tensor] = None, batch: int = 1, M: Optional[int] = None, N: Optional[int] = None,
             K: Optional[int] = None, a_batch=(0, 0), b_batch=(0, 0), c_batch_stride: int = 0) -> torch.Tensor:
    """fp32 ``C[m, n] = sum_k A[m, k] B[n, k]`` on the CUDA cores; the same
    operand views and batching as ``gemm``."""
    for t in (a, b):
        assert t.dim() == 2 and t.stride(1) == 1 and t.dtype == torch.float32, "fp32 GEMM operands: 2-D, unit stride"
    _need_cuda(a, b, out)
    ar, ac, lda = a.shape[0], a.shape[1], a.stride(0)
    br, bc, ldb = b.shape[0], b.shape[1], b.stride(0)
    M = M if M is not None else (ac if a_mn else ar)
    K = K if K is not None else (ar if a_mn else ac)
    N = N if N is not None else (bc if b_mn else br)
    if out is None:
        assert batch == 1
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    assert out.dtype == torch.float32 and out.stride(-1) == 1
    nb = ctypes.c_size_t(0)
    _check(lib().pkm_gemm_f32_workspace(batch, M, N, K, ctypes.byref(nb)), "pkm_gemm_f32_workspace")
    ws = torch.empty(int(nb.value), dtype=torch.uint8, device=a.device) if nb.value else None
    rc = lib().pkm_gemm_f32_ws(_ptr(a), int(a_mn), ar, ac, lda, _ptr(b), int(b_mn), br, bc, ldb, batch, M, N, K,
                               a_batch[0], a_batch[1], b_batch[0], b_batch[1], _ptr(out), out.stride(-2),
                               c_batch_stride, _ptr(ws), 0 if ws is None else ws.numel(), _stream(a.device))
    _check(rc, "pkm_gemm_f32_ws")
    return out


def gemm_swiglu_fwd(x: torch.Tensor, ws: torch.Tensor, bs: Optional[torch.Tensor], a: torch.Tensor):
    """``h = x @ ws.T + bs`` and ``z = a * silu(h)`` in one tensor-core GEMM:
    returns (h, z)."""
    M, K = x.shape
    N = ws.shape[0]
    assert ws.shape == (N, K) and a.shape == (M, N)
    x, ws, a = x.contiguous(), ws.contiguous(), a.contiguous()
    _need_cuda(x, ws, bs, a)
    h = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    z = torch.empty_like(h)
    rc = lib().pkm_gemm_swiglu_fwd(_ptr(x), K, _ptr(ws), _ptr(bs), DT[bs.dtype] if bs is not None else 0, _ptr(a),
                                   M, N, K, _ptr(h), _ptr(z), N, _ptr(err_word(x.device)), _stream(x.device))
    _check(rc, "pkm_gemm_swiglu_fwd")
    return h, z


def gemm_swiglu_bwd(dy: torch.Tensor, wv: torch.Tensor, a: torch.Tensor, h: torch.Tensor, need_da: bool = True):
    """``dz = dy @ wv`` with the gate's backward in the epilogue: returns (da|None, dh)."""
    M, K = dy.shape
    N = wv.shape[1]
    assert wv.shape == (K, N) and a.shape == (M, N) and h.shape == (M, N)
    dy, wv, a, h = dy.contiguous(), wv.contiguous(), a.contiguous(), h.contiguous()
    _need_cuda(dy, wv, a, h)
    dh = torch.empty((M, N), dtype=torch.bfloat16, device=dy.device)
    da = torch.empty_like(dh) if need_da else None
    rc = lib().pkm_gemm_swiglu_bwd(_ptr(dy), K, _ptr(wv), N, _ptr(a), _ptr(h), M, N, K, _ptr(dh), _ptr(da), N,
                                   _ptr(err_word(dy.device)), _stream(dy.device))
    _check(rc, "pkm_gemm_swiglu_bwd")
    return da, dh


def set_wait_limit(polls: int):
    """Test hook: the pipeline wait limit of the GEMM kernel (negative: the
    default; 0: every wait gives up at once)."""
    _check(lib().pkm_debug_set_wait_limit(int(polls)), "pkm_debug_set_wait_limit")


def set_gemm_pair(mode: int):
    """Test hook: the GEMM's form (-1: CTA pairs when M > 128; 0: single
    CTAs; 1: CTA pairs)."""
    _check(lib().pkm_debug_gemm_pair(int(mode)), "pkm_debug_gemm_pair")


TRANSFORM_MODES = {"softmax": 0, "silu": 1, "relu": 2}


def score_transform_fwd(scores: torch.Tensor, temperature: float, mode: str = "softmax") -> torch.Tensor:
    """``score_transform`` of FwPKM on [rows, width] scores: softmax / silu /
    relu of ``scores / temperature`` over each row, in the scores' dtype."""
    assert scores.dim() == 2 and scores.is_contiguous()
    _need_cuda(scores)
    out = torch.empty_like(scores)
    rc = lib().pkm_score_transform_fwd(_ptr(scores), DT[scores.dtype], scores.shape[0], scores.shape[1],
                                       float(temperature), TRANSFORM_MODES[mode], _ptr(out),
                                       _stream(scores.device))
    _check(rc, "pkm_score_transform_fwd")
    return out


def score_transform_bwd(scores: Optional[torch.Tensor], out: Optional[torch.Tensor], grad_out: torch.Tensor,
                        temperature: float, mode: str = "softmax") -> torch.Tensor:
    """Gradient of ``score_transform_fwd`` w.r.t. the scores."""
    grad_out = grad_out.contiguous()
    assert grad_out.dim() == 2
    ref = out if mode == "softmax" else scores
    assert ref is not None and ref.shape == grad_out.shape and ref.is_contiguous()
    if ref.dtype != grad_out.dtype:
        grad_out = grad_out.to(ref.dtype)
    _need_cuda(grad_out, ref)
    ds = torch.empty_like(grad_out)
    rc = lib().pkm_score_transform_bwd(_ptr(scores), _ptr(out), _ptr(grad_out), DT[grad_out.dtype],
                                       grad_out.shape[0], grad_out.shape[1], float(temperature),
                                       TRANSFORM_MODES[mode], _ptr(ds), _stream(grad_out.device))
    _check(rc, "pkm_score_transform_bwd")
    return ds


# ---------------------------------------------------------------------------
# batch normalisation of the query projection
# ---------------------------------------------------------------------------
def batchnorm_workspace(n: int, c: int) -> int:
    nb = ctypes.c_size_t(0)
    _check(lib().pkm_batchnorm_workspace(n, c, ctypes.byref(nb)), "pkm_batchnorm_workspace")
    return int(nb.value)


def batchnorm_fwd(x: torch.Tensor, weight, bias, running_mean, running_var, training: bool, momentum: float,
                  eps: float):
    """``(out, save_mean, save_rstd)`` of ``F.batch_norm`` on a [n, c] tensor;
    the running statistics are updated in place when training."""
    assert x.dim() == 2 and x.is_contiguous()
    n, c = x.shape
    out = torch.empty_like(x)
    mean = torch.empty(c, dtype=torch.float32, device=x.device)
    rstd = torch.empty(c, dtype=torch.float32, device=x.device)
    p = weight if weight is not None else bias
    r = running_mean if running_mean is not None else running_var
    ws = torch.empty(batchnorm_workspace(n, c) if training else 0, dtype=torch.uint8, device=x.device)
    _need_cuda(x, weight, bias, running_mean, running_var)
    _check(lib().pkm_batchnorm_fwd(_ptr(x), DT[x.dtype], n, c, _ptr(weight), _ptr(bias),
                                   DT[p.dtype] if p is not None else 0, _ptr(running_mean), _ptr(running_var),
                                   DT[r.dtype] if r is not None else 0, int(training), float(momentum), float(eps),
                                   _ptr(out), _ptr(mean), _ptr(rstd), _ptr(ws) if ws.numel() else None, ws.numel(),
                                   _stream(x.device)), "pkm_batchnorm_fwd")
    return out, mean, rstd


def batchnorm_bwd(dy: torch.Tensor, x: torch.Tensor, mean: torch.Tensor, rstd: torch.Tensor, weight,
                  need_dx: bool = True, need_dw: bool = True, need_db: bool = True, param_dtype=None):
    """``(dx, dweight, dbias)`` of the training-mode batch normalisation."""
    assert x.dim() == 2 and x.is_contiguous() and dy.shape == x.shape
    dy = dy.contiguous()
    n, c = x.shape
    pdt = param_dtype if param_dtype is not None else (weight.dtype if weight is not None else x.dtype)
    dx = torch.empty_like(x) if need_dx else None
    dw = torch.empty(c, dtype=pdt, device=x.device) if need_dw else None
    db = torch.empty(c, dtype=pdt, device=x.device) if need_db else None
    ws = torch.empty(batchnorm_workspace(n, c), dtype=torch.uint8, device=x.device)
    _need_cuda(dy, x, mean, rstd, weight)
    _check(lib().pkm_batchnorm_bwd(_ptr(dy), _ptr(x), DT[x.dtype], n, c, _ptr(mean), _ptr(rstd), _ptr(weight),
                                   DT[pdt], _ptr(dx), _ptr(dw), _ptr(db), _ptr(ws), ws.numel(), _stream(x.device)),
           "pkm_batchnorm_bwd")
    return dx, dw, db


# ---------------------------------------------------------------------------
# fused FwPKM value update
# ---------------------------------------------------------------------------
def fw_update(values: torch.Tensor, grad: torch.Tensor, indices: torch.Tensor, scale: float, lr: float,
              weight_decay: float, grad_clip: bool, want_scaled: bool = True):
    """``(new_values, scaled_grad, counts)`` of the value branch of
    ``update_fw``; counts are int32 per row."""
    assert values.shape == grad.shape and values.dim() == 2 and values.dtype == grad.dtype
    values, grad = values.contiguous(), grad.contiguous()
    idx = indices.reshape(-1).contiguous()
    assert idx.dtype == torch.long
    _need_cuda(values, grad, idx)
    K, D = values.shape
    new = torch.empty_like(values)
    scaled = torch.empty_like(values) if want_scaled else None
    counts = torch.empty(K, dtype=torch.int32, device=values.device)
    _check(lib().pkm_fw_update(_ptr(values), _ptr(grad), DT[values.dtype], K, D, _ptr(idx), idx.numel(),
                               float(scale), float(lr), float(weight_decay), int(bool(grad_clip)), _ptr(new),
                               _ptr(scaled), _ptr(counts), _ptr(err_word(values.device)), _stream(values.device)),
           "pkm_fw_update")
    return new, scaled, counts


def fw_update_bwd(d_new: torch.Tensor, d_scaled: Optional[torch.Tensor], scaled: Optional[torch.Tensor],
                  counts: torch.Tensor, scale: float, lr: float, weight_decay: float, grad_clip: bool,
                  need_values: bool = True, need_grad: bool = True):
    """``(d_values, d_grad)`` of ``fw_update``."""
    d_new = d_new.contiguous()
    d_scaled = None if d_scaled is None else d_scaled.contiguous().to(d_new.dtype)
    _need_cuda(d_new, d_scaled, scaled, counts)
    K, D = d_new.shape
    dv = torch.empty_like(d_new) if need_values else None
    dg = torch.empty_like(d_new) if need_grad else None
    _check(lib().pkm_fw_update_bwd(_ptr(d_new), _ptr(d_scaled), _ptr(scaled), _ptr(counts), DT[d_new.dtype], K, D,
                                   float(scale), float(lr), float(weight_decay), int(bool(grad_clip)), _ptr(dv),
                                   _ptr(dg), _stream(d_new.device)), "pkm_fw_update_bwd")
    return dv, dg


# ---------------------------------------------------------------------------
# SwiGLU gate and column sums
# ---------------------------------------------------------------------------
def colsum_workspace(n: int, c: int) -> int:
    nb = ctypes.c_size_t(0)
    _check(lib().pkm_colsum_workspace(n, c, ctypes.byref(nb)), "pkm_colsum_workspace")
    return int(nb.value)


def swiglu_fwd(a: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    """``a * silu(h)`` in one pass ([n, c] contiguous, same dtype)."""
    assert a.shape == h.shape and a.dim() == 2 and a.dtype == h.dtype
    a, h = a.contiguous(), h.contiguous()
    _need_cuda(a, h)
    z = torch.empty_like(a)
    _check(lib().pkm_swiglu_fwd(_ptr(a), _ptr(h), DT[a.dtype], a.shape[0], a.shape[1], _ptr(z), _stream(a.device)),
           "pkm_swiglu_fwd")
    return z


def swiglu_bwd(dz: torch.Tensor, a: torch.Tensor, h: torch.Tensor, need_da: bool = True,
               bias_dtype: Optional[torch.dtype] = None):
    """``(da, dh, dbias_h)``; dbias_h (column sums of dh) when bias_dtype is given."""
    dz, a, h = dz.contiguous().to(a.dtype), a.contiguous(), h.contiguous()
    _need_cuda(dz, a, h)
    n, c = a.shape
    da = torch.empty_like(a) if need_da else None
    dh = torch.empty_like(a)
    db = torch.empty(c, dtype=bias_dtype, device=a.device) if bias_dtype is not None else None
    ws = torch.empty(colsum_workspace(n, c) if db is not None else 0, dtype=torch.uint8, device=a.device)
    _check(lib().pkm_swiglu_bwd(_ptr(dz), _ptr(a), _ptr(h), DT[a.dtype], n, c, _ptr(da), _ptr(dh), _ptr(db),
                                DT[bias_dtype] if bias_dtype is not None else 0, _ptr(ws) if ws.numel() else None,
                                ws.numel(), _stream(a.device)), "pkm_swiglu_bwd")
    return da, dh, db


def colsum(x: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Column sums of a [n, c] tensor (fixed order)."""
    x = x.contiguous()
    _need_cuda(x)
    n, c = x.shape
    out = torch.empty(c, dtype=out_dtype or x.dtype, device=x.device)
    ws = torch.empty(colsum_workspace(n, c), dtype=torch.uint8, device=x.device)
    _check(lib().pkm_colsum(_ptr(x), DT[x.dtype], n, c, _ptr(out), DT[out.dtype], _ptr(ws), ws.numel(),
                            _stream(x.device)), "pkm_colsum")
    return out


# ---------------------------------------------------------------------------
# ragged entry lists (row-sharded tables)
# ---------------------------------------------------------------------------
def segment_sum(rows: torch.Tensor, entry_row: torch.Tensor, entry_w: torch.Tensor, seg_offsets: torch.Tensor,
                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``out[s] = sum_{e in segment s} entry_w[e] * rows[entry_row[e]]``."""
    assert rows.dim() == 2 and rows.is_contiguous()
    entry_row = entry_row.to(torch.int32).contiguous()
    entry_w = entry_w.to(torch.float32).contiguous()
    seg_offsets = seg_offsets.to(torch.int64).contiguous()
    _need_cuda(rows, entry_row, entry_w, seg_offsets)
    K, D = rows.shape
    n_segs = seg_offsets.numel() - 1
    out = torch.empty((n_segs, D), dtype=out_dtype or rows.dtype, device=rows.device)
    nb = ctypes.c_size_t(0)
    _check(lib().pkm_segment_sum_workspace(n_segs, ctypes.byref(nb)), "pkm_segment_sum_workspace")
    ws = torch.empty(max(int(nb.value), 1), dtype=torch.uint8, device=rows.device)
    _check(lib().pkm_segment_sum(_ptr(rows), DT[rows.dtype], K, D, _ptr(entry_row), _ptr(entry_w), entry_row.numel(),
                                 _ptr(seg_offsets), n_segs, _ptr(out), DT[out.dtype], _ptr(ws), ws.numel(),
                                 _ptr(err_word(rows.device)), _stream(rows.device)), "pkm_segment_sum")
    return out


def bag_bwd_ragged(row_idx: torch.Tensor, src_of: torch.Tensor, psw: Optional[torch.Tensor], weight: torch.Tensor,
                   grad_rows: torch.Tensor, need_dpsw: bool = True):
    """K4 over a ragged entry list: ``(dW [K, D], dpsw [E] or None)``."""
    row_idx = row_idx.to(torch.int64).contiguous()
    src_of = src_of.to(torch.int32).contiguous()
    grad_rows = grad_rows.to(weight.dtype).contiguous()
    _need_cuda(row_idx, src_of, psw, weight, grad_rows)
    E = row_idx.numel()
    K, D = weight.shape
    dW = torch.empty((K, D), dtype=weight.dtype, device=weight.device)
    if psw is not None:
        psw = psw.contiguous()
    dpsw = torch.empty_like(psw) if (need_dpsw and psw is not None) else None
    ws_bytes = bag_bwd_workspace(E, 1, K, D)
    ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=weight.device)
    _check(lib().pkm_bag_bwd_ragged(_ptr(row_idx), _ptr(src_of), _ptr(psw), DT[psw.dtype] if psw is not None else 0,
                                    _ptr(weight), DT[weight.dtype], _ptr(grad_rows), E, grad_rows.shape[0], K, D,
                                    _ptr(dW), DT[dW.dtype], _ptr(dpsw), DT[dpsw.dtype] if dpsw is not None else 0,
                                    None, _ptr(ws), ws_bytes, _ptr(err_word(weight.device)),
                                    _stream(weight.device)), "pkm_bag_bwd_ragged")
    return dW, dpsw


# ---------------------------------------------------------------------------
# row-sharded routing
# ---------------------------------------------------------------------------
def _ws_query(fn, *args) -> int:
    nb = ctypes.c_size_t(0)
    _check(getattr(lib(), fn)(*args, ctypes.byref(nb)), fn)
    return int(nb.value)


def route_pack(indices: torch.Tensor, psw: Optional[torch.Tensor], shard_rows: int, world: int):
    """Stable partition of the occurrences of ``indices [B, L]`` by owner
    rank: ``(send_counts int64 [world], order, local_row, bag int32 [n],
    weight fp32 [n])``, all on the device."""
    assert indices.dim() == 2 and indices.dtype == torch.long
    indices = indices.contiguous()
    if psw is not None:
        assert psw.shape == indices.shape
        psw = psw.contiguous()
    _need_cuda(indices, psw)
    B, L = indices.shape
    n = B * L
    dev = indices.device
    send = torch.empty(world, dtype=torch.int64, device=dev)
    order = torch.empty(n, dtype=torch.int32, device=dev)
    local_row = torch.empty(n, dtype=torch.int32, device=dev)
    bag = torch.empty(n, dtype=torch.int32, device=dev)
    weight = torch.empty(n, dtype=torch.float32, device=dev)
    ws = torch.empty(max(_ws_query("pkm_route_pack_workspace", n), 1), dtype=torch.uint8, device=dev)
    _check(lib().pkm_route_pack(_ptr(indices), _ptr(psw), DT[psw.dtype] if psw is not None else 0, B, L,
                                int(shard_rows), int(world), _ptr(send), _ptr(order), _ptr(local_row),
                                _ptr(weight), _ptr(bag), _ptr(ws), ws.numel(), _ptr(err_word(dev)), _stream(dev)),
           "pkm_route_pack")
    return send, order, local_row, bag, weight


def route_segments(bag: torch.Tensor, group_counts: torch.Tensor, groups: int):
    """Runs of equal bag inside each group: ``(seg_of int32 [n], seg_start
    int64 [n + 1], seg_bag int32 [n], seg_counts int64 [groups])``; only the
    first ``seg_counts.sum()`` segments (and ``+ 1`` starts) are meaningful."""
    bag = bag.to(torch.int32).contiguous()
    group_counts = group_counts.to(torch.int64).contiguous()
    _need_cuda(bag, group_counts)
    n = bag.numel()
    dev = bag.device
    seg_of = torch.empty(n, dtype=torch.int32, device=dev)
    seg_start = torch.empty(n + 1, dtype=torch.int64, device=dev)
    seg_bag = torch.empty(n, dtype=torch.int32, device=dev)
    seg_counts = torch.empty(groups, dtype=torch.int64, device=dev)
    ws = torch.empty(max(_ws_query("pkm_route_segments_workspace", n), 1), dtype=torch.uint8, device=dev)
    _check(lib().pkm_route_segments(_ptr(bag), n, _ptr(group_counts), int(groups), _ptr(seg_of), _ptr(seg_start),
                                    _ptr(seg_bag), _ptr(seg_counts), _ptr(ws), ws.numel(), _stream(dev)),
           "pkm_route_segments")
    return seg_of, seg_start, seg_bag, seg_counts


def route_combine(partial: torch.Tensor, seg_bag: torch.Tensor, seg_counts: torch.Tensor, groups: int,
                  n_bags: int, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``out [n_bags, D]``: each bag's partial rows summed in group order."""
    assert partial.dim() == 2
    partial = partial.contiguous()
    seg_bag = seg_bag.to(torch.int32).contiguous()
    seg_counts = seg_counts.to(torch.int64).contiguous()
    _need_cuda(partial, seg_bag, seg_counts)
    n_seg, D = partial.shape
    dev = partial.device
    out = torch.empty((n_bags, D), dtype=out_dtype or partial.dtype, device=dev)
    ws = torch.empty(max(_ws_query("pkm_route_combine_workspace", int(groups), int(n_bags)), 1), dtype=torch.uint8,
                     device=dev)
    _check(lib().pkm_route_combine(_ptr(partial), DT[partial.dtype], n_seg, D, _ptr(seg_bag), _ptr(seg_counts),
                                   int(groups), int(n_bags), _ptr(out), DT[out.dtype], _ptr(ws), ws.numel(),
                                   _ptr(err_word(dev)), _stream(dev)), "pkm_route_combine")
    return out


# ---------------------------------------------------------------------------
# addressing statistics
# ---------------------------------------------------------------------------
def addr_stats(indices: torch.Tensor, rows: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """float64 device tensor ``[collided, covered, kl, counted]`` of the slot
    histogram of ``indices`` over ``[0, rows)``; stream-ordered, no sync."""
    idx = indices.reshape(-1).contiguous()
    assert idx.dtype == torch.long
    _need_cuda(idx)
    if idx.numel() == 0:
        raise ValueError("addressing statistics of an empty index set are undefined")
    need = ctypes.c_size_t()
    _check(lib().pkm_addr_stats_workspace(int(rows), ctypes.byref(need)), "pkm_addr_stats_workspace")
    ws = torch.empty(need.value, dtype=torch.uint8, device=idx.device)
    if out is None:
        out = torch.empty(4, dtype=torch.float64, device=idx.device)
    assert out.dtype == torch.float64 and out.numel() >= 4 and out.is_contiguous()
    _check(lib().pkm_addr_stats(_ptr(idx), idx.numel(), int(rows), _ptr(out), _ptr(ws), ws.numel(),
                                _ptr(err_word(idx.device)), _stream(idx.device)), "pkm_addr_stats")
    return out
