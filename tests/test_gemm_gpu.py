"""The tensor-core GEMM (``pkm_gemm_bf16``) against torch's fp32 matmul of
the same bf16 operands: every operand layout (K-major / MN-major A and B),
bias, fp32 and bf16 outputs, ragged M and N, row pitches wider than the
matrix, split K, and the batched forms the scoring backward uses.  fp32
outputs within 1e-5 (only the summation order differs), bf16 outputs within
one bf16 rounding (2^-8) normwise.  Also the bounded-wait path: with a wait
limit of zero polls every pipeline wait gives up, the kernel reports
PKM_DEVERR_TIMEOUT, drains and returns, and the next call is correct.
Each of these runs in both forms of the kernel: single CTAs and CTA pairs
(clusters of two sharing a 256-row MMA tile, forced even where M <= 128)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.fixture(params=[0, 1], ids=["single", "pair"])
def form(request):
    from modelos_b200 import _native
    _native.set_gemm_pair(request.param)
    yield request.param
    _native.set_gemm_pair(-1)


def _operand(rows, cols, g, pitch_extra=0):
    t = torch.randn(rows, cols + pitch_extra, generator=g).to(torch.bfloat16)
    return t[:, :cols].to(DEV)


CASES = [
    # M, N, K, a_mn, b_mn, bias, out dtype, extra row pitch
    (256, 512, 1024, False, False, True, torch.bfloat16, 0),    # forward projection x @ w.T + b
    (300, 264, 192, False, False, True, torch.float32, 8),      # ragged M, N not a tile multiple
    (1000, 1024, 2048, False, True, False, torch.bfloat16, 0),  # data gradient dy @ w
    (2048, 1024, 4096, True, True, False, torch.float32, 0),    # weight gradient dy.T @ x (split K)
    (512, 256, 16384, True, True, True, torch.bfloat16, 16),    # deep K, split and bias in the reduction
    (128, 8, 64, True, False, True, torch.float32, 0),          # one tile, one K block
    (4096, 2048, 1024, False, False, True, torch.bfloat16, 0),  # the query projection's shape
    (1000, 512, 1000, True, True, False, torch.float32, 0),     # weight gradient over 1000 tokens (K tail)
    (200, 136, 104, False, False, True, torch.bfloat16, 0),     # K tail on K-major operands
]


@pytest.mark.parametrize("M,N,K,a_mn,b_mn,bias,dt,pitch", CASES)
def test_gemm_matches_torch(M, N, K, a_mn, b_mn, bias, dt, pitch, form):
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(M + N + K)
    a = _operand(K, M, g, pitch) if a_mn else _operand(M, K, g, pitch)
    b = _operand(K, N, g, pitch) if b_mn else _operand(N, K, g, pitch)
    bv = torch.randn(N, generator=g).to(torch.bfloat16).to(DEV) if bias else None
    c = _native.gemm(a, b, a_mn=a_mn, b_mn=b_mn, bias=bv, out_dtype=dt)
    torch.cuda.synchronize()
    _native.check_device_errors()
    A = (a.T if a_mn else a).float()
    Bm = (b.T if b_mn else b).float()
    ref = A @ Bm.T
    if bias:
        ref = ref + bv.float()
    assert c.shape == (M, N) and c.dtype == dt
    tol = 1e-5 if dt == torch.float32 else 2.0 ** -8
    assert rel_err(c, ref) < tol


def test_gemm_batched_scoring_backward_forms(form):
    """The two batched GEMMs of the scoring backward over (head, half) groups:
    dq[t, g, :] = dS[t, g, :] @ keys_g and dk_g = dS[:, g, :].T @ q[:, g, :]."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(7)
    T, G, n, half = 1000, 8, 512, 256
    dS = torch.randn(T, G * n, generator=g).to(torch.bfloat16).to(DEV)
    keys = torch.randn(G * n, half, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(T, G * half, generator=g).to(torch.bfloat16).to(DEV)
    dq = torch.empty(T, G * half, dtype=torch.bfloat16, device=DEV)
    _native.gemm(dS, keys, b_mn=True, batch=G, M=T, N=half, K=n, a_batch=(n, 0), b_batch=(0, n), out=dq,
                 c_batch_stride=half)
    dk = torch.empty(G * n, half, dtype=torch.float32, device=DEV)
    _native.gemm(dS, q, a_mn=True, b_mn=True, batch=G, M=n, N=half, K=T - T % 64, a_batch=(n, 0),
                 b_batch=(half, 0), out=dk, c_batch_stride=n * half)
    torch.cuda.synchronize()
    _native.check_device_errors()
    dSv = dS.float().view(T, G, n)
    ref_dq = torch.einsum("tgn,gnd->tgd", dSv, keys.float().view(G, n, half)).reshape(T, G * half)
    Tk = T - T % 64
    ref_dk = torch.einsum("tgn,tgd->gnd", dSv[:Tk], q.float().view(T, G, half)[:Tk]).reshape(G * n, half)
    assert rel_err(dq, ref_dq) < 2.0 ** -8
    assert rel_err(dk, ref_dk) < 1e-5


def test_gemm_rejects_bad_arguments():
    from modelos_b200 import _native
    a = torch.zeros(128, 104, dtype=torch.bfloat16, device=DEV)
    b = torch.zeros(64, 104, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="multiple of 64"):
        _native.gemm(a, b, K=72)  # a K tail that is not the operands' edge
    a = torch.zeros(128, 64, dtype=torch.bfloat16, device=DEV)
    b = torch.zeros(12, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        _native.gemm(a, b)  # N = 12


def test_gemm_bounded_waits_time_out_and_recover(form):
    """Zero polls per pipeline wait: the kernel sets PKM_DEVERR_TIMEOUT,
    drains its copies and MMAs, releases TMEM and returns; with the default
    limit restored the same call on the same context is correct again."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(3)
    a = torch.randn(512, 1024, generator=g).to(torch.bfloat16).to(DEV)
    b = torch.randn(256, 1024, generator=g).to(torch.bfloat16).to(DEV)
    _native.read_device_errors()
    try:
        _native.set_wait_limit(0)
        _native.gemm(a, b, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert _native.read_device_errors() & _native.DEVERR_TIMEOUT
    finally:
        _native.set_wait_limit(-1)
    c = _native.gemm(a, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _native.read_device_errors() == 0
    assert rel_err(c, a.float() @ b.float().T) < 1e-5
    assert np.isfinite(c.cpu().numpy()).all()


@pytest.mark.parametrize("M,C,V", [(4096, 1024, 1024), (1000, 256, 200)])
def test_fused_swiglu_gemms_equal_unfused_kernels(form, M, C, V):
    """The gate in the GEMM epilogues (``pkm_gemm_swiglu_fwd/bwd``) gives the
    same bits as the GEMM followed by the standalone gate kernels, and
    matches the reference's op sequence in fp32 within bf16 tolerance.
    Neither shape splits K in the unfused GEMMs (the same summation order);
    the second has boxes at the edges of M and N (direct accesses)."""
    import torch.nn.functional as F

    from modelos_b200 import _native
    g = torch.Generator().manual_seed(11)
    x = torch.randn(M, C, generator=g).to(torch.bfloat16).to(DEV)
    a = (torch.randn(M, V, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    ws = (torch.randn(V, C, generator=g) * C ** -0.5).to(torch.bfloat16).to(DEV)
    bs = (torch.randn(V, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    wv = (torch.randn(C, V, generator=g) * V ** -0.5).to(torch.bfloat16).to(DEV)
    dy = torch.randn(M, C, generator=g).to(torch.bfloat16).to(DEV)
    h, z = _native.gemm_swiglu_fwd(x, ws, bs, a)
    h2 = _native.gemm(x, ws, bias=bs)
    z2 = _native.swiglu_fwd(a, h2)
    assert torch.equal(h, h2) and torch.equal(z, z2)
    da, dh = _native.gemm_swiglu_bwd(dy, wv, a, h)
    dz = _native.gemm(dy, wv, b_mn=True)
    da2, dh2, _ = _native.swiglu_bwd(dz, a, h, need_da=True, bias_dtype=None)
    assert torch.equal(da, da2) and torch.equal(dh, dh2)
    # against the reference's op sequence in fp32
    hr = x.float() @ ws.float().T + bs.float()
    zr = a.float() * F.silu(hr)
    assert rel_err(h, hr) < 2e-2 and rel_err(z, zr) < 2e-2
    dzr = dy.float() @ wv.float()
    sig = torch.sigmoid(hr)
    assert rel_err(da, dzr * F.silu(hr)) < 2e-2
    assert rel_err(dh, dzr * a.float() * sig * (1 + hr * (1 - sig))) < 2e-2


def test_gemm_pair_equals_single_without_split():
    """Where neither form splits K, the pair form's 256-row MMAs sum every
    output in the same K order as the single form's 128-row MMAs: the same
    bits."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(5)
    outs = []
    a = torch.randn(4096, 1024, generator=g).to(torch.bfloat16).to(DEV)
    b = torch.randn(2048, 1024, generator=g).to(torch.bfloat16).to(DEV)
    try:
        for mode in (0, 1):
            _native.set_gemm_pair(mode)
            outs.append(_native.gemm(a, b, out_dtype=torch.float32))
    finally:
        _native.set_gemm_pair(-1)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert torch.equal(outs[0], outs[1])


F32_CASES = [
    # M, N, K, a_mn, b_mn
    (300, 200, 100, False, False),
    (256, 256, 4096, True, True),
    (1000, 136, 512, False, True),
    (7, 5, 3, True, False),
    (512, 256, 8192, True, True),     # few tiles, deep K: split K (workspace, fixed-order reduction)
    (130, 70, 3001, False, False),    # split K with ragged M, N and K
    (257, 129, 1029, True, False),    # odd pitches: scalar loads
]


@pytest.mark.parametrize("M,N,K,a_mn,b_mn", F32_CASES)
def test_gemm_f32_matches_torch(M, N, K, a_mn, b_mn):
    """The fp32 CUDA-core GEMM (``pkm_gemm_f32``) vs torch fp32 (no TF32)."""
    from modelos_b200 import _native
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator().manual_seed(M * 7 + K)
    a = torch.randn((K, M) if a_mn else (M, K), generator=g).to(DEV)
    b = torch.randn((K, N) if b_mn else (N, K), generator=g).to(DEV)
    c = _native.gemm_f32(a, b, a_mn=a_mn, b_mn=b_mn)
    ref = (a.T if a_mn else a).double() @ (b.T if b_mn else b).double().T
    assert rel_err(c, ref) < 1e-5


def test_gemm_f32_batched_split_matches_torch():
    """The fast-weight scoring backward's dK form, batched over (head, half)
    groups with few tiles and a deep K (split K): dk_g = dS[:, g, :].T @ q_g."""
    from modelos_b200 import _native
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator().manual_seed(13)
    T, G, n, half = 4096, 4, 256, 128
    dS = torch.randn(T, G * n, generator=g).to(DEV)
    q = torch.randn(T, G * half, generator=g).to(DEV)
    dk = torch.empty(G * n, half, dtype=torch.float32, device=DEV)
    _native.gemm_f32(dS, q, a_mn=True, b_mn=True, batch=G, M=n, N=half, K=T, a_batch=(n, 0), b_batch=(half, 0),
                     out=dk, c_batch_stride=n * half)
    ref = torch.einsum("tgn,tgh->gnh", dS.double().view(T, G, n), q.double().view(T, G, half)).reshape(G * n, half)
    assert rel_err(dk, ref) < 1e-5


def test_group_mm_second_derivatives_match_einsum():
    """The fast-weight memory's sub-key scores (``SubkeyScores``: sequential
    fp32 kernel forward, ``GroupMM`` backward on the fp32 GEMM) give the
    same first and second derivatives as the reference's einsum formulation
    (``fwpkm/fwpkm.py:861``) evaluated in float64."""
    from modelos_b200.fwpkm.fwpkm import SubkeyScores
    g = torch.Generator().manual_seed(5)
    T, H, n, kd = 96, 4, 64, 128
    q0 = torch.randn(T * H, kd, generator=g)
    k0 = torch.randn(2 * H * n, kd // 2, generator=g) * 0.1
    W = torch.randn(T * H, 2, n, generator=g)
    U = torch.randn(T * H, kd, generator=g)
    V = torch.randn(2 * H * n, kd // 2, generator=g)

    def run(q, k, scores_fn):
        s = scores_fn(q, k)
        gq, gk = torch.autograd.grad((s * W.to(s)).sum(), (q, k), create_graph=True)
        loss2 = (gq * U.to(gq)).sum() + (gk * V.to(gk)).sum() + (s ** 2).sum()
        return [t.double().cpu() for t in (gq, gk, *torch.autograd.grad(loss2, (q, k)))]

    def einsum_scores(q, k):
        return torch.einsum("thpd,hpnd->thpn", q.view(T, H, 2, kd // 2), k.view(H, 2, n, kd // 2)).reshape(-1, 2, n)

    got = run(q0.to(DEV).requires_grad_(True), k0.to(DEV).requires_grad_(True),
              lambda q, k: SubkeyScores.apply(q, k, H))
    ref = run(q0.double().requires_grad_(True), k0.double().requires_grad_(True), einsum_scores)
    for a_, b_ in zip(got, ref):
        assert rel_err(a_, b_) < 1e-5
