"""tcgen05 GEMM numerics against fp32 PyTorch on the same bf16 inputs."""

import pytest
import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.gemm import (
    EPI_ADD_F32, EPI_BF16, EPI_F32, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD, gemm, linear_wgrad,
)

pytestmark = pytest.mark.gpu
dev = "cuda"


def _bf(*shape):
    return (torch.randn(*shape, device=dev) * 0.5).to(torch.bfloat16)


def _close(a, b, tol=2e-2):
    torch.testing.assert_close(a.float(), b.float(), atol=tol * max(1.0, b.abs().max().item() * 0.05), rtol=tol)


@pytest.mark.parametrize("bn", [64, 128, 192, 256])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("mnk", [(256, 512, 256), (200, 136, 72), (1024, 768, 2048)])
def test_gemm_majors(bn, a_mn, b_mn, mnk):
    torch.manual_seed(0)
    m, n, k = mnk
    a = _bf(k, m) if a_mn else _bf(m, k)
    b = _bf(k, n) if b_mn else _bf(n, k)
    A = a.float().t() if a_mn else a.float()
    B = b.float() if b_mn else b.float().t()
    ref = A @ B
    out = torch.empty(m, n, device=dev, dtype=torch.float32)
    gemm(a, b, out, m, n, k, a_mn=a_mn, b_mn=b_mn, epi=EPI_F32, bn=bn)
    _native.check_status()
    _close(out, ref, 1e-2)
    out16 = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    gemm(a, b, out16, m, n, k, a_mn=a_mn, b_mn=b_mn, epi=EPI_BF16, bn=bn)
    _close(out16, ref)


@pytest.mark.parametrize("mode,bn", [(1, 256), (2, 256), (2, 192)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_cta_pair_matches_single_cta(a_mn, b_mn, mode, bn):
    """The 2-SM kernel (256 x 256 tiles on CTA pairs, cta_group::2 MMAs) accumulates
    every output element over K in the same order as the single-CTA kernel: the two
    must agree bit for bit, also with the SwiGLU epilogue (B halves split across the
    pair) and with split-K reduce-adds of exactly representable values."""
    torch.manual_seed(5)
    C = _native.module()
    m, n, k = 1000, 768, 520
    a = _bf(k, m) if a_mn else _bf(m, k)
    b = _bf(k, n) if b_mn else _bf(n, k)
    outs = []
    prev = C.gemm_pair_mode(-1)
    try:
        for md in (mode, 0):
            C.gemm_pair_mode(md)
            out = torch.empty(m, n, device=dev, dtype=torch.float32)
            gemm(a, b, out, m, n, k, a_mn=a_mn, b_mn=b_mn, epi=EPI_F32, bn=bn)
            outs.append(out)
            if not a_mn and not b_mn:
                F = n // 2
                h = torch.empty(m, F, device=dev, dtype=torch.bfloat16)
                gu = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
                gemm(a, b, h, m, n, k, epi=EPI_SWIGLU, aux=gu, bn=bn)
                outs += [h, gu]
        _native.check_status()
    finally:
        C.gemm_pair_mode(prev)
    half = len(outs) // 2
    for x, y in zip(outs[:half], outs[half:]):
        assert torch.equal(x, y)
    A = a.float().t() if a_mn else a.float()
    B = b.float() if b_mn else b.float().t()
    _close(outs[0], A @ B, 1e-2)
    ints = torch.randint(-2, 3, (m, k), device=dev).to(torch.bfloat16)
    intw = torch.randint(-2, 3, (n, k), device=dev).to(torch.bfloat16)
    acc = torch.zeros(m, n, device=dev)
    prev = C.gemm_pair_mode(mode)
    try:
        gemm(ints, intw, acc, m, n, k, epi=EPI_ADD_F32, splits=3, bn=bn)
    finally:
        C.gemm_pair_mode(prev)
    _native.check_status()
    assert torch.equal(acc, ints.float() @ intw.float().t())


def test_gemm_accumulate_and_splitk():
    torch.manual_seed(1)
    m, n, k = 384, 256, 4096
    a, b = _bf(m, k), _bf(n, k)
    ref = a.float() @ b.float().t()
    base = torch.randn(m, n, device=dev)
    out = base.clone()
    gemm(a, b, out, m, n, k, epi=EPI_ADD_F32, bn=128)
    _close(out, base + ref, 1e-2)
    acc = torch.zeros(m, n, device=dev)
    gemm(a, b, acc, m, n, k, epi=EPI_ADD_F32, splits=4, bn=128)
    _close(acc, ref, 1e-2)
    _native.check_status()


@pytest.mark.parametrize("shape", [(8192, 768, 768), (8192, 1280, 768), (8192, 768, 2048), (2048, 32000, 768)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_linear_wgrad_splitk(shape, accumulate):
    torch.manual_seed(4)
    t, n, k = shape
    dy, x = _bf(t, n), _bf(t, k)
    ref = dy.float().t() @ x.float()
    base = torch.randn(n, k, device=dev)
    out = base.clone()
    linear_wgrad(dy, x, out, accumulate=accumulate)
    _native.check_status()
    _close(out, ref + (base if accumulate else 0), 1e-2)


@pytest.mark.parametrize("bn", [64, 128, 192, 256])
def test_gemm_swiglu(bn):
    torch.manual_seed(2)
    m, d, F = 320, 256, 384
    x, w = _bf(m, d), _bf(2 * F, d)
    h = torch.empty(m, F, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(m, 2 * F, device=dev, dtype=torch.bfloat16)
    gemm(x, w, h, m, 2 * F, d, epi=EPI_SWIGLU, aux=gu, bn=bn)
    full = x.float() @ w.float().t()
    _close(gu, full)
    g, u = gu.float()[:, :F], gu.float()[:, F:]
    _close(h, torch.nn.functional.silu(g) * u)
    dh = _bf(m, F)
    dgu = torch.empty(m, 2 * F, device=dev, dtype=torch.bfloat16)
    _native.module().swiglu_bwd_packed(dh, gu, dgu)
    s = torch.sigmoid(g)
    _close(dgu[:, F:], dh.float() * g * s)
    _close(dgu[:, :F], dh.float() * u * s * (1 + g * (1 - s)))
    _native.check_status()


@pytest.mark.parametrize("bn", [64, 128, 192, 256])
def test_gemm_swiglu_bwd_epilogue(bn):
    """Down-projection dgrad with the SwiGLU backward fused: dh = dy @ Wd stays in
    TMEM and [dg | du] is written, against the fp32 chain dy @ Wd -> SwiGLU'."""
    torch.manual_seed(4)
    m, d, F = 300, 256, 416
    dy, wd = _bf(m, d), _bf(d, F)
    gu = _bf(m, 2 * F) * 2
    dgu = torch.full((m, 2 * F), float("nan"), device=dev, dtype=torch.bfloat16)
    gemm(dy, wd, dgu, m, F, d, b_mn=True, epi=EPI_SWIGLU_BWD, aux=gu, bn=bn)
    _native.check_status()
    dh = dy.float() @ wd.float()
    g, u = gu.float()[:, :F], gu.float()[:, F:]
    s = torch.sigmoid(g)
    _close(dgu[:, :F], dh * u * s * (1 + g * (1 - s)))
    _close(dgu[:, F:], dh * g * s)


@pytest.mark.parametrize("hd,bn", [(64, 128), (64, 192), (64, 256), (128, 256), (64, 64)])
def test_gemm_rope_epilogue(hd, bn):
    torch.manual_seed(3)
    t, d, h, hk = 300, 256, 4, 2
    n = (h + 2 * hk) * hd
    x, w = _bf(t, d), _bf(n, d)
    pos = torch.randint(0, 500, (t,), device=dev, dtype=torch.int32)
    inv = 1.0 / (10000 ** (torch.arange(0, hd, 2, device=dev).float() / hd))
    ang = torch.outer(torch.arange(512, device=dev).float(), inv)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    out = torch.empty(t, n, device=dev, dtype=torch.bfloat16)
    gemm(x, w, out, t, n, d, epi=EPI_ROPE, pos=pos, cos=cos, sin=sin, head_dim=hd, n_rope_cols=(h + hk) * hd, bn=bn)
    y = (x.float() @ w.float().t()).view(t, -1, hd)
    c, s = cos[pos.long()][:, None], sin[pos.long()][:, None]
    half = hd // 2
    rot = torch.cat([y[..., :half] * c - y[..., half:] * s, y[..., half:] * c + y[..., :half] * s], -1)
    ref = torch.cat([rot[:, : h + hk], y[:, h + hk :]], 1).reshape(t, n)
    _close(out, ref)
    _native.check_status()


def test_pair_gemm_abort_path_reports_status():
    """The even CTA of every pair stops arming after two of sixteen k-blocks without
    stopping the odd CTA (a test knob, no fault).  The odd CTA loads five stages ahead and
    its bounded wait for the next free stage runs out; it reports the k-blocks it issued,
    the even CTA arms those stages with the odd CTA's bytes and drains them, the MMA
    issuer's wait for the next stage runs out, and the kernel records a status code and
    returns with no load in flight.  The GPU keeps working."""
    C = _native.module()
    torch.manual_seed(1)
    m, n, k = 512, 512, 1024  # 256-wide tiles on CTA pairs, sixteen 64-deep k-blocks
    a, b = _bf(m, k), _bf(n, k)
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    d = torch.cuda.current_device()
    C.status_read(d, True)
    prev_mode = C.gemm_pair_mode(2)
    prev = C.gemm_pair_test_arm_limit(2)
    try:
        gemm(a, b, out, m, n, k, epi=EPI_BF16, bn=256)
        torch.cuda.synchronize()
    finally:
        C.gemm_pair_test_arm_limit(prev)
    code = C.status_read(d, True)
    assert code in (121, 124, 126, 127), code
    gemm(a, b, out, m, n, k, epi=EPI_BF16, bn=256)
    C.gemm_pair_mode(prev_mode)
    _native.check_status()
    _close(out, a.float() @ b.float().t())
