"""Native elementwise / CE / attention kernels against fp32 PyTorch references."""

import math

import pytest
import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.attention import attn_backward_packed, attn_forward_packed, attention_plan
from packbalance_b200.ops.cross_entropy import linear_cross_entropy
from packbalance_b200.ops.reference import chunked_linear_cross_entropy, rmsnorm_reference, swiglu_reference
from packbalance_b200.ops.rmsnorm import rmsnorm
from packbalance_b200.ops.swiglu import swiglu

pytestmark = pytest.mark.gpu
dev = "cuda"


def test_rmsnorm_fwd_bwd():
    torch.manual_seed(0)
    x = torch.randn(333, 768, device=dev)
    w = torch.randn(768, device=dev)
    g = torch.randn(333, 768, device=dev)
    x1, w1 = x.clone().requires_grad_(), w.clone().requires_grad_()
    y1 = rmsnorm_reference(x1, w1, 1e-5)
    y1.backward(g)
    x2, w2 = x.clone().requires_grad_(), w.clone().requires_grad_()
    y2 = rmsnorm(x2, w2, 1e-5)
    y2.backward(g)
    torch.testing.assert_close(y2, y1, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(x2.grad, x1.grad, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(w2.grad, w1.grad, atol=1e-3, rtol=1e-4)
    _native.check_status()


def test_add_rmsnorm():
    torch.manual_seed(0)
    C = _native.module()
    x = torch.randn(300, 768, device=dev)
    delta = torch.randn(300, 768, device=dev).to(torch.bfloat16)
    w = torch.randn(768, device=dev)
    xo, y, rstd = C.add_rmsnorm_fwd(x, delta, w, 1e-5, True)
    ref_x = x + delta.float()
    torch.testing.assert_close(xo, ref_x)
    torch.testing.assert_close(y.float(), rmsnorm_reference(ref_x, w, 1e-5), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(rstd, torch.rsqrt(ref_x.square().mean(-1) + 1e-5), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("n", [256, 512, 768, 1024, 2048, 4096, 800])
def test_rmsnorm_widths_fused_residual(n):
    """Register-resident kernels (n = 128 k) and the generic fallback, with the fused
    residual add (forward) and residual gradient + bf16 copy (backward)."""
    torch.manual_seed(n)
    C = _native.module()
    rows = 1000
    x = torch.randn(rows, n, device=dev)
    delta = torch.randn(rows, n, device=dev).to(torch.bfloat16)
    w = torch.randn(n, device=dev)
    xo, y, rstd = C.add_rmsnorm_fwd(x, delta, w, 1e-5, True)
    ref_x = x + delta.float()
    torch.testing.assert_close(xo, ref_x)
    torch.testing.assert_close(y.float(), rmsnorm_reference(ref_x, w, 1e-5), atol=3e-2, rtol=1e-2)
    dy = torch.randn(rows, n, device=dev)
    dres = torch.randn(rows, n, device=dev)
    xr, wr = ref_x.clone().requires_grad_(), w.clone().requires_grad_()
    rmsnorm_reference(xr, wr, 1e-5).backward(dy)
    dxb = torch.empty(rows, n, device=dev, dtype=torch.bfloat16)
    dw = torch.full((n,), 7.0, device=dev)
    dx = C.rmsnorm_bwd(dy, xo, w, rstd, dres, dxb, dw, False)
    torch.testing.assert_close(dx, xr.grad + dres, atol=1e-3, rtol=1e-4)
    torch.testing.assert_close(dxb.float(), dx, atol=3e-2, rtol=1e-2)
    torch.testing.assert_close(dw, wr.grad, atol=2e-3, rtol=1e-4)
    C.rmsnorm_bwd(dy, xo, w, rstd, None, None, dw, True)  # accumulate
    torch.testing.assert_close(dw, 2 * wr.grad, atol=4e-3, rtol=1e-4)
    _native.check_status()


def test_swiglu_fwd_bwd():
    torch.manual_seed(0)
    g, u, d = (torch.randn(64, 100, device=dev) for _ in range(3))
    g1, u1 = g.clone().requires_grad_(), u.clone().requires_grad_()
    swiglu_reference(g1, u1).backward(d)
    g2, u2 = g.clone().requires_grad_(), u.clone().requires_grad_()
    out = swiglu(g2, u2)
    out.backward(d)
    torch.testing.assert_close(out, swiglu_reference(g, u), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(g2.grad, g1.grad, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(u2.grad, u1.grad, atol=1e-5, rtol=1e-5)


def test_embedding_and_adamw_and_norm():
    torch.manual_seed(0)
    C = _native.module()
    w = torch.randn(100, 32, device=dev)
    ids = torch.randint(0, 100, (77,), device=dev)
    torch.testing.assert_close(C.embedding_fwd(ids, w), w[ids])
    dx = torch.randn(77, 32, device=dev)
    grad = torch.zeros_like(w)
    C.embedding_bwd(ids, dx, grad, False)
    torch.testing.assert_close(grad, torch.zeros_like(w).index_add_(0, ids, dx), atol=1e-5, rtol=1e-5)
    x = torch.randn(1001, device=dev)
    torch.testing.assert_close(C.l2_norm(x), x.norm(), atol=1e-4, rtol=1e-5)
    # AdamW kernel vs torch.optim.AdamW (with clipping by 0.5)
    p = torch.randn(1003, device=dev)
    g = torch.randn(1003, device=dev)
    ref = p.clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    norm = g.norm()
    ref.grad = g * min(1.0, 0.5 / (norm.item() + 1e-6))
    opt.step()
    p0 = p.clone()
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    sh = torch.empty(1003, device=dev, dtype=torch.bfloat16)
    skipped = torch.zeros((), device=dev, dtype=torch.int32)
    C.adamw_step(p, g, m, v, sh, norm, skipped, 1e-2, 0.9, 0.95, 1e-8, 0.1, 0.1, 1 - 0.95, 0.5, True, None)
    torch.testing.assert_close(p, ref.detach(), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(sh.float(), p.to(torch.bfloat16).float())
    # lr and bias corrections from device memory (the CUDA-graph path): same update
    p2, m2, v2 = p0.clone(), torch.zeros_like(p), torch.zeros_like(p)
    hp = torch.tensor([1e-2, 0.1, 1 - 0.95], device=dev)
    C.adamw_step(p2, g, m2, v2, sh, norm, skipped, 0.0, 0.9, 0.95, 1e-8, 0.1, 1.0, 1.0, 0.5, True, hp)
    torch.testing.assert_close(p2, p, atol=0, rtol=0)
    _native.check_status()


@pytest.mark.parametrize("z", [0.0, 0.01])
@pytest.mark.parametrize("shape", [(2, 32, 32, 128), (1, 700, 256, 1000), (1, 2048, 768, 32000)])
def test_fused_linear_ce(z, shape):
    torch.manual_seed(0)
    b, t, d, v = shape
    x = (torch.randn(b, t, d, device=dev) * 0.5).to(torch.bfloat16).float()
    w = (torch.randn(v, d, device=dev) * 0.05).to(torch.bfloat16).float()
    tgt = torch.randint(0, v, (b, t), device=dev)
    tgt[:, ::5] = -100
    x1, w1 = x.clone().requires_grad_(), w.clone().requires_grad_()
    loss1 = chunked_linear_cross_entropy(x1, w1, tgt, chunk_size=1024, z_loss_coeff=z)
    loss1.backward()
    x2, w2 = x.clone().requires_grad_(), w.clone().requires_grad_()
    loss2 = linear_cross_entropy(x2, w2, tgt, chunk_size=1024, z_loss_coeff=z)
    loss2.backward()
    _native.check_status()
    torch.testing.assert_close(loss2, loss1, atol=2e-2 * max(1.0, abs(loss1.item()) * 1e-3), rtol=1e-3)
    torch.testing.assert_close(x2.grad, x1.grad, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(w2.grad, w1.grad, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("z", [0.0, 0.01])
@pytest.mark.parametrize("t,d,v", [(700, 256, 1000), (2048, 768, 32000)])
def test_lmhead_ce_kept_logits(z, t, d, v):
    """Forward keeping the bf16 logits, backward from them (in-place dlogits): loss,
    dx and dW against the chunked fp32 reference, and the kept logits against x @ W.T."""
    from packbalance_b200.ops.cross_entropy import lmhead_ce_backward, lmhead_ce_forward

    torch.manual_seed(1)
    x = (torch.randn(t, d, device=dev) * 0.5).to(torch.bfloat16)
    w = (torch.randn(v, d, device=dev) * 0.05).to(torch.bfloat16)
    tgt = torch.randint(0, v, (t,), device=dev)
    tgt[::7] = -100
    logits = torch.empty(t, v, device=dev, dtype=torch.bfloat16)
    loss, lse = lmhead_ce_forward(x, w, tgt, -100, z, logits_out=logits)
    _native.check_status()
    ref_logits = x.float() @ w.float().t()
    torch.testing.assert_close(logits.float(), ref_logits, atol=2e-2, rtol=2e-2)
    g = torch.tensor(0.5, device=dev)
    dw = torch.empty(v, d, device=dev)
    dx = lmhead_ce_backward(x, w, tgt, lse, g, dw, False, -100, z, logits=logits)
    _native.check_status()
    x1, w1 = x.float().requires_grad_(), w.float().requires_grad_()
    loss1 = chunked_linear_cross_entropy(x1, w1, tgt, chunk_size=1024, z_loss_coeff=z)
    (loss1 * 0.5).backward()
    torch.testing.assert_close(loss, loss1.detach(), atol=2e-2 * max(1.0, abs(loss1.item()) * 1e-3), rtol=1e-3)
    torch.testing.assert_close(dx, x1.grad, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(dw, w1.grad, atol=2e-2, rtol=2e-2)


def _attn_ref(qkv, doc_start, h, hk, d):
    t = qkv.shape[0]
    q = qkv[:, : h * d].float().view(t, h, d)
    k = qkv[:, h * d : (h + hk) * d].float().view(t, hk, d).repeat_interleave(h // hk, 1)
    v = qkv[:, (h + hk) * d :].float().view(t, hk, d).repeat_interleave(h // hk, 1)
    pos = torch.arange(t, device=qkv.device)
    allowed = (pos[None] <= pos[:, None]) & (pos[None] >= doc_start.long()[:, None])
    s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(d)
    s = s.masked_fill(~allowed[None], float("-inf"))
    p = torch.softmax(s, -1)
    return torch.einsum("hqk,khd->qhd", p, v).reshape(t, h * d), torch.logsumexp(s, -1)


def _doc_start(lengths, device=dev):
    starts = []
    off = 0
    for n in lengths:
        starts += [off] * n
        off += n
    return torch.tensor(starts, device=device, dtype=torch.int32)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("lengths", [[1, 127, 128, 300, 17, 1, 450], [2048], [40] * 30 + [5]])
def test_attention_fwd_bwd(d, lengths):
    torch.manual_seed(0)
    h, hk = 4, 2
    ds = _doc_start(lengths)
    t = ds.numel()
    qkv = (torch.randn(t, (h + 2 * hk) * d, device=dev)).to(torch.bfloat16)
    plan = attention_plan(ds, h, hk)
    o, lse = attn_forward_packed(qkv, plan, h, hk, d)
    _native.check_status()
    ref_o, ref_lse = _attn_ref(qkv, ds, h, hk, d)
    torch.testing.assert_close(o.float(), ref_o, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse, ref_lse, atol=1e-2, rtol=1e-3)
    # backward against autograd of the fp32 reference
    do = torch.randn(t, h * d, device=dev).to(torch.bfloat16)
    q32 = qkv.float().requires_grad_()
    ro, _ = _attn_ref(q32, ds, h, hk, d)
    ro.backward(do.float())
    dqkv = attn_backward_packed(qkv, o, do, lse, plan, h, hk, d)
    _native.check_status()
    ref = q32.grad
    for name, sl in (("dq", slice(0, h * d)), ("dk", slice(h * d, (h + hk) * d)), ("dv", slice((h + hk) * d, None))):
        torch.testing.assert_close(dqkv[:, sl].float(), ref[:, sl], atol=3e-2, rtol=3e-2, msg=name)
