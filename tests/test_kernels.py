import pytest
import torch
import torch.nn.functional as F

from packbalance_b200.ops.cross_entropy import linear_cross_entropy
from packbalance_b200.ops.reference import chunked_linear_cross_entropy, rmsnorm_reference, rope_reference, swiglu_reference
from packbalance_b200.ops.rmsnorm import rmsnorm
from packbalance_b200.ops.rope import rope_inplace
from packbalance_b200.ops.swiglu import swiglu


def _full_ce(x, w, t, z=0.0):
    logits = x @ w.t()
    loss = F.cross_entropy(logits, t, ignore_index=-100, reduction="sum")
    if z:
        lse = torch.logsumexp(logits.float(), dim=-1)
        loss = loss + z * lse[t != -100].square().sum()
    return loss


def test_rmsnorm_cpu_matches_reference() -> None:
    torch.manual_seed(0)
    x, w = torch.randn(8, 32), torch.randn(32)
    torch.testing.assert_close(rmsnorm(x, w, 1e-5), rmsnorm_reference(x, w, 1e-5))


def test_swiglu_cpu_matches_reference() -> None:
    torch.manual_seed(0)
    g, u = torch.randn(8, 16), torch.randn(8, 16)
    torch.testing.assert_close(swiglu(g, u), swiglu_reference(g, u))


@pytest.mark.parametrize("z", [0.0, 0.01])
def test_chunked_ce_matches_full(z: float) -> None:
    torch.manual_seed(0)
    x, w = torch.randn(37, 32), torch.randn(64, 32)
    t = torch.randint(0, 64, (37,))
    t[::7] = -100
    x1, w1 = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    _full_ce(x1, w1, t, z).backward()
    x2, w2 = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    loss = linear_cross_entropy(x2, w2, t, chunk_size=8, z_loss_coeff=z)
    loss.backward()
    torch.testing.assert_close(loss, _full_ce(x, w, t, z), atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(x2.grad, x1.grad, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(w2.grad, w1.grad, atol=1e-4, rtol=1e-4)
    loss3 = chunked_linear_cross_entropy(x, w, t, chunk_size=5, z_loss_coeff=z)
    torch.testing.assert_close(loss3, loss.detach(), atol=1e-4, rtol=1e-4)


def test_rope_inverse_roundtrip_cpu() -> None:
    torch.manual_seed(0)
    t, heads, d = 10, 3, 8
    x = torch.randn(t, heads * d)
    pos = torch.arange(t) % 4
    ang = torch.outer(torch.arange(16).float(), 1.0 / 10000 ** (torch.arange(0, d, 2).float() / d))
    cos, sin = ang.cos(), ang.sin()
    y = rope_inplace(x.clone(), pos, cos, sin, heads * d, d)
    ref = rope_reference(x.view(t, heads, d), cos[pos][:, None], sin[pos][:, None]).reshape(t, -1)
    torch.testing.assert_close(y, ref)
    back = rope_inplace(y.clone(), pos, cos, sin, heads * d, d, inverse=True)
    torch.testing.assert_close(back, x, atol=1e-5, rtol=1e-5)
