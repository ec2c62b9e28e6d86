import math

import torch

from packbalance_b200.config import ModelConfig
from packbalance_b200.models.llama import LlamaForCausalLM
from packbalance_b200.parallel.flat import FlatParameters
from packbalance_b200.parallel.optim import FlatAdamW, global_grad_norm


def _batch(cfg, t=16):
    ids = torch.randint(0, cfg.vocab_size, (1, t))
    labels = torch.cat([ids[:, 1:], torch.full((1, 1), -100)], dim=1)
    return ids, labels


def test_params_and_grads_alias_flat_buffers(model_cfg: ModelConfig) -> None:
    torch.manual_seed(0)
    model = LlamaForCausalLM(model_cfg)
    ref = {k: v.clone() for k, v in model.state_dict().items()}
    flat = FlatParameters(model)
    for k, v in model.state_dict().items():
        torch.testing.assert_close(v, ref[k])
    base, gbase = flat.data.data_ptr(), flat.grad.data_ptr()
    end, gend = base + flat.data.numel() * 4, gbase + flat.grad.numel() * 4
    ids, labels = _batch(model_cfg)
    model(ids, labels=labels).loss.backward()
    for s in flat.slots:
        assert base <= s.param.data_ptr() < end
        assert gbase <= s.param.grad.data_ptr() < gend
    assert flat.grad.abs().sum() > 0
    a = model.model.layers[0].self_attn
    qkv = flat.grad_of(a.q_proj.weight, a.k_proj.weight, a.v_proj.weight)
    assert qkv.shape == (model_cfg.d_model + 2 * model_cfg.d_kv, model_cfg.d_model)
    torch.testing.assert_close(qkv[: model_cfg.d_model], a.q_proj.weight.grad)


def test_flat_adamw_matches_torch_adamw(model_cfg: ModelConfig) -> None:
    torch.manual_seed(0)
    m1 = LlamaForCausalLM(model_cfg)
    m2 = LlamaForCausalLM(model_cfg)
    m2.load_state_dict(m1.state_dict())
    flat = FlatParameters(m2)
    o1 = torch.optim.AdamW(m1.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    o2 = FlatAdamW(flat, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for _ in range(3):
        ids, labels = _batch(model_cfg)
        o1.zero_grad(set_to_none=True)
        m1(ids, labels=labels).loss.backward()
        n1 = torch.nn.utils.clip_grad_norm_(m1.parameters(), 0.5)
        o1.step()
        flat.zero_grad()
        m2(ids, labels=labels).loss.backward()
        n2 = global_grad_norm(flat)
        o2.step(grad_norm=n2, max_norm=0.5)
        torch.testing.assert_close(n1, n2, atol=1e-5, rtol=1e-5)
    for (k, a), b in zip(m1.state_dict().items(), m2.state_dict().values()):
        torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5, msg=k)
    sd1, sd2 = o1.state_dict(), o2.state_dict()
    assert sd1["state"].keys() == sd2["state"].keys()
    for k in sd1["state"]:
        torch.testing.assert_close(sd1["state"][k]["exp_avg_sq"], sd2["state"][k]["exp_avg_sq"], atol=1e-6, rtol=1e-4)
    # A torch AdamW state dict loads into FlatAdamW (checkpoint compatibility).
    o3 = FlatAdamW(FlatParameters(LlamaForCausalLM(model_cfg)), lr=1e-2)
    o3.load_state_dict(sd1)
    assert o3.step_count == 3
    torch.testing.assert_close(o3.exp_avg, o2.exp_avg, atol=1e-5, rtol=1e-4)


def test_nonfinite_norm_skips_update(model_cfg: ModelConfig) -> None:
    model = LlamaForCausalLM(model_cfg)
    flat = FlatParameters(model)
    before = flat.data.clone()
    opt = FlatAdamW(flat, lr=1.0)
    flat.grad.fill_(1.0)
    opt.step(grad_norm=torch.tensor(math.inf), max_norm=1.0)
    assert torch.equal(before, flat.data) and int(opt.last_skipped) == 1


def test_claim_protocol(model_cfg: ModelConfig) -> None:
    model = LlamaForCausalLM(model_cfg)
    flat = FlatParameters(model)
    w = model.model.embed_tokens.weight
    flat.begin_window()
    assert flat.claim(w) is False
    assert flat.claim(w) is True
    flat.grad.fill_(3.0)
    flat.finish_window()
    assert float(flat.grad_of(w).abs().sum()) > 0  # claimed slot untouched
    n = model.model.norm.weight
    assert float(flat.grad_of(n).abs().sum()) == 0  # unclaimed slot zeroed
