import torch

from packbalance_b200.config import ModelConfig
from packbalance_b200.models.llama import LlamaForCausalLM, count_parameters
from packbalance_b200.data.cost import FlopModel


def test_forward_backward_and_loss(model_cfg: ModelConfig) -> None:
    torch.manual_seed(0)
    model = LlamaForCausalLM(model_cfg)
    assert count_parameters(model) == FlopModel.from_config(model_cfg).total_params
    ids = torch.randint(0, model_cfg.vocab_size, (1, 16))
    labels = torch.cat([ids[:, 1:], torch.full((1, 1), -100)], dim=1)
    out = model(ids, labels=labels, position_ids=torch.arange(16)[None], doc_ids=torch.zeros_like(ids))
    assert out.loss.ndim == 0 and out.hidden_states.shape == (1, 16, model_cfg.d_model)
    out.loss.backward()
    grads = [p.grad for p in model.parameters() if p.grad is not None]
    assert grads and all(torch.isfinite(g).all() for g in grads)


def test_state_dict_keys_match_reference_layout(model_cfg: ModelConfig) -> None:
    keys = set(LlamaForCausalLM(model_cfg).state_dict())
    assert "model.embed_tokens.weight" in keys and "model.norm.weight" in keys
    for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
        assert f"model.layers.0.self_attn.{name}.weight" in keys
    for name in ("gate_proj", "up_proj", "down_proj"):
        assert f"model.layers.1.mlp.{name}.weight" in keys
    assert not any("rotary" in k for k in keys)
    assert "lm_head.weight" not in keys


def test_overfit_one_tiny_batch(model_cfg: ModelConfig) -> None:
    torch.manual_seed(0)
    model = LlamaForCausalLM(model_cfg)
    ids = torch.randint(0, model_cfg.vocab_size, (1, 32))
    labels = torch.cat([ids[:, 1:], torch.full((1, 1), -100)], dim=1)
    opt = torch.optim.AdamW(model.parameters(), lr=2e-3)
    losses = []
    for _ in range(30):
        opt.zero_grad(set_to_none=True)
        loss = model(ids, labels=labels, position_ids=torch.arange(32)[None], doc_ids=torch.zeros_like(ids)).loss / 31
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0] * 0.85


def test_untied_head(model_cfg: ModelConfig) -> None:
    from dataclasses import replace

    model = LlamaForCausalLM(replace(model_cfg, tie_embeddings=False))
    assert "lm_head.weight" in model.state_dict()
    out = model(torch.randint(0, model_cfg.vocab_size, (1, 8)))
    assert out.logits.shape == (1, 8, model_cfg.vocab_size)


def test_kv_cache_generate_matches_full_recompute(model_cfg: ModelConfig) -> None:
    """Greedy decoding with the KV cache gives the tokens that re-running the whole
    prefix through the module path gives, for a batch of two prompts."""
    torch.manual_seed(3)
    model = LlamaForCausalLM(model_cfg).eval()
    prompt = torch.randint(0, model_cfg.vocab_size, (2, 5))
    out = model.generate(prompt, max_new_tokens=9, temperature=0.0)
    ref = prompt
    with torch.no_grad():
        for _ in range(9):
            nxt = model(ref).logits[:, -1].argmax(-1, keepdim=True)
            ref = torch.cat([ref, nxt], dim=1)
    assert torch.equal(out, ref)


def test_generate_sampling_and_length_cap(model_cfg: ModelConfig) -> None:
    torch.manual_seed(4)
    model = LlamaForCausalLM(model_cfg)
    prompt = torch.randint(0, model_cfg.vocab_size, (1, model_cfg.max_seq_len - 3))
    out = model.generate(prompt, max_new_tokens=10, temperature=0.7, top_k=5)
    assert out.shape == (1, model_cfg.max_seq_len) and torch.equal(out[:, : prompt.shape[1]], prompt)
    assert model.training  # mode restored
    # top_k = 1 at any temperature is greedy
    greedy = model.generate(prompt[:, :6], max_new_tokens=4, temperature=0.0)
    assert torch.equal(model.generate(prompt[:, :6], max_new_tokens=4, temperature=1.3, top_k=1), greedy)
