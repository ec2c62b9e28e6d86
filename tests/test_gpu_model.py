"""The native CUDA model path against the fp32 reference path of the same weights."""

from dataclasses import replace

import pytest
import torch

from packbalance_b200.config import ModelConfig, PackBalanceConfig, TrainConfig
from packbalance_b200.models.llama import LlamaForCausalLM
from packbalance_b200.ops import _native
from packbalance_b200.parallel.flat import FlatParameters

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    base = ModelConfig(vocab_size=1000, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=512, max_seq_len=1024,
                       attention_backend="auto", ce_chunk_size=256)
    return replace(base, **kw)


def _batch(t, vocab, lengths, device="cuda"):
    ids = torch.randint(1, vocab, (t,), device=device)
    doc = torch.cat([torch.full((n,), i, device=device) for i, n in enumerate(lengths)])
    pos = torch.cat([torch.arange(n, device=device) for n in lengths])
    labels = torch.cat([ids[1:], torch.full((1,), -100, device=device)])
    ends = torch.cumsum(torch.tensor(lengths, device=device), 0) - 1
    labels[ends] = -100
    return ids, labels, pos, doc


@pytest.mark.parametrize("keep_logits", [True, False])
@pytest.mark.parametrize("tied", [True, False])
def test_native_model_matches_reference(tied, keep_logits, monkeypatch):
    from packbalance_b200.models import fused

    # the LM head keeps its logits for the backward, or recomputes them
    monkeypatch.setattr(fused, "LOGITS_KEEP_BYTES", (1 << 30) if keep_logits else 0)
    torch.manual_seed(0)
    cfg = _cfg(tie_embeddings=tied)
    lengths = [100, 300, 57, 555]
    ids, labels, pos, doc = _batch(sum(lengths), cfg.vocab_size, lengths)
    ref = LlamaForCausalLM(replace(cfg, attention_backend="eager")).cuda()
    nat = LlamaForCausalLM(cfg).cuda()
    nat.load_state_dict(ref.state_dict())
    flat = FlatParameters(nat)
    nat.flat = flat
    # reference in fp32 on bf16-rounded weights
    with torch.no_grad():
        for p in ref.parameters():
            p.copy_(p.to(torch.bfloat16).float())
        for p in nat.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    flat.refresh_shadow(force=True)
    out_ref = ref(ids[None], labels=labels[None], position_ids=pos[None], doc_ids=doc[None])
    out_ref.loss.backward()
    flat.begin_window()
    out = nat(ids[None], labels=labels[None], position_ids=pos[None], doc_ids=doc[None])
    out.loss.backward()
    flat.finish_window()
    _native.check_status()
    n_tok = int((labels != -100).sum())
    torch.testing.assert_close(out.loss / n_tok, out_ref.loss / n_tok, atol=2e-2, rtol=1e-2)
    for (name, p_ref), p in zip(ref.named_parameters(), nat.parameters()):
        g_ref, g = p_ref.grad, p.grad
        rel = (g - g_ref).norm() / (g_ref.norm() + 1e-12)
        assert rel < 0.08, f"{name}: relative grad error {rel:.3f}"


def test_engine_steps_reduce_loss():
    from packbalance_b200.train.engine import TrainEngine

    torch.manual_seed(0)
    cfg = PackBalanceConfig(model=_cfg(), train=TrainConfig(lr=3e-3, warmup_steps=1, max_steps=30, grad_accum=2))
    eng = TrainEngine(cfg, torch.device("cuda"))
    lengths = [200, 312, 512]
    ids, labels, pos, doc = _batch(1024, cfg.model.vocab_size, lengths, device="cpu")
    from packbalance_b200.data.dataset import doc_starts_from_ids

    batch = dict(input_ids=ids, labels=labels, position_ids=pos, doc_ids=doc,
                 doc_start=torch.from_numpy(doc_starts_from_ids(doc.numpy())))
    toks = 1024
    losses = []
    for _ in range(15):
        out = eng.step([batch, batch], 2 * toks)
        losses.append(float(out["loss_sum"]) / (2 * toks))
    _native.check_status()
    assert losses[-1] < losses[0] * 0.8, losses


def test_cuda_graph_step_matches_eager_step():
    """The captured-and-replayed training step gives the eager step's losses, norms and
    weights (graphs are captured on the third step of an input signature)."""
    from packbalance_b200.data.dataset import doc_starts_from_ids
    from packbalance_b200.train.engine import TrainEngine

    cfg = _cfg()
    g = torch.Generator().manual_seed(5)
    batches = []
    for s in range(6):
        lengths, tot = [], 0
        while tot < 1024:
            n = min(int(torch.randint(20, 400, (1,), generator=g)), 1024 - tot)
            lengths.append(n)
            tot += n
        ids, labels, pos, doc = _batch(1024, cfg.vocab_size, lengths, device="cpu")
        batches.append({"input_ids": ids, "labels": labels, "position_ids": pos, "doc_ids": doc,
                        "doc_start": torch.from_numpy(doc_starts_from_ids(doc.numpy()))})
    engines = []
    for graphs in (False, True):
        torch.manual_seed(0)
        tc = TrainConfig(lr=1e-3, warmup_steps=2, max_steps=20, grad_clip=1.0, cuda_graphs=graphs)
        engines.append(TrainEngine(PackBalanceConfig(model=cfg, train=tc), torch.device("cuda")))
    assert engines[1].use_graphs and not engines[0].use_graphs
    e0, e1 = engines
    for b in batches:
        # same starting state each step, so gradient noise from fp32 atomics is not
        # amplified by Adam over several steps
        for dst, src in ((e1.flat.data, e0.flat.data), (e1.flat.shadow, e0.flat.shadow),
                         (e1.optimizer.exp_avg, e0.optimizer.exp_avg), (e1.optimizer.exp_avg_sq, e0.optimizer.exp_avg_sq)):
            dst.copy_(src)
        e1.flat.mark_shadow_fresh()
        before = e0.flat.data.clone()
        outs = [e.step([b], 900) for e in engines]
        torch.testing.assert_close(outs[1]["loss_sum"], outs[0]["loss_sum"], rtol=1e-5, atol=1e-4)
        torch.testing.assert_close(outs[1]["grad_norm"], outs[0]["grad_norm"], rtol=1e-4, atol=1e-5)
        upd = (e0.flat.data - before).norm()
        err = (e1.flat.data - e0.flat.data).norm()
        assert err <= 0.02 * upd + 1e-6, (float(err), float(upd))
    assert len(e1._graphs) == 1
    _native.check_status()


def test_activation_checkpointing_native_path():
    """With the reference's gradient_checkpointing flag the native path recomputes each
    layer in its backward: same loss and (up to fp32 atomics) the same gradients."""
    torch.manual_seed(0)
    cfg = _cfg()
    lengths = [300, 211, 489]
    ids, labels, pos, doc = _batch(sum(lengths), cfg.vocab_size, lengths)
    model = LlamaForCausalLM(cfg).cuda()
    flat = FlatParameters(model)
    model.flat = flat
    losses, grads = [], []
    for ckpt in (False, True):
        model.model.gradient_checkpointing = ckpt
        flat.begin_window()
        out = model(ids[None], labels=labels[None], position_ids=pos[None], doc_ids=doc[None])
        out.loss.backward()
        flat.finish_window()
        losses.append(float(out.loss))
        grads.append(flat.grad.clone())
    _native.check_status()
    assert abs(losses[0] - losses[1]) <= 1e-6 * abs(losses[0])  # loss sum uses fp32 atomics
    rel = (grads[1] - grads[0]).norm() / grads[0].norm()
    assert rel < 5e-3, float(rel)  # fp32 atomics + bf16 roundings of gradients; a missed recompute is O(1)
