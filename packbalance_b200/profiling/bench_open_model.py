"""The fused LM-head cross-entropy on an open model's hidden states and head.

    python -m packbalance_b200.profiling.bench_open_model [--model HuggingFaceTB/SmolLM-135M]
        [--tokens 1024] [--chunk 512] [--device cuda] [--output artifacts/open_model_bench.json]

Runs the model (``transformers``) on random token ids, takes the last hidden states and
the (tied) output embedding, and times forward + backward of the summed CE three ways:
full ``[T, V]`` logits, the chunked PyTorch reference, and this framework's fused
kernel path (tcgen05 LM-head GEMM with the online log-sum-exp in its epilogue, CUDA
only).  Reports ms (CUDA events, after warm-up), peak memory and each variant's loss
against the full-logits loss.  Same CLI as the reference's
``profiling/bench_open_model.py`` (``main`` 41-111).

Offline machines: when the checkpoint is not in the local Hugging Face cache, the model
is built from its published architecture (SmolLM-135M: 30 layers, d 576, 9/3 heads,
ff 1536, vocab 49152, tied embeddings) with random weights, and the output says so.
"""

from __future__ import annotations

import argparse
import gc
import json
import time
from pathlib import Path

import torch
import torch.nn.functional as F

from packbalance_b200.ops.cross_entropy import linear_cross_entropy
from packbalance_b200.ops.reference import chunked_linear_cross_entropy

SMOLLM_135M = dict(hidden_size=576, num_hidden_layers=30, num_attention_heads=9, num_key_value_heads=3,
                   intermediate_size=1536, vocab_size=49152, max_position_embeddings=2048,
                   tie_word_embeddings=True, rms_norm_eps=1e-5, rope_theta=10000.0)


def load_model(name: str, dtype: torch.dtype):
    from transformers import AutoModelForCausalLM, LlamaConfig, LlamaForCausalLM

    try:
        return AutoModelForCausalLM.from_pretrained(name, dtype=dtype, local_files_only=True), "pretrained"
    except Exception:  # not in the offline cache
        torch.manual_seed(0)
        return LlamaForCausalLM(LlamaConfig(**SMOLLM_135M)).to(dtype), "random init (checkpoint not available offline)"


def timed(fn, device: torch.device, warmup: int = 2, iters: int = 5) -> float:
    for _ in range(warmup):
        fn()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / iters
    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    return (time.perf_counter() - t0) * 1e3 / iters


def main(argv: list[str] | None = None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="HuggingFaceTB/SmolLM-135M")
    ap.add_argument("--tokens", type=int, default=1024)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--output", default="artifacts/open_model_bench.json")
    args = ap.parse_args(argv)
    device = torch.device(args.device)
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    model, weights = load_model(args.model, dtype)
    model.to(device).eval()
    tokens = min(args.tokens, int(getattr(model.config, "max_position_embeddings", args.tokens)))
    vocab = int(model.config.vocab_size)
    ids = torch.randint(0, vocab, (1, tokens), device=device)
    with torch.no_grad():
        hidden = model(ids, output_hidden_states=True).hidden_states[-1].reshape(tokens, -1).detach()
    weight = model.get_output_embeddings().weight.detach()
    targets = torch.randint(0, vocab, (tokens,), device=device)
    del model
    gc.collect()
    if device.type == "cuda":
        torch.cuda.empty_cache()

    losses: dict[str, float] = {}

    def variant(name, f):
        def run():
            x = hidden.clone().requires_grad_(True)
            w = weight.clone().requires_grad_(True)
            loss = f(x, w)
            loss.backward()
            losses[name] = float(loss.detach())
        return run

    variants = [
        ("full_logits", variant("full_logits", lambda x, w: F.cross_entropy((x @ w.t()).float(), targets, reduction="sum"))),
        ("chunked_reference", variant("chunked_reference",
                                      lambda x, w: chunked_linear_cross_entropy(x, w, targets, chunk_size=args.chunk))),
    ]
    if device.type == "cuda":
        variants.append(("fused_sm100", variant("fused_sm100",
                                                lambda x, w: linear_cross_entropy(x, w, targets, chunk_size=args.chunk))))
    rows = []
    for name, fn in variants:
        if device.type == "cuda":
            torch.cuda.reset_peak_memory_stats(device)
        ms = timed(fn, device)
        peak = torch.cuda.max_memory_allocated(device) / 1e9 if device.type == "cuda" else 0.0
        rel = abs(losses[name] - losses["full_logits"]) / abs(losses["full_logits"])
        rows.append({"model": args.model, "weights": weights, "variant": name, "tokens": tokens, "vocab": vocab,
                     "dim": int(hidden.shape[-1]), "ms": ms, "peak_gb": peak, "loss": losses[name],
                     "loss_rel_diff_vs_full": rel})
        print(f"{name:<20} {ms:8.3f} ms  peak {peak:6.2f} GB  loss rel diff {rel:.2e}", flush=True)
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(rows, indent=2), encoding="utf-8")
    print(f"wrote {out} ({weights})")
    return rows


if __name__ == "__main__":
    main()
