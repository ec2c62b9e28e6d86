#!/usr/bin/env bash
# Validation + benchmark suite on a GPU box (B200): build, CPU and GPU tests, kernel
# microbenchmarks with roofline fractions, scheduler ablation, packing-mode training
# bench, a profiled run with its phase report, the open-model CE check, the headline
# bench (ours and the reference), and multi-GPU smoke runs (DDP and sharded) when more
# than one GPU is visible, or 2-rank CPU/gloo runs otherwise.
#   SKIP_CPU_TESTS=1  skip the CPU suite
#   NGPU=N            GPUs to use for the multi-GPU steps (default: all visible)
set -euo pipefail
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)"
cd "$ROOT"
NGPU="${NGPU:-$(python -c 'import torch; print(torch.cuda.device_count())')}"
OUT=artifacts/validate
mkdir -p "$OUT"

python setup.py build_ext --inplace > "$OUT/build.log" 2>&1
python -m packbalance_b200.data.prepare --config configs/tiny.yaml > /dev/null
python -m packbalance_b200.data.prepare --config configs/bench.yaml > /dev/null

if [[ "${SKIP_CPU_TESTS:-0}" != "1" ]]; then
  echo "== CPU tests =="
  python -m pytest tests -m "not gpu" -q
fi
echo "== GPU tests =="
python -m pytest tests -m gpu -q

echo "== kernel microbenchmarks =="
python -m packbalance_b200.profiling.bench_kernels --output "$OUT/kernel_bench.json"
echo "== attention event traces =="
python -m packbalance_b200.profiling.attn_trace --json "$OUT/attn_trace.json"
echo "== scheduler ablation =="
python -m packbalance_b200.profiling.bench_schedule --config configs/bench.yaml --world-size 8 \
  --output "$OUT/schedule_bench.json"
echo "== packing-mode training bench =="
python -m packbalance_b200.profiling.bench_train --config configs/bench.yaml --steps 20 --warmup 5 \
  --device cuda --output "$OUT/train_bench.json"
echo "== profile =="
rm -rf "$OUT/profile"
python -m packbalance_b200.train.train --config configs/bench.yaml --max-steps 8 --profile --output-dir "$OUT/profile"
TRACE="$(ls -t "$OUT"/profile/profile/trace_*.json | head -1)"
python -m packbalance_b200.profiling.analyze_trace --trace "$TRACE" --output "$OUT/profile_report.md"
echo "== open-model LM-head CE =="
python -m packbalance_b200.profiling.bench_open_model --tokens 1024 --output "$OUT/open_model_bench.json"
echo "== headline bench (1 GPU) =="
python bench.py --steps 20 --warmup 5
python bench.py --impl reference --steps 5 --warmup 3

if [[ "$NGPU" -ge 2 ]]; then
  echo "== $NGPU-GPU DDP smoke =="
  timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port 29541 -m packbalance_b200.train.train --config configs/tiny.yaml --max-steps 2 \
    --output-dir "$OUT/ddp_smoke"
  echo "== $NGPU-GPU sharded smoke (persistent weights, then two weight windows) =="
  timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port 29542 -m packbalance_b200.train.train --config configs/tiny.yaml --max-steps 2 --fsdp \
    --output-dir "$OUT/fsdp_smoke"
  timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port 29545 -m packbalance_b200.train.train --config configs/tiny.yaml --max-steps 2 --fsdp \
    --set train.fsdp_weight_windows=2 --output-dir "$OUT/fsdp_windows_smoke"
  echo "== $NGPU-GPU headline bench (fp32 and bf16 gradient wire) =="
  timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port 29546 bench.py --gpus "$NGPU" --steps 20 --warmup 5
  timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port 29547 bench.py --gpus "$NGPU" --steps 20 --warmup 5 --set train.grad_reduce_dtype=bf16
  echo "== collectives =="
  timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port 29543 -m packbalance_b200.profiling.bench_comm
  timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port 29544 -m packbalance_b200.profiling.bench_fsdp
else
  echo "== 2-rank CPU/gloo DDP and FSDP smoke =="
  CUDA_VISIBLE_DEVICES="" timeout -k 30 300 python -m torch.distributed.run --standalone --local-addr 127.0.0.1 \
    --nproc-per-node 2 -m packbalance_b200.train.train --config configs/tiny.yaml --max-steps 1 \
    --output-dir "$OUT/ddp_smoke"
  CUDA_VISIBLE_DEVICES="" timeout -k 30 300 python -m torch.distributed.run --standalone --local-addr 127.0.0.1 \
    --nproc-per-node 2 -m packbalance_b200.train.train --config configs/tiny.yaml --max-steps 1 --fsdp \
    --output-dir "$OUT/fsdp_smoke"
fi
echo "done"
