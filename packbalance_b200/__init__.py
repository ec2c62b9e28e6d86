"""packbalance_b200: packed-sequence LLM pretraining for NVIDIA B200 (sm_100a).

The framework keeps the public surface of DeKodez/packbalance (config schema, data
format, batch dict, model API, checkpoint format, metrics JSONL) and replaces its
execution engine with hand-written sm_100a kernels and a flat-buffer DDP/FSDP engine.

Sub-packages:
  data       corpus builder, token store, cost model, packers, step/rank scheduler, loader
  ops        autograd wrappers over the native kernels (CPU tensors use torch math)
  models     Llama-style decoder assembled from ``ops``
  parallel   process groups, flat parameter buffers, fused all-reduce / FSDP engine
  train      trainer, checkpointing
  profiling  benches, profiler, trace analyser, thesis experiments
"""

__version__ = "0.1.0"
