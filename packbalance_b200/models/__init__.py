"""Llama-style decoder (reference path on CPU, native sm100 path on CUDA)."""
