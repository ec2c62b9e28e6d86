"""Profiler setup, trace analyser, benchmarks and the CPU thesis experiments."""
