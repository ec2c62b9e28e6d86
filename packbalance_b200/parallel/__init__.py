"""Process groups, flat parameter buffers, data-parallel / FSDP engines, fused collectives."""
