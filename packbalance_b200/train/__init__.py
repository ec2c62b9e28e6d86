"""Trainer, training-step engine, checkpointing."""
