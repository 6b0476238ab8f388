"""Optimizer transactions (mirrors src/minifield_training/optimizers/)."""
