"""Checkpoint state I/O in the reference's full-training-state format."""
