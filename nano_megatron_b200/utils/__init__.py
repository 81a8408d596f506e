"""Token streams, checkpoints and timing helpers."""
