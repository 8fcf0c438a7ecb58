"""Verify engine: preallocated KV cache and the per-layer verify forward."""
