"""Helpers around the hot path (synthetic models for tests and benchmarks)."""
