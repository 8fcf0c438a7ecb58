"""MEDUSA heads and the target-model wrapper."""
