"""Operator entry points mirroring tiny_transformer/operators (attention only)."""
