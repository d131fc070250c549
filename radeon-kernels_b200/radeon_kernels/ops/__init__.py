"""Operator front-ends of the dense-contraction hot path."""
