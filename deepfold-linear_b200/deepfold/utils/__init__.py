"""Numerical utilities of the flash-Sinkhorn path."""
