"""Model-side ops of the flash-Sinkhorn path."""
