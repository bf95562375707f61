"""Kernel-facing modules mirroring the reference's actune.kernels package."""
