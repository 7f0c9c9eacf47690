"""Fused decode-step kernels (drop-in for the reference's models/fused)."""
