"""Kernel-level API: w8a16_linear / w4a16_linear and the format helpers."""
