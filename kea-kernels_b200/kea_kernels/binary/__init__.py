"""Kea-B (1-bit) layers on the B200 low-bit GEMM."""
