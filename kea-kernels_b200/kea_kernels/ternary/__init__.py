"""Kea-T (2-bit ternary) layers on the B200 low-bit GEMM."""
