"""kea_kernels for NVIDIA B200 (sm_100a): the low-bit GEMM of kea-kernels' Kea-B / Kea-T encoders.

1-bit (sign) and 2-bit (ternary) packed weights times residual INT8 activations on the tcgen05 tensor cores, behind
the kea-kernels layer and provider API (binary.layer, binary.layer_parts, binary.provider, ternary.runtime). The
device code is the prebuilt C-ABI library libkea_lowbit.so (include/kea_lowbit.h); there is no CPU fallback.
"""
from kea_kernels._lib import LIB_PATH, lib  # noqa: F401

__version__ = "0.1.0"
