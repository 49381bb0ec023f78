"""ExpandedProjection: the Kea-T projection provider (src/kea_kernels/ternary/encoder4.py:77-149).

The reference's default ("expanded") mode keeps an exact INT8 copy of every ternary weight in HBM (about +604 MB)
because its SM120 Triton kernel is fastest on dense INT8. On B200 the expansion happens in shared memory inside the
GEMM, so this provider reads the 2-bit panels directly and holds no extra copy (`bytes` is 0); its arithmetic is the
same residual INT8 path as `int8_matmul`.
"""
from __future__ import annotations

from kea_kernels.ternary.fused_kernels import int8_matmul


class ExpandedProjection:
    def __init__(self, backend: str = "panels", config=None):
        if config is not None:
            raise ValueError("tile configs are chosen by the library's dispatch table")
        self.backend = backend
        self.weights: dict = {}

    @property
    def bytes(self) -> int:
        return 0

    def __call__(self, x, mod, conv=False, components=3, activation="", norm=None, config=None, input_activation=""):
        return int8_matmul(x, mod, conv, components, activation, norm, config, input_activation)
