"""The ternary INT8 provider op (src/kea_kernels/ternary/fused_kernels.py:139-160): `int8_matmul`.

provider semantics (quantized-layer call of the encoder transforms):
    xx = x.transpose(1, 2) if conv else x;  z = input_act(LayerNorm(xx));  y = act(alpha * (W z) + bias)
The reference runs the Triton `_quantize` then `_int8_dot` (in-tile decode of int32 words) and, for split > 1, `_finish`.
Here: the residual INT8 quantizer kernel (LayerNorm / input SiLU fused), then the tcgen05 GEMM reading the 2-bit
panels, whose split-K is reduced exactly in INT32 inside the kernel (no FP32 partials, no finish launch).
"""
from __future__ import annotations

from kea_kernels.ternary.runtime import PackedLinear, matmul


def int8_matmul(x, mod: PackedLinear, conv=False, components=1, activation="", norm=None, config=None,
                input_activation=""):
    if config is not None:
        raise ValueError("tile configs are chosen by the library's dispatch table")
    if components not in (1, 2, 3):
        raise ValueError(f"components must be 1, 2 or 3, got {components!r}")
    y = matmul(x if x.dim() != 2 or conv else x.unsqueeze(0), mod, conv=conv, parts=components,
               activation=activation, norm=norm, input_activation=input_activation)
    return y if x.dim() != 2 or conv else y.view(*x.shape[:-1], mod.out_features)
