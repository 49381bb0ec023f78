"""Int8MmaLayer with 1, 2 or 3 residual activation parts (src/kea_kernels/binary/layer_parts.py:1-138).

`Int8MmaPartsLayer` is Int8MmaLayer with:
  * project(x, *, conv, components, activation, norm, input_activation) honouring components in {1, 2, 3}
    (PartCount overrides it on every provider call);
  * dot(q, qs, ldq, m, y, ..., parts=None): the P-part GEMM, P = q.shape[0] unless given;
  * linear / conv at the variant's fixed part count PARTS: the first PARTS parts of the three-part quantizer, which
    equal the quantizer at PARTS parts (its part loop is sequential).
On B200 the P parts share one expanded weight tile: each part is its own tcgen05 accumulator block in tensor memory,
so x1 reads the same weight bytes as x3 and issues one third of the MMAs.
"""
from __future__ import annotations

import torch
from torch import Tensor

from kea_kernels import lowbit
from kea_kernels.binary import configs
from kea_kernels.binary.layer import Int8MmaLayer, _project, dot


def _round_up(v: int, m: int) -> int:
    return -(-v // m) * m


def m1_quantize_parts(xx: Tensor, parts: int, norm=None, input_activation: str = "") -> tuple[Tensor, Tensor]:
    """The residual INT8 quantizer at `parts` parts on [B, T, K] input (LayerNorm / input SiLU fused)."""
    b, t, k = xx.shape
    q, qs, _ = lowbit.quantize(xx, (xx.stride(0), xx.stride(1), xx.stride(2), t), b * t, k, parts, norm=norm,
                               input_silu=input_activation == "silu")
    return q, qs


class Int8MmaPartsLayer(Int8MmaLayer):
    PARTS = 3

    def dot(self, q: Tensor, qs: Tensor, ldq: int, m: int, y: Tensor, *, silu: bool = False,
            config: configs.DotConfig | None = None, order: int = 0, parts: int | None = None,
            acc: Tensor | None = None) -> None:
        parts = q.shape[0] if parts is None else parts
        if parts not in (1, 2, 3) or q.shape[0] != parts or qs.shape[0] != parts:
            raise ValueError(f"q / qs must hold {parts} parts")
        dot_parts(self, q, qs, ldq, m, y, silu=silu, config=config, order=order, parts=parts, acc=acc)

    def project(self, x: Tensor, *, conv: bool = False, components: int | None = None, activation: str = "",
                norm=None, input_activation: str = "") -> Tensor:
        parts = self.PARTS if components is None else components
        if parts not in (1, 2, 3):
            raise ValueError(f"components must be 1, 2 or 3, got {components!r}")
        return _project(self, x, conv=conv, parts=parts, activation=activation, norm=norm,
                        input_activation=input_activation)


def _aligned(q: Tensor, k: int) -> tuple[Tensor, int]:
    """q [P, M, K] -> rows padded with zeros to a multiple of 16 bytes (TMA row alignment) if needed."""
    if k % 16 == 0 and q.data_ptr() % 16 == 0 and q.stride(1) == k and q.stride(2) == 1:
        return q, k
    ldq = _round_up(k, 16)
    padded = q.new_zeros(q.shape[0], q.shape[1], ldq)
    padded[:, :, :k] = q
    return padded, ldq


def dot_parts(layer: Int8MmaLayer, q: Tensor, qs: Tensor, ldq: int, m: int, y: Tensor, *, silu: bool = False,
              config: configs.DotConfig | None = None, order: int = 0, parts: int = 3,
              acc: Tensor | None = None) -> None:
    """The P-part GEMM + epilogue (src/kea_kernels/binary/layer_parts.py:112-130)."""
    dot(layer, q, qs, ldq, m, y, silu=silu, config=config, order=order, parts=parts, acc=acc)


def variant(parts: int):
    """The layer class whose linear / conv run at `parts` activation parts."""
    return type(f"Int8MmaX{parts}Layer", (Int8MmaPartsLayer,), {"PARTS": parts})


LAYERS = {parts: variant(parts) for parts in (1, 2, 3)}
