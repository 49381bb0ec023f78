"""Export formats the kernels read: the 2-bit ternary codes and the constants of the two export kinds.

  * parakeet-binary-v1 (Kea-B): `<name>.codes` uint8 [N, ceil(K/8)], 1 bit per weight (see binary.bits) plus
    `<name>.scale` FP32 [N];
  * parakeet-ternary-v1 (Kea-T): `<name>.codes` uint8 [N, ceil(K/4)], 2 bits per weight: 00 = 0, 01 = +1, 10 = -1,
    code k at bits 2 * (k % 4) of byte k // 4; the pattern 11 is invalid; plus `<name>.scale` FP32 [N].
Both layouts are kea-kernels' (src/kea_kernels/formats.py:1-16,62-81) and are read unchanged.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor

BINARY_FORMAT = "parakeet-binary-v1"
TERNARY_FORMAT = "parakeet-ternary-v1"
BUNDLE_FORMAT = "keab-8bit-v1"
FILE = "export.safetensors"
MANIFEST = "manifest.json"

LAYERS = 24
PER_LAYER = ("feed_forward1.linear1", "feed_forward1.linear2", "feed_forward2.linear1", "feed_forward2.linear2",
             "self_attn.linear_q", "self_attn.linear_k", "self_attn.linear_v", "self_attn.linear_out",
             "self_attn.linear_pos", "conv.pointwise_conv1", "conv.pointwise_conv2")
EXPECTED_MODULES = LAYERS * len(PER_LAYER)

# Modes per export kind; the first is the default.
BINARY_MODES = ("x2", "x3", "x1")
TERNARY_MODES = ("x2", "x3", "compact")

_FIELD_SHIFTS = torch.tensor([0, 2, 4, 6], dtype=torch.uint8)


def packed_row_bytes(in_features: int, wbits: int) -> int:
    return math.ceil(in_features * wbits / 8)


def pack_ternary(codes: Tensor) -> Tensor:
    """int8 [out, in] in {-1, 0, 1} -> uint8 [out, ceil(in/4)] (0 -> 00, +1 -> 01, -1 -> 10)."""
    if codes.dtype != torch.int8 or codes.dim() != 2 or bool(((codes < -1) | (codes > 1)).any()):
        raise ValueError("expected 2-D int8 codes in {-1, 0, 1}")
    rows, k = codes.shape
    width = math.ceil(k / 4)
    fields = torch.zeros(rows, 4 * width, dtype=torch.uint8, device=codes.device)
    fields[:, :k] = codes.eq(1).to(torch.uint8) + 2 * codes.eq(-1).to(torch.uint8)
    shifted = fields.view(rows, width, 4) << _FIELD_SHIFTS.to(codes.device)
    return shifted.sum(dim=2).to(torch.uint8)  # disjoint 2-bit fields: the sum is their OR


def ternary_fields(packed: Tensor) -> Tensor:
    """uint8 [out, B] -> the 2-bit fields uint8 [out, 4 B] in code order."""
    return ((packed.unsqueeze(-1) >> _FIELD_SHIFTS.to(packed.device)) & 3).reshape(packed.shape[0], -1)


def unpack_ternary(packed: Tensor, in_features: int) -> Tensor:
    """Inverse of pack_ternary; rejects the unused 11 pattern and nonzero tail padding."""
    width = math.ceil(in_features / 4)
    if packed.dtype != torch.uint8 or packed.dim() != 2 or packed.shape[1] != width:
        raise ValueError(f"expected uint8 [out, {width}], got {packed.dtype} {tuple(packed.shape)}")
    fields = ternary_fields(packed)
    if bool(fields.eq(3).any()) or bool(fields[:, in_features:].any()):
        raise ValueError("invalid packed codes")
    fields = fields[:, :in_features]
    return fields.eq(1).to(torch.int8) - fields.eq(2).to(torch.int8)


def validate_ternary(packed: Tensor, scale: Tensor, bias: Tensor | None, in_features: int) -> tuple[int, int]:
    """(N, K) after the checks PackedLinear makes (src/kea_kernels/ternary/runtime.py:17-30); ValueError otherwise."""
    if not isinstance(in_features, int) or isinstance(in_features, bool) or in_features < 1:
        raise ValueError("weight dimensions must be positive")
    if packed.dim() != 2 or packed.shape[0] < 1:
        raise ValueError("weight dimensions must be positive")
    if packed.device != scale.device or (bias is not None and bias.device != packed.device):
        raise ValueError("codes, scales, and bias must be on the same device")
    unpack_ternary(packed, in_features)
    n = packed.shape[0]
    if tuple(scale.shape) != (n,) or scale.dtype != torch.float32 or not bool(torch.isfinite(scale).all()):
        raise ValueError("scale must be finite FP32 [N]")
    if bias is not None and (tuple(bias.shape) != (n,) or bias.dtype != torch.float32
                             or not bool(torch.isfinite(bias).all())):
        raise ValueError("bias must be finite FP32 [N]")
    return n, in_features
