"""1-bit weight codes (the parakeet-binary-v1 export layout): packing, checks and dequantization.

Layout (kept from kea-kernels, src/kea_kernels/binary/bits.py:3-5): uint8 [N, ceil(K/8)]; code k of a row is bit
k % 8 of byte k // 8, least significant bit first; 1 means +1, 0 means -1; the unused tail bits of the last byte are 0.
One FP32 scale per row gives W = alpha * sign. Every function here runs on any torch device.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor

_BIT_WEIGHTS = torch.tensor([1, 2, 4, 8, 16, 32, 64, 128], dtype=torch.uint8)


def packed_row_bytes(in_features: int) -> int:
    return math.ceil(in_features / 8)


def _tail_bits_set(codes: Tensor, in_features: int) -> bool:
    unused = 8 * codes.shape[1] - in_features
    if unused == 0:
        return False
    keep = (1 << (8 - unused)) - 1           # bits of the last byte that hold codes
    return bool((codes[:, -1] & ~keep & 0xFF).any())


def validate_weights(codes: Tensor, scale: Tensor, bias: Tensor | None, in_features: int) -> tuple[int, int]:
    """(N, K) after the checks a layer's prepare() makes; ValueError otherwise (src/kea_kernels/binary/bits.py:21-38).
    Synchronizes when the tensors live on a GPU."""
    if not isinstance(in_features, int) or isinstance(in_features, bool) or in_features < 1:
        raise ValueError(f"in_features must be a positive int, got {in_features!r}")
    width = packed_row_bytes(in_features)
    if codes.dtype != torch.uint8 or codes.dim() != 2 or codes.shape[0] < 1 or codes.shape[1] != width:
        raise ValueError(f"codes must be uint8 [N, {width}], got {codes.dtype} {tuple(codes.shape)}")
    n = codes.shape[0]
    if _tail_bits_set(codes, in_features):
        raise ValueError("invalid packed codes: nonzero tail padding")
    if scale.dtype != torch.float32 or tuple(scale.shape) != (n,) or not bool(torch.isfinite(scale).all()):
        raise ValueError("scale must be finite FP32 [N]")
    if bias is not None and (bias.dtype != torch.float32 or tuple(bias.shape) != (n,)
                             or not bool(torch.isfinite(bias).all())):
        raise ValueError("bias must be None or finite FP32 [N]")
    if scale.device != codes.device or (bias is not None and bias.device != codes.device):
        raise ValueError("codes, scale and bias must be on one device")
    return n, in_features


def unpack_bits(codes: Tensor, in_features: int) -> Tensor:
    """uint8 [N, ceil(K/8)] -> uint8 {0, 1} [N, K] (1 = +1); rejects nonzero tail bits."""
    width = packed_row_bytes(in_features)
    if codes.dtype != torch.uint8 or codes.dim() != 2 or codes.shape[1] != width:
        raise ValueError(f"expected uint8 [N, {width}], got {codes.dtype} {tuple(codes.shape)}")
    if _tail_bits_set(codes, in_features):
        raise ValueError("invalid packed codes: nonzero tail padding")
    weights = _BIT_WEIGHTS.to(codes.device)
    bits = (codes.unsqueeze(-1) & weights).ne(0).to(torch.uint8)   # [N, bytes, 8], bit j of byte b = code 8b + j
    return bits.reshape(codes.shape[0], -1)[:, :in_features].contiguous()


def unpack_signs(codes: Tensor, in_features: int) -> Tensor:
    """uint8 [N, ceil(K/8)] -> int8 {-1, +1} [N, K]."""
    return unpack_bits(codes, in_features).to(torch.int8).mul_(2).sub_(1)


def pack_signs(signs: Tensor) -> Tensor:
    """int8 {-1, +1} [N, K] -> packed codes uint8 [N, ceil(K/8)]."""
    if signs.dtype != torch.int8 or signs.dim() != 2 or bool(((signs != 1) & (signs != -1)).any()):
        raise ValueError("expected 2-D int8 signs in {-1, +1}")
    rows, k = signs.shape
    width = packed_row_bytes(k)
    bits = torch.zeros(rows, 8 * width, dtype=torch.uint8, device=signs.device)
    bits[:, :k] = signs.eq(1).to(torch.uint8)
    weights = _BIT_WEIGHTS.to(signs.device)
    # distinct powers of two: a byte's sum is the OR of its bits (at most 255)
    return (bits.view(rows, width, 8) * weights).sum(dim=2).to(torch.uint8)


def dense_weight(codes: Tensor, scale: Tensor, in_features: int, dtype: torch.dtype = torch.float64) -> Tensor:
    """Dequantized [N, K] = sign * scale[:, None] (exact in FP32 and FP64), on codes.device."""
    signs = unpack_signs(codes, in_features).to(dtype)
    return signs * scale.to(device=codes.device, dtype=dtype).unsqueeze(1)


def resident_bytes(*tensors: Tensor | None) -> int:
    """Sum of the distinct CUDA storages' sizes (a view counts its whole storage once)."""
    sizes: dict[int, int] = {}
    for t in tensors:
        if t is None or not t.is_cuda:
            continue
        storage = t.untyped_storage()
        key = storage.data_ptr()
        sizes[key] = max(sizes.get(key, 0), storage.nbytes())
    return sum(sizes.values())
