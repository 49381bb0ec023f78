"""PackedLinear: a ternary (2-bit) layer resident on a B200 as packed panels (src/kea_kernels/ternary/runtime.py:12-49).

The reference keeps the codes as int32 decode words [ceil(K/16), N] and multiplies FP32 input by split-float Triton
GEMMs (bf16x3 / tf32x3). Here the codes stay at 2 bits per weight in the B200 panel layout (`packed_t`, 0.25 bytes
per weight; no expanded INT8 copy in HBM) and the product is the INT8 path: the input is split into `parts` residual
INT8 parts (3 by default, relative error far below the reference's 1e-5 contract) and multiplied on the tcgen05 INT8
tensor cores with exact INT32 accumulation.
"""
from __future__ import annotations

import torch
from torch import nn

from kea_kernels import formats, lowbit

MODES = {"x1": 1, "x2": 2, "x3": 3}


class PackedLinear(nn.Module):
    WBITS = 2

    def __init__(self, packed: torch.Tensor, scale: torch.Tensor, in_features: int,
                 bias: torch.Tensor | None = None, *, mode: str = "x3", device=None):
        super().__init__()
        n, k = formats.validate_ternary(packed, scale, bias, in_features)
        if mode not in MODES:
            raise ValueError(f"unknown mode {mode!r} (expected one of {tuple(MODES)})")
        self.in_features, self.out_features, self.mode = k, n, mode
        device = torch.device(device) if device is not None else packed.device
        if device.type == "cuda":
            if device.index is None:
                device = torch.device("cuda", torch.cuda.current_device())
            panels = lowbit.prepare_panels(packed.to(device), self.WBITS, n, k)
        else:
            # Host-resident until .cuda(): keep the export codes; panels are built on the first CUDA move.
            panels = packed.detach().clone().contiguous()
        self.register_buffer("packed_t", panels)
        self.register_buffer("scale", scale.to(device).contiguous())
        self.register_buffer("bias", bias.to(device).contiguous() if bias is not None else None)
        self._panels_ready = device.type == "cuda"
        self.eval()

    def _apply(self, fn, recurse=True):
        out = super()._apply(fn, recurse)
        if not self._panels_ready and self.packed_t.is_cuda:
            # first move to a GPU: the buffer still holds the export codes; re-lay them into panels there
            self.packed_t = lowbit.prepare_panels(self.packed_t, self.WBITS, self.out_features, self.in_features)
            self._panels_ready = True
        return out

    @property
    def parts(self) -> int:
        return MODES[self.mode]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return matmul(x, self, conv=False, parts=self.parts)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, mode={self.mode!r}"


class PackedPointwiseConv1d(PackedLinear):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return matmul(x, self, conv=True, parts=self.parts)


def matmul(x: torch.Tensor, mod: PackedLinear, *, conv: bool = False, parts: int = 3, activation: str = "",
           norm=None, input_activation: str = "") -> torch.Tensor:
    """Linear [..., K] or pointwise convolution [B, K, T] through the INT8 residual path (FP32 output)."""
    if not mod._panels_ready or not mod.packed_t.is_cuda:
        raise ValueError("move the layer to a CUDA device first")
    if not isinstance(x, torch.Tensor) or not x.is_cuda or x.device != mod.packed_t.device or x.dtype != torch.float32:
        raise ValueError("expected FP32 CUDA input on the weight device")
    if torch.is_grad_enabled() and x.requires_grad:
        raise RuntimeError("packed kernels are inference-only; use torch.inference_mode()")
    if activation not in ("", "silu") or input_activation not in ("", "silu"):
        raise ValueError(f"unknown activation {activation!r} / {input_activation!r}")
    k, n = mod.in_features, mod.out_features
    if conv:
        if x.dim() != 3 or x.shape[1] != k:
            raise ValueError(f"expected [B,{k},T] convolution input")
        xx = x.transpose(1, 2)
    else:
        if x.dim() < 1 or x.shape[-1] != k:
            raise ValueError(f"expected [...,{k}] linear input")
        xx = x if x.dim() == 3 else x.reshape(1, -1, k)
    b, t, _ = xx.shape
    m = b * t
    y = torch.empty(b, t, n, device=x.device, dtype=torch.float32)
    if m:
        q, qs, ldq = lowbit.quantize(xx, (xx.stride(0), xx.stride(1), xx.stride(2), t), m, k, parts, norm=norm,
                                     input_silu=input_activation == "silu")
        lowbit.gemm(q, qs, ldq, m, mod.packed_t, mod.WBITS, n, k, mod.scale, mod.bias, y.view(m, n), parts=parts,
                    silu=activation == "silu")
    if conv:
        return y.transpose(1, 2)
    return y.view(*x.shape[:-1], n)
