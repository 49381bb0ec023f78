"""Int8MmaLayer: 1-bit weights expanded to INT8 on chip, residual INT8 activations, tcgen05 INT32 accumulation.

The B200 counterpart of the reference's Int8MmaLayer (src/kea_kernels/binary/layer.py:29-209), with the same methods,
argument meaning and errors:
  * prepare(codes, scale, bias, in_features, device): validate (binary.bits.validate_weights), then re-lay the export
    codes on the device into panels (kea_lowbit_prepare), once per layer;
  * dot(q, qs, ldq, m, y, *, silu, config, order): the GEMM + epilogue on prequantized activations and caller-owned
    outputs (three residual parts, like the reference's b1_dot x3); y may be FP32 (the reference's output) or FP16;
  * linear(x) / conv(x): quantize (three residual INT8 parts) + dot, FP32 output;
  * project(x, *, conv, components, activation, norm, input_activation): the fused provider op (LayerNorm and input
    SiLU fused into the quantizer, SiLU fused into the GEMM epilogue).
Every call enqueues work on torch.cuda.current_stream() and never synchronizes. There is no fallback kernel: the
panel layout pads N and K to 128 only, so every shape runs on the tensor-core kernel (`fast` is always True).
"""
from __future__ import annotations

import math

import torch
from torch import Tensor

from kea_kernels import lowbit
from kea_kernels.binary import bits as api
from kea_kernels.binary import configs


def _round_up(v: int, m: int) -> int:
    return -(-v // m) * m


class Int8MmaLayer:
    """One layer resident as B200 panels (1 bit per weight) plus FP32 scale / bias."""

    WBITS = 1
    PARTS = 3

    def __init__(self, n: int, k: int, device: torch.device, panels: Tensor, scale: Tensor, bias: Tensor | None):
        self.out_features, self.in_features, self.device = n, k, device
        self.panels, self.scale, self.bias = panels, scale, bias

    @classmethod
    def prepare(cls, codes: Tensor, scale: Tensor, bias: Tensor | None, in_features: int, device) -> "Int8MmaLayer":
        n, k = api.validate_weights(codes, scale, bias, in_features)
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("Int8MmaLayer runs on CUDA devices only")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        with torch.no_grad():
            panels = lowbit.prepare_panels(codes.to(device), cls.WBITS, n, k)
            scale = scale.to(device=device, dtype=torch.float32, copy=True).contiguous()
            bias = None if bias is None else bias.to(device=device, dtype=torch.float32, copy=True).contiguous()
        return cls(n, k, device, panels, scale, bias)

    @property
    def fast(self) -> bool:
        return True

    def weight_bytes(self) -> int:
        return api.resident_bytes(self.panels, self.scale, self.bias)

    # --- calls ------------------------------------------------------------------------------------
    # Where each entry point keeps the K features: the last axis of a token-major input, or axis 1 of [B, K, T].
    _FEATURE_AXIS = {"linear": (-1, "[..., {k}]"), "conv": (1, "[B, {k}, T]")}

    def _check(self, x: Tensor, kind: str) -> None:
        """Checks every entry point makes (the reference layer's messages): an FP32 tensor on this layer's device
        with its features where `kind` puts them, and no autograd."""
        axis, form = self._FEATURE_AXIS[kind]
        if not isinstance(x, Tensor):
            problem = ValueError("input must be a tensor")
        elif x.dtype != torch.float32:
            problem = ValueError(f"expected FP32 input, got {x.dtype}")
        elif x.device != self.device:
            problem = ValueError(f"input on {x.device}, layer on {self.device}")
        elif x.dim() < 1 or (kind == "conv" and x.dim() != 3) or x.shape[axis] != self.in_features:
            problem = ValueError(f"expected {form.format(k=self.in_features)} input, got {tuple(x.shape)}")
        elif torch.is_grad_enabled() and x.requires_grad:
            problem = RuntimeError("Int8MmaLayer is inference only: input requires grad")
        else:
            return
        raise problem

    def linear(self, x: Tensor) -> Tensor:
        self._check(x, "linear")
        return self._token_rows_product(x).view(*x.shape[:-1], self.out_features)

    def conv(self, x: Tensor) -> Tensor:
        self._check(x, "conv")
        b, _, t = x.shape
        # [B, K, T] read through its transposed view: the token rows are its T positions
        return self._token_rows_product(x.transpose(1, 2)).view(b, t, self.out_features).transpose(1, 2)

    def _token_rows_product(self, xt: Tensor) -> Tensor:
        """xt [..., K] -> FP32 [rows, N]: its token rows quantized into the layer's PARTS residual INT8 parts, then
        the GEMM."""
        y = torch.empty(math.prod(xt.shape[:-1]), self.out_features, device=self.device, dtype=torch.float32)
        if y.shape[0]:
            rows, layout = token_rows(xt)
            q, qs, ldq = quantize(rows, layout, y.shape[0], self.in_features, self.PARTS)
            self.dot(q, qs, ldq, y.shape[0], y)
        return y

    def dot(self, q: Tensor, qs: Tensor, ldq: int, m: int, y: Tensor, *, silu: bool = False,
            config: configs.DotConfig | None = None, order: int = 0, acc: Tensor | None = None) -> None:
        """y[:m] (row-major, row stride y.stride(0), FP32 or FP16) from q int8 [3, m, ldq] and qs FP32 [3, m].
        acc, when given, receives the exact INT32 accumulators int32 [3, m, N]."""
        if q.dim() != 3 or q.shape[0] != 3 or qs.dim() != 2 or qs.shape[0] != 3:
            raise ValueError("q / qs must hold 3 parts")
        dot(self, q, qs, ldq, m, y, silu=silu, config=config, order=order, parts=3, acc=acc)

    def project(self, x: Tensor, *, conv: bool = False, components: int = 3, activation: str = "",
                norm=None, input_activation: str = "") -> Tensor:
        """The fused provider op (src/kea_kernels/binary/layer.py:118-151): y = act(alpha * (W z) + bias) with
        z = input_act(LayerNorm(x)), z quantized into `components` residual INT8 parts."""
        if components != 3:
            raise ValueError("Int8MmaLayer implements INT8x3 arithmetic only (components=3)")
        return _project(self, x, conv=conv, parts=3, activation=activation, norm=norm,
                        input_activation=input_activation)


def _project(layer, x: Tensor, *, conv: bool, parts: int, activation: str, norm, input_activation: str) -> Tensor:
    if activation not in ("", "silu") or input_activation not in ("", "silu"):
        raise ValueError(f"unsupported activation {activation!r} / {input_activation!r}")
    xx = x.transpose(1, 2) if conv else x
    layer._check(xx, "linear")
    if xx.dim() == 2:
        xx = xx.unsqueeze(0)
    if xx.dim() != 3:
        raise ValueError("project expects [B, T, K] (or [T, K]) input")
    b, t, k = xx.shape
    m, n = b * t, layer.out_features
    y = torch.empty(b, t, n, device=layer.device, dtype=torch.float32)
    if m:
        q, qs, ldq = lowbit.quantize(xx, (xx.stride(0), xx.stride(1), xx.stride(2), t), m, k, parts, norm=norm,
                                     input_silu=input_activation == "silu")
        dot(layer, q, qs, ldq, m, y.view(m, n), silu=activation == "silu", parts=parts)
    if conv:
        return y.transpose(1, 2)
    return y if x.dim() == 3 else y.view(*x.shape[:-1], n)


def token_rows(x: Tensor) -> tuple[Tensor, tuple[int, int, int, int]]:
    """x [..., K] (at least one token) -> (x3 [B, T, K], (XB, XT, XK, T)): the quantizer's addressing of x's token
    rows, row r at (r // T) * XB + (r % T) * XT. The leading dimensions fold into B with reshape, which copies only
    when their strides cannot be merged."""
    x3 = x.reshape(1, 1, x.shape[0]) if x.dim() == 1 else x.reshape(-1, x.shape[-2], x.shape[-1])
    return x3, (x3.stride(0), x3.stride(1), x3.stride(2), x3.shape[1])


def quantize(x: Tensor, rows: tuple, m: int, k: int, parts: int = 3) -> tuple[Tensor, Tensor, int]:
    """(x, (XB, XT, XK, T)) -> q int8 [parts, m, ldq] (zero padded), qs FP32 [parts, m], ldq = roundup(k, 16).

    The residual INT8 quantizer of kea-kernels (b1_quantize, src/kea_kernels/binary/kernels.py:567-617): per part,
    s = max(amax / 127, 1e-30), q = rint(r / s), r -= q * s; here every division is IEEE round-to-nearest."""
    return lowbit.quantize(x, rows, m, k, parts)


def m1_quantize(xx: Tensor, norm=None, input_activation: str = "") -> tuple[Tensor, Tensor]:
    """The fused quantizer at three parts on [B, T, K] input (LayerNorm / input SiLU fused): q [3, m, ldq], qs."""
    b, t, k = xx.shape
    q, qs, _ = lowbit.quantize(xx, (xx.stride(0), xx.stride(1), xx.stride(2), t), b * t, k, 3, norm=norm,
                               input_silu=input_activation == "silu")
    return q, qs


def dot(layer: Int8MmaLayer, q: Tensor, qs: Tensor, ldq: int, m: int, y: Tensor, *, silu: bool = False,
        config: configs.DotConfig | None = None, order: int = 0, parts: int = 3, acc: Tensor | None = None,
        pdl: bool = False) -> None:
    """order selects the epilogue's first FP32 contraction for parts >= 2 (fma(a0, s0, a1 * s1) or
    fma(a1, s1, a0 * s0)), as the reference's flags bit 1 does (src/kea_kernels/binary/kernels.py:73-84)."""
    lowbit.gemm(q, qs, ldq, m, layer.panels, layer.WBITS, layer.out_features, layer.in_features, layer.scale,
                layer.bias, y, parts=parts, silu=silu, order=order, acc=acc, config=config, pdl=pdl)
