"""The three device operations every layer object here is built from, each one C-ABI call on the current stream:

  * prepare_panels - export codes (1- or 2-bit) -> the B200 panel layout, with the code checks on the device;
  * quantize       - FP32 rows -> P residual INT8 parts + per-row part scales (optional LayerNorm / input SiLU);
  * gemm           - INT8 parts x packed weights -> exact INT32 accumulators -> the FP32 epilogue -> FP32 / FP16.

They replace the reference's per-kernel NVRTC launches (src/kea_kernels/binary/layer.py:154-209,
src/kea_kernels/binary/layer_parts.py:112-130) and Triton launches (src/kea_kernels/ternary/fused_kernels.py:139-160).
No call allocates on the launch path except where a function returns new tensors (quantize, prepare_panels); gemm
writes caller-owned outputs, so it can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes
import math

import torch
from torch import Tensor

from kea_kernels import _lib


def _round_up(v: int, m: int) -> int:
    return -(-v // m) * m


def _require_cuda(t: Tensor, name: str) -> None:
    if not isinstance(t, Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def prepare_panels(codes: Tensor, wbits: int, n: int, k: int) -> Tensor:
    """codes uint8 [n, ceil(k * wbits / 8)] on a CUDA device -> panels uint8 [panel_bytes] on that device.
    Raises ValueError for nonzero tail bits or (2-bit) a 0b11 field. Synchronizes (like the reference's checks)."""
    _require_cuda(codes, "codes")
    width = -(-k * wbits // 8)
    if codes.dtype != torch.uint8 or codes.dim() != 2 or tuple(codes.shape) != (n, width):
        raise ValueError(f"codes must be uint8 [{n}, {width}], got {codes.dtype} {tuple(codes.shape)}")
    codes = codes.contiguous()
    panels = torch.empty(_lib.panel_bytes(wbits, n, k), dtype=torch.uint8, device=codes.device)
    err = torch.zeros(1, dtype=torch.int32, device=codes.device)
    with torch.cuda.device(codes.device):
        _lib.check(_lib.lib().kea_lowbit_prepare(codes.data_ptr(), wbits, n, k, panels.data_ptr(), err.data_ptr(),
                                                 _lib.stream_handle(codes.device)), "prepare")
    bad = int(err.item())
    if bad:
        raise ValueError("invalid packed codes" + (": nonzero tail padding" if bad & _lib.DEVERR_TAIL_BITS else ""))
    return panels


def quantize(x: Tensor, rows: tuple[int, int, int, int], m: int, k: int, parts: int, *, ldq: int | None = None,
             norm=None, input_silu: bool = False, pdl: bool = False, pre_norm=None,
             normed: Tensor | None = None, narrow_rows: bool = False) -> tuple[Tensor, Tensor, int]:
    """x[m', kk] at x + (m' // T) * XB + (m' % T) * XT + kk * XK for rows = (XB, XT, XK, T) ->
    (q int8 [parts, m, ldq] zero-padded past k, qs FP32 [parts, m], ldq). pdl lets the kernel start while the
    previous kernel on the stream finishes (it waits for that kernel's results before reading x).
    `pre_norm` (a LayerNorm) is applied first and its output written to `normed` (FP32 [m, k] rows, unit stride; may
    be x itself): a layer's output norm folded into the next projection's quantizer. narrow_rows: as few threads per
    row as registers allow (one warp up to K = 1024), the reduction order of project()'s fused quantizer."""
    _require_cuda(x, "x")
    if x.dtype != torch.float32:
        raise ValueError(f"expected FP32 input, got {x.dtype}")
    ldq = _round_up(k, 16) if ldq is None else ldq
    q = torch.empty(parts, m, ldq, device=x.device, dtype=torch.int8)
    qs = torch.empty(parts, m, device=x.device, dtype=torch.float32)
    if m == 0:
        return q, qs, ldq
    d = _quant_desc(x, rows, m, k, parts, q, qs, ldq, norm=norm, input_silu=input_silu, pdl=pdl, pre_norm=pre_norm,
                    normed=normed, narrow=narrow_rows)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().kea_lowbit_quantize(ctypes.byref(d), _lib.stream_handle(x.device)), "quantize")
    return q, qs, ldq


def _quant_desc(x: Tensor, rows, m: int, k: int, parts: int, q: Tensor, qs: Tensor, ldq: int, *, norm, input_silu,
                pdl, pre_norm, normed, narrow) -> _lib.QuantizeDesc:
    xb, xt, xk, t = rows
    d = _lib.QuantizeDesc()
    d.x, d.xb, d.xt, d.xk, d.t = x.data_ptr(), xb, xt, xk, max(t, 1)
    d.m, d.k, d.parts = m, k, parts
    d.q, d.q_part_stride, d.ldq = q.data_ptr(), m * ldq, ldq
    d.qs, d.qs_part_stride = qs.data_ptr(), m
    if norm is not None:
        d.norm_weight = norm.weight.data_ptr()
        d.norm_bias = None if norm.bias is None else norm.bias.data_ptr()
        d.eps = float(norm.eps)
    if pre_norm is not None:
        if normed is None or normed.dtype != torch.float32 or normed.dim() != 2 or normed.shape[0] < m \
                or normed.shape[1] < k or normed.stride(1) != 1:
            raise ValueError("pre_norm needs `normed`, an FP32 [m, k] tensor with unit-stride rows")
        _require_cuda(normed, "normed")
        d.pre_norm_weight = pre_norm.weight.data_ptr()
        d.pre_norm_bias = None if pre_norm.bias is None else pre_norm.bias.data_ptr()
        d.pre_eps = float(pre_norm.eps)
        d.normed, d.ld_normed = normed.data_ptr(), normed.stride(0)
    d.flags = (_lib.QUANT_INPUT_SILU if input_silu else 0) | (_lib.QUANT_PDL if pdl else 0) \
        | (_lib.QUANT_NARROW_ROWS if narrow else 0)
    return d


def gemm(q: Tensor, qs: Tensor, ldq: int, m: int, panels: Tensor, wbits: int, n: int, k: int, alpha: Tensor,
         bias: Tensor | None, y: Tensor, *, parts: int, silu: bool = False, order: int = 0, acc: Tensor | None = None,
         config=None, pdl: bool = False, error_word: Tensor | None = None, pair: bool = True,
         force_pair: bool = False, residual: Tensor | None = None, residual_scale: float = 1.0,
         workspace: Tensor | None = None, swap: bool = True, wait_clocks: int = 0, test_stall: bool = False,
         resident_weights: bool = True, reg: bool = True) -> None:
    """y[:m] (row stride y.stride(0); FP32 or FP16) from q int8 [parts, m, ldq] and qs FP32 [parts, m].
    acc, when given, receives the exact INT32 accumulators as int32 [parts, m, n] (any row / part strides).
    `config` forces the per-tile kernel's tiles, or (tile_m <= 16, m <= 16) the CUDA-core kernel's channels per CTA;
    a pair config from the table forces nothing. pair=False keeps the dispatch table away from the persistent
    CTA-pair kernel; force_pair=True takes it wherever its shape allows (also below the table's tile threshold).
    residual (FP32 [m, n], unit column stride; may be y itself) makes the epilogue write residual + residual_scale *
    value, rounded as the unfused `residual + residual_scale * y` (FP32 y only). workspace: scratch for the pair
    kernel's split-K (few tiles, long K): None takes _lib.workspace_bytes of it from PyTorch's allocator when the
    shape splits; a caller's uint8 CUDA tensor is used as given (an empty one runs the GEMM unsplit). swap=False keeps
    the table away from the small-M swapped-operand kernel; a SWAP config (kernel == 3) forces it with its splits and
    stages. wait_clocks bounds each wait of the swap kernel (0: the library's default); test_stall (tests only, with a
    forced SWAP config) makes the kernel withhold its activation copies so that a wait runs out. resident_weights=False
    keeps the pair kernel re-expanding every tile's weights where it would keep them resident (one part, K <= 1024).
    reg=False keeps the table away from the small-M register-operand kernel; a REG config (kernel == 4) forces it
    with its channels, rows and K-slices per CTA."""
    if m == 0:
        return
    d, keep = _gemm_desc(q, qs, ldq, m, panels, wbits, n, k, alpha, bias, y, parts=parts, silu=silu, order=order,
                         acc=acc, config=config, pdl=pdl, error_word=error_word, pair=pair, force_pair=force_pair,
                         residual=residual, residual_scale=residual_scale, workspace=workspace, swap=swap,
                         wait_clocks=wait_clocks, test_stall=test_stall, resident_weights=resident_weights, reg=reg)
    with torch.cuda.device(y.device):
        _lib.check(_lib.lib().kea_lowbit_gemm(ctypes.byref(d), _lib.stream_handle(y.device)), "gemm")


def _gemm_desc(q, qs, ldq, m, panels, wbits, n, k, alpha, bias, y, *, parts, silu=False, order=0, acc=None,
               config=None, pdl=False, error_word=None, pair=True, force_pair=False, residual=None,
               residual_scale=1.0, workspace=None, swap=True, wait_clocks=0, test_stall=False,
               resident_weights=True, reg=True):
    """The C descriptor of gemm()'s arguments (checked), and the workspace tensor it points into (keep it alive
    until the launch)."""
    if parts not in (1, 2, 3):
        raise ValueError(f"parts must be 1, 2 or 3, got {parts!r}")
    if order not in (0, 1):
        raise ValueError("order must be 0 or 1")
    for t, name in ((q, "q"), (qs, "qs"), (y, "y")):
        _require_cuda(t, name)
    if q.dtype != torch.int8 or q.dim() != 3 or q.shape[0] < parts or q.shape[1] < m:
        raise ValueError(f"q must be int8 [{parts}, {m}, ldq]")
    if ldq % 16 or q.stride(1) != ldq or q.stride(2) != 1 or q.data_ptr() % 16 or ldq < k:
        raise ValueError("fast path needs 16-byte aligned rows of q")
    if parts > 1 and q.stride(0) % 16:
        raise ValueError("fast path needs 16-byte aligned parts of q")
    if qs.dtype != torch.float32 or qs.dim() != 2 or qs.shape[0] < parts or qs.shape[1] < m or qs.stride(1) != 1:
        raise ValueError(f"qs must be FP32 [{parts}, {m}] with unit column stride")
    if y.dtype not in (torch.float32, torch.float16) or y.dim() != 2 or y.shape[0] < m or y.shape[1] < n \
            or y.stride(1) != 1:
        raise ValueError(f"y must be FP32 / FP16 [{m}, {n}] with unit column stride")
    if not (q.device == qs.device == y.device == panels.device):
        raise ValueError("q, qs, y and the layer must be on one device")
    if acc is not None and (acc.dtype != torch.int32 or acc.dim() != 3 or acc.shape[0] < parts
                            or acc.shape[1] < m or acc.shape[2] < n or acc.stride(2) != 1 or acc.device != y.device):
        raise ValueError(f"acc must be int32 [{parts}, {m}, {n}] with unit column stride")
    if residual is not None:
        _require_cuda(residual, "residual")
        if residual.dtype != torch.float32 or residual.dim() != 2 or residual.shape[0] < m or residual.shape[1] < n \
                or residual.stride(1) != 1 or residual.device != y.device or y.dtype != torch.float32:
            raise ValueError(f"residual must be FP32 [{m}, {n}] with unit column stride, with an FP32 y")
    d = _lib.GemmDesc()
    d.q, d.q_part_stride, d.ldq, d.parts = q.data_ptr(), q.stride(0), ldq, parts
    if residual is not None:
        d.residual, d.ld_residual, d.residual_scale = residual.data_ptr(), residual.stride(0), float(residual_scale)
    d.qs, d.qs_part_stride = qs.data_ptr(), qs.stride(0)
    d.panels, d.wbits, d.n, d.k = panels.data_ptr(), wbits, n, k
    d.alpha, d.bias = alpha.data_ptr(), (None if bias is None else bias.data_ptr())
    d.y, d.ldy = y.data_ptr(), y.stride(0)
    d.y_dtype = _lib.OUT_F16 if y.dtype == torch.float16 else _lib.OUT_F32
    if acc is not None:
        d.acc, d.ld_acc, d.acc_part_stride = acc.data_ptr(), acc.stride(1), acc.stride(0)
    d.m = m
    d.flags = (_lib.FLAG_SILU if silu else 0) | (_lib.FLAG_ORDER1 if order else 0) | (_lib.FLAG_PDL if pdl else 0) \
        | (0 if pair else _lib.FLAG_NO_PAIR) | (_lib.FLAG_FORCE_PAIR if force_pair else 0) \
        | (0 if swap else _lib.FLAG_NO_SWAP) | (_lib.FLAG_TEST_STALL if test_stall else 0) \
        | (0 if resident_weights else _lib.FLAG_NO_RESIDENT_WEIGHTS)
    kernel = getattr(config, "kernel", 0) if config is not None else None
    if not reg and kernel != 4:
        d.flags |= _lib.FLAG_NO_REG
    if kernel == 4:   # the register kernel with this config's channels, rows and K-slices per CTA (0: the table's)
        d.flags |= _lib.FLAG_FORCE_REG
        d.tile_m, d.tile_n, d.splits = config.tile_m, config.tile_n, config.splits
    elif kernel == 3:   # the swap kernel with this config's token tile, split and stages (0: the table's)
        d.flags |= _lib.FLAG_FORCE_SWAP
        d.tile_m, d.splits, d.stages = config.tile_m, config.splits, config.stages
    elif config is not None and kernel != 1:   # a pair config from the table forces nothing
        d.tile_m, d.tile_n, d.splits, d.stages = config.tile_m, config.tile_n, config.splits, config.stages
    d.wait_clocks = int(wait_clocks)
    if error_word is not None:
        d.error_word = error_word.data_ptr()
    if workspace is None and pair and d.tile_m == 0:
        need = _lib.workspace_bytes(m, n, k, wbits, parts)
        if need:
            workspace = torch.empty(need, dtype=torch.uint8, device=y.device)
    if workspace is not None and workspace.numel():
        if workspace.device != y.device or not workspace.is_contiguous():
            raise ValueError("workspace must be a contiguous tensor on y's device")
        d.workspace, d.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    return d, workspace


def project(x: Tensor, rows: tuple[int, int, int, int], m: int, k: int, panels: Tensor, wbits: int, n: int,
            alpha: Tensor, bias: Tensor | None, y: Tensor, *, parts: int, norm=None, input_silu: bool = False,
            pre_norm=None, normed: Tensor | None = None, ldq: int | None = None, quant_pdl: bool = False,
            fuse: bool = False, require_fused: bool = False, **gemm_options) -> tuple[Tensor, Tensor, int]:
    """quantize() then gemm() in one call (the reference's Int8MmaLayer.project): x rows as quantize() takes them ->
    y[:m] with gemm()'s epilogue options (silu, residual, acc, pdl, ...). By default the two kernels run back to back
    (quantize with quant_pdl, then the GEMM; the faster form measured on B200). fuse=True asks for one kernel whose
    thread-block clusters quantize the rows themselves where the shape allows (one part, 33 <= m <= 128, k a
    multiple of 128 up to 1024: one warp a row, quantize(..., narrow_rows=True)'s arithmetic, bit for bit);
    require_fused=True demands it (ValueError where it does not apply). Returns the parts it multiplied
    (q int8 [parts, m, ldq], qs FP32 [parts, m], ldq)."""
    _require_cuda(x, "x")
    if x.dtype != torch.float32:
        raise ValueError(f"expected FP32 input, got {x.dtype}")
    ldq = _round_up(k, 16) if ldq is None else ldq
    q = torch.empty(parts, m, ldq, device=x.device, dtype=torch.int8)
    qs = torch.empty(parts, m, device=x.device, dtype=torch.float32)
    if m == 0:
        return q, qs, ldq
    pd = _lib.ProjectDesc()
    pd.quant = _quant_desc(x, rows, m, k, parts, q, qs, ldq, norm=norm, input_silu=input_silu, pdl=quant_pdl,
                           pre_norm=pre_norm, normed=normed, narrow=False)
    g, keep = _gemm_desc(q, qs, ldq, m, panels, wbits, n, k, alpha, bias, y, parts=parts, **gemm_options)
    pd.gemm = g
    fuse = fuse or require_fused
    pd.flags = _lib.PROJECT_FUSE if fuse else 0
    need = _lib.lib().kea_lowbit_project_scratch_bytes(m, n, k, wbits, parts) if fuse else 0
    scratch = torch.empty(need, dtype=torch.uint8, device=x.device) if need else None
    if scratch is not None:
        pd.scratch, pd.scratch_bytes = scratch.data_ptr(), need
    with torch.cuda.device(y.device):
        if require_fused:
            route = _lib.lib().kea_lowbit_project_fuses(ctypes.byref(pd))
            if route < 0:
                _lib.check(-route, "project")
            if route != 1:
                raise ValueError("the fused quantizer does not apply to this projection")
        _lib.check(_lib.lib().kea_lowbit_project(ctypes.byref(pd), _lib.stream_handle(y.device)), "project")
    return q, qs, ldq


def glu_depthwise(h: Tensor, weight: Tensor, bias: Tensor | None = None, lengths: Tensor | None = None, *,
                  pdl: bool = False) -> Tensor:
    """The convolution module's middle in one kernel: h FP32 [B, T, 2C] (pw1's output) -> GLU (first half times
    sigmoid of the second), zero at frames t >= lengths[b], depthwise conv along time with weight FP32 [C, kw]
    (BatchNorm folded in) and bias [C], zero padding -> FP32 [B, T, C]."""
    _require_cuda(h, "h")
    if h.dtype != torch.float32 or h.dim() != 3 or h.shape[2] % 2 or not h.is_contiguous():
        raise ValueError("h must be contiguous FP32 [B, T, 2C]")
    b, t, c2 = h.shape
    c = c2 // 2
    if weight.dim() == 3:
        weight = weight.reshape(weight.shape[0], weight.shape[-1])
    if weight.dtype != torch.float32 or weight.shape[0] != c or weight.device != h.device:
        raise ValueError(f"weight must be FP32 [{c}, kw] on {h.device}")
    weight = weight.contiguous()
    if bias is not None and (bias.dtype != torch.float32 or tuple(bias.shape) != (c,) or bias.device != h.device):
        raise ValueError(f"bias must be FP32 [{c}] on {h.device}")
    if lengths is not None:
        if tuple(lengths.shape) != (b,) or lengths.device != h.device:
            raise ValueError(f"lengths must be [{b}] on {h.device}")
        lengths = lengths.to(torch.int32).contiguous()
    y = torch.empty(b, t, c, device=h.device, dtype=torch.float32)
    d = _lib.ConvDesc(h=h.data_ptr(), y=y.data_ptr(), weight=weight.data_ptr(), bias=_lib.ptr(bias),
                      lengths=_lib.ptr(lengths), b=b, t=t, c=c, kw=weight.shape[1], flags=_lib.CONV_PDL if pdl else 0)
    with torch.cuda.device(h.device):
        _lib.check(_lib.lib().kea_lowbit_glu_depthwise(ctypes.byref(d), _lib.stream_handle(h.device)), "glu_depthwise")
    return y


def glu_depthwise_quantized(h: Tensor, weight: Tensor, bias: Tensor | None, lengths: Tensor | None, parts: int, *,
                            silu: bool = True, ldq: int | None = None, pdl: bool = False) -> tuple[Tensor, Tensor, int]:
    """glu_depthwise with the next projection's quantizer fused in: the conv output y [B, T, C] (never written) ->
    (q int8 [parts, B*T, ldq], qs FP32 [parts, B*T], ldq), bit for bit quantize(y, input_silu=silu). Kernel width 9,
    C % 4 == 0 and C <= 1024 (the Parakeet conv module); other shapes raise ValueError."""
    _require_cuda(h, "h")
    if h.dtype != torch.float32 or h.dim() != 3 or h.shape[2] % 2 or not h.is_contiguous():
        raise ValueError("h must be contiguous FP32 [B, T, 2C]")
    b, t, c2 = h.shape
    c = c2 // 2
    if weight.dim() == 3:
        weight = weight.reshape(weight.shape[0], weight.shape[-1])
    if weight.dtype != torch.float32 or weight.shape[0] != c or weight.device != h.device:
        raise ValueError(f"weight must be FP32 [{c}, kw] on {h.device}")
    if weight.shape[1] != 9 or c % 4 or c > 1024:
        raise ValueError("the fused conv quantizer needs kernel width 9 and C % 4 == 0, C <= 1024")
    weight = weight.contiguous()
    if bias is not None and (bias.dtype != torch.float32 or tuple(bias.shape) != (c,) or bias.device != h.device):
        raise ValueError(f"bias must be FP32 [{c}] on {h.device}")
    if lengths is not None:
        if tuple(lengths.shape) != (b,) or lengths.device != h.device:
            raise ValueError(f"lengths must be [{b}] on {h.device}")
        lengths = lengths.to(torch.int32).contiguous()
    m = b * t
    ldq = _round_up(c, 16) if ldq is None else ldq
    q = torch.empty(parts, m, ldq, device=h.device, dtype=torch.int8)
    qs = torch.empty(parts, m, device=h.device, dtype=torch.float32)
    if m == 0:
        return q, qs, ldq
    flags = (_lib.CONV_PDL if pdl else 0) | (_lib.CONV_QUANT_SILU if silu else 0)
    d = _lib.ConvDesc(h=h.data_ptr(), y=None, weight=weight.data_ptr(), bias=_lib.ptr(bias),
                      lengths=_lib.ptr(lengths), b=b, t=t, c=c, kw=weight.shape[1], flags=flags, q=q.data_ptr(),
                      q_part_stride=m * ldq, ldq=ldq, qs=qs.data_ptr(), qs_part_stride=m, parts=parts)
    with torch.cuda.device(h.device):
        _lib.check(_lib.lib().kea_lowbit_glu_depthwise(ctypes.byref(d), _lib.stream_handle(h.device)),
                   "glu_depthwise_quantized")
    return q, qs, ldq


def rel_attention(qkv: Tensor, pos: Tensor, bias_u: Tensor, bias_v: Tensor, heads: int,
                  lengths: Tensor | None = None, *, pdl: bool = False) -> Tensor:
    """Relative-position self-attention in one kernel: qkv FP32 [B, T, 3 * H * DK] (q, k, v of each token, heads
    inside), pos FP32 [2T - 1, H * DK] (the position projection of relative positions T - 1 .. -(T - 1)),
    bias_u / bias_v [H, DK] -> ctx FP32 [B, T, H * DK]; keys at frames >= lengths[b] are masked."""
    _require_cuda(qkv, "qkv")
    if qkv.dtype != torch.float32 or qkv.dim() != 3 or not qkv.is_contiguous() or qkv.shape[2] % (3 * heads):
        raise ValueError("qkv must be contiguous FP32 [B, T, 3 * H * DK]")
    b, t, w3 = qkv.shape
    d = w3 // 3
    dk = d // heads
    pos = pos.reshape(-1, d)
    if pos.dtype != torch.float32 or pos.shape[0] != max(0, 2 * t - 1) or pos.device != qkv.device:
        raise ValueError(f"pos must be FP32 [{2 * t - 1}, {d}] on {qkv.device}")
    pos = pos.contiguous()
    bu, bv = bias_u.contiguous(), bias_v.contiguous()
    for name, x in (("bias_u", bu), ("bias_v", bv)):
        if x.dtype != torch.float32 or x.numel() != d or x.device != qkv.device:
            raise ValueError(f"{name} must be FP32 [{heads}, {dk}] on {qkv.device}")
    if lengths is not None:
        if tuple(lengths.shape) != (b,) or lengths.device != qkv.device:
            raise ValueError(f"lengths must be [{b}] on {qkv.device}")
        lengths = lengths.to(torch.int32).contiguous()
    ctx = torch.empty(b, t, d, device=qkv.device, dtype=torch.float32)
    desc = _lib.AttentionDesc(qkv=qkv.data_ptr(), pos=pos.data_ptr(), bias_u=bu.data_ptr(), bias_v=bv.data_ptr(),
                              lengths=_lib.ptr(lengths), ctx=ctx.data_ptr(), b=b, t=t, h=heads, dk=dk,
                              scale=1.0 / math.sqrt(dk), flags=_lib.CONV_PDL if pdl else 0)
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.lib().kea_lowbit_rel_attention(ctypes.byref(desc), _lib.stream_handle(qkv.device)),
                   "rel_attention")
    return ctx
