"""A random-init FastConformer encoder (Parakeet-TDT-0.6B shapes) whose low-bit projections run on the B200 kernels,
plus the TDT joint's projections: the call sites of the low-bit GEMM for one clip or a batch of clips.

kea-kernels swaps the NeMo encoder's quantised linears for its projection provider and fuses their neighbours into
the calls (src/kea_kernels/ternary/transforms.py:45-97, src/kea_kernels/ternary/layer_fusions4.py:52-94):
  * FF1 / FF2 (macaron halves): LayerNorm fused into the quantizer, 1024 -> 4096 with SiLU fused into the epilogue,
    4096 -> 1024, residual + 0.5 * ff;
  * attention: LayerNorm fused, Q, K, V as one 1024 -> 3072 projection, relative-position attention whose
    linear_pos projection of the position table is computed once per clip length and cached, out 1024 -> 1024;
  * convolution: LayerNorm fused, pointwise 1024 -> 2048, GLU, depthwise conv (kernel 9, BatchNorm folded into it),
    SiLU fused into the next quantizer as its input activation, pointwise 1024 -> 1024.
Everything else (subsampling, attention arithmetic, GLU, depthwise conv, residuals, the final LayerNorm) is plain
FP32 PyTorch, as in the reference, where only the 264 encoder linears are quantised (src/kea_kernels/formats.py:39-46).
NeMo is not a dependency: this module builds the same layer structure with random weights (1-bit signs drawn with
p = 0.5, or ternary codes with p = {0.3, 0.4, 0.3}) so the GEMM call sequence and shapes are those of a real clip.

Per layer that is 8 low-bit GEMMs at M = frames (QKV, out, 2 x FF up, 2 x FF down, pw1, pw2), plus linear_pos at
M = 2 T - 1 when a new clip length is first seen.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from kea_kernels import formats, lowbit
from kea_kernels.binary import bits

# The low-bit projections of one layer in call order (linear_pos runs once per clip length and is cached).
LAYER_LINEARS = ("ff1_up", "ff1_down", "qkv", "out", "pw1", "pw2", "ff2_up", "ff2_down")


def layer_linear_shapes(d: int, ff: int) -> dict[str, tuple[int, int]]:
    """(out_features, in_features) of every low-bit projection of a layer."""
    return {"ff1_up": (ff, d), "ff1_down": (d, ff), "qkv": (3 * d, d), "out": (d, d), "pw1": (2 * d, d),
            "pw2": (d, d), "ff2_up": (ff, d), "ff2_down": (d, ff), "linear_pos": (d, d)}


class LowBitLinear(nn.Module):
    """One low-bit projection resident as B200 panels: quantize (optional fused LayerNorm / input SiLU) into `parts`
    residual INT8 parts, then the tcgen05 GEMM with the FP32 epilogue (optional SiLU). FP32 in, FP32 out."""

    def __init__(self, codes: Tensor, wbits: int, scale: Tensor, bias: Tensor | None, in_features: int, *,
                 parts: int, device: torch.device, pdl: bool = True):
        super().__init__()
        n = codes.shape[0]
        self.in_features, self.out_features, self.wbits, self.parts, self.pdl = in_features, n, wbits, parts, pdl
        self.quant_pdl = False   # launch this projection's quantizer with programmatic dependent launch
        self.panels = lowbit.prepare_panels(codes.to(device), wbits, n, in_features)
        self.scale = scale.to(device=device, dtype=torch.float32).contiguous()
        self.bias = None if bias is None else bias.to(device=device, dtype=torch.float32).contiguous()

    def forward(self, x: Tensor, *, norm: nn.LayerNorm | None = None, input_silu: bool = False,
                silu: bool = False, residual: Tensor | None = None, residual_scale: float = 1.0,
                pre_norm: nn.LayerNorm | None = None, normed: Tensor | None = None) -> Tensor:
        """x [B, T, K] (any strides) -> [B, T, N]; with `residual` ([B, T, N] contiguous FP32) the GEMM's epilogue
        returns residual + residual_scale * projection (the layer's skip connection, same roundings as unfused).
        `pre_norm`: a LayerNorm applied to x before `norm`, its output written to `normed` ([B, T, K] contiguous;
        x itself allowed, which keeps the quantizer out of the GEMM kernel) - the previous layer's output norm folded
        into this quantizer."""
        b, t, k = x.shape
        m = b * t
        y = torch.empty(b, t, self.out_features, device=x.device, dtype=torch.float32)
        if m == 0:
            return y
        # one call: the library runs the quantizer inside the GEMM kernel where the shape allows, else the two
        # kernels back to back. The quantizer is launched plainly unless `quant_pdl` is set: with programmatic
        # dependent launch its CTAs sit on the SMs while the previous kernel drains, which measured slower on the
        # clip after most kernels (3.234 -> 3.371 ms per clip with every quantizer so launched) but faster after the
        # FF up projections' one-CTA-per-SM GEMMs (3.234 -> 3.209 ms with the FF down quantizers alone); the GEMM
        # after a quantizer always uses it
        res = None if residual is None else residual.reshape(m, self.out_features)
        lowbit.project(x, (x.stride(0), x.stride(1), x.stride(2), t), m, k, self.panels, self.wbits,
                       self.out_features, self.scale, self.bias, y.view(m, self.out_features), parts=self.parts,
                       norm=norm, input_silu=input_silu, pre_norm=pre_norm,
                       normed=None if normed is None else normed.view(m, k), silu=silu, pdl=self.pdl, residual=res,
                       residual_scale=residual_scale, quant_pdl=self.pdl and self.quant_pdl)
        return y

    def from_quantized(self, q: Tensor, qs: Tensor, ldq: int, b: int, t: int, *, silu: bool = False,
                       residual: Tensor | None = None, residual_scale: float = 1.0) -> Tensor:
        """The GEMM on activations already quantized into `parts` INT8 parts (q [parts, b*t, ldq], qs [parts, b*t])
        -> FP32 [b, t, N], with forward's epilogue options."""
        m = b * t
        y = torch.empty(b, t, self.out_features, device=q.device, dtype=torch.float32)
        if m == 0:
            return y
        res = None if residual is None else residual.reshape(m, self.out_features)
        lowbit.gemm(q, qs, ldq, m, self.panels, self.wbits, self.out_features, self.in_features, self.scale,
                    self.bias, y.view(m, self.out_features), parts=self.parts, silu=silu, pdl=self.pdl, residual=res,
                    residual_scale=residual_scale)
        return y


class RandomLowBitWeights:
    """Seeded export-format codes for one projection: 1-bit signs (bits.pack_signs) or ternary codes
    (formats.pack_ternary), with per-channel scales (FP16 values stored as FP32) of about 1 / sqrt(K E[w^2]), so a
    random-init stack keeps its activations in range."""

    def __init__(self, n: int, k: int, wbits: int, gen: torch.Generator, *, keep_dense: bool = False):
        dev = gen.device
        if wbits == 1:
            w = torch.where(torch.rand(n, k, generator=gen, device=dev) < 0.5, -1, 1).to(torch.int8)
            self.codes = bits.pack_signs(w)
        else:
            u = torch.rand(n, k, generator=gen, device=dev)
            w = torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8)
            self.codes = formats.pack_ternary(w)
        self.w = w if keep_dense else None
        # variance-preserving scale for random init: alpha ~ 1 / sqrt(k * E[w^2])
        base = 1.0 / math.sqrt(k * (1.0 if wbits == 1 else 0.6))
        self.scale = ((torch.rand(n, generator=gen, device=dev) * 0.8 + 0.6) * base).half().float()

    def dense(self) -> Tensor:
        if self.w is None:
            raise RuntimeError("built without keep_dense=True")
        return self.w.float() * self.scale[:, None]


def rel_shift(x: Tensor) -> Tensor:
    """[B, H, T, 2T - 1] relative-position scores -> [B, H, T, T] aligned to absolute positions (Transformer-XL)."""
    b, h, t, p = x.shape
    x = F.pad(x, (1, 0))
    x = x.view(b, h, p + 1, t)[:, :, 1:].reshape(b, h, t, p)
    return x[:, :, :, : t]


def torch_rel_attention(qkv: Tensor, pos: Tensor, bias_u: Tensor, bias_v: Tensor, heads: int,
                        lengths: Tensor | None = None) -> Tensor:
    """The relative-position attention as PyTorch FP32 ops (NeMo's RelPositionMultiHeadAttention math): the same
    function as lowbit.rel_attention, used where that kernel measured slower (one clip: too few CTAs; long clips)."""
    b, t, w3 = qkv.shape
    d = w3 // 3
    dk = d // heads
    q, k, v = qkv.view(b, t, 3, heads, dk).unbind(2)                   # [b, t, h, dk]
    p = pos.view(2 * t - 1, heads, dk)
    ac = torch.matmul((q + bias_u).transpose(1, 2), k.permute(0, 2, 3, 1))            # [b, h, t, t]
    bd = rel_shift(torch.matmul((q + bias_v).transpose(1, 2), p.permute(1, 2, 0)))   # [b, h, t, t]
    scores = (ac + bd) * (1.0 / math.sqrt(dk))
    if lengths is not None:
        keys = torch.arange(t, device=qkv.device)[None, :] < lengths.to(qkv.device)[:, None]
        scores = scores.masked_fill(~keys[:, None, None, :], float("-inf"))
    attn = torch.softmax(scores, dim=-1)
    return torch.matmul(attn, v.transpose(1, 2)).transpose(1, 2).reshape(b, t, d)


# The fused FP32 attention kernel measured faster than the PyTorch sequence from 16 (clip, head) pairs on (B200, 125
# frames: 1.6-2.1x at 2-4 clips, 1.4x at 256; 85 clips of 375 frames: 1.03x); one clip ties at 125 frames and loses
# at 375 (too few CTAs), so a single clip takes the PyTorch sequence.
FUSED_ATTENTION_MIN_ROWS, FUSED_ATTENTION_MAX_T = 16, 1 << 30


def rel_positions(t: int, d: int, device) -> Tensor:
    """Sinusoidal table for relative positions t - 1 ... -(t - 1): [2 t - 1, d]."""
    pos = torch.arange(t - 1, -t, -1, device=device, dtype=torch.float32)[:, None]
    div = torch.exp(torch.arange(0, d, 2, device=device, dtype=torch.float32) * (-math.log(10000.0) / d))
    pe = torch.zeros(2 * t - 1, d, device=device)
    pe[:, 0::2] = torch.sin(pos * div)
    pe[:, 1::2] = torch.cos(pos * div)
    return pe


class ConformerLayer(nn.Module):
    def __init__(self, d: int, heads: int, ff: int, kernel: int, wbits: int, parts: int, gen: torch.Generator,
                 device: torch.device, pdl: bool, keep_dense: bool,
                 projections: dict[str, LowBitLinear] | None = None):
        """`projections`: loaded low-bit projections by this module's names (an export); the others are random."""
        super().__init__()
        self.d, self.heads, self.dk = d, heads, d // heads
        self.lin = nn.ModuleDict()
        self.weights = {}
        rnd = lambda *shape: torch.randn(*shape, generator=gen, device=device)
        for name, (n, k) in layer_linear_shapes(d, ff).items():
            if projections is not None and name in projections:
                lin = projections[name]
                if (lin.out_features, lin.in_features) != (n, k):
                    raise ValueError(f"{name}: projection is {lin.out_features} x {lin.in_features}, expected {n} x {k}")
                self.lin[name] = lin
                continue
            w = RandomLowBitWeights(n, k, wbits, gen, keep_dense=keep_dense)
            bias = rnd(n) * 0.02 if name != "linear_pos" else None
            self.weights[name] = (w, bias)
            self.lin[name] = LowBitLinear(w.codes, wbits, w.scale, bias, k, parts=parts, device=device, pdl=pdl)
        for name in ("ff1_down", "ff2_down"):   # their quantizers follow the FF up GEMMs: launched early (forward)
            self.lin[name].quant_pdl = True
        self.norms = nn.ModuleDict({n: nn.LayerNorm(d) for n in ("ff1", "att", "conv", "ff2", "out")}).to(device)
        with torch.no_grad():
            for norm in self.norms.values():
                norm.weight.copy_(1.0 + 0.1 * rnd(d))
                norm.bias.copy_(0.05 * rnd(d))
        self.pos_bias_u = 0.02 * rnd(heads, self.dk)
        self.pos_bias_v = 0.02 * rnd(heads, self.dk)
        # depthwise conv with BatchNorm (eval) folded into its weight and bias
        self.dw_weight = rnd(d, 1, kernel) / math.sqrt(kernel)
        self.dw_bias = 0.02 * rnd(d)
        self.kernel = kernel
        self._pos_cache: dict[int, Tensor] = {}

    def positions(self, t: int, device) -> Tensor:
        """linear_pos(position table) for clip length t, cached (the reference caches it per length too)."""
        p = self._pos_cache.get(t)
        if p is None:
            table = rel_positions(t, self.d, device)[None]
            p = self.lin["linear_pos"](table)[0]
            self._pos_cache[t] = p
        return p

    def attention(self, x: Tensor, lengths: Tensor | None = None) -> Tensor:
        """Relative-position MHSA: LayerNorm fused into the QKV quantizer, the attention itself one FP32 kernel
        (both position biases, the shifted position scores, key masking past `lengths`, online softmax) reading the
        QKV GEMM's rows and writing the out projection's, whose epilogue adds the skip connection."""
        b, t, _ = x.shape
        qkv = self.lin["qkv"](x, norm=self.norms["att"])                # [b, t, 3 d]: q, k, v by heads
        attend = lowbit.rel_attention if (b * self.heads >= FUSED_ATTENTION_MIN_ROWS and
                                          t <= FUSED_ATTENTION_MAX_T) else torch_rel_attention
        ctx = attend(qkv, self.positions(t, x.device), self.pos_bias_u, self.pos_bias_v, self.heads, lengths)
        return self.lin["out"](ctx, residual=x)                          # x + out(ctx)

    def conv(self, x: Tensor, lengths: Tensor | None = None) -> Tensor:
        """lengths: optional int32 [b] frames per clip (later frames are padding, zeroed before the depthwise conv).
        GLU, padding mask and the depthwise conv (BatchNorm folded in) are one kernel between the two GEMMs, reading
        and writing token-major rows, so pw2's quantizer (with the conv module's SiLU fused) reads unit-stride rows."""
        h = self.lin["pw1"](x, norm=self.norms["conv"])                 # [b, t, 2d]
        pw2 = self.lin["pw2"]
        if self.kernel == 9 and self.d % 4 == 0 and self.d <= 1024:
            # pw2's quantizer (input SiLU) fused into the conv kernel: the FP32 conv output is never written
            q, qs, ldq = lowbit.glu_depthwise_quantized(h, self.dw_weight, self.dw_bias, lengths, pw2.parts)
            return pw2.from_quantized(q, qs, ldq, x.shape[0], x.shape[1], residual=x)   # x + pw2(...)
        h = lowbit.glu_depthwise(h, self.dw_weight, self.dw_bias, lengths)   # [b, t, d]
        return pw2(h, input_silu=True, residual=x)                      # SiLU in the quantizer; x + pw2(...)

    def forward(self, x: Tensor, lengths: Tensor | None = None) -> Tensor:
        return self.norms["out"](self.body(x, lengths))

    def body(self, x: Tensor, lengths: Tensor | None = None, pre_norm: nn.LayerNorm | None = None) -> Tensor:
        """The layer without its output LayerNorm. `pre_norm` (the previous layer's output norm) is applied to x
        inside FF1's quantizer, which writes the normalized rows out: the skip connection's input."""
        # every skip connection is added in the epilogue of the GEMM that ends its branch (x + 0.5 ff, x + att, ...)
        xn = torch.empty_like(x, memory_format=torch.contiguous_format) if pre_norm is not None else None
        h = self.lin["ff1_up"](x, norm=self.norms["ff1"], silu=True, pre_norm=pre_norm, normed=xn)
        if xn is not None:
            x = xn
        x = self.lin["ff1_down"](h, residual=x, residual_scale=0.5)
        x = self.attention(x, lengths)
        x = self.conv(x, lengths)
        return self.lin["ff2_down"](self.lin["ff2_up"](x, norm=self.norms["ff2"], silu=True), residual=x,
                                    residual_scale=0.5)


class Subsampling(nn.Module):
    """8x time reduction of log-mel frames (three stride-2 3x3 convolutions, depthwise-separable after the first),
    then a linear map to d_model: [B, 128, T] -> [B, ceil(T / 8), d]. FP32, not quantised."""

    def __init__(self, n_mels: int, d: int, channels: int, gen: torch.Generator, device):
        super().__init__()
        c = channels
        self.conv = nn.Sequential(
            nn.Conv2d(1, c, 3, 2, 1), nn.ReLU(),
            nn.Conv2d(c, c, 3, 2, 1, groups=c), nn.Conv2d(c, c, 1), nn.ReLU(),
            nn.Conv2d(c, c, 3, 2, 1, groups=c), nn.Conv2d(c, c, 1), nn.ReLU())
        f = n_mels
        for _ in range(3):
            f = (f - 1) // 2 + 1
        self.out = nn.Linear(c * f, d)
        self.to(device)
        with torch.no_grad():
            for mod in self.modules():
                if isinstance(mod, (nn.Conv2d, nn.Linear)):
                    fan_in = mod.weight[0].numel()
                    mod.weight.copy_(torch.randn(mod.weight.shape, generator=gen, device=device) * math.sqrt(2.0 / fan_in))
                    mod.bias.copy_(0.01 * torch.randn(mod.bias.shape, generator=gen, device=device))

    def forward(self, mel: Tensor) -> Tensor:
        h = self.conv(mel.unsqueeze(1).transpose(2, 3))                 # [b, c, t/8, f/8]
        b, c, t, f = h.shape
        return self.out(h.permute(0, 2, 1, 3).reshape(b, t, c * f))


class FastConformerEncoder(nn.Module):
    """24 x (FF1, rel-pos MHSA, conv, FF2) over 8x-subsampled log-mel, d_model 1024, 8 heads, FF 4096, conv kernel 9:
    the Parakeet-TDT-0.6B encoder shapes, random weights, low-bit projections on the B200 kernels."""

    def __init__(self, *, layers: int = 24, d_model: int = 1024, heads: int = 8, ff: int = 4096, conv_kernel: int = 9,
                 n_mels: int = 128, sub_channels: int = 256, wbits: int = 1, parts: int = 1, seed: int = 0,
                 device=None, pdl: bool = True, keep_dense: bool = False,
                 projections: list[dict[str, LowBitLinear]] | None = None):
        """`projections`: per layer, loaded low-bit projections (kea_kernels.export); random weights otherwise."""
        super().__init__()
        device = torch.device(device if device is not None else "cuda")
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=device).manual_seed(seed)
        self.d_model, self.wbits, self.parts = d_model, wbits, parts
        self.pre = Subsampling(n_mels, d_model, sub_channels, gen, device)
        if projections is not None and len(projections) != layers:
            raise ValueError(f"projections for {len(projections)} layers, expected {layers}")
        self.layers = nn.ModuleList(ConformerLayer(d_model, heads, ff, conv_kernel, wbits, parts, gen, device, pdl,
                                                   keep_dense, None if projections is None else projections[i])
                                    for i in range(layers))

    def frames(self, t: int) -> int:
        for _ in range(3):
            t = (t - 1) // 2 + 1
        return t

    @torch.inference_mode()
    def forward(self, mel: Tensor, lengths: Tensor | None = None) -> Tensor:
        """mel FP32 [B, 128, T] -> encoder states FP32 [B, frames(T), d_model]. With `lengths` (int [B], encoder
        frames of each clip; the rest of its row is padding) padded frames are masked out as attention keys and
        zeroed before the depthwise convolution, so a clip's real frames do not depend on the padding (the
        length-bucketed batches of mixed-length clips)."""
        x = self.pre(mel)
        lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32)
        # each layer's output LayerNorm runs inside the next layer's first quantizer; the last one here
        pre = None
        for layer in self.layers:
            x = layer.body(x, lens, pre)
            pre = layer.norms["out"]
        return pre(x) if pre is not None else x

    def gemm_shapes(self, batch: int, t: int) -> list[tuple[str, int, int, int]]:
        """(name, M, N, K) of every low-bit GEMM one forward issues once linear_pos is cached."""
        m = batch * self.frames(t)
        out = []
        for i, layer in enumerate(self.layers):
            for name in LAYER_LINEARS:
                lin = layer.lin[name]
                out.append((f"{i}.{name}", m, lin.out_features, lin.in_features))
        return out

    def weight_bytes(self) -> int:
        return sum(l.panels.numel() + 4 * l.scale.numel() for layer in self.layers for l in layer.lin.values())


class TDTJoint(nn.Module):
    """The TDT joint's projections (encoder 1024 -> 640, prediction 640 -> 640, joint 640 -> vocab + blank +
    durations = 1030), random FP32 weights, as the reference keeps them (src/kea_kernels/ternary/decoder_kernels.py:
    139-157). `greedy` scores every encoder frame against a fixed prediction state and returns the arg-max label per
    frame: a frame-synchronous stand-in for the TDT search, enough to produce per-clip token rows to gather."""

    def __init__(self, d_model: int = 1024, hidden: int = 640, vocab: int = 1024, durations: int = 5, seed: int = 1,
                 device=None):
        super().__init__()
        device = torch.device(device if device is not None else "cuda")
        gen = torch.Generator().manual_seed(seed)
        self.enc = nn.Linear(d_model, hidden)
        self.pred = nn.Linear(hidden, hidden)
        self.out = nn.Linear(hidden, vocab + 1 + durations)
        self.vocab = vocab
        with torch.no_grad():
            for p in self.parameters():
                p.copy_(torch.randn(p.shape, generator=gen) / math.sqrt(max(1, p.shape[-1])))
        self.to(device)
        self.state = torch.randn(hidden, generator=gen).to(device)

    @torch.inference_mode()
    def greedy(self, enc: Tensor) -> Tensor:
        """enc [B, T, d] -> int32 labels [B, T] (vocab + 1 = blank)."""
        h = torch.relu(self.enc(enc) + self.pred(self.state))
        return self.out(h)[..., : self.vocab + 1].argmax(-1).to(torch.int32)
