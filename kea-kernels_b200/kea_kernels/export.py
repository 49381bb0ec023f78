"""Loading a Kea-B / Kea-T export onto the B200 kernels, without NeMo.

The reference builds a NeMo model from the export's config and swaps its 264 quantized modules for packed ones
(src/kea_kernels/binary/provider.py:212-262 for parakeet-binary-v1, fusing Q/K/V; src/kea_kernels/ternary/
runtime.py:52-82 for parakeet-ternary-v1). NeMo is not a dependency here: `load_export` validates the directory
(formats.describe / formats.check_export: manifest, SHA-256 of every file, layer names, dtypes, shapes), prepares
every quantized layer's codes as device panels (`LowBitLinear`: the only GPU copy of codes, scales and biases;
ternary codes stay at 2 bits in HBM in every mode, where the reference's Kea-T x2 default keeps an expanded INT8
copy, src/kea_kernels/ternary/encoder4.py:77-149), fuses Q/K/V into one projection per layer, and returns the other
tensors as FP32. `FastConformerEncoder.from_export`-style assembly is `build_encoder`: the loaded projections plus
the export's LayerNorms, relative-position biases, depthwise convolution (its BatchNorm folded in) and subsampling,
under their NeMo state-dict names.

Modes (the residual INT8 parts of every activation): binary x2 (default), x3, x1 (Kea-B 0.1's default); ternary x2
(default), x3, compact (three parts; the same 2-bit panels as x3 here).
"""
from __future__ import annotations

import dataclasses
from pathlib import Path

import torch
from torch import Tensor

from kea_kernels import formats
from kea_kernels.encoder import FastConformerEncoder, LowBitLinear

MODE_PARTS = {"x1": 1, "x2": 2, "x3": 3, "compact": 3}
QKV = ("self_attn.linear_q", "self_attn.linear_k", "self_attn.linear_v")
# export module suffix -> this package's projection name (per encoder layer; Q/K/V fuse into "qkv")
PROJECTIONS = {"feed_forward1.linear1": "ff1_up", "feed_forward1.linear2": "ff1_down",
               "feed_forward2.linear1": "ff2_up", "feed_forward2.linear2": "ff2_down",
               "self_attn.linear_out": "out", "self_attn.linear_pos": "linear_pos",
               "conv.pointwise_conv1": "pw1", "conv.pointwise_conv2": "pw2"}
# NeMo LayerNorm names of a ConformerLayer -> this package's
NORMS = {"norm_feed_forward1": "ff1", "norm_self_att": "att", "norm_conv": "conv", "norm_feed_forward2": "ff2",
         "norm_out": "out"}
BATCH_NORM_EPS = 1e-5


@dataclasses.dataclass
class LoadedExport:
    model: formats.ModelDir
    mode: str
    parts: int
    wbits: int
    manifest: dict
    layers: list[dict[str, LowBitLinear]]   # per encoder layer, by this package's projection names
    tensors: dict[str, Tensor]              # every other tensor of the export, FP32 (CPU)

    def weight_bytes(self) -> int:
        """Device bytes of the quantized layers: panels + scales + biases."""
        total = 0
        for layer in self.layers:
            for lin in layer.values():
                total += lin.panels.numel() + 4 * lin.scale.numel() + (0 if lin.bias is None else 4 * lin.bias.numel())
        return total


def load_export(directory, *, device="cuda", mode: str | None = None, fuse_qkv: bool = True,
                verify_hashes: bool = True, pdl: bool = True) -> LoadedExport:
    """A validated export's quantized layers as device panels (Q/K/V fused per layer when `fuse_qkv`, as the
    reference's loader does by default) and its other tensors as FP32. ValueError for an invalid directory, export,
    mode or codes (tail bits past K, the unused ternary pattern 11)."""
    from safetensors.torch import load_file
    md = formats.describe(directory)
    manifest = formats.check_export(md.export_dir, md.kind, verify_hashes=verify_hashes)
    modes = formats.BINARY_MODES if md.kind == "binary" else formats.TERNARY_MODES
    mode = md.default_mode if mode is None else mode
    if mode not in modes:
        raise ValueError(f"mode {mode!r} is not one of {modes} for a {md.kind} export")
    parts, wbits = MODE_PARTS[mode], (1 if md.kind == "binary" else 2)
    device = torch.device(device)
    tensors = load_file(str(md.export_dir / formats.FILE))
    info = manifest["quantized_layers"]

    def take(name):
        return tensors.pop(f"{name}.codes"), tensors.pop(f"{name}.scale"), \
            tensors.pop(f"{name}.bias") if info[name].get("bias") else None

    def projection(codes, scale, bias, k):
        return LowBitLinear(codes, wbits, scale.float(), None if bias is None else bias.float(), k, parts=parts,
                            device=device, pdl=pdl)

    layers: list[dict[str, LowBitLinear]] = []
    for i in range(formats.LAYERS):
        prefix = f"encoder.layers.{i}."
        lins: dict[str, LowBitLinear] = {}
        if fuse_qkv:
            names = [prefix + q for q in QKV]
            shapes = {tuple(info[n]["shape"]) for n in names}
            kinds = {info[n]["kind"] for n in names}
            biased = {bool(info[n].get("bias")) for n in names}
            if len(shapes) != 1 or kinds != {"linear"} or len(biased) != 1:
                raise ValueError(f"{prefix}self_attn: Q/K/V must be equal-shape linear layers with matching biases")
            k = shapes.pop()[1]
            got = [take(n) for n in names]
            bias = torch.cat([g[2] for g in got]) if biased.pop() else None
            lins["qkv"] = projection(torch.cat([g[0] for g in got]), torch.cat([g[1] for g in got]), bias, k)
        else:
            for q in QKV:
                lins[q.rsplit(".", 1)[1]] = projection(*take(prefix + q), info[prefix + q]["shape"][1])
        for suffix, ours in PROJECTIONS.items():
            name = prefix + suffix
            lins[ours] = projection(*take(name), info[name]["shape"][1])
        layers.append(lins)
    rest = {key: (v.float() if v.is_floating_point() else v) for key, v in tensors.items()}
    return LoadedExport(md, mode, parts, wbits, manifest, layers, rest)


def _assign(dst: Tensor, src: Tensor, name: str) -> None:
    if tuple(dst.shape) != tuple(src.shape):
        raise ValueError(f"{name}: export shape {tuple(src.shape)}, expected {tuple(dst.shape)}")
    with torch.no_grad():
        dst.copy_(src.to(device=dst.device, dtype=dst.dtype))


def build_encoder(loaded: LoadedExport, *, device="cuda", strict: bool = True, seed: int = 0) -> FastConformerEncoder:
    """The encoder on the loaded projections, with the export's non-quantized encoder tensors under their NeMo
    names: per layer the five LayerNorms (`norm_feed_forward1`, `norm_self_att`, `norm_conv`, `norm_feed_forward2`,
    `norm_out`), `self_attn.pos_bias_u/v`, `conv.depthwise_conv` with `conv.batch_norm` folded in (eval statistics);
    the subsampling `pre_encode.conv.{0,2,3,5,6}` and `pre_encode.out`. With strict, every one must be present;
    otherwise missing ones keep their seeded random values. Dimensions come from the projections' shapes."""
    if any("qkv" not in layer for layer in loaded.layers):
        raise ValueError("build_encoder needs Q/K/V fused (load_export(fuse_qkv=True))")
    device = torch.device(device)
    t = loaded.tensors
    first = loaded.layers[0]
    d, ff = first["out"].out_features, first["ff1_up"].out_features
    heads = t["encoder.layers.0.self_attn.pos_bias_u"].shape[0] if "encoder.layers.0.self_attn.pos_bias_u" in t else 8
    kernel = t["encoder.layers.0.conv.depthwise_conv.weight"].shape[-1] \
        if "encoder.layers.0.conv.depthwise_conv.weight" in t else 9
    sub = t["encoder.pre_encode.conv.0.weight"].shape[0] if "encoder.pre_encode.conv.0.weight" in t else 256
    n_mels = 128
    if "encoder.pre_encode.out.weight" in t:
        f = t["encoder.pre_encode.out.weight"].shape[1] // sub   # frequency bins after three stride-2 convs
        n_mels = f * 8   # the largest mel count giving f bins; the count itself does not change any weight
    enc = FastConformerEncoder(layers=len(loaded.layers), d_model=d, heads=heads, ff=ff, conv_kernel=kernel,
                               n_mels=n_mels, sub_channels=sub, wbits=loaded.wbits, parts=loaded.parts, seed=seed,
                               device=device, projections=loaded.layers)
    missing = []

    def get(name):
        if name in t:
            return t[name]
        missing.append(name)
        return None

    for i, layer in enumerate(enc.layers):
        p = f"encoder.layers.{i}."
        for nemo, ours in NORMS.items():
            for field in ("weight", "bias"):
                v = get(f"{p}{nemo}.{field}")
                if v is not None:
                    _assign(getattr(layer.norms[ours], field), v, f"{p}{nemo}.{field}")
        for field in ("pos_bias_u", "pos_bias_v"):
            v = get(f"{p}self_attn.{field}")
            if v is not None:
                _assign(getattr(layer, field), v, f"{p}self_attn.{field}")
        w, b = get(f"{p}conv.depthwise_conv.weight"), t.get(f"{p}conv.depthwise_conv.bias")
        bn = {f: get(f"{p}conv.batch_norm.{f}") for f in ("weight", "bias", "running_mean", "running_var")}
        if w is not None and all(v is not None for v in bn.values()):
            inv = bn["weight"] / torch.sqrt(bn["running_var"] + BATCH_NORM_EPS)
            bias = b if b is not None else torch.zeros_like(bn["running_mean"])
            _assign(layer.dw_weight, w * inv[:, None, None], f"{p}conv.depthwise_conv.weight")
            _assign(layer.dw_bias, (bias - bn["running_mean"]) * inv + bn["bias"], f"{p}conv.batch_norm")
    for idx in (0, 2, 3, 5, 6):
        for field in ("weight", "bias"):
            v = get(f"encoder.pre_encode.conv.{idx}.{field}")
            if v is not None:
                _assign(getattr(enc.pre.conv[idx], field), v, f"encoder.pre_encode.conv.{idx}.{field}")
    for field in ("weight", "bias"):
        v = get(f"encoder.pre_encode.out.{field}")
        if v is not None:
            _assign(getattr(enc.pre.out, field), v, f"encoder.pre_encode.out.{field}")
    if strict and missing:
        raise ValueError(f"the export lacks {len(missing)} encoder tensors, e.g. {missing[:4]}")
    return enc
