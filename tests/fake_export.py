"""Structurally valid parakeet-*-v1 export directories at a small, consistent encoder size, for the loader tests.

The 264 quantized layer names of the Parakeet encoder with seeded codes (1-bit signs or ternary fields) and scales,
plus, optionally, the encoder's other tensors under their NeMo names (LayerNorms, relative-position biases,
depthwise conv and its BatchNorm, subsampling). Written with safetensors, a manifest with every file's SHA-256, a
tokenizer file, as the reference's own test fixture does for its loader (tests/conftest.py:31-53).
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import torch

from kea_kernels import formats
from kea_kernels.binary import bits


def projection_shapes(d: int, ff: int) -> dict[str, tuple[int, int, bool]]:
    """Export module suffix -> (N, K, has bias)."""
    return {"feed_forward1.linear1": (ff, d, True), "feed_forward1.linear2": (d, ff, True),
            "feed_forward2.linear1": (ff, d, True), "feed_forward2.linear2": (d, ff, True),
            "self_attn.linear_q": (d, d, False), "self_attn.linear_k": (d, d, False),
            "self_attn.linear_v": (d, d, False), "self_attn.linear_out": (d, d, True),
            "self_attn.linear_pos": (d, d, False), "conv.pointwise_conv1": (2 * d, d, True),
            "conv.pointwise_conv2": (d, d, True)}


def random_codes(kind: str, n: int, k: int, g: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
    """(export codes, dense int8 weights)."""
    if kind == "binary":
        w = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
        return bits.pack_signs(w), w
    u = torch.rand(n, k, generator=g)
    w = torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8)
    return formats.pack_ternary(w), w


def write_export(directory: Path, kind: str, *, d: int = 64, ff: int = 128, heads: int = 2, kernel: int = 9,
                 sub: int = 8, n_mels: int = 64, encoder_tensors: bool = True, extra: dict | None = None,
                 seed: int = 0, tamper=None) -> Path:
    """`tamper(layers, tensors)` may edit the manifest's layer table and the tensors before they are written."""
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    directory.mkdir(parents=True, exist_ok=True)
    layers, tensors = {}, {}
    for i in range(formats.LAYERS):
        for suffix, (n, k, has_bias) in projection_shapes(d, ff).items():
            name = f"encoder.layers.{i}.{suffix}"
            layers[name] = {"kind": "pointwise_conv1d" if "pointwise" in suffix else "linear", "shape": [n, k],
                            "bias": has_bias}
            codes, _ = random_codes(kind, n, k, g)
            tensors[f"{name}.codes"] = codes
            tensors[f"{name}.scale"] = ((torch.rand(n, generator=g) * 0.5 + 0.75) / math.sqrt(k)).float()
            if has_bias:
                tensors[f"{name}.bias"] = (torch.randn(n, generator=g) * 0.02).float()
        if encoder_tensors:
            p = f"encoder.layers.{i}."
            for norm in ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"):
                tensors[f"{p}{norm}.weight"] = (1 + 0.1 * torch.randn(d, generator=g)).half()
                tensors[f"{p}{norm}.bias"] = (0.05 * torch.randn(d, generator=g)).half()
            tensors[f"{p}self_attn.pos_bias_u"] = (0.02 * torch.randn(heads, d // heads, generator=g)).half()
            tensors[f"{p}self_attn.pos_bias_v"] = (0.02 * torch.randn(heads, d // heads, generator=g)).half()
            tensors[f"{p}conv.depthwise_conv.weight"] = (torch.randn(d, 1, kernel, generator=g) / 3).half()
            tensors[f"{p}conv.depthwise_conv.bias"] = (0.02 * torch.randn(d, generator=g)).half()
            tensors[f"{p}conv.batch_norm.weight"] = (1 + 0.1 * torch.randn(d, generator=g)).half()
            tensors[f"{p}conv.batch_norm.bias"] = (0.05 * torch.randn(d, generator=g)).half()
            tensors[f"{p}conv.batch_norm.running_mean"] = (0.1 * torch.randn(d, generator=g)).half()
            tensors[f"{p}conv.batch_norm.running_var"] = (1 + 0.2 * torch.rand(d, generator=g)).half()
    if encoder_tensors:
        f = n_mels
        for _ in range(3):
            f = (f - 1) // 2 + 1
        shapes = {0: (sub, 1, 3, 3), 2: (sub, 1, 3, 3), 3: (sub, sub, 1, 1), 5: (sub, 1, 3, 3), 6: (sub, sub, 1, 1)}
        for idx, shape in shapes.items():
            fan = shape[1] * shape[2] * shape[3]
            tensors[f"encoder.pre_encode.conv.{idx}.weight"] = (torch.randn(*shape, generator=g) / math.sqrt(fan)).half()
            tensors[f"encoder.pre_encode.conv.{idx}.bias"] = (0.01 * torch.randn(sub, generator=g)).half()
        tensors["encoder.pre_encode.out.weight"] = (torch.randn(d, sub * f, generator=g) / math.sqrt(sub * f)).half()
        tensors["encoder.pre_encode.out.bias"] = (0.01 * torch.randn(d, generator=g)).half()
    if tamper is not None:
        tamper(layers, tensors)
    fmt = formats.BINARY_FORMAT if kind == "binary" else formats.TERNARY_FORMAT
    save_file(tensors, str(directory / formats.FILE), metadata={"format": fmt})
    (directory / formats.TOKENIZER_DIR).mkdir(exist_ok=True)
    (directory / formats.TOKENIZER_DIR / "vocab.txt").write_text("a\nb\n")
    files = {rel: formats.sha256_file(directory / rel) for rel in (formats.FILE, "tokenizer/vocab.txt")}
    manifest = {"format": fmt, "file": formats.FILE, "sha256": files[formats.FILE], "files": files,
                "config": {"target": formats.MODEL_TARGET}, "quantized_layers": layers, "extra": extra or {}}
    (directory / formats.MANIFEST).write_text(json.dumps(manifest))
    return directory
