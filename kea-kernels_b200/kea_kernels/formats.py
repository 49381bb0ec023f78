"""Export formats the kernels read: the 2-bit ternary codes and the constants of the two export kinds.

  * parakeet-binary-v1 (Kea-B): `<name>.codes` uint8 [N, ceil(K/8)], 1 bit per weight (see binary.bits) plus
    `<name>.scale` FP32 [N];
  * parakeet-ternary-v1 (Kea-T): `<name>.codes` uint8 [N, ceil(K/4)], 2 bits per weight: 00 = 0, 01 = +1, 10 = -1,
    code k at bits 2 * (k % 4) of byte k // 4; the pattern 11 is invalid; plus `<name>.scale` FP32 [N].
Both layouts are kea-kernels' (src/kea_kernels/formats.py:1-16,62-81) and are read unchanged.

An export directory holds `export.safetensors` (the codes and scales above; every other tensor FP16, the feature
window and filterbank FP32), `manifest.json` (format, SHA-256 of every file, the model config, the 264 quantized
layers with kind / shape / bias) and `tokenizer/`. A downloaded Kea-B 0.1 directory is an 8-bit bundle whose
`compat/` directory is a parakeet-binary-v1 export of the same weights. `describe` says which model a directory
holds and `check_export` validates one without loading its tensors, as the reference does
(src/kea_kernels/formats.py:95-172); loading onto the GPU is kea_kernels.export.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import math
import re
from pathlib import Path

import torch
from torch import Tensor

BINARY_FORMAT = "parakeet-binary-v1"
TERNARY_FORMAT = "parakeet-ternary-v1"
BUNDLE_FORMAT = "keab-8bit-v1"
FILE = "export.safetensors"
MANIFEST = "manifest.json"
COMPAT_DIR = "compat"
TOKENIZER_DIR = "tokenizer"
MODEL_TARGET = "nemo.collections.asr.models.rnnt_bpe_models.EncDecRNNTBPEModel"

LAYERS = 24
PER_LAYER = ("feed_forward1.linear1", "feed_forward1.linear2", "feed_forward2.linear1", "feed_forward2.linear2",
             "self_attn.linear_q", "self_attn.linear_k", "self_attn.linear_v", "self_attn.linear_out",
             "self_attn.linear_pos", "conv.pointwise_conv1", "conv.pointwise_conv2")
EXPECTED_MODULES = LAYERS * len(PER_LAYER)
# the quantized module names of an export: encoder.layers.<i>.<one of PER_LAYER>
QUANTIZED_NAME = re.compile(r"encoder\.layers\.(\d+)\.(" + "|".join(re.escape(p) for p in PER_LAYER) + r")")
LAYER_KINDS = ("linear", "pointwise_conv1d")

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


# ---- export directories ------------------------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class ModelDir:
    """What a downloaded directory holds: model name, export kind, the export directory and its default mode."""
    model: str          # "kea-b-0.1", "kea-b" or "kea-t"
    kind: str           # "binary" or "ternary"
    export_dir: Path
    default_mode: str   # "x1", "x2", ...


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def read_manifest(directory) -> dict:
    path = Path(directory) / MANIFEST
    if not path.is_file():
        raise ValueError(f"{directory}: no {MANIFEST} (expected a downloaded Kea-B or Kea-T model directory)")
    try:
        return json.loads(path.read_text())
    except json.JSONDecodeError as e:
        raise ValueError(f"{path}: not JSON ({e})") from None


def describe(directory) -> ModelDir:
    """Which model `directory` holds: a Kea-B 0.1 bundle (its compat/ binary export, measured in x1), a Kea-B
    binary export (x2) or a Kea-T ternary export (x2). ValueError for anything else."""
    directory = Path(directory).expanduser().resolve()
    manifest = read_manifest(directory)
    fmt = manifest.get("format")
    if fmt == BUNDLE_FORMAT:
        compat = directory / COMPAT_DIR
        if not (compat / MANIFEST).is_file():
            raise ValueError(f"{directory}: a {BUNDLE_FORMAT} bundle without its {COMPAT_DIR}/ export")
        inner = describe(compat)
        if inner.kind != "binary":
            raise ValueError(f"{compat}: expected a {BINARY_FORMAT} export")
        recorded = ((read_manifest(compat).get("extra") or {}).get("keab") or {}).get("bundle_sha256")
        if recorded != manifest.get("sha256"):
            raise ValueError(f"{compat}: its manifest does not record this directory's bundle")
        return inner
    if fmt == BINARY_FORMAT:
        if (manifest.get("extra") or {}).get("keab"):
            return ModelDir("kea-b-0.1", "binary", directory, "x1")
        return ModelDir("kea-b", "binary", directory, "x2")
    if fmt == TERNARY_FORMAT:
        return ModelDir("kea-t", "ternary", directory, "x2")
    raise ValueError(f"{directory}: unsupported format {fmt!r} (expected {BINARY_FORMAT}, {TERNARY_FORMAT} or "
                     f"{BUNDLE_FORMAT})")


def check_export(directory, kind: str, *, verify_hashes: bool = True) -> dict:
    """The manifest of an intact `kind` ("binary" / "ternary") export, checked without loading its tensors: the
    format (manifest and safetensors metadata), the SHA-256 of every listed file, the model target, the 264
    quantized layer names and kinds, and each layer's codes / scale dtype and shape and bias presence.
    ValueError otherwise."""
    from safetensors import safe_open
    if kind not in ("binary", "ternary"):
        raise ValueError(f"unknown export kind {kind!r}")
    directory = Path(directory)
    manifest = read_manifest(directory)
    fmt = BINARY_FORMAT if kind == "binary" else TERNARY_FORMAT
    if manifest.get("format") != fmt:
        raise ValueError(f"{directory}: export format {manifest.get('format')!r}, expected {fmt!r}")
    files = manifest.get("files") or {}
    if manifest.get("file") != FILE or FILE not in files:
        raise ValueError(f"{directory}: the manifest does not list {FILE}")
    if verify_hashes:
        for rel, digest in files.items():
            path = directory / rel
            if not path.is_file() or sha256_file(path) != digest:
                raise ValueError(f"{path} does not match the manifest SHA-256")
    if (manifest.get("config") or {}).get("target") != MODEL_TARGET:
        raise ValueError(f"{directory}: unexpected model target {(manifest.get('config') or {}).get('target')!r}")
    layers = manifest.get("quantized_layers") or {}
    if len(layers) != EXPECTED_MODULES or not all(QUANTIZED_NAME.fullmatch(n) for n in layers):
        raise ValueError(f"{directory}: expected the {EXPECTED_MODULES} Parakeet quantized layers, got {len(layers)}")
    wbits = 1 if kind == "binary" else 2
    with safe_open(str(directory / FILE), framework="pt") as f:
        if (f.metadata() or {}).get("format") != fmt:
            raise ValueError(f"{directory}: the safetensors metadata format is not {fmt!r}")
        keys = set(f.keys())
        for name, info in layers.items():
            if info.get("kind") not in LAYER_KINDS:
                raise ValueError(f"{name}: unknown kind {info.get('kind')!r}")
            n, k = info["shape"]
            if f"{name}.weight" in keys:
                raise ValueError(f"{name}: dense weight present in a quantized export")
            if f"{name}.codes" not in keys or f"{name}.scale" not in keys:
                raise ValueError(f"{name}: codes or scale missing")
            codes, scale = f.get_slice(f"{name}.codes"), f.get_slice(f"{name}.scale")
            if codes.get_dtype() != "U8" or list(codes.get_shape()) != [n, packed_row_bytes(k, wbits)]:
                raise ValueError(f"{name}: codes must be uint8 [{n}, {packed_row_bytes(k, wbits)}]")
            if scale.get_dtype() != "F32" or list(scale.get_shape()) != [n]:
                raise ValueError(f"{name}: scale must be FP32 [{n}]")
            if bool(info.get("bias")) != (f"{name}.bias" in keys):
                raise ValueError(f"{name}: bias presence differs from the manifest")
    return manifest
