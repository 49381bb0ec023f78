"""The 1-bit layers at the projection-provider seam (src/kea_kernels/binary/provider.py:1-209).

The encoder transforms route every quantized-layer call through one `projection` object, called as

    provider(x, mod, conv=False, components=3, activation="", norm=None, config=None, input_activation="")

with these semantics:
    xx = x.transpose(1, 2) if conv else x           # conv: [B, K, T] -> [B, T, K] view
    z  = LayerNorm(norm)(xx) if norm else xx        # fused input normalization
    z  = z * sigmoid(z) if input_activation == "silu" else z
    y  = alpha * (W z) + bias                       # the quantized layer, [B, T, N]
    y  = y * sigmoid(y) if activation == "silu" else y
    return y.transpose(1, 2) if conv else y          # conv returns a [B, N, T] view
`components` is the number of INT8 residual activation parts (3 unless PartCount overrides it).

A module resolves to its layer through a CPU int64 row handle [1, N] (`packed_t`): global row ids in a Table of
prepared layers, so Q, K and V can be one fused [3072, 1024] layer whose modules are row slices of it. Model
construction from an export (NeMo) is not part of this package.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import Tensor, nn


@dataclass
class Entry:
    """One prepared 1-bit layer and the global handle range of its rows."""
    name: str
    layer: object
    kind: str            # "linear" or "conv"
    out_features: int
    in_features: int
    start: int           # first global row id
    members: tuple = ()  # for a fused entry (e.g. QKV): the module names


@dataclass
class Table:
    entries: list[Entry] = field(default_factory=list)
    next_row: int = 0

    def add(self, name, layer, kind, n, k, members=()) -> Entry:
        entry = Entry(name, layer, kind, n, k, self.next_row, tuple(members))
        self.entries.append(entry)
        self.next_row += n
        return entry

    def resolve(self, start: int, count: int) -> tuple[Entry, int]:
        for entry in self.entries:
            if entry.start <= start < entry.start + entry.out_features:
                if start + count > entry.start + entry.out_features:
                    raise ValueError("handle range crosses layers")
                return entry, start - entry.start
        raise KeyError(f"no layer owns row handle {start}")

    def weight_bytes(self) -> int:
        return sum(e.layer.weight_bytes() for e in self.entries)


def handle(start: int, n: int) -> Tensor:
    """The CPU row handle of rows [start, start + n) of a Table."""
    return torch.arange(start, start + n, dtype=torch.int64).view(1, n)


class BinaryLinear(nn.Module):
    """A module standing for rows [offset, offset + n) of a Table entry (a whole layer or a fused member)."""

    def __init__(self, entry: Entry, offset: int, n: int, k: int, scale_cpu: Tensor, bias_cpu: Tensor | None):
        super().__init__()
        self.in_features, self.out_features, self.mode = k, n, "binary"
        self._entry, self._offset = entry, offset
        object.__setattr__(self, "packed_t", handle(entry.start + offset, n))
        object.__setattr__(self, "scale", scale_cpu.detach().clone().contiguous())
        object.__setattr__(self, "bias", None if bias_cpu is None else bias_cpu.detach().clone().contiguous())
        self.eval()

    def _run(self, x: Tensor, conv: bool) -> Tensor:
        e = self._entry
        y = e.layer.conv(x) if conv else e.layer.linear(x)
        if self.out_features == e.out_features:
            return y
        sl = slice(self._offset, self._offset + self.out_features)
        return y[:, sl] if conv else y[..., sl]

    def forward(self, x: Tensor) -> Tensor:
        return self._run(x, False)


class BinaryPointwiseConv1d(BinaryLinear):
    def forward(self, x: Tensor) -> Tensor:
        return self._run(x, True)


class BinaryProjection:
    """The provider object handed to the encoder transforms (module docstring)."""

    def __init__(self, table: Table, names: dict[int, str] | None = None):
        self.table = table
        self._resolved: dict[tuple, tuple[Entry, int, int]] = {}
        self.names = names or {}

    @property
    def bytes(self) -> int:
        return self.table.weight_bytes()

    def _lookup(self, mod) -> tuple[Entry, int, int]:
        h = mod.packed_t
        key = (h.data_ptr(), tuple(h.shape))
        hit = self._resolved.get(key)
        if hit is None:
            if h.is_cuda or h.dtype != torch.int64 or h.dim() != 2 or h.shape[0] != 1:
                raise TypeError("BinaryProjection serves BinaryLinear / BinaryPointwiseConv1d handles only")
            start, count = int(h[0, 0]), h.shape[1]
            if not torch.equal(h[0], torch.arange(start, start + count)):
                raise ValueError("non-contiguous row handle")
            entry, offset = self.table.resolve(start, count)
            hit = (entry, offset, count)
            self._resolved[key] = hit
        return hit

    def __call__(self, x, mod, conv=False, components=3, activation="", norm=None, config=None, input_activation=""):
        if config is not None:
            raise ValueError("BinaryProjection takes no tile config")
        if activation not in ("", "silu") or input_activation not in ("", "silu"):
            raise ValueError(f"unsupported activation {activation!r} / {input_activation!r}")
        entry, offset, count = self._lookup(mod)
        layer = entry.layer
        if hasattr(layer, "project"):
            y = layer.project(x, conv=conv, components=components, activation=activation, norm=norm,
                              input_activation=input_activation)
        else:
            z = x.transpose(1, 2) if conv else x
            if norm is not None:
                z = F.layer_norm(z, norm.normalized_shape, norm.weight, norm.bias, norm.eps)
            if input_activation == "silu":
                z = F.silu(z)
            y = layer.linear(z)
            if activation == "silu":
                y = F.silu(y)
            if conv:
                y = y.transpose(1, 2)
        if count != entry.out_features:
            y = y[:, offset:offset + count] if conv else y[..., offset:offset + count]
        return y


class PartCount:
    """Wraps a projection provider and sets `components` (the INT8 activation part count) to n on every call;
    attribute writes other than its own (provider, n) reach the wrapped provider, reads fall through to it
    (src/kea_kernels/binary/provider.py:185-209)."""

    OWN = ("provider", "n")

    def __init__(self, provider, n: int):
        if n not in (1, 2, 3):
            raise ValueError("n must be 1, 2 or 3")
        object.__setattr__(self, "provider", provider)
        object.__setattr__(self, "n", n)

    def __setattr__(self, name, value):
        if name in PartCount.OWN:
            object.__setattr__(self, name, value)
        else:
            setattr(self.provider, name, value)

    def __call__(self, x, mod, conv=False, components=3, activation="", norm=None, config=None, input_activation=""):
        return self.provider(x, mod, conv, self.n, activation, norm, config, input_activation)

    def __getattr__(self, name):
        return getattr(self.provider, name)
