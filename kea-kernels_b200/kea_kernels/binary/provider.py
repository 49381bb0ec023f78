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

import bisect
from typing import NamedTuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn


class LayerRows(NamedTuple):
    """A prepared layer registered in a Table: its rows hold the global row ids first .. first + rows - 1."""
    name: str
    layer: object
    kind: str            # "linear" or "conv"
    first: int
    rows: int            # output features
    cols: int            # input features
    members: tuple = ()  # a fused layer's module names (e.g. Q, K, V)


class Table:
    """Global row ids -> prepared layers. Each added layer takes the next block of ids; a handle's first id is looked
    up by bisection over the blocks' first ids (they are added in increasing order)."""

    def __init__(self):
        self._firsts: list[int] = []
        self._layers: list[LayerRows] = []

    @property
    def entries(self) -> list[LayerRows]:
        return list(self._layers)

    def add(self, name, layer, kind, n, k, members=()) -> LayerRows:
        first = self._firsts[-1] + self._layers[-1].rows if self._layers else 0
        rec = LayerRows(name, layer, kind, first, n, k, tuple(members))
        self._firsts.append(first)
        self._layers.append(rec)
        return rec

    def resolve(self, start: int, count: int) -> tuple[LayerRows, int]:
        """(layer, row offset inside it) of the handle rows start .. start + count - 1, all in one layer."""
        i = bisect.bisect_right(self._firsts, start) - 1
        rec = self._layers[i] if i >= 0 else None
        if rec is None or start >= rec.first + rec.rows:
            raise KeyError(f"no layer owns row handle {start}")
        if start + count > rec.first + rec.rows:
            raise ValueError("handle range crosses layers")
        return rec, start - rec.first

    def weight_bytes(self) -> int:
        return sum(rec.layer.weight_bytes() for rec in self._layers)


def handle(start: int, n: int) -> Tensor:
    """The CPU int64 row handle [1, n] (a module's `packed_t`) of global rows start .. start + n - 1."""
    return torch.arange(start, start + n, dtype=torch.int64)[None, :]


class BinaryLinear(nn.Module):
    """A module standing for rows [offset, offset + n) of a Table entry (a whole layer or a fused member)."""

    def __init__(self, entry: LayerRows, offset: int, n: int, k: int, scale_cpu: Tensor, bias_cpu: Tensor | None):
        super().__init__()
        self.in_features, self.out_features, self.mode = k, n, "binary"
        self._entry, self._offset = entry, offset
        object.__setattr__(self, "packed_t", handle(entry.first + offset, n))
        object.__setattr__(self, "scale", scale_cpu.detach().clone().contiguous())
        object.__setattr__(self, "bias", None if bias_cpu is None else bias_cpu.detach().clone().contiguous())
        self.eval()

    def _run(self, x: Tensor, conv: bool) -> Tensor:
        e = self._entry
        y = e.layer.conv(x) if conv else e.layer.linear(x)
        if self.out_features == e.rows:
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
        self._resolved: dict[tuple, tuple[LayerRows, int, int]] = {}
        self.names = names or {}

    @property
    def bytes(self) -> int:
        return self.table.weight_bytes()

    def _lookup(self, mod) -> tuple[LayerRows, int, int]:
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
        if count != entry.rows:
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
