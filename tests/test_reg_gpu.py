"""GPU parity of the small-M register-operand kernel (warp-level INT8 MMAs whose weight fragments are expanded from
the panels in registers), called through the C ABI: bit for bit the oracle's accumulators and outputs for every
instantiated warp tile, K-slice count, part count, ragged edge and epilogue, and bitwise equal to the tcgen05
kernels on the same inputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
from kea_kernels import _lib, lowbit
from kea_kernels.binary import configs
from test_gemm_gpu import DEV, _activations, _channel, _check, _codes, _run

pytestmark = pytest.mark.gpu

# (rows, channels, K-slices): every instantiated warp tile (channel groups x row groups = 1x4, 2x4, 2x2, 4x2)
TILES = [(32, 16, 8), (32, 32, 8), (16, 32, 8), (16, 64, 8), (32, 32, 4), (32, 64, 4), (16, 64, 4), (16, 128, 4),
         (32, 64, 2), (32, 128, 2), (16, 128, 2), (32, 128, 1)]


def _reg(rows: int, cn: int, ks: int) -> configs.DotConfig:
    return configs.DotConfig(rows, cn, ks, 0, configs.REG)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [1, 2, 3])
@pytest.mark.parametrize("rows,cn,ks", TILES)
def test_forced_tiles(wbits, parts, rows, cn, ks):
    """Every warp tile and K split gives the oracle's bits, with the rows of a CTA shared among the parts of its
    tokens (rows / parts tokens per CTA, the last CTA's rows past M reading zero)."""
    n, k, m = 384, 1024, 45
    seed = wbits * 101 + parts * 13 + rows + cn + ks
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, config=_reg(rows, cn, ks))
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m,parts", [(5, 300, 3, 2), (200, 21, 7, 1), (130, 4097, 1, 1), (129, 129, 129, 3),
                                         (1, 128, 33, 1), (300, 1000, 250, 1), (4096, 1024, 125, 1),
                                         (1024, 4096, 125, 1), (1000, 40, 17, 2)])
@pytest.mark.parametrize("tile", [(32, 32, 8), (16, 64, 4)])
def test_ragged_edges(wbits, n, k, m, parts, tile):
    """N not a multiple of the CTA's channels, K not a multiple of the 32-wide k-step (the last step's codes past K
    weigh zero), K-slices longer than the k-steps (idle warps), a single token."""
    seed = wbits * 31 + n + k + m + parts + tile[1]
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, config=_reg(*tile))
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("k", [20, 100, 1000])
def test_columns_past_k_are_ignored(wbits, k):
    """Activation bytes between K and the row stride are not zero here: the kernel must weigh them zero (a 1-bit
    zero code expands to -1, so the weights past K are masked, not just the activations)."""
    n, m, parts = 96, 37, 1
    seed = wbits + k
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed, ldq=-(-k // 16) * 16 + 32)
    q[:, :, k:] = 77
    alpha, bias = _channel(n, seed, False)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, config=_reg(32, 32, 8))
    want, want_acc = oracle.reference(np.ascontiguousarray(q[:, :, :k]), qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [1, 2, 3])
@pytest.mark.parametrize("flags", [0, 1, 2, 3])
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_epilogues(wbits, parts, flags, out):
    """SiLU, the other P = 2 contraction order, FP16 output, with and without bias."""
    n, k, m = 256, 512, 29
    seed = wbits * 5 + parts * 7 + flags * 11 + (out == torch.float16)
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, flags < 2)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, out=out, config=_reg(32, 64, 4))
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, flags)
    _check(y, acc, want, want_acc, flags)


@pytest.mark.parametrize("wbits", [1, 2])
def test_residual_in_place(wbits):
    """y = residual + scale * value with y the residual itself (every element read before it is written, by the
    same thread), as the tcgen05 kernels write it."""
    n, k, m, parts = 320, 1024, 40, 1
    codes, w = _codes(wbits, n, k, 3 + wbits)
    q, qs = _activations(parts, m, k, 3 + wbits)
    alpha, bias = _channel(n, 3 + wbits, True)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), wbits, n, k)
    qd, qsd = torch.from_numpy(q).to(DEV), torch.from_numpy(qs).to(DEV)
    ad, bd = torch.from_numpy(alpha).to(DEV), torch.from_numpy(bias).to(DEV)
    res = torch.randn(m, n, generator=torch.Generator().manual_seed(wbits)).to(DEV)
    y_reg = res.clone()
    lowbit.gemm(qd, qsd, k, m, panels, wbits, n, k, ad, bd, y_reg, parts=parts, residual=y_reg, residual_scale=0.5,
                config=_reg(16, 64, 8))
    y_tile = res.clone()
    lowbit.gemm(qd, qsd, k, m, panels, wbits, n, k, ad, bd, y_tile, parts=parts, residual=y_tile, residual_scale=0.5,
                reg=False)
    plain = torch.empty(m, n, device=DEV)
    lowbit.gemm(qd, qsd, k, m, panels, wbits, n, k, ad, bd, plain, parts=parts, config=_reg(16, 64, 8))
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    want, _ = oracle.reference(q, qs, w, alpha, bias)
    assert np.array_equal(plain.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert torch.equal(y_reg.view(torch.int32), (res + 0.5 * plain).view(torch.int32))
    assert torch.equal(y_reg.view(torch.int32), y_tile.view(torch.int32))


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [1, 3])
@pytest.mark.parametrize("n,k,m", [(4096, 1024, 125), (1024, 4096, 125), (1024, 1024, 16), (2048, 1024, 64)])
def test_equals_the_tcgen05_kernels(wbits, parts, n, k, m):
    """At the Parakeet shapes the register kernel and the tcgen05 kernels give the same bits, with programmatic
    dependent launch on."""
    seed = wbits + parts + n + k + m
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    y_reg, acc_reg = _run(codes, wbits, n, k, q, qs, alpha, bias, config=_reg(32, 64, 4), pdl=True)
    y_tc, acc_tc = _run(codes, wbits, n, k, q, qs, alpha, bias, config=None, reg=False)
    assert np.array_equal(acc_reg, acc_tc)
    assert torch.equal(y_reg.view(torch.int32), y_tc.view(torch.int32))


def test_forced_config_errors():
    """Tiles the kernel does not have are refused before launch."""
    n, k, m, wbits = 128, 256, 8, 1
    codes, _ = _codes(wbits, n, k, 1)
    q, qs = _activations(1, m, k, 1)
    alpha, _ = _channel(n, 1, False)
    for bad in [(32, 48, 8), (24, 32, 8), (32, 32, 3), (32, 256, 8), (16, 16, 8), (32, 64, 8), (16, 128, 8)]:
        with pytest.raises((ValueError, RuntimeError)):
            _run(codes, wbits, n, k, q, qs, alpha, None, config=_reg(*bad))
    # more token tiles than a grid's y dimension holds (65535 x 16 tokens)
    m = 65535 * 16 + 1
    qd = torch.zeros(1, m, k, dtype=torch.int8, device=DEV)
    qsd = torch.ones(1, m, device=DEV)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), wbits, n, k)
    y = torch.empty(m, n, device=DEV)
    with pytest.raises((ValueError, RuntimeError)):
        lowbit.gemm(qd, qsd, k, m, panels, wbits, n, k, torch.from_numpy(alpha).to(DEV), None, y, parts=1,
                    config=_reg(16, 32, 8))
    assert _lib.read_device_error() == 0
