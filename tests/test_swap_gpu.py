"""GPU parity of the small-M swapped-operand kernel (weights on the tcgen05 M axis, every part's tokens on N),
called through the C ABI: bit for bit the oracle's accumulators and outputs for every split, pipeline depth, part
count, token tiling, ragged edge and epilogue, bitwise equal to the 128-token-tile kernel, and its bounded waits."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
from kea_kernels import _lib, lowbit
from kea_kernels.binary import configs
from test_gemm_gpu import DEV, _activations, _channel, _check, _codes, _run

pytestmark = pytest.mark.gpu


def _swap(splits: int, stages: int) -> configs.DotConfig:
    return configs.DotConfig(0, 128, splits, stages, configs.SWAP)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [1, 2, 3])
@pytest.mark.parametrize("splits,stages", [(1, 1), (1, 3), (1, 5), (2, 2), (3, 1), (4, 2), (8, 1), (16, 1), (5, 3)])
def test_forced_splits_and_stages(wbits, parts, splits, stages):
    """Every split of K over the cluster (ranks own round-robin units) and every pipeline depth (a ring of stages
    refilled after the MMAs free them, or every k-block resident at once) gives the oracle's bits."""
    n, k, m = 640, 2048, 45
    seed = wbits * 101 + parts * 13 + splits * 7 + stages
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, config=_swap(splits, stages))
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts,m,splits", [(1, 256, 2), (1, 600, 1), (2, 256, 1), (2, 300, 1), (3, 200, 1),
                                            (3, 368, 2), (1, 17, 4), (3, 1, 2), (2, 128, 2)])
@pytest.mark.parametrize("flags", [0, 2])
def test_token_tiles(wbits, parts, m, splits, flags):
    """Tokens beyond one tile (256 tokens, or 512 / P TMEM columns) are cut into equal tiles of a multiple of 16;
    the MMA's N splits in two above 256 stacked rows; a split-K receive buffer too large to sit beside the stages
    reuses their area (3 parts x 128 tokens over 2 ranks)."""
    n, k = 512, 1024
    seed = wbits * 3 + parts * 5 + m + flags
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, flags == 0)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, config=_swap(splits, 2))
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, flags)
    _check(y, acc, want, want_acc, flags)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts,m", [(1, 125), (3, 38), (2, 64)])
@pytest.mark.parametrize("tile,splits", [(16, 1), (16, 4), (32, 2), (48, 1)])
def test_forced_token_tiles(wbits, parts, m, tile, splits):
    """A caller's token tile (a multiple of 16; the last tile ragged) with or without a K split gives the oracle's
    bits: the grid's token-tile axis, out-of-range rows of the last tile read as zero and clipped on store."""
    n, k = 384, 1024
    seed = wbits * 7 + parts * 11 + m + tile + splits
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias,
                  config=configs.DotConfig(tile, 128, splits, 0, configs.SWAP))
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m,parts", [(5, 300, 3, 2), (200, 21, 7, 1), (130, 4097, 1, 1), (129, 129, 129, 3),
                                         (1, 128, 33, 1), (300, 1000, 250, 1), (4096, 1024, 125, 1)])
@pytest.mark.parametrize("splits", [1, 3])
def test_ragged_edges(wbits, n, k, m, parts, splits):
    """N not a multiple of 128, K not a multiple of 128 (activation boxes per part with columns past K read as
    zero), a single token, splits that do not divide the k-blocks."""
    splits = min(splits, -(-k // 128))
    seed = wbits + n + k + m + parts + splits
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    for out in (torch.float32, torch.float16):
        y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, out=out, config=_swap(splits, 1))
        want, want_acc = oracle.reference(q, qs, w, alpha, bias)
        _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m,parts", [(4096, 1024, 125, 1), (1024, 4096, 125, 1), (3072, 1024, 16, 1),
                                         (1024, 1024, 38, 3), (4096, 1024, 126, 3), (1024, 4096, 200, 2),
                                         (4096, 1024, 256, 3), (1024, 4096, 368, 3)])
@pytest.mark.parametrize("flags", [0, 1, 2])
def test_equals_per_tile_kernel_bitwise(wbits, n, k, m, parts, flags):
    """The swap kernel (its table split) and the 128-token-tile kernel give the same bits, SiLU included (the same
    epilogue arithmetic)."""
    seed = wbits * 11 + n + k + m + parts + flags
    codes, _ = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    y0, acc0 = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, config=_swap(0, 0))
    y1, acc1 = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, swap=False)
    assert np.array_equal(acc0, acc1)
    assert np.array_equal(y0.numpy().view(np.uint32), y1.numpy().view(np.uint32))


def test_pdl_chain_matches():
    """Back-to-back swap launches with programmatic dependent launch (codes fetched and expanded before the wait for
    the previous kernel): every launch gives the first launch's bits."""
    n, k, m = 4096, 1024, 125
    codes, w = _codes(1, n, k, 61)
    q, qs = _activations(1, m, k, 62)
    alpha, _ = _channel(n, 63, False)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), 1, n, k)
    qd, qsd, ad = (torch.from_numpy(v).to(DEV) for v in (q, qs, alpha))
    outs = []
    for _ in range(4):
        y = torch.empty(m, n, device=DEV, dtype=torch.float16)
        acc = torch.empty(1, m, n, device=DEV, dtype=torch.int32)
        lowbit.gemm(qd, qsd, q.shape[2], m, panels, 1, n, k, ad, None, y, parts=1, acc=acc, pdl=True)
        outs.append((y, acc))
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    want, want_acc = oracle.reference(q, qs, w, alpha)
    for y, acc in outs:
        _check(y.cpu(), acc.cpu().numpy(), want, want_acc, 0)


def test_bounded_wait_expires_and_the_context_stays_usable():
    """A wait that nothing will satisfy (the test hook withholds every activation copy) runs out after wait_clocks,
    the kernel reports KEA_DEVERR_TIMEOUT and returns; the host raises RuntimeError; the next GEMM is exact."""
    n, k, m = 1024, 1024, 64
    codes, w = _codes(1, n, k, 71)
    q, qs = _activations(1, m, k, 72)
    alpha, _ = _channel(n, 73, False)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), 1, n, k)
    qd, qsd, ad = (torch.from_numpy(v).to(DEV) for v in (q, qs, alpha))
    y = torch.empty(m, n, device=DEV)
    word = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert _lib.read_device_error() == 0
    lowbit.gemm(qd, qsd, q.shape[2], m, panels, 1, n, k, ad, None, y, parts=1, config=_swap(2, 1),
                error_word=word, wait_clocks=200_000, test_stall=True)
    torch.cuda.synchronize()
    bits = int(word.item())
    assert bits == _lib.DEVERR_TIMEOUT
    with pytest.raises(RuntimeError, match="timed out"):
        _lib.raise_device_errors(bits)
    # the library's own word (no caller word) takes the same report
    lowbit.gemm(qd, qsd, q.shape[2], m, panels, 1, n, k, ad, None, y, parts=1, config=_swap(1, 1),
                wait_clocks=200_000, test_stall=True)
    with pytest.raises(RuntimeError, match="timed out"):
        _lib.raise_device_errors()
    _lib.raise_device_errors()   # read and cleared
    y, acc = _run(codes, 1, n, k, q, qs, alpha, None)
    want, want_acc = oracle.reference(q, qs, w, alpha)
    _check(y, acc, want, want_acc, 0)


def test_stall_hook_needs_the_forced_swap_kernel():
    n, k, m = 256, 256, 8
    codes, _ = _codes(1, n, k, 81)
    q, qs = _activations(1, m, k, 82)
    alpha, _ = _channel(n, 83, False)
    with pytest.raises(ValueError, match="invalid"):
        panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), 1, n, k)
        lowbit.gemm(torch.from_numpy(q).to(DEV), torch.from_numpy(qs).to(DEV), q.shape[2], m, panels, 1, n, k,
                    torch.from_numpy(alpha).to(DEV), None, torch.empty(m, n, device=DEV), parts=1, test_stall=True)
