"""GPU parity: the sm_100a library (called through its C ABI) against the CPU oracle and the reference's fixtures.

Bar: INT32 accumulators bit-exact; FP32 outputs bit-exact without SiLU (every epilogue operation is one IEEE
rounding on both sides); FP16 outputs bit-exact without SiLU (round-to-nearest-even of the same FP32 value); with
SiLU (hardware ex2.approx / div.full on the GPU) FP32 within rtol 2e-6 / atol 1e-6 - the reference's own GPU-test
tolerance (tests/test_kernels_gpu.py:44) - and FP16 within 1e-3 relative.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
from conftest import golden_cases
from kea_kernels import _lib, formats, lowbit
from kea_kernels.binary import bits, configs
from kea_kernels.binary import layer as L
from kea_kernels.binary import layer_parts
from kea_kernels.ternary.runtime import PackedLinear, PackedPointwiseConv1d

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _codes(wbits: int, n: int, k: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """(export codes, dense int8 weights) drawn like the reference's tests / BASELINE configs 0-1."""
    g = torch.Generator().manual_seed(seed)
    if wbits == 1:
        w = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
        return bits.pack_signs(w).numpy(), w.numpy()
    u = torch.rand(n, k, generator=g)
    w = torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8)
    return formats.pack_ternary(w).numpy(), w.numpy()


def _activations(parts: int, m: int, k: int, seed: int, ldq: int | None = None):
    g = torch.Generator().manual_seed(seed + 17)
    ldq = -(-k // 16) * 16 if ldq is None else ldq
    q = torch.zeros(parts, m, ldq, dtype=torch.int8)
    q[:, :, :k] = torch.randint(-127, 128, (parts, m, k), generator=g, dtype=torch.int8)
    qs = (torch.rand(parts, m, generator=g) * 0.015 + 0.005).float()
    return q.numpy(), qs.numpy()


def _channel(n: int, seed: int, bias: bool):
    g = torch.Generator().manual_seed(seed + 29)
    alpha = (torch.rand(n, generator=g) * 0.04 + 0.01).half().float().numpy()
    b = (torch.randn(n, generator=g) * 0.1).float().numpy() if bias else None
    return alpha, b


def _run(codes, wbits, n, k, q, qs, alpha, bias, *, flags=0, out=torch.float32, config=None, pdl=False, pair=True,
         pair_only=False, swap=True, reg=False):
    parts, m, ldq = q.shape
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), wbits, n, k)
    qd, qsd = torch.from_numpy(q).to(DEV), torch.from_numpy(qs).to(DEV)
    ad = torch.from_numpy(alpha).to(DEV)
    bd = None if bias is None else torch.from_numpy(bias).to(DEV)
    y = torch.full((m, n), float("nan"), device=DEV, dtype=out)
    acc = torch.full((parts, m, n), -7, device=DEV, dtype=torch.int32)
    lowbit.gemm(qd, qsd, ldq, m, panels, wbits, n, k, ad, bd, y, parts=parts, silu=bool(flags & 1),
                order=(flags >> 1) & 1, acc=acc, config=config, pdl=pdl, pair=pair, force_pair=pair_only, swap=swap,
                reg=reg)
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    return y.cpu(), acc.cpu().numpy()


def _check(y, acc, want_y, want_acc, flags):
    assert np.array_equal(acc, want_acc), f"{(acc != want_acc).sum()} accumulators differ"
    if y.dtype == torch.float16:
        want16 = oracle.to_f16(want_y)
        if flags & 1:
            np.testing.assert_allclose(y.float().numpy(), want16.astype(np.float32), rtol=1e-3, atol=1e-5)
        else:
            assert np.array_equal(y.numpy().view(np.uint16), want16.view(np.uint16))
    else:
        if flags & 1:
            np.testing.assert_allclose(y.numpy(), want_y, rtol=2e-6, atol=1e-6)
        else:
            assert np.array_equal(y.numpy().view(np.uint32), want_y.view(np.uint32)), \
                f"{(y.numpy() != want_y).sum()} outputs differ"


# ---- panels ---------------------------------------------------------------------------------------------------

@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k", [(4096, 1024), (1024, 4096), (5, 300), (200, 21), (130, 136)])
def test_device_panels_equal_the_oracle_layout(wbits, n, k):
    codes, _ = _codes(wbits, n, k, seed=n + k)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), wbits, n, k)
    assert panels.numel() == _lib.panel_bytes(wbits, n, k)
    assert np.array_equal(panels.cpu().numpy(), oracle.panels(codes, wbits, n, k))


def test_device_prepare_rejects_invalid_codes():
    bad = torch.zeros(2, 2, dtype=torch.uint8)
    bad[0, 1] = 0x80  # bit 15 set for K = 12
    with pytest.raises(ValueError, match="tail"):
        lowbit.prepare_panels(bad.to(DEV), 1, 2, 12)
    t = torch.zeros(3, 1, dtype=torch.uint8)
    t[1, 0] = 0b11 << 2
    with pytest.raises(ValueError):
        lowbit.prepare_panels(t.to(DEV), 2, 3, 4)
    with pytest.raises(ValueError, match="tail"):
        L.Int8MmaLayer.prepare(bad, torch.ones(2), None, 12, DEV)


# ---- the reference's fixtures ------------------------------------------------------------------------------------

@pytest.mark.parametrize("index", range(8))
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_gemm_equals_golden_fixtures(golden, index, out):
    case = golden_cases(golden)[index]
    k, n = case["k"], case["n"]
    ldq = -(-k // 16) * 16
    q = np.zeros((case["parts"], case["m"], ldq), dtype=np.int8)
    q[:, :, :k] = case["q"]
    y, acc = _run(case["codes"], case["wbits"], n, k, q, case["qs"], case["alpha"], case["bias"], out=out)
    assert np.array_equal(acc, case["acc"])                       # the reference's int64 accumulators
    w = oracle.unpack(case["codes"], case["wbits"], k)
    want, _ = oracle.reference(q, case["qs"], w, case["alpha"], case["bias"])
    _check(y, acc, want, case["acc"], 0)
    if out == torch.float32:                                      # the reference test's own tolerance vs FP64
        np.testing.assert_allclose(y.double().numpy(), case["y64"], rtol=2e-6, atol=1e-6)


# ---- shape sweep (config-1 M sweep and the Parakeet encoder shapes) ----------------------------------------------

SHAPES = [(4096, 1024), (1024, 4096), (3072, 1024), (2048, 1024), (1024, 1024)]


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 16, 38, 125, 300, 512])
def test_gemm_x1_fp16_sweep(wbits, n, k, m):
    seed = wbits * 7919 + n + k + m
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(1, m, k, seed)
    alpha, _ = _channel(n, seed, False)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, None, out=torch.float16)
    want, want_acc = oracle.reference(q, qs, w, alpha)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [2, 3])
@pytest.mark.parametrize("n,k,m", [(4096, 1024, 125), (1024, 4096, 38), (3072, 1024, 300), (2048, 1024, 77)])
@pytest.mark.parametrize("flags", [0, 2])
def test_gemm_parts_and_order(wbits, parts, n, k, m, flags):
    seed = wbits * 131 + parts * 17 + n + k + m + flags
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, flags)
    _check(y, acc, want, want_acc, flags)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [2, 3])
@pytest.mark.parametrize("n,k,m", [(1024, 1024, 38), (4096, 1024, 40), (3072, 1024, 17), (2048, 1024, 64),
                                   (1024, 4096, 1), (1024, 1024, 5), (512, 256, 33), (1024, 1024, 126),
                                   (4096, 1024, 368), (1024, 4096, 257), (640, 512, 511)])
@pytest.mark.parametrize("flags", [0, 2, 1])
@pytest.mark.parametrize("swap", [True, False])
def test_stacked_parts_small_m(wbits, parts, n, k, m, flags, swap):
    """M <= 512 with 2 or 3 parts, both small-M kernels: the swap kernel stacks the parts along the MMA's N (token)
    axis; the 128-token-tile kernel (swap=False) cuts the tokens into tiles of mp tokens whose parts are stacked along
    one 128-row tile, with and without split-K. Bit for bit the oracle's results."""
    seed = wbits * 31 + parts * 7 + n + k + m + flags
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, flags != 2)
    out = torch.float16 if flags == 2 else torch.float32
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, out=out, swap=swap)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, flags)
    _check(y, acc, want, want_acc, flags)


def _gemv_fits(rows: int, ch: int = 8) -> bool:
    """The CUDA-core kernel's slice sums ([8 warps][rows][channels] INT32) fit its 48 KB of shared memory."""
    return 8 * rows * ch * 4 <= 48 * 1024


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [1, 2, 3])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 13, 16])
@pytest.mark.parametrize("n,k,flags", [(4096, 1024, 0), (1024, 4096, 2), (3072, 1024, 1), (200, 300, 0),
                                       (1000, 21, 2), (130, 4097, 1), (8, 129, 0)])
def test_gemv_small_m_equals_oracle(wbits, parts, m, n, k, flags):
    """The CUDA-core kernel (dp4a over expanded codes), forced for every M <= 16 (the table takes it up to 4
    activation rows = tokens x parts): bit for bit the oracle's results, for every token-count bucket (1, <= 4,
    <= 16), part count, epilogue and ragged K / N."""
    rows, fits = m * parts, _gemv_fits(m * parts)
    assert (configs.choose(m, n, k, wbits, parts).kernel == configs.GEMV) == (rows <= 4 and fits)
    seed = wbits * 53 + parts * 11 + m + n + k + flags
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, flags != 2)
    out = torch.float16 if flags == 2 else torch.float32
    config = configs.DotConfig(m, 8, 1, 1, configs.GEMV)
    if not fits:
        with pytest.raises(ValueError, match="unsupported"):
            _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, out=out, config=config)
        return
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, out=out, config=config)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, flags)
    _check(y, acc, want, want_acc, flags)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [1, 3])
@pytest.mark.parametrize("flags", [0, 1, 2])
def test_gemv_equals_tensor_core_kernel_bitwise(wbits, parts, flags):
    """The CUDA-core and tensor-core kernels give the same bits, SiLU included (same epilogue code)."""
    n, k, m = 2048, 1024, 7
    codes, _ = _codes(wbits, n, k, 77 + flags)
    q, qs = _activations(parts, m, k, 78)
    alpha, bias = _channel(n, 79, True)
    y0, acc0 = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags)
    y1, acc1 = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, config=configs.DotConfig(128, 64, 2, 4))
    assert np.array_equal(acc0, acc1)
    assert np.array_equal(y0.numpy().view(np.uint32), y1.numpy().view(np.uint32))
    for ch in (8, 16, 32):   # every forced channels-per-CTA width of the CUDA-core kernel
        y2, acc2 = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags,
                        config=configs.DotConfig(m, ch, 1, 1, configs.GEMV))
        assert np.array_equal(acc0, acc2)
        assert np.array_equal(y0.numpy().view(np.uint32), y2.numpy().view(np.uint32))


def test_forced_gemv_config_is_refused_above_16_tokens():
    codes, _ = _codes(1, 512, 1024, 3)
    q, qs = _activations(1, 17, 1024, 3)
    alpha, _ = _channel(512, 3, False)
    with pytest.raises(ValueError, match="unsupported"):
        _run(codes, 1, 512, 1024, q, qs, alpha, None, config=configs.DotConfig(16, 32, 1, 1, configs.GEMV))
    q, qs = _activations(1, 16, 1024, 3)
    with pytest.raises(ValueError, match="unsupported"):        # channels per CTA: 8, 16 or 32
        _run(codes, 1, 512, 1024, q, qs, alpha, None, config=configs.DotConfig(16, 64, 1, 1, configs.GEMV))


def test_gemv_pdl_chain_matches():
    """Back-to-back CUDA-core launches with programmatic dependent launch: the second reads the first's output."""
    n, k, m = 1024, 1024, 4
    codes, w = _codes(1, n, k, 91)
    q, qs = _activations(1, m, k, 92)
    alpha, _ = _channel(n, 93, False)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), 1, n, k)
    qd, qsd, ad = (torch.from_numpy(v).to(DEV) for v in (q, qs, alpha))
    ref = None
    for pdl in (False, True):
        outs = []
        for _ in range(3):
            y = torch.empty(m, n, device=DEV)
            acc = torch.empty(1, m, n, device=DEV, dtype=torch.int32)
            lowbit.gemm(qd, qsd, q.shape[2], m, panels, 1, n, k, ad, None, y, parts=1, acc=acc, pdl=pdl)
            outs.append((y, acc))
        torch.cuda.synchronize()
        got = [(y.cpu().numpy(), a.cpu().numpy()) for y, a in outs]
        ref = ref or got[0]
        for y, a in got:
            assert np.array_equal(a, ref[1]) and np.array_equal(y.view(np.uint32), ref[0].view(np.uint32))
    want, want_acc = oracle.reference(q, qs, w, alpha)
    _check(torch.from_numpy(ref[0]), ref[1], want, want_acc, 0)


@pytest.mark.parametrize("config", [(128, 32, 1, 8), (128, 64, 2, 4), (128, 128, 4, 2), (128, 32, 4, 2),
                                    (128, 256, 8, 1), (128, 64, 1, 1)])
@pytest.mark.parametrize("parts", [2, 3])
def test_stacked_parts_forced_configs(config, parts):
    n, k, m = 512, 2048, 38
    codes, w = _codes(1, n, k, 13)
    q, qs = _activations(parts, m, k, 13)
    alpha, bias = _channel(n, 13, True)
    y, acc = _run(codes, 1, n, k, q, qs, alpha, bias, config=configs.DotConfig(*config))
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("out", [torch.float32, torch.float16])
@pytest.mark.parametrize("parts", [1, 3])
def test_gemm_silu_epilogue(out, parts):
    n, k, m = 1024, 1024, 125
    codes, w = _codes(1, n, k, 5)
    q, qs = _activations(parts, m, k, 5)
    alpha, bias = _channel(n, 5, True)
    y, acc = _run(codes, 1, n, k, q, qs, alpha, bias, flags=1, out=out)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, 1)
    _check(y, acc, want, want_acc, 1)


@pytest.mark.parametrize("config", [(128, 128, 1, 1), (128, 128, 2, 2), (128, 128, 4, 1), (128, 128, 8, 1),
                                    (128, 128, 1, 4), (256, 128, 1, 2), (128, 128, 16, 1), (128, 128, 3, 2),
                                    (256, 256, 1, 3), (256, 128, 2, 2), (128, 256, 5, 3), (128, 256, 1, 3),
                                    (256, 256, 1, 1), (128, 128, 1, 6), (128, 32, 1, 4), (128, 64, 2, 3),
                                    (256, 32, 4, 2), (128, 32, 16, 1), (256, 64, 1, 4)])
@pytest.mark.parametrize("wbits", [1, 2])
def test_forced_tile_configs(config, wbits):
    """Every token / channel tile, cluster split and pipeline depth gives the same bits."""
    n, k, m = 512, 2048, 300
    codes, w = _codes(wbits, n, k, 11)
    q, qs = _activations(1, m, k, 11)
    alpha, _ = _channel(n, 11, False)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, None, config=configs.DotConfig(*config))
    want, want_acc = oracle.reference(q, qs, w, alpha)
    _check(y, acc, want, want_acc, 0)


def test_oversized_config_is_refused():
    codes, _ = _codes(1, 512, 2048, 11)
    q, qs = _activations(1, 200, 2048, 11)
    alpha, _ = _channel(512, 11, False)
    with pytest.raises(ValueError, match="unsupported"):
        _run(codes, 1, 512, 2048, q, qs, alpha, None, config=configs.DotConfig(256, 256, 1, 8))   # > smem
    codes384, _ = _codes(1, 384, 2048, 12)
    with pytest.raises(ValueError, match="unsupported"):        # 256-channel tiles need an even tile count
        _run(codes384, 1, 384, 2048, q, qs, alpha[:384], None, config=configs.DotConfig(128, 256, 1, 2))
    with pytest.raises(ValueError, match="unsupported"):        # the split-K exchange would not fit
        _run(codes, 1, 512, 2048, q, qs, alpha, None, config=configs.DotConfig(256, 256, 2, 1))


@pytest.mark.parametrize("n,k,m", [(5, 300, 3), (200, 21, 7), (130, 4097, 1), (1, 128, 257), (129, 129, 129)])
@pytest.mark.parametrize("wbits", [1, 2])
def test_ragged_edges(n, k, m, wbits):
    codes, w = _codes(wbits, n, k, n * k + m)
    q, qs = _activations(2, m, k, n + m)
    alpha, bias = _channel(n, k, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


def test_zero_rows_is_a_no_op():
    layer = L.Int8MmaLayer.prepare(*_binary_layer(256, 128), None, 128, DEV)
    y = torch.full((4, 256), 3.0, device=DEV)
    q = torch.zeros(3, 4, 128, dtype=torch.int8, device=DEV)
    qs = torch.ones(3, 4, device=DEV)
    layer.dot(q, qs, 128, 0, y)
    torch.cuda.synchronize()
    assert bool((y == 3.0).all())


@pytest.mark.parametrize("wbits", [1, 2])
def test_full_size_m8192_rows_sampled(wbits):
    """Config-1's largest M at full size: the accumulators of 96 sampled rows and a checksum of every row."""
    n, k, m = 4096, 1024, 8192
    codes, w = _codes(wbits, n, k, 8192 + wbits)
    q, qs = _activations(1, m, k, 99)
    alpha, _ = _channel(n, 3, False)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, None, out=torch.float16)
    rows = np.random.default_rng(0).choice(m, size=96, replace=False)
    want, want_acc = oracle.reference(q[:, rows], qs[:, rows], w, alpha)
    _check(y[rows], acc[:, rows], want, want_acc, 0)
    # checksum of checksums: sum_n acc[m, n] = q[m] . (sum_n w[n]) exactly, for every row
    colsum = w.astype(np.int64).sum(axis=0)
    assert np.array_equal(acc[0].astype(np.int64).sum(axis=1), q[0, :, :k].astype(np.int64) @ colsum)


# ---- the persistent CTA-pair kernel (large M) ---------------------------------------------------------------------

PAIR_SHAPES = [(256, 128, 257), (512, 2048, 300), (768, 136, 513), (256, 200, 700), (1024, 4096, 1100),
               (4096, 1024, 2048), (2048, 1024, 611)]


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m", PAIR_SHAPES)
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_pair_kernel_equals_oracle(wbits, n, k, m, out):
    """Ragged K (zero-filled boxes), ragged M (clipped stores), one to several tiles per pair of SMs."""
    assert configs.choose(m, n, k, wbits, 1).kernel == configs.PAIR
    seed = wbits * 977 + n + k + m
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(1, m, k, seed)
    alpha, bias = _channel(n, seed, m % 2 == 1)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, out=out)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_pair_kernel_silu_epilogue(out):
    n, k, m = 1024, 1024, 777
    codes, w = _codes(2, n, k, 41)
    q, qs = _activations(1, m, k, 41)
    alpha, bias = _channel(n, 41, True)
    y, acc = _run(codes, 2, n, k, q, qs, alpha, bias, flags=1, out=out)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, 1)
    _check(y, acc, want, want_acc, 1)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m", [(4096, 1024, 8192), (1024, 4096, 8192), (3072, 1024, 32000)])
def test_pair_kernel_equals_per_tile_kernel_bitwise(wbits, n, k, m):
    """At full BASELINE sizes (7 and more tiles per pair, both accumulator buffers reused many times) the pair kernel
    and the per-tile kernel give identical FP16 outputs and INT32 accumulators."""
    codes, _ = _codes(wbits, n, k, m + n)
    q, qs = _activations(1, m, k, 5)
    alpha, _ = _channel(n, 5, False)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, None, out=torch.float16)
    y2, acc2 = _run(codes, wbits, n, k, q, qs, alpha, None, out=torch.float16, pair=False)
    assert np.array_equal(acc, acc2)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m", [(256, 128, 257), (512, 2048, 300), (768, 136, 513), (1024, 4096, 1000),
                                   (2048, 1024, 611), (4096, 1024, 2000)])
@pytest.mark.parametrize("flags,out", [(0, torch.float32), (2, torch.float32), (0, torch.float16),
                                       (2, torch.float16), (1, torch.float32)])
def test_pair_kernel_two_parts_equals_oracle(wbits, n, k, m, flags, out):
    """Two residual parts on the pair kernel (both parts' boxes per load slot, one accumulator per part): both
    combination orders, SiLU, bias, both output types, the accumulators of both parts, ragged K and M. The table
    takes the pair kernel for two parts from 32 pair tiles on; smaller shapes run it through pair_only."""
    tiles = -(-m // 256) * (n // 256)
    assert (configs.choose(m, n, k, wbits, 2).kernel == configs.PAIR) == (tiles >= 32)
    seed = wbits * 433 + n + k + m + flags
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(2, m, k, seed)
    alpha, bias = _channel(n, seed, m % 2 == 1)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, out=out, pair_only=True)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias, flags)
    _check(y, acc, want, want_acc, flags)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("flags", [0, 2])
def test_pair_kernel_two_parts_equals_per_tile_kernel_bitwise(wbits, flags):
    """Kea-T's x2 mode at config-4 size (M = 32000 frames): pair and per-tile kernels agree bit for bit."""
    n, k, m = 4096, 1024, 32000
    codes, _ = _codes(wbits, n, k, 31 + flags)
    q, qs = _activations(2, m, k, 32)
    alpha, bias = _channel(n, 33, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, out=torch.float16)
    y2, acc2 = _run(codes, wbits, n, k, q, qs, alpha, bias, flags=flags, out=torch.float16, pair=False)
    assert np.array_equal(acc, acc2)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


def test_pair_kernel_pdl_chain_matches():
    n, k, m = 1024, 1024, 1024
    codes, w = _codes(1, n, k, 8)
    q, qs = _activations(1, m, k, 8)
    alpha, _ = _channel(n, 8, False)
    y, acc = _run(codes, 1, n, k, q, qs, alpha, None, pdl=True)
    want, want_acc = oracle.reference(q, qs, w, alpha)
    _check(y, acc, want, want_acc, 0)


def test_pdl_launch_chain_matches():
    n, k, m = 1024, 1024, 125
    codes, w = _codes(1, n, k, 3)
    q, qs = _activations(1, m, k, 3)
    alpha, _ = _channel(n, 3, False)
    y, acc = _run(codes, 1, n, k, q, qs, alpha, None, pdl=True)
    want, want_acc = oracle.reference(q, qs, w, alpha)
    _check(y, acc, want, want_acc, 0)


# ---- the quantizer ---------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,k", [(125, 1024), (38, 4096), (7, 300), (1, 21), (3000, 1024), (1500, 4096), (999, 300)])
@pytest.mark.parametrize("parts", [1, 2, 3])
def test_quantizer_equals_oracle_bitwise(m, k, parts):
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g) * torch.rand(m, 1, generator=g) * 5
    x[0, :] = 0.0
    q, qs, ldq = lowbit.quantize(x.to(DEV), (0, x.stride(0), x.stride(1), m), m, k, parts)
    torch.cuda.synchronize()
    want_q, want_qs = oracle.quantize(x.numpy(), parts, ldq)
    assert np.array_equal(q.cpu().numpy(), want_q)
    assert np.array_equal(qs.cpu().numpy().view(np.uint32), want_qs.view(np.uint32))


@pytest.mark.parametrize("m", [3, 700])
def test_quantizer_half_integer_quotients_are_exact(m):
    """Values whose quotient by the row scale lies within a few ulps of a half-integer: rint of the IEEE quotient
    must come out bit for bit (the kernel divides exactly only where a reciprocal product could round differently)."""
    g = torch.Generator().manual_seed(m)
    k = 1024
    amax = (torch.rand(m, 1, generator=g) * 3 + 0.1)
    s = (amax / 127).float()
    j = torch.randint(-126, 126, (m, k), generator=g).float() + 0.5
    x = (j * s).float()
    ulps = torch.randint(-4, 5, (m, k), generator=g).to(torch.int32)
    x = (x.view(torch.int32) + ulps).view(torch.float32)          # a few ulps either side of (j + 1/2) s
    x[:, 0] = amax[:, 0]
    q, qs, ldq = lowbit.quantize(x.to(DEV), (0, x.stride(0), x.stride(1), m), m, k, 2)
    torch.cuda.synchronize()
    want_q, want_qs = oracle.quantize(x.numpy(), 2, ldq)
    assert np.array_equal(qs.cpu().numpy().view(np.uint32), want_qs.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), want_q)


@pytest.mark.parametrize("b,k,t", [(2, 300, 19), (16, 1024, 125)])
def test_quantizer_strided_conv_input(b, k, t):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(b, k, t, generator=g)             # [B, K, T]: the conv layout, read through strides
    xd = x.to(DEV)
    q, qs, ldq = lowbit.quantize(xd, (xd.stride(0), xd.stride(2), xd.stride(1), t), b * t, k, 3)
    want_q, want_qs = oracle.quantize(x.transpose(1, 2).reshape(b * t, k).numpy(), 3, ldq)
    assert np.array_equal(q.cpu().numpy(), want_q) and np.array_equal(qs.cpu().numpy(), want_qs)


def test_quantizer_fused_norm_and_silu_match_torch():
    g = torch.Generator().manual_seed(6)
    x = torch.randn(3, 41, 1024, generator=g)
    norm = torch.nn.LayerNorm(1024)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(1024, generator=g) + 0.5)
        norm.bias.copy_(torch.randn(1024, generator=g) * 0.1)
    z = torch.nn.functional.silu(norm(x)).detach()
    normd = norm.to(DEV)
    xd = x.to(DEV)
    q, qs = layer_parts.m1_quantize_parts(xd, 3, normd, "silu")
    deq = (q.float()[:, :, :1024] * qs[:, :, None]).sum(0).cpu().view(3, 41, 1024)
    assert (deq - z).abs().max() < 1e-5 * z.abs().max()


def _norm(k, seed):
    g = torch.Generator().manual_seed(seed)
    norm = torch.nn.LayerNorm(k)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(k, generator=g) + 0.5)
        norm.bias.copy_(torch.randn(k, generator=g) * 0.1)
    return norm


@pytest.mark.parametrize("m,k,parts", [(125, 1024, 1), (250, 1024, 3), (37, 4096, 2), (3000, 1024, 1)])
@pytest.mark.parametrize("main_norm", [False, True])
@pytest.mark.parametrize("in_place", [False, True])
@torch.inference_mode()
def test_quantizer_pre_norm_equals_the_unfused_passes(m, k, parts, main_norm, in_place):
    """The layer's output LayerNorm folded into the next quantizer: its normalized rows (written out as the next
    skip connection's input) match PyTorch's LayerNorm within FP32 summation order, and the codes and scales equal
    the plain quantizer run on those rows afterwards, bit for bit - and, without a second norm, the oracle's."""
    g = torch.Generator().manual_seed(m + k + parts)
    x = (torch.randn(m, k, generator=g) * 3 + 0.5).to(DEV)
    pre, norm = _norm(k, 1).to(DEV), _norm(k, 2).to(DEV) if main_norm else None
    xin = x.clone()
    normed = xin if in_place else torch.full((m, k), float("nan"), device=DEV)
    q, qs, ldq = lowbit.quantize(xin, (0, k, 1, m), m, k, parts, norm=norm, pre_norm=pre, normed=normed)
    torch.cuda.synchronize()
    want = torch.nn.functional.layer_norm(x, (k,), pre.weight, pre.bias, pre.eps)
    assert (normed - want).abs().max().item() <= 1e-5 * want.abs().max().item()
    q2, qs2, _ = lowbit.quantize(normed.clone(), (0, k, 1, m), m, k, parts, norm=norm)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(qs.view(torch.int32), qs2.view(torch.int32))
    if not main_norm:
        want_q, want_qs = oracle.quantize(normed.cpu().numpy(), parts, ldq)
        assert np.array_equal(q.cpu().numpy(), want_q)
        assert np.array_equal(qs.cpu().numpy().view(np.uint32), want_qs.view(np.uint32))


def test_quantizer_pre_norm_needs_its_output():
    x = torch.randn(4, 1024, device=DEV)
    with pytest.raises(ValueError):
        lowbit.quantize(x, (0, 1024, 1, 4), 4, 1024, 1, pre_norm=_norm(1024, 1).to(DEV))


# ---- the layer API (the reference's GPU contract tests, tests/test_kernels_gpu.py:30-105) ------------------------

def _binary_layer(n, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    signs = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
    scale = torch.rand(n, generator=g) * 0.02 + 0.001
    return bits.pack_signs(signs), scale.float()


@pytest.mark.parametrize("parts", [1, 2, 3])
@pytest.mark.parametrize("n,k", [(1024, 1024), (4096, 1024), (1024, 4096), (3072, 1024)])
@pytest.mark.parametrize("m", [38, 126, 300])
@torch.inference_mode()
def test_b1_dot_equals_exact_integer_reference(parts, n, k, m):
    codes, scale = _binary_layer(n, k, seed=n + k + m)
    layer = layer_parts.LAYERS[parts].prepare(codes, scale, None, k, DEV)
    assert layer.fast
    x = torch.randn(m, k, device=DEV)
    q, qs, ldq = L.quantize(x, (0, x.stride(0), x.stride(1), m), m, k)
    y = torch.empty(m, n, device=DEV)
    layer.dot(q[:parts], qs[:parts], ldq, m, y, parts=parts)
    torch.cuda.synchronize()
    signs = bits.unpack_signs(codes, k).to(torch.int64)
    acc = [q[c, :, :k].cpu().to(torch.int64) @ signs.t() for c in range(parts)]
    ref = sum(a.double() * qs[c].cpu().double()[:, None] for c, a in enumerate(acc)) * scale.double()[None, :]
    torch.testing.assert_close(y.cpu().double(), ref, rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize("parts,tol", [(1, 2e-2), (2, 1e-4), (3, 1e-6)])
@torch.inference_mode()
def test_linear_matches_dense_fp64_within_activation_precision(parts, tol):
    n, k, m = 1024, 4096, 126
    codes, scale = _binary_layer(n, k, seed=7)
    layer = layer_parts.LAYERS[parts].prepare(codes, scale, None, k, DEV)
    x = torch.randn(2, m // 2, k, device=DEV)
    y = layer.linear(x).cpu().double()
    ref = x.cpu().double() @ bits.dense_weight(codes, scale, k).t()
    assert (y - ref).norm() / ref.norm() < tol


@torch.inference_mode()
def test_conv_and_project_paths():
    n, k = 2048, 1024
    codes, scale = _binary_layer(n, k, seed=9)
    bias = torch.randn(n) * 0.1
    layer = layer_parts.LAYERS[3].prepare(codes, scale, bias, k, DEV)
    dense = bits.dense_weight(codes, scale, k)
    x = torch.randn(2, k, 33, device=DEV)
    y = layer.conv(x)
    assert y.shape == (2, n, 33)
    ref = torch.einsum("bkt,nk->bnt", x.cpu().double(), dense) + bias.double()[None, :, None]
    assert (y.cpu().double() - ref).norm() / ref.norm() < 1e-6
    xt = torch.randn(2, 33, k, device=DEV)
    yp = layer.project(xt, components=3, activation="silu")
    refp = torch.nn.functional.silu(xt.cpu().double() @ dense.t() + bias.double())
    assert (yp.cpu().double() - refp).norm() / refp.norm() < 1e-5
    yc = layer.project(x, conv=True, components=2)
    refc = ref
    assert yc.shape == (2, n, 33) and (yc.cpu().double() - refc).norm() / refc.norm() < 1e-4


@torch.inference_mode()
def test_ternary_packed_linear_matches_dense_fp64():
    n, k, m = 1024, 1024, 64
    g = torch.Generator().manual_seed(3)
    codes = torch.randint(-1, 2, (n, k), generator=g, dtype=torch.int8)
    scale = torch.rand(n, generator=g) * 0.02 + 0.001
    module = PackedLinear(formats.pack_ternary(codes), scale.float(), k).cuda()
    x = torch.randn(m, k, device=DEV)
    y = module(x).cpu().double()
    ref = x.cpu().double() @ (codes.double() * scale.double()[:, None]).t()
    assert (y - ref).norm() / ref.norm() < 1e-5
    conv = PackedPointwiseConv1d(formats.pack_ternary(codes), scale.float(), k, device=DEV)
    xc = torch.randn(1, k, 40, device=DEV)
    yc = conv(xc).cpu().double()
    refc = torch.einsum("bkt,nk->bnt", xc.cpu().double(), codes.double() * scale.double()[:, None])
    assert (yc - refc).norm() / refc.norm() < 1e-5


@torch.inference_mode()
def test_graph_capture_replays_bitwise():
    n, k, m = 4096, 1024, 125
    codes, scale = _binary_layer(n, k, seed=12)
    layer = layer_parts.LAYERS[1].prepare(codes, scale, None, k, DEV)
    q = torch.randint(-127, 128, (1, m, k), dtype=torch.int8, device=DEV)
    qs = torch.rand(1, m, device=DEV) * 0.01 + 0.005
    y = torch.empty(m, n, device=DEV, dtype=torch.float16)
    layer.dot(q, qs, k, m, y, parts=1)       # first call on the device: one-time set-up outside capture
    torch.cuda.synchronize()
    first = y.clone()
    graph = torch.cuda.CUDAGraph()
    y.zero_()
    with torch.cuda.graph(graph):
        layer.dot(q, qs, k, m, y, parts=1)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, first)


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m,parts,kernel", [(1024, 1024, 2, 1, configs.GEMV), (4096, 1024, 125, 1, configs.PER_TILE),
                                                (1024, 4096, 38, 1, configs.PER_TILE),
                                                (1024, 1024, 40, 3, configs.PER_TILE),
                                                (300, 200, 77, 2, configs.PER_TILE), (4096, 1024, 16, 1, configs.REG),
                                                (1024, 4096, 16, 1, configs.REG), (1024, 1024, 125, 1, configs.REG),
                                                (1024, 4096, 256, 3, configs.SWAP),
                                                (2048, 1024, 256, 2, configs.SWAP), (1024, 1024, 200, 1, configs.SWAP), (4096, 1024, 2048, 1, configs.PAIR),
                                                (4096, 1024, 8192, 2, configs.PAIR)])
@pytest.mark.parametrize("scale", [1.0, 0.5])
def test_residual_epilogue_equals_unfused(wbits, n, k, m, parts, kernel, scale):
    """The skip connection in the epilogue (CUDA-core, register-operand, swap with and without split-K, per-tile
    with and without split-K and stacked parts, pair with one and two parts): bit for bit PyTorch's
    `residual + scale * y`, also written in place over the residual."""
    swap, reg = kernel not in (configs.PER_TILE, configs.REG), kernel == configs.REG
    if kernel != configs.PER_TILE:
        assert configs.choose(m, n, k, wbits, parts).kernel == kernel
    seed = wbits * 7 + n + k + m + parts
    codes, _ = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, True)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), wbits, n, k)
    qd, qsd = torch.from_numpy(q).to(DEV), torch.from_numpy(qs).to(DEV)
    ad, bd = torch.from_numpy(alpha).to(DEV), torch.from_numpy(bias).to(DEV)
    res = torch.randn(m, n, generator=torch.Generator().manual_seed(seed)).to(DEV)
    y = torch.empty(m, n, device=DEV)
    lowbit.gemm(qd, qsd, q.shape[2], m, panels, wbits, n, k, ad, bd, y, parts=parts, swap=swap, reg=reg)
    want = res + scale * y
    fused = torch.empty(m, n, device=DEV)
    lowbit.gemm(qd, qsd, q.shape[2], m, panels, wbits, n, k, ad, bd, fused, parts=parts, residual=res,
                residual_scale=scale, swap=swap, reg=reg)
    inplace = res.clone()
    lowbit.gemm(qd, qsd, q.shape[2], m, panels, wbits, n, k, ad, bd, inplace, parts=parts, residual=inplace,
                residual_scale=scale, swap=swap, reg=reg)
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    assert torch.equal(fused.view(torch.int32), want.view(torch.int32))
    assert torch.equal(inplace.view(torch.int32), want.view(torch.int32))


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m,parts", [(1024, 4096, 512, 1), (1024, 8192, 1000, 1), (512, 4096, 700, 1),
                                         (1024, 4096, 300, 2), (256, 2100, 600, 1)])
@pytest.mark.parametrize("flags,out,extras", [(0, torch.float16, False), (2, torch.float32, True),
                                              (1, torch.float32, True), (0, torch.float32, False)])
def test_pair_split_k_equals_unsplit(wbits, n, k, m, parts, flags, out, extras):
    """Few pair tiles, long K: the K range is cut into slices whose INT32 partial sums go through the scratch
    workspace and a finishing kernel - bit for bit the unsplit pair kernel, accumulators and residual included."""
    need = 8 * parts * m * n * 4                                  # at most 8 slices of INT32 partial sums
    seed = wbits * 5 + n + k + m + parts + flags
    codes, _ = _codes(wbits, n, k, seed)
    q, qs = _activations(parts, m, k, seed)
    alpha, bias = _channel(n, seed, extras)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), wbits, n, k)
    qd, qsd = torch.from_numpy(q).to(DEV), torch.from_numpy(qs).to(DEV)
    ad = torch.from_numpy(alpha).to(DEV)
    bd = None if bias is None else torch.from_numpy(bias).to(DEV)
    res = torch.randn(m, n, generator=torch.Generator().manual_seed(seed)).to(DEV) if out == torch.float32 and extras \
        else None

    def run(ws):
        y = torch.full((m, n), float("nan"), device=DEV, dtype=out)
        acc = torch.full((parts, m, n), -7, device=DEV, dtype=torch.int32) if extras else None
        lowbit.gemm(qd, qsd, q.shape[2], m, panels, wbits, n, k, ad, bd, y, parts=parts, silu=bool(flags & 1),
                    order=(flags >> 1) & 1, acc=acc, force_pair=True, residual=res, workspace=ws)
        return y, acc

    ws = torch.full((need,), 0x5A, dtype=torch.uint8, device=DEV)   # stale contents must not matter
    y_split, acc_split = run(ws)
    y_one, acc_one = run(torch.empty(0, dtype=torch.uint8, device=DEV))
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    bits_of = (lambda t: t.view(torch.int16)) if out == torch.float16 else (lambda t: t.view(torch.int32))
    assert torch.equal(bits_of(y_split), bits_of(y_one))
    if extras:
        assert torch.equal(acc_split, acc_one)


@pytest.mark.parametrize("wbits", [1, 2])
def test_pair_split_k_equals_oracle(wbits):
    n, k, m = 2048, 4096, 512
    assert _lib.workspace_bytes(m, n, k, wbits, 1) > 0       # the table's own split, workspace from gemm
    codes, w = _codes(wbits, n, k, 404)
    q, qs = _activations(1, m, k, 405)
    alpha, bias = _channel(n, 406, True)
    y, acc = _run(codes, wbits, n, k, q, qs, alpha, bias)
    want, want_acc = oracle.reference(q, qs, w, alpha, bias)
    _check(y, acc, want, want_acc, 0)


# ---- config-size cases recorded from the reference (golden_config.npz) -------------------------------------------

@pytest.mark.parametrize("name", ["config0_b1_n4096_k1024_m125", "config1_t2_n1024_k4096_m2048"])
@pytest.mark.parametrize("route", ["table", "swap", "tile"])
def test_gemm_equals_the_reference_at_config_size(golden_config, name, route):
    """BASELINE config 0 (1-bit, M 125, N 4096, K 1024) and config 1's FF-down point (2-bit, M 2048, N 1024, K 4096):
    the library's INT32 accumulators hash to the reference's own int64 accumulators (make_golden.py ran the
    reference's pack / unpack and its test oracle on the same draw), and the FP16 / FP32 outputs equal the oracle's
    epilogue of them bit for bit, within the reference test's tolerance of its FP64 outputs."""
    from config_cases import CONFIG_CASES, SAMPLE_ROWS, draw
    from conftest import sha256
    _, wbits, n, k, m, parts = {c[0]: c for c in CONFIG_CASES}[name]
    w, q, qs, alpha = (t.numpy() for t in draw(wbits, n, k, m, parts))
    codes = oracle.pack_signs(w) if wbits == 1 else oracle.pack_ternary(w)
    config = configs.DotConfig(0, 128, 0, 0, configs.SWAP) if route == "swap" else None
    if route == "swap" and m > 256:
        config = configs.DotConfig(0, 128, 4, 0, configs.SWAP)
    for out in (torch.float16, torch.float32):
        y, acc = _run(codes, wbits, n, k, q, qs, alpha, None, out=out, config=config, swap=route != "tile",
                      pair=route != "tile")
        assert np.array_equal(sha256(acc), golden_config[f"{name}/acc_sha256"]), "accumulators differ from the reference"
        want = oracle.finish(acc, qs, alpha)
        _check(y, acc, want, acc, 0)
        np.testing.assert_allclose(y.double().numpy()[list(SAMPLE_ROWS)], golden_config[f"{name}/y64_rows"],
                                   rtol=2e-6 if out == torch.float32 else 1e-3, atol=1e-6 if out == torch.float32 else 1e-4)


# ---- the weight-stationary pair kernel (one part, K <= 1024) ------------------------------------------------------

@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("n,k,m", [(4096, 1024, 8192), (4096, 1024, 2048), (256, 1024, 300), (1024, 1024, 1000),
                                   (512, 640, 1500), (768, 136, 513), (2048, 384, 3000)])
@pytest.mark.parametrize("flags,out,extras", [(0, torch.float16, False), (2, torch.float32, True),
                                              (1, torch.float32, True)])
def test_pair_resident_weights_equal_streamed_and_oracle(wbits, n, k, m, flags, out, extras):
    """Runs of tiles that keep a channel tile's expanded weights resident (re-expanded when the run reaches the next
    channel tile, odd k-block counts included) give the bits of the kernel that re-expands every tile, accumulators,
    bias, SiLU and the residual included; and the oracle's (rows sampled at the largest M)."""
    assert configs.choose(m, n, k, wbits, 1).kernel == configs.PAIR
    seed = wbits * 5 + n + k + m + flags
    codes, w = _codes(wbits, n, k, seed)
    q, qs = _activations(1, m, k, seed)
    alpha, bias = _channel(n, seed, extras)
    panels = lowbit.prepare_panels(torch.from_numpy(codes).to(DEV), wbits, n, k)
    qd, qsd = torch.from_numpy(q).to(DEV), torch.from_numpy(qs).to(DEV)
    ad = torch.from_numpy(alpha).to(DEV)
    bd = None if bias is None else torch.from_numpy(bias).to(DEV)
    res = torch.randn(m, n, generator=torch.Generator().manual_seed(seed)).to(DEV) if extras else None
    outs = []
    for resident in (True, False):
        y = torch.full((m, n), float("nan"), device=DEV, dtype=out)
        acc = torch.full((1, m, n), -7, device=DEV, dtype=torch.int32)
        lowbit.gemm(qd, qsd, q.shape[2], m, panels, wbits, n, k, ad, bd, y, parts=1, silu=bool(flags & 1),
                    order=(flags >> 1) & 1, acc=acc, residual=res, residual_scale=0.5, resident_weights=resident)
        outs.append((y, acc))
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    (y0, a0), (y1, a1) = outs
    assert torch.equal(a0, a1)
    view = torch.int16 if out == torch.float16 else torch.int32
    assert torch.equal(y0.view(view), y1.view(view))
    rows = np.unique(np.linspace(0, m - 1, 48).astype(int)) if m > 2048 else np.arange(m)
    want, want_acc = oracle.reference(q[:, rows], qs[:, rows], w, alpha, bias, flags)
    if res is not None:
        want = (res.cpu().numpy()[rows] + np.float32(0.5) * want).astype(np.float32)
    _check(y0.cpu()[rows], a0.cpu().numpy()[:, rows], want, want_acc, flags)
