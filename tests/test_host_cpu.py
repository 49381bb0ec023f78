"""CPU: the C-ABI library loads and exports what include/kea_lowbit.h declares; host-side logic (dispatch table,
argument checks, layer / provider plumbing, export-code checks) behaves like the reference's (no GPU work here)."""
from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import ROOT
from kea_kernels import _lib, formats, lowbit
from kea_kernels.binary import bits, configs
from kea_kernels.binary import layer as L
from kea_kernels.binary.provider import BinaryLinear, BinaryProjection, PartCount, Table, handle


def test_library_exports_every_declared_symbol():
    header = (ROOT / "include" / "kea_lowbit.h").read_text()
    declared = set(re.findall(r"^\s*(?:int|size_t|const char \*)\s*(kea_lowbit_\w+)\s*\(", header, re.M))
    assert declared == set(_lib.EXPORTS)
    lib = _lib.lib()
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.kea_lowbit_version() == 5
    assert lib.kea_lowbit_status_string(0) == b"success"
    assert lib.kea_lowbit_status_string(4) == b"invalid packed codes"


def test_panel_bytes():
    assert _lib.panel_bytes(1, 4096, 1024) == 4096 * 1024 // 8           # no padding at Parakeet shapes
    assert _lib.panel_bytes(2, 4096, 1024) == 4096 * 1024 // 4
    assert _lib.panel_bytes(1, 5, 300) == 1 * 3 * 2048
    assert _lib.panel_bytes(2, 129, 129) == 2 * 2 * 2 * 2048
    assert _lib.panel_bytes(3, 8, 8) == 0 and _lib.panel_bytes(1, 0, 8) == 0


PARAKEET = [(1024, 1024), (1024, 4096), (2048, 1024), (3072, 1024), (4096, 1024)]


@pytest.mark.parametrize("n,k", PARAKEET)
@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts", [1, 2, 3])
def test_every_shape_has_a_valid_config(n, k, wbits, parts):
    kb = -(-k // 128)
    for m in (1, 16, 38, 125, 126, 249, 256, 368, 400, 512, 1500, 2048, 8192, 32000):
        c = _lib.choose_config(m, n, k, wbits, parts)
        assert (c.kernel == configs.GEMV) == (m * parts <= 4)
        if c.kernel == configs.GEMV:   # the CUDA-core kernel: tile_m = the tokens, tile_n = channels per CTA
            assert c.tile_m == m and c.tile_n in (8, 16, 32)
            assert c.splits == 1 and 0 < c.smem_bytes <= 48 * 1024
            cfg = configs.choose(m, n, k, wbits, parts)
            cfg.validate(parts)
            assert cfg.grid(m, n)[0] * cfg.tile_n >= n
            continue
        rows = m * parts   # the register kernel: up to 160 K output rows x channels, or narrow long-K layers
        reg = (rows <= 256 and rows * n <= 160 * 1024) or (n >= 2048 and k <= 1024 and rows * n <= 256 * 1024) or (n <= 1024 and k >= 4096 and (rows <= 128 or (parts == 3 and rows <= 400)))
        assert (c.kernel == configs.REG) == reg
        if c.kernel == configs.REG:   # tile_m activation rows x tile_n channels per CTA, K-slices among 8 warps
            cfg = configs.choose(m, n, k, wbits, parts)
            cfg.validate(parts)
            gx, gy, _ = cfg.grid(m, n, parts)
            assert gx * cfg.tile_n >= n and gy * (cfg.tile_m // parts) >= m
            assert 0 < c.smem_bytes <= 48 * 1024
            continue
        if c.kernel == configs.PAIR:   # 256 x 256 pair tiles, one 256-column accumulator per part
            assert c.tile_m == 256 and c.tile_n == 256 and parts <= 2 and c.splits == 1
            assert c.smem_bytes <= 227 * 1024
            continue
        swap = m <= 32 or 128 < m <= 256 if parts == 1 else (parts * -(-m // 16) * 16 >= 512 and m <= 512
                                                                and (n >= 2048 or k >= 4096))
        assert (c.kernel == configs.SWAP) == (swap and not (c.kernel == configs.PAIR))
        if c.kernel == configs.SWAP:   # 128 channels x tile_m tokens of every part (<= 512 TMEM columns)
            assert c.tile_n == 128 and c.tile_m % 16 == 0 and c.tile_m <= 256 and parts * c.tile_m <= 512
            assert c.tile_m * -(-m // c.tile_m) >= m and c.tile_m < m + 16 * -(-m // c.tile_m)
            assert 1 <= c.splits <= min(kb, 8) and 1 <= c.stages <= 8 and c.smem_bytes <= 227 * 1024
            cfg = configs.choose(m, n, k, wbits, parts)
            cfg.validate(parts)
            gx, gy, gz = cfg.grid(m, n)
            assert gx * gy * gz <= 148 or gz == 1      # K is split only while the grid stays within one wave
            continue
        assert c.tile_m in (128, 256) and c.tile_n in (32, 64, 128, 256)
        assert (c.tile_m // 128) * parts * c.tile_n <= 512
        assert 1 <= c.splits <= min(kb, 16) and 1 <= c.stages <= 8
        assert c.smem_bytes <= 227 * 1024
        if c.splits > 1:
            per = -(-(c.tile_n // 4) // c.splits)
            assert c.splits * (c.tile_m // 128) * parts * per * 128 * 16 <= c.smem_bytes
        cfg = configs.choose(m, n, k, wbits, parts)
        cfg.validate(parts)
        gx, gy, gz = cfg.grid(m, n)
        assert gx * gy * gz >= min(74, gx * gy)   # small grids are split along K to cover the SMs


def test_small_m_splits_k_and_large_m_does_not():
    c = _lib.choose_config(125, 4096, 1024, 1, 1)       # 32-channel tiles already give 128 CTAs
    assert (c.kernel, c.tile_m, c.tile_n, c.splits) == (configs.PER_TILE, 128, 32, 1)
    c = _lib.choose_config(125, 1024, 4096, 1, 1)       # register kernel: 32 channels x 16 tokens, 256 CTAs
    assert (c.kernel, c.tile_m, c.tile_n, c.splits) == (configs.REG, 16, 32, 8)
    c = _lib.choose_config(16, 4096, 1024, 1, 1)        # 16 channels x 32 rows: 256 CTAs
    assert (c.kernel, c.tile_m, c.tile_n, c.splits) == (configs.REG, 32, 16, 8)
    c = _lib.choose_config(125, 2048, 1024, 1, 1)       # 64 channels x 16 tokens: 256 CTAs
    assert (c.kernel, c.tile_m, c.tile_n, c.splits) == (configs.REG, 16, 64, 8)
    c = _lib.choose_config(125, 3072, 1024, 1, 1)       # wider: the tcgen05 per-tile kernel
    assert c.kernel == configs.PER_TILE
    c = _lib.choose_config(378, 1024, 4096, 1, 1)       # one part past 128 rows: the tcgen05 table
    assert c.kernel != configs.REG
    c = _lib.choose_config(126, 1024, 4096, 1, 3)       # 378 rows of three parts: 32 rows x 32 channels
    assert (c.kernel, c.tile_m, c.tile_n, c.splits) == (configs.REG, 32, 32, 8)
    c = _lib.choose_config(256, 4096, 1024, 1, 3)       # three parts stacked along the MMA's N: 3 x 128 tokens x 2
    assert (c.kernel, c.tile_m, c.splits) == (configs.SWAP, 128, 1)
    c = _lib.choose_config(8192, 4096, 1024, 1, 1)
    assert c.splits == 1


def _desc(**kw):
    d = _lib.GemmDesc()
    header = (ROOT / "include" / "kea_lowbit.h").read_text()
    body = header[header.index("typedef struct KeaGemmDesc"):header.index("} KeaGemmDesc;")]
    declared = re.findall(r"^\s+[\w ]+?\**\s*\**(\w+)(?:,\s*(\w+))?;", body, re.M)
    names = [n for pair in declared for n in pair if n]
    assert [f[0] for f in d._fields_] == names   # the ctypes mirror is the header's struct, field for field
    d.q, d.ldq, d.parts, d.qs, d.panels, d.wbits, d.n, d.k = 16, 1024, 1, 16, 16, 1, 4096, 1024
    d.alpha, d.y, d.ldy, d.y_dtype, d.m = 16, 16, 4096, 0, 125
    for key, value in kw.items():
        setattr(d, key, value)
    return d


def test_c_abi_argument_errors_are_reported_before_any_device_work():
    lib = _lib.lib()
    assert lib.kea_lowbit_gemm(None, None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(wbits=3)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(parts=4)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(y_dtype=2)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(m=0)), None) == _lib.OK          # empty: a no-op
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(q=24)), None) == _lib.ALIGNMENT
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(ldq=1000)), None) == _lib.INVALID_VALUE   # ldq < k
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(ldq=1032, k=1030)), None) == _lib.ALIGNMENT  # ldq % 16
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=2048)), None) == _lib.INVALID_VALUE
    # the register kernel takes no stages and no contradictory kernel flags
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=_lib.FLAG_FORCE_REG, stages=2)), None) == _lib.INVALID_VALUE
    for other in (_lib.FLAG_NO_REG, _lib.FLAG_FORCE_SWAP, _lib.FLAG_FORCE_PAIR):
        assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=_lib.FLAG_FORCE_REG | other)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=_lib.FLAG_TEST_STALL)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=_lib.FLAG_FORCE_SWAP, tile_m=100)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=_lib.FLAG_FORCE_SWAP, tile_n=32)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=_lib.FLAG_FORCE_SWAP | _lib.FLAG_NO_SWAP)), None) == \
        _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(wait_clocks=-1)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(residual=16, ld_residual=4095)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(residual=16, ld_residual=4096, y_dtype=1)), None) == \
        _lib.INVALID_VALUE                                # a residual needs FP32 output
    both = _lib.FLAG_NO_PAIR | _lib.FLAG_FORCE_PAIR   # contradictory pair flags
    assert lib.kea_lowbit_gemm(ctypes.byref(_desc(flags=both)), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_prepare(None, 1, 4, 8, None, None, None) == _lib.INVALID_VALUE
    with pytest.raises(ValueError):
        _lib.check(_lib.ALIGNMENT, "gemm")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.CUDA, "gemm")


def _qdesc(**kw):
    """A quantizer descriptor with plausible (never dereferenced) addresses: 125 unit-stride rows of 1024."""
    d = _lib.QuantizeDesc()
    d.x, d.xb, d.xt, d.xk, d.t, d.m, d.k, d.parts = 1 << 20, 0, 1024, 1, 125, 125, 1024, 1
    d.q, d.q_part_stride, d.ldq, d.qs, d.qs_part_stride = 2 << 20, 125 * 1024, 1024, 3 << 20, 125
    for key, value in kw.items():
        setattr(d, key, value)
    return d


def test_quantizer_pre_norm_argument_errors_are_reported_before_any_device_work():
    lib = _lib.lib()
    pre = dict(pre_norm_weight=4 << 20, pre_eps=1e-5, normed=5 << 20, ld_normed=1024)
    assert lib.kea_lowbit_quantize(ctypes.byref(_qdesc(**pre, m=0)), None) == _lib.OK        # empty: a no-op
    assert lib.kea_lowbit_quantize(ctypes.byref(_qdesc(**{**pre, "normed": 0})), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_quantize(ctypes.byref(_qdesc(**{**pre, "normed": (5 << 20) + 4})), None) == _lib.ALIGNMENT
    assert lib.kea_lowbit_quantize(ctypes.byref(_qdesc(**{**pre, "ld_normed": 1022})), None) == _lib.ALIGNMENT
    assert lib.kea_lowbit_quantize(ctypes.byref(_qdesc(**{**pre, "ld_normed": 1020})), None) == _lib.ALIGNMENT
    assert lib.kea_lowbit_quantize(ctypes.byref(_qdesc(**{**pre, "pre_norm_weight": (4 << 20) + 8})), None) == \
        _lib.ALIGNMENT
    # the pre-norm keeps rows in registers: the strided (conv layout) path refuses it
    assert lib.kea_lowbit_quantize(ctypes.byref(_qdesc(**pre, xt=1, xk=125)), None) == _lib.UNSUPPORTED


def test_project_argument_errors_are_reported_before_any_device_work():
    lib = _lib.lib()
    p = _lib.ProjectDesc()
    p.gemm = _desc()
    p.quant = _qdesc(m=p.gemm.m, k=p.gemm.k, q=p.gemm.q, ldq=p.gemm.ldq, qs=p.gemm.qs,
                     q_part_stride=p.gemm.q_part_stride, qs_part_stride=p.gemm.qs_part_stride)
    assert lib.kea_lowbit_project(None, None) == _lib.INVALID_VALUE
    p.flags = 2                                                    # unknown flag
    assert lib.kea_lowbit_project(ctypes.byref(p), None) == _lib.INVALID_VALUE
    assert lib.kea_lowbit_project_fuses(ctypes.byref(p)) == -_lib.INVALID_VALUE
    p.flags = _lib.PROJECT_FUSE
    p.quant.qs = p.gemm.qs + 64                                    # the quantizer's output is not the GEMM's input
    assert lib.kea_lowbit_project(ctypes.byref(p), None) == _lib.INVALID_VALUE
    p.quant.qs = p.gemm.qs
    p.quant.m = p.gemm.m + 1
    assert lib.kea_lowbit_project(ctypes.byref(p), None) == _lib.INVALID_VALUE
    p.quant.m = p.gemm.m
    p.quant.flags = 64                                             # the quantizer's own checks apply
    assert lib.kea_lowbit_project(ctypes.byref(p), None) == _lib.INVALID_VALUE
    # the fused form's scratch: one part, M <= 128, K a multiple of 128 up to 1024
    assert lib.kea_lowbit_project_scratch_bytes(125, 4096, 1024, 1, 1) == 16 * 128 * (1024 + 4)
    for shape in ((129, 4096, 1024, 1, 1), (125, 4096, 1024, 1, 2), (125, 4096, 1000, 1, 1), (125, 1024, 4096, 1, 1)):
        assert lib.kea_lowbit_project_scratch_bytes(*shape) == 0, shape


def test_fused_conv_quantizer_argument_errors_are_reported_before_any_device_work():
    lib = _lib.lib()

    def conv(**kw):
        base = dict(h=1 << 20, y=0, weight=2 << 20, b=1, t=125, c=1024, kw=9, flags=0, q=3 << 20,
                    q_part_stride=125 * 1024, ldq=1024, qs=4 << 20, qs_part_stride=125, parts=1)
        base.update(kw)
        return lib.kea_lowbit_glu_depthwise(ctypes.byref(_lib.ConvDesc(**base)), None)

    assert conv(q=0) == _lib.INVALID_VALUE                                  # neither y nor q
    assert conv(q=0, y=5 << 20, flags=_lib.CONV_QUANT_SILU) == _lib.INVALID_VALUE   # SiLU flag without q
    assert conv(qs=0) == _lib.INVALID_VALUE
    assert conv(parts=4) == _lib.INVALID_VALUE
    assert conv(ldq=1020) == _lib.INVALID_VALUE                             # ldq < c
    assert conv(q=(3 << 20) + 2) == _lib.ALIGNMENT
    assert conv(ldq=1030) == _lib.ALIGNMENT
    assert conv(h=(1 << 20) + 4) == _lib.ALIGNMENT
    assert conv(c=1022, ldq=1024) == _lib.UNSUPPORTED                       # c % 4
    assert conv(c=1028, ldq=1040) == _lib.UNSUPPORTED                       # c > 1024
    assert conv(kw=3) == _lib.UNSUPPORTED                                   # the fused form is built for width 9
    assert conv(b=0) == _lib.OK                                             # empty: a no-op


def test_python_boundary_refuses_host_tensors():
    q = torch.zeros(1, 4, 16, dtype=torch.int8)
    with pytest.raises(ValueError, match="CUDA"):
        lowbit.gemm(q, torch.ones(1, 4), 16, 4, torch.zeros(2048, dtype=torch.uint8), 1, 8, 16, torch.ones(8), None,
                    torch.zeros(4, 8), parts=1)
    with pytest.raises(ValueError, match="CUDA"):
        lowbit.prepare_panels(torch.zeros(8, 2, dtype=torch.uint8), 1, 8, 16)
    codes = bits.pack_signs(torch.ones(8, 16, dtype=torch.int8))
    with pytest.raises(ValueError, match="CUDA devices only"):
        L.Int8MmaLayer.prepare(codes, torch.ones(8), None, 16, "cpu")


def test_validate_weights_rejections():
    codes = torch.zeros(2, 2, dtype=torch.uint8)
    codes[0, 1] = 0x80
    with pytest.raises(ValueError, match="tail"):
        bits.validate_weights(codes, torch.ones(2), None, 12)
    good = torch.zeros(2, 2, dtype=torch.uint8)
    assert bits.validate_weights(good, torch.ones(2), None, 12) == (2, 12)
    with pytest.raises(ValueError, match="finite"):
        bits.validate_weights(good, torch.tensor([1.0, float("nan")]), None, 12)
    with pytest.raises(ValueError, match="codes must be"):
        bits.validate_weights(good, torch.ones(2), None, 20)
    with pytest.raises(ValueError, match="bias"):
        bits.validate_weights(good, torch.ones(2), torch.ones(3), 12)
    with pytest.raises(ValueError, match="in_features"):
        bits.validate_weights(good, torch.ones(2), None, True)


def test_dot_config_validation():
    configs.DotConfig(128, 128, 4, 2).validate(1)
    with pytest.raises(ValueError):
        configs.DotConfig(100, 128, 1, 1).validate(1)
    with pytest.raises(ValueError):
        configs.DotConfig(256, 256, 1, 1).validate(3)
    with pytest.raises(ValueError):
        configs.DotConfig(128, 128, 17, 1).validate(1)
    assert configs.DotConfig(128, 128, 4, 2).label() == "m128_n128_c4_s2"
    # register kernel: channels x rows x K-slices must name an instantiated warp tile
    for rows, cn, ks in ((32, 32, 8), (16, 64, 4), (32, 16, 8), (32, 128, 1)):
        configs.DotConfig(rows, cn, ks, 0, configs.REG).validate(3)
    for rows, cn, ks, parts in ((24, 32, 8, 1), (32, 48, 8, 1), (32, 32, 3, 1), (16, 16, 8, 1), (32, 256, 8, 1),
                                (32, 64, 8, 1), (16, 128, 8, 1)):
        with pytest.raises(ValueError):
            configs.DotConfig(rows, cn, ks, 0, configs.REG).validate(parts)
    assert configs.DotConfig(32, 64, 4, 0, configs.REG).label() == "reg_r32_n64_k4"
    assert configs.DotConfig(30, 64, 4, 0, configs.REG).grid(125, 1000, 3) == (16, 13, 1)


def test_part_count_overrides_components_and_forwards_writes():
    calls = []

    class Provider:
        defer_epilogue = False

        def __call__(self, x, mod, conv=False, components=3, activation="", norm=None, config=None,
                     input_activation=""):
            calls.append(components)
            return x

    inner = Provider()
    wrapped = PartCount(inner, 2)
    wrapped(torch.zeros(1), None, components=3)
    assert calls == [2]
    wrapped.defer_epilogue = True
    assert inner.defer_epilogue is True and wrapped.n == 2
    with pytest.raises(ValueError):
        PartCount(inner, 4)


def test_table_handles_resolve_fused_rows():
    class FakeLayer:
        def __init__(self, n):
            self.n = n

        def weight_bytes(self):
            return self.n

        def project(self, x, **kw):
            return torch.arange(x.shape[-2] * self.n, dtype=torch.float32).view(1, x.shape[-2], self.n)

    table = Table()
    qkv = table.add("qkv", FakeLayer(12), "linear", 12, 4, members=("q", "k", "v"))
    out = table.add("out", FakeLayer(4), "linear", 4, 4)
    assert table.resolve(4, 4) == (qkv, 4) and table.resolve(12, 4) == (out, 0)
    with pytest.raises(ValueError):
        table.resolve(10, 4)
    with pytest.raises(KeyError):
        table.resolve(16, 1)
    k_mod = BinaryLinear(qkv, 4, 4, 4, torch.ones(4), None)
    provider = BinaryProjection(table)
    y = provider(torch.zeros(1, 3, 4), k_mod)
    assert y.shape == (1, 3, 4) and y[0, 0].tolist() == [4.0, 5.0, 6.0, 7.0]
    assert provider.bytes == 16
    with pytest.raises(ValueError):
        provider(torch.zeros(1, 3, 4), k_mod, config=(1, 2))
    bad = BinaryLinear(qkv, 0, 4, 4, torch.ones(4), None)
    object.__setattr__(bad, "packed_t", handle(0, 4).flip(1))
    with pytest.raises(ValueError, match="non-contiguous"):
        provider(torch.zeros(1, 3, 4), bad)


def test_ternary_validation_matches_the_reference_errors():
    packed = formats.pack_ternary(torch.zeros(4, 8, dtype=torch.int8))
    assert formats.validate_ternary(packed, torch.ones(4), None, 8) == (4, 8)
    with pytest.raises(ValueError, match="finite"):
        formats.validate_ternary(packed, torch.full((4,), float("inf")), None, 8)
    with pytest.raises(ValueError):
        formats.validate_ternary(torch.tensor([[0b11, 0]], dtype=torch.uint8), torch.ones(1), None, 8)
    with pytest.raises(ValueError, match="positive"):
        formats.validate_ternary(packed, torch.ones(4), None, 0)


def test_encoder_layer_shapes_are_the_parakeet_linears():
    """BASELINE config 2's per-layer GEMMs (QKV, out, two macaron FF pairs, conv pw1 / pw2) plus linear_pos."""
    from kea_kernels import encoder as E
    shapes = E.layer_linear_shapes(1024, 4096)
    assert [shapes[n] for n in E.LAYER_LINEARS] == [(4096, 1024), (1024, 4096), (3072, 1024), (1024, 1024),
                                                    (2048, 1024), (1024, 1024), (4096, 1024), (1024, 4096)]
    assert shapes["linear_pos"] == (1024, 1024)
    assert sum(n * k for n, k in (shapes[x] for x in E.LAYER_LINEARS)) == 24_117_248   # 2.875 MiB of signs per layer


def test_split_k_workspace_only_where_pair_tiles_are_few():
    """Pair tiles filling at most a quarter of the SM pairs, with >= 16 k-blocks, split K through scratch: slices x
    parts x M x N INT32; every other shape needs none."""
    assert _lib.workspace_bytes(512, 2048, 4096, 1, 1) == 4 * 512 * 2048 * 4       # 16 tiles, 32 k-blocks: 4 slices
    assert _lib.workspace_bytes(1000, 1024, 8192, 2, 1) == 4 * 1000 * 1024 * 4     # 16 tiles: 4 slices
    assert _lib.workspace_bytes(600, 256, 2100, 1, 1) == 4 * 600 * 256 * 4         # 3 tiles, 17 k-blocks: 4 slices
    # (512, 1024, 4096), (300, 1024, 4096): a narrow layer just above the pair kernel's M runs on the per-tile kernel
    for shape in ((8192, 4096, 1024), (2048, 1024, 4096), (512, 4096, 1024), (125, 4096, 1024), (1, 1024, 4096),
                  (512, 1024, 1024), (512, 1024, 4096), (300, 1024, 4096)):
        assert _lib.workspace_bytes(*shape, 1, 1) == 0, shape
