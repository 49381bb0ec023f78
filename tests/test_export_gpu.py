"""Loading an export onto the B200 kernels (kea_kernels.export): the device panels hold exactly the export's codes
(exact INT32 accumulators against the unpacked weights, Q/K/V in order), fused Q/K/V equals the three separate
projections bit for bit, the encoder picks up the export's LayerNorms, position biases, depthwise conv with its
BatchNorm folded in and subsampling, and modes / strictness / invalid codes behave as documented."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
from fake_export import projection_shapes, write_export
from kea_kernels import export, formats, lowbit
from kea_kernels.binary import bits

pytestmark = pytest.mark.gpu
DEV = "cuda"
D, FF = 64, 128


def formats_panel_bytes(wbits: int, n: int, k: int) -> int:
    """Panels: ceil(N / 128) x ceil(K / 128) x wbits x 2048 bytes."""
    return -(-n // 128) * -(-k // 128) * wbits * 2048


def _dense(kind: str, codes: torch.Tensor, k: int) -> np.ndarray:
    w = bits.unpack_signs(codes, k) if kind == "binary" else formats.unpack_ternary(codes, k)
    return w.to(torch.int8).numpy()


def _acc(lin, q: np.ndarray) -> np.ndarray:
    m, k = q.shape[1], lin.in_features
    ldq = q.shape[2]
    qd = torch.from_numpy(q).to(DEV)
    qs = torch.ones(q.shape[0], m, device=DEV)
    y = torch.empty(m, lin.out_features, device=DEV)
    acc = torch.empty(q.shape[0], m, lin.out_features, device=DEV, dtype=torch.int32)
    lowbit.gemm(qd, qs, ldq, m, lin.panels, lin.wbits, lin.out_features, k, lin.scale, lin.bias, y,
                parts=q.shape[0], acc=acc)
    torch.cuda.synchronize()
    return acc.cpu().numpy()


@pytest.mark.parametrize("kind", ["binary", "ternary"])
def test_loaded_panels_hold_the_export_codes(tmp_path, kind):
    from safetensors.torch import load_file
    d = write_export(tmp_path / "m", kind, d=D, ff=FF)
    loaded = export.load_export(d, device=DEV)
    raw = load_file(str(d / formats.FILE))
    g = np.random.default_rng(1)
    for i in (0, 23):
        p = f"encoder.layers.{i}."
        lins = loaded.layers[i]
        for suffix, ours in list(export.PROJECTIONS.items()) + [("qkv", "qkv")]:
            if suffix == "qkv":
                names = [p + q for q in export.QKV]
                w = np.concatenate([_dense(kind, raw[f"{n}.codes"], D) for n in names])
            else:
                n_, k_, _ = projection_shapes(D, FF)[suffix]
                w = _dense(kind, raw[f"{p}{suffix}.codes"], k_)
            k = w.shape[1]
            q = np.zeros((1, 37, -(-k // 16) * 16), dtype=np.int8)
            q[:, :, :k] = g.integers(-127, 128, (1, 37, k), dtype=np.int8)
            assert np.array_equal(_acc(lins[ours], q), oracle.int_acc(q, w)), f"{p}{suffix}"


def test_fused_qkv_equals_the_separate_projections(tmp_path):
    d = write_export(tmp_path / "m", "ternary", d=D, ff=FF)
    fused = export.load_export(d, device=DEV)
    split = export.load_export(d, device=DEV, fuse_qkv=False)
    x = torch.randn(2, 29, D, device=DEV)
    for i in (0, 5):
        y = fused.layers[i]["qkv"](x)
        parts = [split.layers[i][n](x) for n in ("linear_q", "linear_k", "linear_v")]
        assert torch.equal(y, torch.cat(parts, dim=-1))
    with pytest.raises(ValueError, match="fused"):
        export.build_encoder(split, device=DEV)


@pytest.mark.parametrize("kind,mode,parts", [("binary", None, 2), ("binary", "x1", 1), ("binary", "x3", 3),
                                             ("ternary", None, 2), ("ternary", "compact", 3)])
def test_modes_set_the_activation_parts(tmp_path, kind, mode, parts):
    d = write_export(tmp_path / "m", kind, d=D, ff=FF, encoder_tensors=False)
    loaded = export.load_export(d, device=DEV, mode=mode)
    assert loaded.parts == parts and all(l.parts == parts for l in loaded.layers[0].values())
    assert loaded.wbits == (1 if kind == "binary" else 2)
    shapes = [(3 * D, D, False)] + [projection_shapes(D, FF)[s] for s in export.PROJECTIONS]   # Q/K/V fused
    per_layer = sum(formats_panel_bytes(loaded.wbits, n, k) + 4 * n + (4 * n if b else 0) for n, k, b in shapes)
    assert loaded.weight_bytes() == formats.LAYERS * per_layer
    with pytest.raises(ValueError, match="mode"):
        export.load_export(d, device=DEV, mode="x4")


def test_encoder_takes_the_export_tensors(tmp_path):
    d = write_export(tmp_path / "m", "binary", d=D, ff=FF, heads=2, sub=8, n_mels=64)
    loaded = export.load_export(d, device=DEV)
    t = dict(loaded.tensors)
    enc = export.build_encoder(loaded, device=DEV)
    layer = enc.layers[3]
    p = "encoder.layers.3."
    assert torch.equal(layer.norms["att"].weight.cpu(), t[f"{p}norm_self_att.weight"])
    assert torch.equal(layer.pos_bias_v.cpu(), t[f"{p}self_attn.pos_bias_v"])
    inv = t[f"{p}conv.batch_norm.weight"] / torch.sqrt(t[f"{p}conv.batch_norm.running_var"] + 1e-5)
    want_w = t[f"{p}conv.depthwise_conv.weight"] * inv[:, None, None]
    want_b = (t[f"{p}conv.depthwise_conv.bias"] - t[f"{p}conv.batch_norm.running_mean"]) * inv + \
        t[f"{p}conv.batch_norm.bias"]
    torch.testing.assert_close(layer.dw_weight.cpu(), want_w, rtol=0, atol=0)
    torch.testing.assert_close(layer.dw_bias.cpu(), want_b, rtol=0, atol=0)
    # the folded conv equals depthwise conv then eval BatchNorm
    h = torch.randn(2, D, 40)
    conv = torch.nn.functional.conv1d(h, t[f"{p}conv.depthwise_conv.weight"], t[f"{p}conv.depthwise_conv.bias"],
                                      padding=4, groups=D)
    bn = torch.nn.functional.batch_norm(conv, t[f"{p}conv.batch_norm.running_mean"],
                                        t[f"{p}conv.batch_norm.running_var"], t[f"{p}conv.batch_norm.weight"],
                                        t[f"{p}conv.batch_norm.bias"], training=False, eps=1e-5)
    folded = torch.nn.functional.conv1d(h, want_w, want_b, padding=4, groups=D)
    torch.testing.assert_close(folded, bn, rtol=1e-5, atol=1e-5)
    assert torch.equal(enc.pre.conv[5].weight.cpu(), t["encoder.pre_encode.conv.5.weight"])
    mel = torch.randn(2, 64, 160, device=DEV)
    y = enc(mel)
    assert y.shape == (2, 20, D) and bool(torch.isfinite(y).all())


def test_strict_build_needs_the_encoder_tensors(tmp_path):
    d = write_export(tmp_path / "m", "binary", d=D, ff=FF, encoder_tensors=False)
    loaded = export.load_export(d, device=DEV)
    with pytest.raises(ValueError, match="lacks"):
        export.build_encoder(loaded, device=DEV)
    enc = export.build_encoder(loaded, device=DEV, strict=False)
    assert len(enc.layers) == formats.LAYERS


def test_invalid_ternary_codes_are_rejected_at_load(tmp_path):
    def bad(layers, tensors):
        name = next(iter(layers))
        tensors[f"{name}.codes"][0, 0] = 0b11
    d = write_export(tmp_path / "m", "ternary", d=D, ff=FF, encoder_tensors=False, tamper=bad)
    with pytest.raises(ValueError):
        export.load_export(d, device=DEV)
