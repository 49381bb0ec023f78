"""The FastConformer call sites of the low-bit GEMM (the clip workload of BASELINE configs 2-4) against a plain
PyTorch FP32 forward of the same layers with dense weights (codes x scale): the only differences are the residual
INT8 activation quantization and the exact INT32 accumulation, so the relative error is set by the number of parts
(x3: ~1e-6 per projection; x1: ~1e-2)."""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from kea_kernels import encoder as E

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _dense_linear(layer, name, x, *, norm=None, input_silu=False, silu=False):
    w, bias = layer.weights[name]
    if norm is not None:
        x = F.layer_norm(x, (x.shape[-1],), norm.weight, norm.bias, norm.eps)
    if input_silu:
        x = F.silu(x)
    y = F.linear(x, w.dense(), bias)
    return F.silu(y) if silu else y


def _dense_layer(layer, x):
    b, t, d = x.shape
    lin = lambda name, h, **kw: _dense_linear(layer, name, h, **kw)
    x = x + 0.5 * lin("ff1_down", lin("ff1_up", x, norm=layer.norms["ff1"], silu=True))
    qkv = lin("qkv", x, norm=layer.norms["att"]).view(b, t, 3, layer.heads, layer.dk)
    q, k, v = qkv.unbind(2)
    p = lin("linear_pos", E.rel_positions(t, d, x.device)[None])[0].view(2 * t - 1, layer.heads, layer.dk)
    ac = torch.matmul((q + layer.pos_bias_u).transpose(1, 2), k.permute(0, 2, 3, 1))
    bd = E.rel_shift(torch.matmul((q + layer.pos_bias_v).transpose(1, 2), p.permute(1, 2, 0)))
    attn = torch.softmax((ac + bd) / math.sqrt(layer.dk), dim=-1)
    x = x + lin("out", torch.matmul(attn, v.transpose(1, 2)).transpose(1, 2).reshape(b, t, d))
    h = F.glu(lin("pw1", x, norm=layer.norms["conv"]), dim=-1).transpose(1, 2)
    h = F.conv1d(h, layer.dw_weight, layer.dw_bias, padding=layer.kernel // 2, groups=d)
    x = x + lin("pw2", h.transpose(1, 2), input_silu=True)
    x = x + 0.5 * lin("ff2_down", lin("ff2_up", x, norm=layer.norms["ff2"], silu=True))
    n = layer.norms["out"]
    return F.layer_norm(x, (d,), n.weight, n.bias, n.eps)


def _dense_forward(enc, mel):
    x = enc.pre(mel)
    for layer in enc.layers:
        x = _dense_layer(layer, x)
    return x


@pytest.mark.parametrize("wbits", [1, 2])
@pytest.mark.parametrize("parts,tol", [(3, 2e-4), (1, 5e-2)])
@torch.inference_mode()
def test_encoder_matches_dense_fp32_forward(wbits, parts, tol):
    enc = E.FastConformerEncoder(layers=2, wbits=wbits, parts=parts, seed=wbits, device=DEV, keep_dense=True)
    g = torch.Generator().manual_seed(3)
    mel = torch.randn(2, 128, 400, generator=g).to(DEV)
    y = enc(mel)
    assert y.shape == (2, 50, 1024) and bool(torch.isfinite(y).all())
    ref = _dense_forward(enc, mel)
    rel = ((y - ref).norm() / ref.norm()).item()
    assert rel < tol, rel


@torch.inference_mode()
def test_clip_gemm_sequence_is_config2():
    """One 10 s clip: 1000 log-mel frames -> 125 encoder frames; 8 low-bit GEMMs per layer at M = 125 with the
    BASELINE config-2 shapes, and the large-M batch (config 3: 256 clips) at M = 32000 through the same layers."""
    enc = E.FastConformerEncoder(layers=1, device=DEV)
    shapes = enc.gemm_shapes(1, 1000)
    assert [(n, k) for _, m, n, k in shapes] == [(4096, 1024), (1024, 4096), (3072, 1024), (1024, 1024),
                                                (2048, 1024), (1024, 1024), (4096, 1024), (1024, 4096)]
    assert {m for _, m, _, _ in shapes} == {125}
    assert {m for _, m, _, _ in enc.gemm_shapes(256, 1000)} == {32000}
    mel = torch.randn(1, 128, 1000, device=DEV)
    assert enc(mel).shape == (1, 125, 1024)


@torch.inference_mode()
def test_encoder_forward_replays_in_a_cuda_graph():
    enc = E.FastConformerEncoder(layers=2, device=DEV)
    mel = torch.randn(1, 128, 1000, device=DEV)
    first = enc(mel).clone()           # warm-up: one-time set-up and the linear_pos cache outside the capture
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = enc(mel)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)


@torch.inference_mode()
def test_joint_greedy_labels():
    joint = E.TDTJoint(device=DEV)
    enc = torch.randn(3, 125, 1024, device=DEV)
    lab = joint.greedy(enc)
    assert lab.shape == (3, 125) and lab.dtype == torch.int32
    assert int(lab.min()) >= 0 and int(lab.max()) <= 1024


@torch.inference_mode()
def test_padded_bucket_matches_clip_alone():
    """Config 4's length buckets: a short clip padded to its bucket's longest clip (padding masked as attention
    keys and zeroed before the depthwise conv) gives its own frames as when run alone."""
    enc = E.FastConformerEncoder(layers=2, wbits=2, parts=3, seed=4, device=DEV)
    g = torch.Generator().manual_seed(5)
    long_mel, short_mel = torch.randn(1, 128, 400, generator=g), torch.randn(1, 128, 288, generator=g)
    batch = torch.zeros(2, 128, 400)
    batch[0], batch[1, :, :288] = long_mel[0], short_mel[0]
    lengths = torch.tensor([enc.frames(400), enc.frames(288)])
    y = enc(batch.to(DEV), lengths.to(DEV))
    alone_short, alone_long = enc(short_mel.to(DEV))[0], enc(long_mel.to(DEV))[0]
    n = int(lengths[1])
    assert alone_short.shape[0] == n
    for got, want in ((y[1, :n], alone_short), (y[0], alone_long)):
        rel = ((got - want).norm() / want.norm()).item()
        assert rel < 2e-4, rel


@pytest.mark.parametrize("b,t,c", [(3, 125, 1024), (1, 7, 40), (2, 1, 300), (4, 200, 1024)])
@pytest.mark.parametrize("kw", [9, 3, 31])
@pytest.mark.parametrize("masked", [False, True])
@torch.inference_mode()
def test_glu_depthwise_matches_torch(b, t, c, kw, masked):
    """GLU + padding mask + depthwise conv in one kernel against F.glu -> mask -> F.conv1d (FP32; the kernel sums
    the taps in its own order with FMAs, so within FP32 rounding of the conv)."""
    from kea_kernels import lowbit
    g = torch.Generator().manual_seed(b * 1000 + t + c + kw)
    h = torch.randn(b, t, 2 * c, generator=g).to(DEV)
    w = (torch.randn(c, 1, kw, generator=g) / math.sqrt(kw)).to(DEV)
    bias = (0.1 * torch.randn(c, generator=g)).to(DEV) if kw != 3 else None
    lengths = torch.randint(1, t + 1, (b,), generator=g).to(DEV) if masked else None
    y = lowbit.glu_depthwise(h, w, bias, lengths)
    gl = F.glu(h, dim=-1)
    if masked:
        gl = gl * (torch.arange(t, device=DEV)[None, :] < lengths[:, None])[:, :, None]
    want = F.conv1d(gl.transpose(1, 2), w, bias, padding=kw // 2, groups=c).transpose(1, 2)
    torch.testing.assert_close(y, want, rtol=2e-5, atol=2e-5)


def test_glu_depthwise_rejects_bad_arguments():
    from kea_kernels import lowbit
    h = torch.randn(1, 4, 8, device=DEV)
    with pytest.raises(ValueError):
        lowbit.glu_depthwise(h, torch.randn(4, 1, 4, device=DEV))     # even width
    with pytest.raises(ValueError):
        lowbit.glu_depthwise(h, torch.randn(3, 1, 9, device=DEV))     # channel count
    with pytest.raises(ValueError):
        lowbit.glu_depthwise(h.transpose(1, 2), torch.randn(4, 1, 9, device=DEV))


@pytest.mark.parametrize("b,t,c", [(1, 125, 1024), (3, 37, 1000), (40, 125, 256), (2, 1, 4)])
@pytest.mark.parametrize("parts", [1, 3])
@pytest.mark.parametrize("silu,masked", [(True, True), (True, False), (False, True)])
@torch.inference_mode()
def test_glu_depthwise_with_fused_quantizer_equals_the_two_kernels(b, t, c, parts, silu, masked):
    """pw2's quantizer fused into the conv kernel: the INT8 parts and scales equal glu_depthwise followed by the
    quantizer (input SiLU) bit for bit - four and eight frames per CTA (40 clips take the wider chunks), ragged C
    (padding columns of ldq zeroed), padded frames, one and three parts; the FP32 output, when the C ABI is given
    one, equals glu_depthwise's."""
    import ctypes
    from kea_kernels import _lib, lowbit
    g = torch.Generator().manual_seed(b * 1000 + t + c + parts)
    h = torch.randn(b, t, 2 * c, generator=g).to(DEV)
    w = (torch.randn(c, 1, 9, generator=g) / 3).to(DEV)
    bias = (0.1 * torch.randn(c, generator=g)).to(DEV)
    lengths = torch.randint(1, t + 1, (b,), generator=g).to(DEV) if masked else None
    q, qs, ldq = lowbit.glu_depthwise_quantized(h, w, bias, lengths, parts, silu=silu)
    y = lowbit.glu_depthwise(h, w, bias, lengths)
    q2, qs2, ldq2 = lowbit.quantize(y, (y.stride(0), y.stride(1), 1, t), b * t, c, parts, input_silu=silu)
    torch.cuda.synchronize()
    assert ldq == ldq2
    assert torch.equal(q, q2)
    assert torch.equal(qs.view(torch.int32), qs2.view(torch.int32))
    # through the C ABI with the FP32 output requested as well
    yf = torch.full_like(y, float("nan"))
    q3 = torch.full_like(q, 7)
    qs3 = torch.empty_like(qs)
    wc = w.reshape(c, 9).contiguous()
    lens32 = None if lengths is None else lengths.to(torch.int32).contiguous()
    d = _lib.ConvDesc(h=h.data_ptr(), y=yf.data_ptr(), weight=wc.data_ptr(), bias=bias.data_ptr(),
                      lengths=_lib.ptr(lens32), b=b, t=t, c=c, kw=9, flags=_lib.CONV_QUANT_SILU if silu else 0,
                      q=q3.data_ptr(), q_part_stride=b * t * ldq, ldq=ldq, qs=qs3.data_ptr(), qs_part_stride=b * t,
                      parts=parts)
    assert _lib.lib().kea_lowbit_glu_depthwise(ctypes.byref(d), _lib.stream_handle(h.device)) == _lib.OK
    torch.cuda.synchronize()
    assert torch.equal(yf.view(torch.int32), y.view(torch.int32))
    assert torch.equal(q3, q) and torch.equal(qs3.view(torch.int32), qs.view(torch.int32))


def test_glu_depthwise_fused_quantizer_rejects_other_shapes():
    from kea_kernels import lowbit
    h = torch.randn(1, 4, 12, device=DEV)
    with pytest.raises(ValueError):
        lowbit.glu_depthwise_quantized(h, torch.randn(6, 1, 9, device=DEV), None, None, 1)    # C % 4
    with pytest.raises(ValueError):
        lowbit.glu_depthwise_quantized(torch.randn(1, 4, 16, device=DEV), torch.randn(8, 1, 3, device=DEV), None,
                                       None, 1)                                                  # width 3


def _torch_rel_attention(qkv, pos, u, v, heads, lengths=None):
    b, t, w3 = qkv.shape
    d = w3 // 3
    dk = d // heads
    q, k, vv = qkv.view(b, t, 3, heads, dk).unbind(2)
    p = pos.view(2 * t - 1, heads, dk)
    ac = torch.matmul((q + u).transpose(1, 2), k.permute(0, 2, 3, 1))
    bd = E.rel_shift(torch.matmul((q + v).transpose(1, 2), p.permute(1, 2, 0)))
    s = (ac + bd) * (1.0 / math.sqrt(dk))
    if lengths is not None:
        s = s.masked_fill(~(torch.arange(t, device=qkv.device)[None, :] < lengths[:, None])[:, None, None, :],
                          float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), vv.transpose(1, 2)).transpose(1, 2).reshape(b, t, d)


@pytest.mark.parametrize("b,t,heads,dk", [(2, 125, 8, 128), (1, 7, 2, 32), (3, 33, 4, 64), (1, 375, 8, 128),
                                          (2, 64, 1, 32), (16, 125, 8, 128), (40, 70, 4, 64)])
@pytest.mark.parametrize("masked", [False, True])
@torch.inference_mode()
def test_rel_attention_matches_torch(b, t, heads, dk, masked):
    """The fused relative-position attention against the torch sequence it replaces (bias adds, two score matmuls,
    Transformer-XL shift, scale, key mask, softmax, context matmul), FP32 within summation-order rounding."""
    from kea_kernels import lowbit
    g = torch.Generator().manual_seed(b * 100 + t + heads + dk)
    d = heads * dk
    qkv = torch.randn(b, t, 3 * d, generator=g).to(DEV)
    pos = torch.randn(2 * t - 1, d, generator=g).to(DEV)
    u, v = (0.1 * torch.randn(heads, dk, generator=g)).to(DEV), (0.1 * torch.randn(heads, dk, generator=g)).to(DEV)
    lengths = torch.randint(1, t + 1, (b,), generator=g).to(DEV) if masked else None
    got = lowbit.rel_attention(qkv, pos, u, v, heads, lengths)
    want = _torch_rel_attention(qkv, pos, u, v, heads, lengths)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=2e-5)
    # the encoder's own PyTorch route (small batches, long clips) is the same function
    torch.testing.assert_close(E.torch_rel_attention(qkv, pos, u, v, heads, lengths), want, rtol=1e-5, atol=1e-6)
