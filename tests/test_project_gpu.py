"""kea_lowbit_project: quantize + GEMM in one call (the reference's Int8MmaLayer.project, src/kea_kernels/binary/
layer.py:118-151). Asked to fuse, where the shape allows, the quantizer runs inside the GEMM kernel: thread-block
clusters of 8 CTAs quantize the token rows one warp a row into a scratch block and read it back as their activation
boxes (by default the quantizer kernel and the GEMM run back to back, the faster form measured on B200). The fused
form must give, bit for bit, the parts of the quantizer kernel with KEA_QUANT_NARROW_ROWS (its reduction order) and
the GEMM of those parts - codes, scales, pre-norm output, INT32 accumulators and outputs - and, without a LayerNorm
(whose FP32 sums depend on the order), the oracle's quantizer and exact product. Shapes outside the fused form run
the two kernels and equal the two plain calls."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
from kea_kernels import _lib, lowbit
from kea_kernels import formats
from kea_kernels.binary import bits

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(wbits, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    if wbits == 1:
        w = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
        codes = bits.pack_signs(w)
    else:
        u = torch.rand(n, k, generator=g)
        w = torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8)
        codes = formats.pack_ternary(w)
    panels = lowbit.prepare_panels(codes.to(DEV), wbits, n, k)
    alpha = (torch.rand(n, generator=g) * 0.04 + 0.01).to(DEV)
    bias = (torch.randn(n, generator=g) * 0.1).to(DEV)
    return w, panels, alpha, bias


def _norm(k, seed):
    g = torch.Generator().manual_seed(seed)
    norm = torch.nn.LayerNorm(k)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(k, generator=g) + 0.5)
        norm.bias.copy_(torch.randn(k, generator=g) * 0.1)
    return norm.to(DEV)


def _bits(t):
    return t.view(torch.int16) if t.dtype == torch.float16 else t.view(torch.int32)


CASES = [  # (wbits, n, k, m, options)
    (1, 4096, 1024, 125, dict(norm=True, silu=True)),
    (1, 3072, 1024, 125, dict(norm=True)),
    (1, 2048, 1024, 128, dict(norm=True, pre=True)),
    (1, 1024, 1024, 125, dict(input_silu=True, residual=True)),
    (2, 4096, 1024, 37, dict(norm=True, f16=True)),
    (2, 1024, 512, 33, dict(pre=True)),   # the per-tile route starts above 32 tokens (swap / CUDA-core below)
    (1, 2048, 256, 64, dict(norm=True, residual=True)),
    (1, 4096, 1024, 100, dict(t=50)),   # two clips of 50 frames: rows through the batch stride
    (1, 1000, 1024, 125, dict(norm=True)),   # ragged N: 32 channel tiles, the last one partly past N
]


@pytest.mark.parametrize("wbits,n,k,m,opt", CASES)
@torch.inference_mode()
def test_fused_project_equals_narrow_quantizer_and_gemm(wbits, n, k, m, opt):
    seed = wbits * 7 + n + k + m
    w, panels, alpha, bias = _layer(wbits, n, k, seed)
    g = torch.Generator().manual_seed(seed + 1)
    t = opt.get("t", m)
    x = (torch.randn(m // t, t, k, generator=g) * 2 + 0.3).to(DEV)
    if t != m:   # a strided batch: every clip's rows 2 k apart
        big = torch.zeros(m // t, t, 2 * k, device=DEV)
        big[:, :, :k] = x
        x = big[:, :, :k]
    rows = (x.stride(0), x.stride(1), 1, t)
    norm = _norm(k, 3) if opt.get("norm") else None
    pre = _norm(k, 4) if opt.get("pre") else None
    res = torch.randn(m, n, generator=g).to(DEV) if opt.get("residual") else None
    out = torch.float16 if opt.get("f16") else torch.float32
    kw = dict(norm=norm, input_silu=opt.get("input_silu", False), pre_norm=pre)
    ep = dict(silu=opt.get("silu", False), residual=res, residual_scale=0.5 if res is not None else 1.0)

    normed = torch.full((m, k), float("nan"), device=DEV) if pre is not None else None
    y = torch.full((m, n), float("nan"), device=DEV, dtype=out)
    acc = torch.full((1, m, n), -7, device=DEV, dtype=torch.int32)
    q, qs, ldq = lowbit.project(x, rows, m, k, panels, wbits, n, alpha, bias, y, parts=1, normed=normed, acc=acc,
                                require_fused=True, **kw, **ep)

    normed2 = torch.full((m, k), float("nan"), device=DEV) if pre is not None else None
    q2, qs2, ldq2 = lowbit.quantize(x, rows, m, k, 1, narrow_rows=True, normed=normed2, **kw)
    y2 = torch.full((m, n), float("nan"), device=DEV, dtype=out)
    acc2 = torch.full((1, m, n), -7, device=DEV, dtype=torch.int32)
    lowbit.gemm(q2, qs2, ldq2, m, panels, wbits, n, k, alpha, bias, y2, parts=1, acc=acc2, **ep)
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    assert ldq == ldq2 and torch.equal(q, q2)
    assert torch.equal(qs.view(torch.int32), qs2.view(torch.int32))
    if pre is not None:
        assert torch.equal(normed.view(torch.int32), normed2.view(torch.int32))
    assert torch.equal(acc, acc2)
    assert torch.equal(_bits(y), _bits(y2))
    # and the accumulators are the exact product of the parts
    want = oracle.int_acc(q[:, :, :k].cpu().numpy(), w.numpy())
    assert np.array_equal(acc.cpu().numpy(), want)


@pytest.mark.parametrize("m,n", [(125, 4096), (40, 2048)])
@torch.inference_mode()
def test_fused_project_without_layernorm_equals_the_oracle(m, n):
    k = 1024
    w, panels, alpha, _ = _layer(1, n, k, m + n)
    x = (torch.randn(m, k, generator=torch.Generator().manual_seed(m)) * torch.rand(m, 1) * 4).to(DEV)
    y = torch.empty(m, n, device=DEV)
    acc = torch.empty(1, m, n, device=DEV, dtype=torch.int32)
    q, qs, ldq = lowbit.project(x, (0, k, 1, m), m, k, panels, 1, n, alpha, None, y, parts=1, acc=acc,
                                require_fused=True)
    torch.cuda.synchronize()
    want_q, want_qs = oracle.quantize(x.cpu().numpy(), 1, ldq)
    assert np.array_equal(q.cpu().numpy(), want_q)
    assert np.array_equal(qs.cpu().numpy().view(np.uint32), want_qs.view(np.uint32))
    want_acc = oracle.int_acc(want_q[:, :, :k], w.numpy())
    assert np.array_equal(acc.cpu().numpy(), want_acc)
    want_y = oracle.finish(want_acc, want_qs, alpha.cpu().numpy(), None)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want_y.view(np.uint32))


@pytest.mark.parametrize("wbits,n,k,m,parts", [(1, 4096, 1024, 300, 1), (1, 1024, 4096, 125, 1), (2, 4096, 1024, 125, 2),
                                               (1, 4096, 1000, 125, 1), (1, 1056, 1024, 125, 1), (1, 4096, 1024, 16, 1)])
@torch.inference_mode()
def test_project_outside_the_fused_form_equals_the_two_calls(wbits, n, k, m, parts):
    """M above one token tile, K above 1024 or not a multiple of 128, two parts, channel tiles that do not fill
    clusters, the swapped-operand route at M 16: quantizer then GEMM, the plain calls' bits."""
    w, panels, alpha, bias = _layer(wbits, n, k, n + k + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + k)).to(DEV)
    norm = _norm(k, 5)
    y = torch.full((m, n), float("nan"), device=DEV)
    with pytest.raises(ValueError):
        lowbit.project(x, (0, k, 1, m), m, k, panels, wbits, n, alpha, bias, y, parts=parts, norm=norm,
                       require_fused=True)
    q, qs, ldq = lowbit.project(x, (0, k, 1, m), m, k, panels, wbits, n, alpha, bias, y, parts=parts, norm=norm)
    q2, qs2, ldq2 = lowbit.quantize(x, (0, k, 1, m), m, k, parts, norm=norm)
    y2 = torch.full((m, n), float("nan"), device=DEV)
    lowbit.gemm(q2, qs2, ldq2, m, panels, wbits, n, k, alpha, bias, y2, parts=parts)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(qs.view(torch.int32), qs2.view(torch.int32))
    assert torch.equal(y.view(torch.int32), y2.view(torch.int32))


@torch.inference_mode()
def test_project_takes_the_two_kernels_unless_asked_to_fuse():
    """The default form is the quantizer kernel then the GEMM (the faster on B200): on a shape the fused form serves,
    project() without fuse gives the plain calls' bits, including the quantizer's own LayerNorm reduction order."""
    wbits, n, k, m = 1, 3072, 1024, 125
    _, panels, alpha, bias = _layer(wbits, n, k, 77)
    x = (torch.randn(m, k, generator=torch.Generator().manual_seed(78)) * 3 + 1).to(DEV)
    norm = _norm(k, 8)
    y = torch.empty(m, n, device=DEV)
    q, qs, ldq = lowbit.project(x, (0, k, 1, m), m, k, panels, wbits, n, alpha, bias, y, parts=1, norm=norm, pdl=True)
    q2, qs2, ldq2 = lowbit.quantize(x, (0, k, 1, m), m, k, 1, norm=norm)
    y2 = torch.empty(m, n, device=DEV)
    lowbit.gemm(q2, qs2, ldq2, m, panels, wbits, n, k, alpha, bias, y2, parts=1, pdl=True)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(qs.view(torch.int32), qs2.view(torch.int32))
    assert torch.equal(y.view(torch.int32), y2.view(torch.int32))


@torch.inference_mode()
def test_fused_projects_back_to_back_under_pdl_and_in_a_graph():
    """A chain of fused projections on one stream with programmatic dependent launch - each reading the previous
    one's output - captured in a CUDA graph and replayed: the same bits as the chain run call by call without PDL."""
    k = n = 1024
    m = 125
    layers = [_layer(1, n, k, 50 + i) for i in range(4)]
    norm = _norm(k, 6)
    x0 = torch.randn(m, k, generator=torch.Generator().manual_seed(9)).to(DEV)

    def chain(pdl):
        x = x0
        for _, panels, alpha, bias in layers:
            y = torch.empty(m, n, device=DEV)
            lowbit.project(x, (0, k, 1, m), m, k, panels, 1, n, alpha, bias, y, parts=1, norm=norm, pdl=pdl,
                           require_fused=True)
            x = y
        return x

    want = chain(False)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        chain(True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            got = chain(True)
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
