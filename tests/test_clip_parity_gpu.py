"""Accumulator parity of a whole clip: one synthetic 10 s clip (log-mel N(0, 1) [1, 128, 1000] ->
125 encoder frames) through the 24-layer random-init 1-bit FastConformer. Every low-bit GEMM the clip issues - 8 per
layer at M = 125 (fused QKV, out, 2 x FF up, 2 x FF down, conv pw1, pw2) plus linear_pos at M = 249, 216 in all - is
recorded with its INT8 parts and scales (the quantizer's output as the GEMM consumed them: from the quantizer inside
the GEMM kernel where the library fuses it, from the conv kernel for pw2, else from the quantizer kernel) and its INT32
accumulators, and checked on the host:
  * the accumulators equal the reference's exact integer product of those parts and the layer's codes bit for bit
    (its GPU test oracle `_exact_epilogue`, tests/test_kernels_gpu.py:23-27, restated by the oracle and pinned to the
    reference's own outputs at config size by the golden fixtures);
  * the outputs equal the oracle's FP32 epilogue of those accumulators bit for bit (SiLU epilogues within rtol 2e-6,
    the reference test's tolerance), with each skip connection added as the unfused residual + scale * y.
The call sites follow the reference's fusions (src/kea_kernels/ternary/transforms.py:69-97, layer_fusions4.py:52-94)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
from kea_kernels import encoder as E
from kea_kernels import lowbit

pytestmark = pytest.mark.gpu
DEV = "cuda"


@torch.inference_mode()
def test_config2_clip_accumulators_are_bit_exact(monkeypatch):
    enc = E.FastConformerEncoder(layers=24, wbits=1, parts=1, seed=0, device=DEV, keep_dense=True)
    layers = {}
    for i, layer in enumerate(enc.layers):
        for name, (w, bias) in layer.weights.items():
            lin = layer.lin[name]
            layers[lin.panels.data_ptr()] = (f"{i}.{name}", w.w.cpu().numpy(), lin.scale.cpu().numpy(),
                                             None if lin.bias is None else lin.bias.cpu().numpy())
    records = []
    real_gemm = lowbit.gemm

    def recording_gemm(q, qs, ldq, m, panels, wbits, n, k, alpha, bias, y, *, parts, silu=False, residual=None,
                       residual_scale=1.0, **kw):
        assert kw.get("acc") is None
        acc = torch.empty(parts, m, n, dtype=torch.int32, device=y.device)
        res = None if residual is None else residual[:m, :n].clone()
        real_gemm(q, qs, ldq, m, panels, wbits, n, k, alpha, bias, y, parts=parts, silu=silu, acc=acc,
                  residual=residual, residual_scale=residual_scale, **kw)
        records.append(dict(panels=panels.data_ptr(), q=q[:, :m, :k].clone(), qs=qs[:, :m].clone(), acc=acc,
                            y=y[:m, :n].clone(), res=res, scale=residual_scale, silu=silu))

    real_project = lowbit.project

    def recording_project(x, rows, m, k, panels, wbits, n, alpha, bias, y, *, parts, silu=False, residual=None,
                          residual_scale=1.0, **kw):
        assert kw.get("acc") is None
        acc = torch.empty(parts, m, n, dtype=torch.int32, device=y.device)
        res = None if residual is None else residual[:m, :n].clone()
        q, qs, ldq = real_project(x, rows, m, k, panels, wbits, n, alpha, bias, y, parts=parts, silu=silu, acc=acc,
                                  residual=residual, residual_scale=residual_scale, **kw)
        records.append(dict(panels=panels.data_ptr(), q=q[:, :m, :k].clone(), qs=qs[:, :m].clone(), acc=acc,
                            y=y[:m, :n].clone(), res=res, scale=residual_scale, silu=silu))
        return q, qs, ldq

    monkeypatch.setattr(lowbit, "gemm", recording_gemm)
    monkeypatch.setattr(lowbit, "project", recording_project)
    mel = torch.randn(1, 128, 1000, generator=torch.Generator().manual_seed(2)).to(DEV)
    out = enc(mel)
    torch.cuda.synchronize()
    assert out.shape == (1, 125, 1024) and bool(torch.isfinite(out).all())
    assert len(records) == 24 * 9                      # 8 GEMMs per layer + linear_pos (first use of this length)
    seen = set()
    for r in records:
        name, w, alpha, bias = layers[r["panels"]]
        seen.add(name)
        q, qs, acc = r["q"].cpu().numpy(), r["qs"].cpu().numpy(), r["acc"].cpu().numpy()
        m = q.shape[1]
        assert m == (249 if name.endswith("linear_pos") else 125), name
        want_acc = oracle.int_acc(q, w)
        assert np.array_equal(acc, want_acc), f"{name}: {(acc != want_acc).sum()} accumulators differ"
        want = oracle.finish(want_acc, qs, alpha, bias, oracle.SILU if r["silu"] else 0)
        if r["res"] is not None:
            res = r["res"].cpu().numpy()
            want = (res + np.float32(r["scale"]) * want).astype(np.float32)   # two FP32 roundings, as unfused
        y = r["y"].cpu().numpy()
        if r["silu"]:
            np.testing.assert_allclose(y, want, rtol=2e-6, atol=1e-6, err_msg=name)
        else:
            assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), \
                f"{name}: {(y != want).sum()} outputs differ"
    assert len(seen) == 24 * 9                          # every projection of every layer was checked
