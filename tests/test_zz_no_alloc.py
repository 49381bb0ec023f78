"""The GEMM entry point that allocates nothing (kea_lowbit_gemm_noalloc), for callers that may not call cudaMalloc:
a real-time recognizer's request path (cudaMalloc can wait for the whole device, with no bound on its latency) or a
host that runs the library inside its own device-memory budget. Its split-K partial sums live in the library's
static 16 MiB device buffer instead of a caller's workspace.

Called through the C ABI and checked against kea_lowbit_gemm (the existing entry point, with a workspace it is
given) on two calls in a row - bit for bit, the tolerance of the other GEMM parity tests without SiLU - at a shape
that splits K through the scratch and at two that do not (a tcgen05 and a register-operand route); two split calls back to back on one stream (programmatic
dependent launch, FP32 output with a residual) against the unsplit GEMM and the oracle; and a shape whose split would
need more than the buffer is refused. This file is collected last, so a run that stops at the first failure has run every other test first.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from kea_kernels import _lib, lowbit
from kea_kernels.binary import bits

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _operands(n: int, k: int, m: int, parts: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    signs = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
    panels = lowbit.prepare_panels(bits.pack_signs(signs).to(DEV), 1, n, k)
    q = torch.randint(-127, 128, (parts, m, k), generator=g, dtype=torch.int8).to(DEV)
    qs = (torch.rand(parts, m, generator=g) * 0.015 + 0.005).to(DEV)
    alpha = (torch.rand(n, generator=g) * 0.04 + 0.01).to(DEV)
    bias = (torch.randn(n, generator=g) * 0.1).to(DEV)
    return panels, q, qs, alpha, bias


def _noalloc(panels, q, qs, alpha, bias, n, k, m, parts, y, acc, flags=0, residual=None, residual_scale=1.0) -> int:
    """kea_lowbit_gemm_noalloc through ctypes on the current stream; returns its status."""
    d = _lib.GemmDesc()
    d.q, d.q_part_stride, d.ldq, d.parts = q.data_ptr(), q.stride(0), q.stride(1), parts
    d.qs, d.qs_part_stride = qs.data_ptr(), qs.stride(0)
    d.panels, d.wbits, d.n, d.k = panels.data_ptr(), 1, n, k
    d.alpha, d.bias = alpha.data_ptr(), bias.data_ptr()
    d.y, d.ldy, d.y_dtype = y.data_ptr(), y.stride(0), _lib.OUT_F16 if y.dtype == torch.float16 else _lib.OUT_F32
    d.acc, d.ld_acc, d.acc_part_stride = acc.data_ptr(), acc.stride(1), acc.stride(0)
    d.m, d.flags = m, flags
    if residual is not None:
        d.residual, d.ld_residual, d.residual_scale = residual.data_ptr(), residual.stride(0), residual_scale
    with torch.cuda.device(y.device):
        return _lib.lib().kea_lowbit_gemm_noalloc(ctypes.byref(d), _lib.stream_handle(y.device))


@pytest.mark.parametrize("n,k,m", [(2048, 4096, 384), (4096, 1024, 125), (1024, 1024, 125)])
def test_noalloc_gemm_equals_gemm_on_two_calls(n, k, m):
    splits = _lib.workspace_bytes(m, n, k, 1, 1) > 0
    assert splits == (m == 384)                        # the first shape goes through the static scratch
    for call in range(2):                              # the second call finds the first call's partial sums
        panels, q, qs, alpha, bias = _operands(n, k, m, 1, 100 * call + m)
        y_free = torch.full((m, n), float("nan"), device=DEV, dtype=torch.float16)
        acc_free = torch.full((1, m, n), -7, device=DEV, dtype=torch.int32)
        assert _noalloc(panels, q, qs, alpha, bias, n, k, m, 1, y_free, acc_free) == _lib.OK
        y_ref = torch.full((m, n), float("nan"), device=DEV, dtype=torch.float16)
        acc_ref = torch.full((1, m, n), -7, device=DEV, dtype=torch.int32)
        lowbit.gemm(q, qs, k, m, panels, 1, n, k, alpha, bias, y_ref, parts=1, acc=acc_ref)   # its own workspace
        torch.cuda.synchronize()
        assert _lib.read_device_error() == 0
        assert torch.equal(acc_free, acc_ref), f"call {call}: accumulators differ"
        assert torch.equal(y_free.view(torch.int16), y_ref.view(torch.int16)), f"call {call}: outputs differ"


def test_noalloc_back_to_back_split_calls_with_residual_and_pdl():
    """Two split-K calls back to back on one stream, programmatic dependent launch on, FP32 output with a residual:
    the second call's partial sums overwrite the first's in the shared scratch only after the first call's finishing
    kernel has read them (stream order, griddepcontrol.wait). Both equal the unsplit GEMM and the oracle bit for bit."""
    import numpy as np
    import kea_oracle as oracle
    n, k, m = 2048, 4096, 384
    assert _lib.workspace_bytes(m, n, k, 1, 1) > 0      # this shape splits K through the scratch
    ops = [_operands(n, k, m, 1, 300 + i) for i in range(2)]
    res = [torch.randn(m, n, generator=torch.Generator().manual_seed(400 + i)).to(DEV) for i in range(2)]
    ys = [torch.full((m, n), float("nan"), device=DEV) for _ in range(2)]
    accs = [torch.full((1, m, n), -7, device=DEV, dtype=torch.int32) for _ in range(2)]
    for i in range(2):                                    # no synchronization between the two calls
        panels, q, qs, alpha, bias = ops[i]
        assert _noalloc(panels, q, qs, alpha, bias, n, k, m, 1, ys[i], accs[i], flags=_lib.FLAG_PDL,
                        residual=res[i], residual_scale=0.5) == _lib.OK
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    for i in range(2):
        panels, q, qs, alpha, bias = ops[i]
        y_unsplit = torch.empty(m, n, device=DEV)
        lowbit.gemm(q, qs, k, m, panels, 1, n, k, alpha, bias, y_unsplit, parts=1, residual=res[i], residual_scale=0.5,
                    workspace=torch.empty(0, dtype=torch.uint8, device=DEV))   # no workspace: the GEMM runs unsplit
        torch.cuda.synchronize()
        assert torch.equal(ys[i].view(torch.int32), y_unsplit.view(torch.int32)), f"call {i}: differs from unsplit"
        w = oracle.unpack(bits.pack_signs(torch.where(torch.rand(n, k, generator=torch.Generator().manual_seed(
            300 + i)) < 0.5, -1, 1).to(torch.int8)).numpy(), 1, k)
        qn, qsn = q.cpu().numpy(), qs.cpu().numpy()
        want_acc = oracle.int_acc(qn, w)
        assert np.array_equal(accs[i].cpu().numpy(), want_acc)
        want = oracle.finish(want_acc, qsn, alpha.cpu().numpy(), bias.cpu().numpy())
        want = (res[i].cpu().numpy() + np.float32(0.5) * want).astype(np.float32)
        assert np.array_equal(ys[i].cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_noalloc_gemm_refuses_a_split_beyond_its_scratch():
    n, k, m, parts = 1024, 8192, 1024, 2                # forced pair, 4 slices x 2 parts x M x N x 4 B = 32 MiB
    panels, q, qs, alpha, bias = _operands(n, k, m, parts, 7)
    y = torch.empty(m, n, device=DEV)
    acc = torch.empty(parts, m, n, device=DEV, dtype=torch.int32)
    status = _noalloc(panels, q, qs, alpha, bias, n, k, m, parts, y, acc, flags=_lib.FLAG_FORCE_PAIR)
    assert status == _lib.SCRATCH_LIMIT
    assert b"16 MiB" in _lib.lib().kea_lowbit_status_string(status)
