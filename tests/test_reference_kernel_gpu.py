"""The reference's own b1_dot kernels as a checker on the B200: its SM120 mma.sync sources, written by its own
generator and tile table and compiled unchanged for sm_100a (oracle/ref_kernels.py, into oracle/_ref/), run on the
same signs, INT8 parts and scales as this library, through the reference's own argument list. Their FP32 outputs -
the reference's comb<P> epilogue (src/kea_kernels/binary/kernels_parts.py:30-45), with and without bias - must equal
the library's bit for bit: config 0 at one part, one-part shapes with split K, and tuned three-part shapes with and
without the reference's cluster split-K exchange (src/kea_kernels/binary/configs.py:17-36).

Skipped when the kernels were not built (they are built, beside the library, where the reference's sources are
mounted: `python oracle/ref_kernels.py build --reference <root>`, also run by __graft_entry__.build())."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kea_oracle as oracle
import ref_kernels
from kea_kernels import _lib, lowbit
from kea_kernels.binary import bits

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = [(1, 4096, 1024, 125), (1, 1024, 4096, 125), (1, 4096, 1024, 16), (3, 1024, 4096, 126), (3, 1024, 4096, 38),
         (3, 4096, 1024, 368), (3, 1024, 1024, 38), (3, 2048, 1024, 256)]


def _case(parts, n, k, m):
    for c in ref_kernels.cases():
        if (c["parts"], c["n"], c["k"], c["m"]) == (parts, n, k, m):
            return c
    pytest.skip("the reference's kernels were not built here (oracle/ref_kernels.py build)")


@pytest.mark.parametrize("parts,n,k,m", CASES)
@pytest.mark.parametrize("with_bias", [False, True])
@torch.inference_mode()
def test_reference_kernel_equals_the_library_bitwise(parts, n, k, m, with_bias):
    case = _case(parts, n, k, m)
    g = torch.Generator().manual_seed(parts * 1000 + n + k + m)
    signs = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
    ldq = -(-k // 16) * 16
    q = torch.zeros(parts, m, ldq, dtype=torch.int8)
    q[:, :, :k] = torch.randint(-127, 128, (parts, m, k), generator=g, dtype=torch.int8)
    qs = (torch.rand(parts, m, generator=g) * 0.015 + 0.005).float()
    alpha = (torch.rand(n, generator=g) * 0.04 + 0.01).half().float()
    bias = (torch.randn(n, generator=g) * 0.1).float() if with_bias else None
    qd, qsd, ad = q.to(DEV), qs.to(DEV), alpha.to(DEV)
    bd = None if bias is None else bias.to(DEV)

    words = torch.from_numpy(ref_kernels.relayout(signs.numpy())).to(DEV)
    ws = torch.zeros(case["workspace_ints"], dtype=torch.int32, device=DEV) if case["workspace_ints"] else None
    y_ref = torch.full((m, n), float("nan"), device=DEV)
    kernel = ref_kernels.RefKernel(case)
    kernel.launch(qd, qsd, words, ad, bd, y_ref, m, n, k, ws, torch.cuda.current_stream().cuda_stream)

    panels = lowbit.prepare_panels(bits.pack_signs(signs).to(DEV), 1, n, k)
    y = torch.full((m, n), float("nan"), device=DEV)
    lowbit.gemm(qd, qsd, ldq, m, panels, 1, n, k, ad, bd, y, parts=parts)
    torch.cuda.synchronize()
    assert _lib.read_device_error() == 0
    assert torch.equal(y_ref.view(torch.int32), y.view(torch.int32)), \
        f"{case['name']}: {(y_ref != y).sum().item()} outputs differ"
    # and both equal the oracle's epilogue of the exact accumulators
    want = oracle.reference(q[:, :, :k].numpy(), qs.numpy(), signs.numpy(), alpha.numpy(),
                            None if bias is None else bias.numpy())[0]
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
