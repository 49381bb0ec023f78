"""Generates tests/golden/golden.npz from the kea-kernels reference itself (run here, where the reference is mounted).

The reference's CPU arithmetic for the low-bit GEMM path is its own Python:
  * bits.pack_signs / bits.unpack_signs (src/kea_kernels/binary/bits.py:41-64),
  * formats.pack_ternary / formats.unpack_ternary (src/kea_kernels/formats.py:62-81),
  * the GPU test's oracle `_exact_epilogue` (tests/test_kernels_gpu.py:23-27): integer accumulators from an int64
    matmul of the unpacked codes, then sum_c acc_c * s_c * alpha in FP64;
  * kernels.relayout (src/kea_kernels/binary/kernels.py:726-742), the fragment layout its b1_dot kernels read.
This script imports exactly those functions, draws seeded inputs the way the reference's tests do
(tests/test_kernels_gpu.py:16-20: torch.Generator().manual_seed, signs with p = 0.5), and stores codes, activations,
scales, the reference's int64 accumulators and its FP64 outputs. The oracle (oracle/kea_oracle.py) is checked
against these fixtures by tests/test_oracle_golden.py; the GPU tests check the CUDA library against both.

Two files are written: golden.npz (small cases in full) and golden_config.npz (config-size cases from
config_cases.py: the inputs are redrawn from their seeds by the tests, so only SHA-256 digests of the reference's
codes, INT32 accumulators and FP64 outputs, per-row accumulator sums and a few sampled rows are stored).

Usage: python tests/golden/make_golden.py REFERENCE_ROOT   (or KEA_REFERENCE_ROOT in the environment; the root of a
kea-kernels checkout; needs only torch + numpy)
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "golden.npz"
OUT_CONFIG = HERE / "golden_config.npz"
sys.path.insert(0, str(HERE))
from config_cases import CONFIG_CASES, SAMPLE_ROWS, draw  # noqa: E402

# (name, wbits, n, k, m, parts, bias): config-0/1 style cases at reduced N, ragged shapes, every part count.
CASES = [
    ("b1_n256_k1024_m38_p1", 1, 256, 1024, 38, 1, False),
    ("b1_n128_k1024_m125_p1", 1, 128, 1024, 125, 1, False),
    ("b1_n200_k300_m7_p3", 1, 200, 300, 7, 3, False),
    ("b1_n130_k4096_m16_p2_bias", 1, 130, 4096, 16, 2, True),
    ("b1_n5_k21_m3_p1", 1, 5, 21, 3, 1, False),
    ("t2_n256_k1024_m38_p1", 2, 256, 1024, 38, 1, False),
    ("t2_n136_k520_m19_p3_bias", 2, 136, 520, 19, 3, True),
    ("t2_n64_k13_m1_p2", 2, 64, 13, 1, 2, False),
]


def load_reference(root: Path):
    src = root / "src"
    sys.path.insert(0, str(src))
    from kea_kernels import formats  # noqa: E402  (the reference package)
    from kea_kernels.binary import bits  # noqa: E402
    spec = importlib.util.spec_from_file_location("ref_test_kernels_gpu", root / "tests" / "test_kernels_gpu.py")
    test_mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(test_mod)
    return bits, formats, test_mod._exact_epilogue


def main(root: Path) -> None:
    bits, formats, exact_epilogue = load_reference(root)
    out: dict[str, np.ndarray] = {}
    # Known-answer layout vectors of the reference's own tests (tests/test_formats.py:19-22,51-52).
    one = torch.full((1, 8), -1, dtype=torch.int8)
    one[0, 3] = 1
    out["kat_sign_codes"] = bits.pack_signs(one).numpy()
    out["kat_sign_signs"] = one.numpy()
    tern = torch.tensor([[0, 1, -1, 1]], dtype=torch.int8)
    out["kat_ternary_codes"] = formats.pack_ternary(tern).numpy()
    out["kat_ternary_values"] = tern.numpy()
    # Round trips at odd widths (tests/test_formats.py:14-18,46-50).
    g = torch.Generator().manual_seed(1)
    s = torch.where(torch.rand(5, 21, generator=g) < 0.5, -1, 1).to(torch.int8)
    out["rt_sign_signs"], out["rt_sign_codes"] = s.numpy(), bits.pack_signs(s).numpy()
    t = torch.randint(-1, 2, (4, 13), generator=g, dtype=torch.int8)
    out["rt_ternary_values"], out["rt_ternary_codes"] = t.numpy(), formats.pack_ternary(t).numpy()
    # The reference's mma fragment layout of sign bits (src/kea_kernels/binary/kernels.py:726-742), which its own
    # b1_dot kernels read: ragged N and K (padding), pinning oracle/ref_kernels.py's restatement.
    from kea_kernels.binary import kernels as ref_kernels  # noqa: E402  (the reference package)
    lay = torch.where(torch.rand(20, 300, generator=g) < 0.5, -1, 1).to(torch.int8)
    out["relayout_signs"] = lay.numpy()
    out["relayout_words"] = ref_kernels.relayout((lay > 0).to(torch.uint8)).numpy()

    names = []
    for name, wbits, n, k, m, parts, has_bias in CASES:
        g = torch.Generator().manual_seed(wbits * 100003 + n * 1009 + k * 31 + m * 7 + parts)
        if wbits == 1:
            w = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
            codes = bits.pack_signs(w)
            dense = bits.unpack_signs(codes, k)
        else:
            u = torch.rand(n, k, generator=g)
            w = torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8)
            codes = formats.pack_ternary(w)
            dense = formats.unpack_ternary(codes, k)
        assert torch.equal(dense, w)
        q = torch.randint(-127, 128, (parts, m, k), generator=g, dtype=torch.int8)
        qs = (torch.rand(parts, m, generator=g) * 0.015 + 0.005).float()
        alpha = (torch.rand(n, generator=g) * 0.04 + 0.01).half().float()   # fp16-valued, stored as FP32
        bias = (torch.randn(n, generator=g) * 0.1).float() if has_bias else None
        acc = torch.stack([q[c].to(torch.int64) @ dense.to(torch.int64).t() for c in range(parts)])
        y64 = exact_epilogue(q, qs, dense, alpha, parts)          # the reference test's FP64 oracle
        if bias is not None:
            y64 = y64 + bias.double()[None, :]
        names.append(name)
        out[f"{name}/codes"] = codes.numpy()
        out[f"{name}/q"] = q.numpy()
        out[f"{name}/qs"] = qs.numpy()
        out[f"{name}/alpha"] = alpha.numpy()
        if bias is not None:
            out[f"{name}/bias"] = bias.numpy()
        out[f"{name}/acc"] = acc.to(torch.int32).numpy()
        out[f"{name}/y64"] = y64.numpy()
        out[f"{name}/meta"] = np.array([wbits, n, k, m, parts, int(has_bias)], dtype=np.int64)
    out["cases"] = np.array(names)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(names)} GEMM cases)")
    config_fixtures(bits, formats, exact_epilogue)


def digest(a: np.ndarray) -> np.ndarray:
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), dtype=np.uint8)


def config_fixtures(bits, formats, exact_epilogue) -> None:
    out: dict[str, np.ndarray] = {}
    for name, wbits, n, k, m, parts in CONFIG_CASES:
        w, q, qs, alpha = draw(wbits, n, k, m, parts)
        codes = bits.pack_signs(w) if wbits == 1 else formats.pack_ternary(w)
        dense = bits.unpack_signs(codes, k) if wbits == 1 else formats.unpack_ternary(codes, k)
        assert torch.equal(dense, w)
        acc = torch.stack([q[c].to(torch.int64) @ dense.to(torch.int64).t() for c in range(parts)])
        y64 = exact_epilogue(q, qs, dense, alpha, parts)
        acc32 = acc.to(torch.int32).numpy()
        out[f"{name}/meta"] = np.array([wbits, n, k, m, parts], dtype=np.int64)
        out[f"{name}/codes_sha256"] = digest(codes.numpy())
        out[f"{name}/acc_sha256"] = digest(acc32)
        out[f"{name}/y64_sha256"] = digest(y64.numpy())
        out[f"{name}/acc_rowsum"] = acc.sum(dim=2).numpy()
        out[f"{name}/acc_rows"] = acc32[:, list(SAMPLE_ROWS)]
        out[f"{name}/y64_rows"] = y64.numpy()[list(SAMPLE_ROWS)]
        print(f"{name}: reference accumulators and FP64 outputs recorded")
    out["cases"] = np.array([c[0] for c in CONFIG_CASES])
    np.savez_compressed(OUT_CONFIG, **out)
    print(f"wrote {OUT_CONFIG} ({OUT_CONFIG.stat().st_size} bytes)")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KEA_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (or set KEA_REFERENCE_ROOT)")
    main(Path(root))
