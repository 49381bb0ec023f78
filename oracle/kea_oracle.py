"""ORACLE - TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, never by the product
(kea-kernels_b200/). It restates kea-kernels' low-bit GEMM arithmetic on the CPU, as the checker of the CUDA library:

  * numpy restatements of the export codes (src/kea_kernels/binary/bits.py:41-64: 1-bit signs, LSB first, 1 = +1;
    src/kea_kernels/formats.py:62-81: 2-bit fields 00 / 01 / 10 = 0 / +1 / -1) and of the exact integer product
    (tests/test_kernels_gpu.py:23-27: an integer matmul of the unpacked codes; here float64 BLAS, exact because every
    partial sum is an integer below 2^53);
  * the FP32 epilogue comb<P> (src/kea_kernels/binary/kernels_parts.py:30-45) and the residual INT8 quantizer
    (src/kea_kernels/ternary/fused_kernels.py:31-50), through the plain-C restatement in kea_oracle.c
    (correctly rounded fmaf, no contraction), with a numpy restatement for P = 1 to cross-check it;
  * the B200 panel layout, to check the device relayout byte for byte.
Pinned against the reference: tests/golden/make_golden.py runs the reference's own bits.py / formats.py and its test
oracle `_exact_epilogue` and stores the results as fixtures; tests/test_oracle_golden.py checks this module on them.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libkea_oracle.so"

SILU, ORDER1 = 1, 2


def build(force: bool = False) -> Path:
    src = HERE / "kea_oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-f", str(HERE / "Makefile")] + (["-B"] if force else []), check=True)
    return LIB


_c = None


def clib() -> ctypes.CDLL:
    global _c
    if _c is None:
        build()
        lib = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        lib.kea_oracle_unpack.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        lib.kea_oracle_unpack.restype = ctypes.c_int
        lib.kea_oracle_panels.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        lib.kea_oracle_panels.restype = None
        lib.kea_oracle_gemm.argtypes = [P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P, ctypes.c_long, P,
                                        ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int]
        lib.kea_oracle_gemm.restype = None
        lib.kea_oracle_quantize.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P]
        lib.kea_oracle_quantize.restype = ctypes.c_int
        lib.kea_oracle_finish_all.argtypes = [P, P, ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P,
                                              ctypes.c_int, P]
        lib.kea_oracle_finish_all.restype = None
        lib.kea_oracle_finish.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_float, P]
        lib.kea_oracle_finish.restype = ctypes.c_float
        _c = lib
    return _c


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---- codes ----------------------------------------------------------------------------------------------------

def pack_signs(signs: np.ndarray) -> np.ndarray:
    """int8 {-1, +1} [N, K] -> uint8 [N, ceil(K/8)], code k at bit k % 8 of byte k // 8."""
    if signs.dtype != np.int8 or signs.ndim != 2 or not np.isin(signs, (-1, 1)).all():
        raise ValueError("expected 2-D int8 signs in {-1, +1}")
    return np.packbits(signs == 1, axis=1, bitorder="little")


def unpack_signs(codes: np.ndarray, k: int) -> np.ndarray:
    bits = np.unpackbits(codes, axis=1, bitorder="little")
    if bits[:, k:].any():
        raise ValueError("invalid packed codes: nonzero tail padding")
    return (2 * bits[:, :k].astype(np.int8) - 1).astype(np.int8)


def pack_ternary(codes: np.ndarray) -> np.ndarray:
    """int8 {-1, 0, 1} [N, K] -> uint8 [N, ceil(K/4)]: 0 -> 00, +1 -> 01, -1 -> 10 at bits 2 (k % 4)."""
    if codes.dtype != np.int8 or codes.ndim != 2 or not np.isin(codes, (-1, 0, 1)).all():
        raise ValueError("expected 2-D int8 codes in {-1, 0, 1}")
    n, k = codes.shape
    width = -(-k // 4)
    fields = np.zeros((n, 4 * width), dtype=np.uint8)
    fields[:, :k] = np.where(codes == 1, 1, np.where(codes == -1, 2, 0))
    f = fields.reshape(n, width, 4)
    return (f[..., 0] | (f[..., 1] << 2) | (f[..., 2] << 4) | (f[..., 3] << 6)).astype(np.uint8)


def unpack_ternary(packed: np.ndarray, k: int) -> np.ndarray:
    f = np.stack([(packed >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(packed.shape[0], -1)
    if (f == 3).any() or f[:, k:].any():
        raise ValueError("invalid packed codes")
    f = f[:, :k]
    return ((f == 1).astype(np.int8) - (f == 2).astype(np.int8)).astype(np.int8)


def unpack(codes: np.ndarray, wbits: int, k: int) -> np.ndarray:
    return unpack_signs(codes, k) if wbits == 1 else unpack_ternary(codes, k)


def unpack_c(codes: np.ndarray, wbits: int, n: int, k: int) -> tuple[np.ndarray, int]:
    w = np.zeros((n, k), dtype=np.int8)
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    status = clib().kea_oracle_unpack(_p(codes), wbits, n, k, _p(w))
    return w, status


def panels(codes: np.ndarray, wbits: int, n: int, k: int) -> np.ndarray:
    nt, kb = -(-n // 128), -(-k // 128)
    out = np.zeros(nt * kb * wbits * 128 * 16, dtype=np.uint8)
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    clib().kea_oracle_panels(_p(codes), wbits, n, k, _p(out))
    return out


# ---- the product ----------------------------------------------------------------------------------------------

def int_acc(q: np.ndarray, w: np.ndarray) -> np.ndarray:
    """q int8 [P, M, >=K], w int8 [N, K] -> exact INT32 [P, M, N] via float64 BLAS (partial sums < 2^53)."""
    k = w.shape[1]
    wt = w.astype(np.float64).T
    out = np.stack([q[p, :, :k].astype(np.float64) @ wt for p in range(q.shape[0])])
    return out.astype(np.int64).astype(np.int32)


def int_acc_f32(q: np.ndarray, w: np.ndarray) -> np.ndarray:
    """The same exact INT32 [P, M, N] through FP32 BLAS (numpy's sgemm, every host thread): exact because each
    product and every partial sum is an integer of magnitude <= 128 K < 2^24 (K <= 131072), which FP32 holds exactly in
    any summation order. The strong CPU baseline of the reference's arithmetic."""
    k = w.shape[1]
    if k > 131072:
        raise ValueError("FP32 accumulation is exact only for K <= 131072")
    wt = np.ascontiguousarray(w.astype(np.float32).T)
    out = np.stack([q[p, :, :k].astype(np.float32) @ wt for p in range(q.shape[0])])
    return out.astype(np.int32)


def gemm_blas(codes: np.ndarray, wbits: int, q: np.ndarray, qs: np.ndarray, alpha: np.ndarray) -> np.ndarray:
    """The reference's CPU path for one part without bias - unpack the export codes, exact integer GEMM, the comb<1>
    epilogue, FP16 output - as the strong CPU baseline: the GEMM in FP32 BLAS (exact, as int_acc_f32) and the epilogue
    as two in-place FP32 multiplies (one IEEE rounding each, as epilogue_x1), both in PyTorch's multi-threaded CPU
    kernels (torch.get_num_threads() threads). Returns y FP16 [M, N]."""
    import torch
    k = q.shape[2]
    w = torch.from_numpy(unpack(codes, wbits, k)).to(torch.float32)
    acc = torch.from_numpy(q[0, :, :k]).to(torch.float32) @ w.t()          # exact integers in FP32
    acc.mul_(torch.from_numpy(qs[0]).to(torch.float32)[:, None]).mul_(torch.from_numpy(alpha).to(torch.float32)[None, :])
    return acc.half().numpy()


def gemm(q: np.ndarray, qs: np.ndarray, w: np.ndarray, alpha: np.ndarray, bias: np.ndarray | None = None,
         flags: int = 0, threads: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """(y FP32 [M, N], acc INT32 [P, M, N]) from q int8 [P, M, ldq], qs FP32 [P, M], w int8 [N, K]."""
    parts, m, ldq = q.shape
    n, k = w.shape
    q = np.ascontiguousarray(q, dtype=np.int8)
    qs = np.ascontiguousarray(qs, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.int8)
    alpha = np.ascontiguousarray(alpha, dtype=np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.zeros((m, n), dtype=np.float32)
    acc = np.zeros((parts, m, n), dtype=np.int32)
    clib().kea_oracle_gemm(_p(q), m * ldq, ldq, parts, _p(qs), m, _p(w), n, k, _p(alpha), _p(bias), m, flags, _p(y),
                           _p(acc), threads)
    return y, acc


def finish(acc: np.ndarray, qs: np.ndarray, alpha: np.ndarray, bias: np.ndarray | None = None,
           flags: int = 0) -> np.ndarray:
    """The FP32 epilogue alone: acc INT32 [P, M, N], qs FP32 [P, M] -> y FP32 [M, N] (kea_oracle.c)."""
    parts, m, n = acc.shape
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    qs = np.ascontiguousarray(qs[:parts, :m], dtype=np.float32)
    alpha = np.ascontiguousarray(alpha, dtype=np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.zeros((m, n), dtype=np.float32)
    clib().kea_oracle_finish_all(_p(acc), _p(qs), m, parts, m, n, _p(alpha), _p(bias), flags, _p(y))
    return y


def reference(q: np.ndarray, qs: np.ndarray, w: np.ndarray, alpha: np.ndarray, bias: np.ndarray | None = None,
              flags: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(y FP32 [M, N], acc INT32 [P, M, N]): BLAS-exact accumulators + the C epilogue (fast for large shapes)."""
    acc = int_acc(q, w)
    return finish(acc, qs, alpha, bias, flags), acc


def epilogue_x1(acc0: np.ndarray, qs0: np.ndarray, alpha: np.ndarray) -> np.ndarray:
    """comb<1> without bias in numpy: RN(RN(float(acc) * s) * alpha), each product one FP32 rounding."""
    r = acc0.astype(np.float32) * qs0.astype(np.float32)[:, None]
    return (r * alpha.astype(np.float32)[None, :]).astype(np.float32)


def quantize(x: np.ndarray, parts: int, ldq: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """x FP32 [M, K] -> (q int8 [parts, M, ldq], qs FP32 [parts, M]) with IEEE division (kea_oracle.c)."""
    m, k = x.shape
    ldq = -(-k // 16) * 16 if ldq is None else ldq
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.zeros((parts, m, ldq), dtype=np.int8)
    qs = np.zeros((parts, m), dtype=np.float32)
    if clib().kea_oracle_quantize(_p(x), m, k, parts, _p(q), ldq, _p(qs)) != 0:
        raise MemoryError("oracle quantize")
    return q, qs


def quantize_np(x: np.ndarray, parts: int, ldq: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """The same quantizer in numpy float32 (cross-check of the C restatement)."""
    m, k = x.shape
    ldq = -(-k // 16) * 16 if ldq is None else ldq
    r = x.astype(np.float32).copy()
    q = np.zeros((parts, m, ldq), dtype=np.int8)
    qs = np.zeros((parts, m), dtype=np.float32)
    for p in range(parts):
        amax = np.abs(r).max(axis=1)
        s = np.maximum(amax / np.float32(127.0), np.float32(1e-30)).astype(np.float32)
        v = np.rint(r / s[:, None]).astype(np.float32)
        q[p, :, :k] = v.astype(np.int8)
        qs[p] = s
        r = (r - (v * s[:, None]).astype(np.float32)).astype(np.float32)
    return q, qs


def to_f16(y: np.ndarray) -> np.ndarray:
    """FP32 -> FP16 round-to-nearest-even (numpy's cast)."""
    return y.astype(np.float16)
