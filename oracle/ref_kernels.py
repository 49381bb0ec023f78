"""TEST INFRASTRUCTURE ONLY: the reference's own b1_dot kernels, built for the B200 and run beside the library as a
checker and a baseline - never as the product, which neither imports nor loads anything here.

The reference compiles its SM120 kernels at run time with NVRTC (src/kea_kernels/_nvrtc.py:81-100) from sources its
generator writes (src/kea_kernels/binary/kernels.py:702-715 for the three-part b1_dot that layer.dot launches,
src/kea_kernels/binary/kernels_parts.py:115 for the P-part variant of layer_parts.dot_parts). Its tile table
(src/kea_kernels/binary/configs.py:16-58) picks a DotConfig per shape; the launch geometry (grid, threads, shared
bytes, split-K workspace) comes from that DotConfig (kernels.py:640-700).

Build (only where the reference's sources are mounted; the GPU box receives the built files):
    python oracle/ref_kernels.py build --reference <reference project root>
runs the reference's own generator and table for every case below, writes each source and an nvcc-built cubin
(-gencode arch=compute_100a,code=sm_100a, the reference's options --std=c++17 --fmad=false; the kernels use the
legacy mma.sync INT8 path, which sm_100a still executes) and a manifest of launch geometries into oracle/_ref/b1dot/,
which git ignores. Nothing of the reference is copied into the repository.

At run time (tests/test_reference_kernel_gpu.py, oracle/time_ref_kernels.py): `cases()` reads the manifest,
`RefKernel` loads a cubin through the CUDA driver and launches it with the reference's argument list
(src/kea_kernels/binary/layer.py:196-203), and `relayout` restates the reference's weight layout
(kernels.py:726-742: sign bits -> int32 mma fragment words [ceil(N/8)][ceil(K/128)][32]) so both kernels multiply the
same signs.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import shutil
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "b1dot"
MANIFEST = OUT / "manifest.json"

# (parts, n, k, m): the reference's 20 tuned x3 shapes (configs.py:17-36), config 0, the config-1 M sweep at one
# part, and the clip's other one-part shapes at M = 125.
X3_SHAPES = [(n, k, m) for n, k in ((1024, 1024), (1024, 4096), (2048, 1024), (3072, 1024), (4096, 1024))
             for m in (38, 126, 256, 368)]
X1_SHAPES = [(4096, 1024, m) for m in (16, 125, 512, 2048, 8192)] + [(1024, 4096, m) for m in (16, 125, 512, 2048, 8192)] \
    + [(3072, 1024, 125), (2048, 1024, 125), (1024, 1024, 125)]


def _round_up(v: int, m: int) -> int:
    return -(-v // m) * m


# ---- build (needs the reference's sources) ---------------------------------------------------------------------
def _generate(reference: Path) -> list[dict]:
    """Runs the reference's own table and generator (in a separate interpreter: its package shares this library's
    name) and returns [{name, source, parts, n, k, m, grid, threads, shared_bytes, workspace_ints, label}]."""
    script = r'''
import dataclasses, json, sys
sys.path.insert(0, sys.argv[1])
from kea_kernels.binary import configs, kernels, kernels_parts
out = []
for parts, n, k, m in json.loads(sys.argv[2]):
    config = configs.choose(m, n, k)
    if config.xchg == 3 and 127 * k >= 2**20:            # as layer.dot / dot_parts adjust it
        config = dataclasses.replace(config, xchg=1)
    if parts == 3:
        cfg = config
        source, name = kernels.dot_source(cfg, False, 0)
    else:
        cfg = kernels_parts.PartsConfig.of(config, parts)
        source, name = kernels_parts.dot_source(cfg, False, 0, parts)
    out.append(dict(name=name, source=source, parts=parts, n=n, k=k, m=m, grid=list(cfg.grid(m, n)),
                    threads=cfg.threads, shared_bytes=cfg.shared_bytes, workspace_ints=cfg.workspace_ints(m, n),
                    label=config.label()))
print(json.dumps(out))
'''
    shapes = [(3, n, k, m) for n, k, m in X3_SHAPES] + [(1, n, k, m) for n, k, m in X1_SHAPES]
    res = subprocess.run([sys.executable, "-c", script, str(reference / "src"), json.dumps(shapes)],
                         capture_output=True, text=True, check=True)
    return json.loads(res.stdout.strip().splitlines()[-1])


def build(reference: Path, nvcc: str = "nvcc") -> Path:
    if not (reference / "src" / "kea_kernels" / "binary" / "kernels.py").is_file():
        raise FileNotFoundError(f"no reference sources under {reference}")
    OUT.mkdir(parents=True, exist_ok=True)
    entries = []
    for e in _generate(reference):
        stem = f"{e['name']}_n{e['n']}_k{e['k']}_m{e['m']}"
        src, cubin = OUT / f"{stem}.cu", OUT / f"{stem}.cubin"
        src.write_text(e.pop("source"))
        subprocess.run([nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "--std=c++17", "-fmad=false",
                        "-O3", "-o", str(cubin), str(src)], check=True)
        e["cubin"] = cubin.name
        entries.append(e)
    MANIFEST.write_text(json.dumps(entries, indent=1))
    return MANIFEST


# ---- run time --------------------------------------------------------------------------------------------------
def cases() -> list[dict]:
    """The built kernels (empty when they were not built here)."""
    return json.loads(MANIFEST.read_text()) if MANIFEST.is_file() else []


def relayout(signs: np.ndarray) -> np.ndarray:
    """Signs {-1, +1} int8 [N, K] -> the reference's int32 fragment words [ceil(N/8)][ceil(K/128)][32]
    (kernels.py:730-742): word 4 g + s of (t, b) holds at bit 8 i + 2 j + r the sign of row 8 t + g, column
    128 b + 32 j + 16 r + 4 s + i (g < 8, s < 4, i < 4, j < 4, r < 2); a set bit means +1, padding is 0."""
    n, k = signs.shape
    nt, kb = -(-n // 8), -(-k // 128)
    padded = np.zeros((nt * 8, kb * 128), dtype=np.int64)
    padded[:n, :k] = (signs > 0).astype(np.int64)
    # axes [t, g, b, j, r, s, i] -> [t, b, g, s, i, j, r]: the last three (i, j, r) are the word's bits 8 i + 2 j + r
    v = padded.reshape(nt, 8, kb, 4, 2, 4, 4).transpose(0, 2, 1, 5, 6, 3, 4).reshape(nt, kb, 32, 32)
    words = (v << np.arange(32, dtype=np.int64)).sum(axis=-1)
    return (words - (words >= 2**31) * 2**32).astype(np.int32)


class _Driver:
    """The few CUDA driver calls a cubin launch needs (libcuda, through ctypes)."""

    def __init__(self):
        self.lib = ctypes.CDLL("libcuda.so.1")
        self.lib.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        self.lib.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
        self.lib.cuFuncSetAttribute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        self.lib.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 7 + [ctypes.c_void_p] * 3

    def check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what} failed with CUresult {rc}")


_DRIVER = None


class RefKernel:
    """One built reference kernel, loaded into the current CUDA context (create it after torch has made its
    context current, e.g. after a first CUDA tensor)."""

    def __init__(self, case: dict):
        global _DRIVER
        _DRIVER = _DRIVER or _Driver()
        self.case = case
        image = (OUT / case["cubin"]).read_bytes()
        self._image = ctypes.create_string_buffer(image, len(image))
        mod, fn = ctypes.c_void_p(), ctypes.c_void_p()
        _DRIVER.check(_DRIVER.lib.cuModuleLoadData(ctypes.byref(mod), self._image), "cuModuleLoadData")
        _DRIVER.check(_DRIVER.lib.cuModuleGetFunction(ctypes.byref(fn), mod, case["name"].encode()),
                      "cuModuleGetFunction")
        self.fn = fn
        if case["shared_bytes"] >= 48 * 1024:   # CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES
            _DRIVER.check(_DRIVER.lib.cuFuncSetAttribute(fn, 8, case["shared_bytes"]), "cuFuncSetAttribute")

    def launch(self, q, qs, words, scale, bias, y, m: int, n: int, k: int, workspace, stream_handle: int) -> None:
        """The reference's dot() argument list (layer.py:196-203): q int8 [P][M][ldq], qs FP32 [P][M], fragment
        words, channel scale / bias FP32 [N], y FP32 [M][ldy], split-K workspace (int32, or None)."""
        c = self.case
        holders = [ctypes.c_void_p(q.data_ptr()), ctypes.c_int64(q.stride(0)), ctypes.c_int32(q.stride(1)),
                   ctypes.c_int32(_round_up(k, 16)), ctypes.c_void_p(qs.data_ptr()), ctypes.c_int32(qs.stride(0)),
                   ctypes.c_void_p(words.data_ptr()), ctypes.c_int32(words.shape[0]), ctypes.c_int32(words.shape[1]),
                   ctypes.c_void_p(scale.data_ptr()), ctypes.c_void_p(0 if bias is None else bias.data_ptr()),
                   ctypes.c_void_p(y.data_ptr()), ctypes.c_int32(y.stride(0)), ctypes.c_int32(m), ctypes.c_int32(n),
                   ctypes.c_void_p(0 if workspace is None else workspace.data_ptr())]
        args = (ctypes.c_void_p * len(holders))(*[ctypes.cast(ctypes.byref(h), ctypes.c_void_p) for h in holders])
        gx, gy, gz = c["grid"]
        _DRIVER.check(_DRIVER.lib.cuLaunchKernel(self.fn, gx, gy, gz, c["threads"], 1, 1, c["shared_bytes"],
                                                 ctypes.c_void_p(stream_handle), args, None), f"launch {c['name']}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("cmd", choices=("build", "clean"))
    ap.add_argument("--reference", type=Path, default=None)
    a = ap.parse_args()
    if a.cmd == "clean":
        shutil.rmtree(OUT, ignore_errors=True)
    else:
        if a.reference is None:
            raise SystemExit("--reference <reference project root> is required")
        print(build(a.reference))
