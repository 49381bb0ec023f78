"""ctypes binding of libkea_lowbit.so, the sm_100a C-ABI library (include/kea_lowbit.h).

This module replaces the reference's NVRTC launch runtime (src/kea_kernels/_nvrtc.py:50-149): there is no run-time
compilation; the library is built ahead of time by kea-kernels_b200/build.py and loaded here. Status codes map to
ValueError (argument errors) and RuntimeError (CUDA failures), as the reference's launcher raised RuntimeError for a
nonzero CUresult (_nvrtc.py:123-124). There is no CPU fallback: without the library every call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("KEA_LOWBIT_LIB", Path(__file__).resolve().parent / "libkea_lowbit.so"))

OK, INVALID_VALUE, ALIGNMENT, UNSUPPORTED, INVALID_CODES, CUDA, NO_DEVICE, DEVICE_TIMEOUT, CAPTURE, SCRATCH_LIMIT = range(10)
OUT_F32, OUT_F16 = 0, 1
FLAG_SILU, FLAG_ORDER1, FLAG_PDL, FLAG_NO_PAIR, FLAG_FORCE_PAIR = 1, 2, 4, 8, 16
FLAG_FORCE_SWAP, FLAG_NO_SWAP, FLAG_TEST_STALL, FLAG_NO_RESIDENT_WEIGHTS = 32, 64, 128, 256
FLAG_FORCE_REG, FLAG_NO_REG = 512, 1024
QUANT_INPUT_SILU, QUANT_PDL, QUANT_NARROW_ROWS = 1, 2, 4
PROJECT_FUSE = 1
DEVERR_TIMEOUT, DEVERR_TAIL_BITS, DEVERR_TERNARY_11 = 1, 2, 4

# Every symbol include/kea_lowbit.h declares.
EXPORTS = ("kea_lowbit_gemm", "kea_lowbit_gemm_noalloc", "kea_lowbit_choose_config", "kea_lowbit_panel_bytes", "kea_lowbit_workspace_bytes",
           "kea_lowbit_prepare",
           "kea_lowbit_quantize", "kea_lowbit_project", "kea_lowbit_project_fuses", "kea_lowbit_project_scratch_bytes", "kea_lowbit_glu_depthwise", "kea_lowbit_rel_attention", "kea_lowbit_read_error",
           "kea_lowbit_status_string", "kea_lowbit_version")
CONV_PDL, CONV_QUANT_SILU = 1, 2


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("q_part_stride", ctypes.c_int64), ("ldq", ctypes.c_int32), ("parts", ctypes.c_int32),
        ("qs", ctypes.c_void_p), ("qs_part_stride", ctypes.c_int64),
        ("panels", ctypes.c_void_p), ("wbits", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
        ("alpha", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64), ("y_dtype", ctypes.c_int32),
        ("acc", ctypes.c_void_p), ("ld_acc", ctypes.c_int64), ("acc_part_stride", ctypes.c_int64),
        ("m", ctypes.c_int32), ("flags", ctypes.c_int32),
        ("tile_m", ctypes.c_int32), ("tile_n", ctypes.c_int32), ("splits", ctypes.c_int32),
        ("stages", ctypes.c_int32), ("error_word", ctypes.c_void_p),
        ("residual", ctypes.c_void_p), ("ld_residual", ctypes.c_int64), ("residual_scale", ctypes.c_float),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_int64), ("wait_clocks", ctypes.c_int64),
    ]


class GemmConfig(ctypes.Structure):
    _fields_ = [("tile_m", ctypes.c_int32), ("tile_n", ctypes.c_int32), ("splits", ctypes.c_int32),
                ("stages", ctypes.c_int32), ("smem_bytes", ctypes.c_int32), ("kernel", ctypes.c_int32)]


class QuantizeDesc(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("xb", ctypes.c_int64), ("xt", ctypes.c_int64), ("xk", ctypes.c_int64),
        ("t", ctypes.c_int32), ("m", ctypes.c_int32), ("k", ctypes.c_int32), ("parts", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_part_stride", ctypes.c_int64), ("ldq", ctypes.c_int32),
        ("qs", ctypes.c_void_p), ("qs_part_stride", ctypes.c_int64),
        ("norm_weight", ctypes.c_void_p), ("norm_bias", ctypes.c_void_p), ("eps", ctypes.c_float),
        ("flags", ctypes.c_int32),
        ("pre_norm_weight", ctypes.c_void_p), ("pre_norm_bias", ctypes.c_void_p), ("pre_eps", ctypes.c_float),
        ("normed", ctypes.c_void_p), ("ld_normed", ctypes.c_int64),
    ]


class ProjectDesc(ctypes.Structure):
    _fields_ = [("gemm", GemmDesc), ("quant", QuantizeDesc), ("scratch", ctypes.c_void_p),
                ("scratch_bytes", ctypes.c_size_t), ("flags", ctypes.c_int32)]


class ConvDesc(ctypes.Structure):
    _fields_ = [("h", ctypes.c_void_p), ("y", ctypes.c_void_p), ("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("lengths", ctypes.c_void_p), ("b", ctypes.c_int32), ("t", ctypes.c_int32), ("c", ctypes.c_int32),
                ("kw", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("q", ctypes.c_void_p), ("q_part_stride", ctypes.c_int64), ("ldq", ctypes.c_int32),
                ("qs", ctypes.c_void_p), ("qs_part_stride", ctypes.c_int64), ("parts", ctypes.c_int32)]


class AttentionDesc(ctypes.Structure):
    _fields_ = [("qkv", ctypes.c_void_p), ("pos", ctypes.c_void_p), ("bias_u", ctypes.c_void_p),
                ("bias_v", ctypes.c_void_p), ("lengths", ctypes.c_void_p), ("ctx", ctypes.c_void_p),
                ("b", ctypes.c_int32), ("t", ctypes.c_int32), ("h", ctypes.c_int32), ("dk", ctypes.c_int32),
                ("scale", ctypes.c_float), ("flags", ctypes.c_int32)]


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises RuntimeError (never falls back) when it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python kea-kernels_b200/build.py` "
                               "(kea_kernels has no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        handle.kea_lowbit_gemm.argtypes = [ctypes.POINTER(GemmDesc), ctypes.c_void_p]
        handle.kea_lowbit_gemm.restype = ctypes.c_int
        handle.kea_lowbit_gemm_noalloc.argtypes = [ctypes.POINTER(GemmDesc), ctypes.c_void_p]
        handle.kea_lowbit_gemm_noalloc.restype = ctypes.c_int
        handle.kea_lowbit_choose_config.argtypes = [ctypes.c_int32] * 5 + [ctypes.POINTER(GemmConfig)]
        handle.kea_lowbit_choose_config.restype = ctypes.c_int
        handle.kea_lowbit_panel_bytes.argtypes = [ctypes.c_int32] * 3
        handle.kea_lowbit_panel_bytes.restype = ctypes.c_size_t
        handle.kea_lowbit_workspace_bytes.argtypes = [ctypes.c_int32] * 5
        handle.kea_lowbit_workspace_bytes.restype = ctypes.c_size_t
        handle.kea_lowbit_prepare.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        handle.kea_lowbit_prepare.restype = ctypes.c_int
        handle.kea_lowbit_quantize.argtypes = [ctypes.POINTER(QuantizeDesc), ctypes.c_void_p]
        handle.kea_lowbit_quantize.restype = ctypes.c_int
        handle.kea_lowbit_project.argtypes = [ctypes.POINTER(ProjectDesc), ctypes.c_void_p]
        handle.kea_lowbit_project.restype = ctypes.c_int
        handle.kea_lowbit_project_fuses.argtypes = [ctypes.POINTER(ProjectDesc)]
        handle.kea_lowbit_project_fuses.restype = ctypes.c_int
        handle.kea_lowbit_project_scratch_bytes.argtypes = [ctypes.c_int32] * 5
        handle.kea_lowbit_project_scratch_bytes.restype = ctypes.c_size_t
        handle.kea_lowbit_glu_depthwise.argtypes = [ctypes.POINTER(ConvDesc), ctypes.c_void_p]
        handle.kea_lowbit_glu_depthwise.restype = ctypes.c_int
        handle.kea_lowbit_rel_attention.argtypes = [ctypes.POINTER(AttentionDesc), ctypes.c_void_p]
        handle.kea_lowbit_rel_attention.restype = ctypes.c_int
        handle.kea_lowbit_read_error.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        handle.kea_lowbit_read_error.restype = ctypes.c_int
        handle.kea_lowbit_status_string.argtypes = [ctypes.c_int]
        handle.kea_lowbit_status_string.restype = ctypes.c_char_p
        handle.kea_lowbit_version.argtypes = []
        handle.kea_lowbit_version.restype = ctypes.c_int
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status == OK:
        return
    text = lib().kea_lowbit_status_string(status).decode()
    if status in (INVALID_VALUE, ALIGNMENT, UNSUPPORTED, INVALID_CODES, SCRATCH_LIMIT):
        raise ValueError(f"{what}: {text}")
    raise RuntimeError(f"{what}: {text} (status {status})")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def panel_bytes(wbits: int, n: int, k: int) -> int:
    return int(lib().kea_lowbit_panel_bytes(wbits, n, k))


def workspace_bytes(m: int, n: int, k: int, wbits: int, parts: int) -> int:
    """Scratch bytes the dispatch table's split-K uses at this shape (0: none)."""
    return int(lib().kea_lowbit_workspace_bytes(m, n, k, wbits, parts))


def choose_config(m: int, n: int, k: int, wbits: int, parts: int) -> GemmConfig:
    out = GemmConfig()
    check(lib().kea_lowbit_choose_config(m, n, k, wbits, parts, ctypes.byref(out)), "choose_config")
    return out


def read_device_error() -> int:
    """Reads and clears the library's own device error word (synchronizes the current device)."""
    v = ctypes.c_uint32(0)
    check(lib().kea_lowbit_read_error(ctypes.byref(v)), "read_error")
    return int(v.value)


def raise_device_errors(word: int | None = None) -> None:
    """Raises RuntimeError when a kernel reported an expired wait (KEA_DEVERR_TIMEOUT) - in `word` (a caller's error
    word, already read back) or, when None, in the library's own word (read and cleared; synchronizes). The
    reference raised RuntimeError for a failed launch (_nvrtc.py:123-124); a wait that ran out is this library's
    equivalent, reported after the kernel has returned."""
    bits = read_device_error() if word is None else int(word)
    if bits & DEVERR_TIMEOUT:
        raise RuntimeError(f"kernel: {lib().kea_lowbit_status_string(DEVICE_TIMEOUT).decode()} "
                           f"(device error bits {bits:#x})")
