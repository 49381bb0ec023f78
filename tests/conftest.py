"""Shared test set-up. GPU tests carry the `gpu` marker and are skipped unless an sm_100 (B200-class) GPU is visible."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT / "kea-kernels_b200", ROOT / "oracle"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = ROOT / "tests" / "golden" / "golden.npz"
GOLDEN_CONFIG = ROOT / "tests" / "golden" / "golden_config.npz"
if str(ROOT / "tests" / "golden") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests" / "golden"))


def sm100() -> bool:
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA sm_100 GPU (B200)")


def pytest_collection_modifyitems(config, items):
    if sm100():
        return
    skip = pytest.mark.skip(reason="needs an NVIDIA sm_100 GPU (B200)")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def golden_config():
    with np.load(GOLDEN_CONFIG) as data:
        return {k: data[k] for k in data.files}


def sha256(a: np.ndarray) -> np.ndarray:
    import hashlib
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), dtype=np.uint8)


def golden_cases(golden):
    out = []
    for name in golden["cases"]:
        wbits, n, k, m, parts, has_bias = (int(v) for v in golden[f"{name}/meta"])
        out.append(dict(name=str(name), wbits=wbits, n=n, k=k, m=m, parts=parts,
                        codes=golden[f"{name}/codes"], q=golden[f"{name}/q"], qs=golden[f"{name}/qs"],
                        alpha=golden[f"{name}/alpha"], bias=golden.get(f"{name}/bias") if has_bias else None,
                        acc=golden[f"{name}/acc"], y64=golden[f"{name}/y64"]))
    return out
