"""Config-size GEMM cases (BASELINE config 0 and one config-1 M-sweep point), drawn from seeded torch generators so
that the fixtures need only hashes and a few sampled rows: make_golden.py draws them and stores what the reference's
own functions produce; the tests draw the same inputs and compare against those records."""
from __future__ import annotations

import torch

# (name, wbits, n, k, m, parts)
CONFIG_CASES = [
    ("config0_b1_n4096_k1024_m125", 1, 4096, 1024, 125, 1),
    ("config1_t2_n1024_k4096_m2048", 2, 1024, 4096, 2048, 1),  # the FF down shape at M = 2048
]
SAMPLE_ROWS = (0, 1, 63, 124)   # rows of acc / y64 stored in full (all < every case's m)


def draw(wbits: int, n: int, k: int, m: int, parts: int):
    """(dense int8 weights [n, k], q int8 [parts, m, k], qs FP32 [parts, m], alpha FP32 [n]) with the BASELINE
    distributions: signs p = 0.5, ternary {-1, 0, +1} p = {0.3, 0.4, 0.3}, activations uniform in [-127, 127], row
    scales in [0.005, 0.02], fp16-valued channel scales in [0.01, 0.05]."""
    g = torch.Generator().manual_seed(wbits * 1_000_003 + n * 101 + k * 7 + m + parts)
    if wbits == 1:
        w = torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8)
    else:
        u = torch.rand(n, k, generator=g)
        w = torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8)
    q = torch.randint(-127, 128, (parts, m, k), generator=g, dtype=torch.int8)
    qs = (torch.rand(parts, m, generator=g) * 0.015 + 0.005).float()
    alpha = (torch.rand(n, generator=g) * 0.04 + 0.01).half().float()
    return w, q, qs, alpha
