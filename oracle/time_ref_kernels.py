"""TEST INFRASTRUCTURE ONLY: times the reference's own b1_dot kernels (built by oracle/ref_kernels.py) beside this
library on one B200, on every built shape, and prints one JSON line per shape plus a summary line.

Both sides run the same shapes on the same kind of inputs (signs with p = 0.5, INT8 parts uniform in [-127, 127],
row scales in [0.005, 0.02], FP32 output as the reference's dot writes it), each through its own launch path: the
reference's kernel with its own table's config, grid, block and shared bytes and plain cuLaunchKernel (its launcher,
src/kea_kernels/_nvrtc.py:116-125), the library through lowbit.gemm with its table (with and without programmatic
dependent launch). A step is a chain of CHAIN launches captured in a CUDA graph over 4 weight sets in rotation (each
launch reads weights the previous did not), replayed after a warm-up; the figure is the best of 5 replays divided by
CHAIN (microseconds per GEMM). The reference's outputs are checked against the library's, bit for bit, on the first
launch of every shape.

Usage (on a GPU box, after `python oracle/ref_kernels.py build --reference <root>` where the sources are mounted):
    python oracle/time_ref_kernels.py [--chain 48]
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent / "kea-kernels_b200"))
import ref_kernels  # noqa: E402
from kea_kernels import lowbit  # noqa: E402
from kea_kernels.binary import bits  # noqa: E402


def graph_time(body, stream, reps: int = 5) -> float:
    with torch.cuda.stream(stream):
        body()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            body()
        g.replay()
        stream.synchronize()
        best = math.inf
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            stream.synchronize()
            best = min(best, e0.elapsed_time(e1))
    return best


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--chain", type=int, default=48)
    a = ap.parse_args()
    cases = ref_kernels.cases()
    if not cases:
        raise SystemExit("the reference's kernels are not built (oracle/ref_kernels.py build)")
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    rows = []
    for c in cases:
        parts, n, k, m = c["parts"], c["n"], c["k"], c["m"]
        g = torch.Generator().manual_seed(n + k + m + parts)
        ldq = -(-k // 16) * 16
        q = torch.zeros(parts, m, ldq, dtype=torch.int8)
        q[:, :, :k] = torch.randint(-127, 128, (parts, m, k), generator=g, dtype=torch.int8)
        q = q.to(dev)
        qs = (torch.rand(parts, m, generator=g) * 0.015 + 0.005).to(dev)
        alpha = (torch.rand(n, generator=g) * 0.04 + 0.01).half().float().to(dev)
        signs = [torch.where(torch.rand(n, k, generator=g) < 0.5, -1, 1).to(torch.int8) for _ in range(4)]
        words = [torch.from_numpy(ref_kernels.relayout(s.numpy())).to(dev) for s in signs]
        panels = [lowbit.prepare_panels(bits.pack_signs(s).to(dev), 1, n, k) for s in signs]
        ws = torch.zeros(max(1, c["workspace_ints"]), dtype=torch.int32, device=dev) if c["workspace_ints"] else None
        kernel = ref_kernels.RefKernel(c)
        y_ref, y = torch.empty(m, n, device=dev), torch.empty(m, n, device=dev)
        kernel.launch(q, qs, words[0], alpha, None, y_ref, m, n, k, ws, torch.cuda.current_stream().cuda_stream)
        lowbit.gemm(q, qs, ldq, m, panels[0], 1, n, k, alpha, None, y, parts=parts)
        torch.cuda.synchronize()
        same = bool(torch.equal(y_ref.view(torch.int32), y.view(torch.int32)))

        def ref_body():
            h = torch.cuda.current_stream().cuda_stream
            for i in range(a.chain):
                kernel.launch(q, qs, words[i % 4], alpha, None, y_ref, m, n, k, ws, h)

        def ours_body(pdl):
            def run():
                for i in range(a.chain):
                    lowbit.gemm(q, qs, ldq, m, panels[i % 4], 1, n, k, alpha, None, y, parts=parts, pdl=pdl)
            return run

        t_ref = graph_time(ref_body, stream) * 1e3 / a.chain
        t_ours = graph_time(ours_body(False), stream) * 1e3 / a.chain
        t_pdl = graph_time(ours_body(True), stream) * 1e3 / a.chain
        row = dict(parts=parts, n=n, k=k, m=m, ref_config=c["label"], ref_us=round(t_ref, 3), ours_us=round(t_ours, 3),
                   ours_pdl_us=round(t_pdl, 3), speedup=round(t_ref / min(t_ours, t_pdl), 3), outputs_equal=same)
        rows.append(row)
        print(json.dumps(row), flush=True)
    gm = math.exp(sum(math.log(r["speedup"]) for r in rows) / len(rows))
    print(json.dumps({"summary": "reference b1_dot (sm_100a build of its SM120 source) vs this library, same B200",
                      "shapes": len(rows), "geomean_speedup": round(gm, 3),
                      "wins": sum(r["speedup"] > 1 for r in rows), "all_outputs_equal": all(r["outputs_equal"] for r in rows),
                      "chain": a.chain}))


if __name__ == "__main__":
    main()
