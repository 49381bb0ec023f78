"""Benchmark of the B200 low-bit GEMM on BASELINE config 1: the M sweep {1, 16, 125, 512, 2048, 8192} at
(N, K) = (4096, 1024) and (1024, 4096), for 1-bit (sign) and 2-bit (ternary) weights x one INT8 activation part.

A step is one pass over the 24 GEMMs of that sweep (fp16 outputs), replayed as one CUDA graph. Every GEMM reads a
weight set and activations from rotating pools, and a step writes about 220 MB of outputs, so each step streams
more than the 126 MB L2. `value` is the whole job's effective INT8 rate, sum(2 M N K) / time, over all ranks
(replicas: each rank runs the full sweep on its own GPU; weak scaling). `e2e` is the same rate through the C-ABI call
with host buffers (pinned host -> device activations, device -> pinned host outputs, inside the timed region).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the reference's CPU algorithm (unpack the packed codes, exact integer GEMM, FP32 epilogue,
fp16 out) on the same workload - every step one pass over the whole sweep - with every host core: the strong
restatement of that arithmetic through FP32 BLAS (exact: every partial sum is an integer below 2^24), oracle.gemm_blas.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kea-kernels_b200"))

METRIC = "1-bit GEMM effective TOPS and % of HBM/INT8 roofline; ms per synthetic 10 s clip"
UNIT = "TOPS"
SHAPES = [(4096, 1024), (1024, 4096)]
MS = [1, 16, 125, 512, 2048, 8192]
CASES = [(wbits, n, k, m) for wbits in (1, 2) for (n, k) in SHAPES for m in MS]
POOL = 4                                 # distinct weight / activation sets per case in the step graphs
COLD_BYTES = 512 << 20                   # per (wbits, N, K): distinct weights swept by the per-case cold timing
L2_BYTES = 126 << 20
# dram__bytes_read.sum + dram__bytes_write.sum of one cold launch, from the committed ncu captures of those cases
# (keyed by (wbits, N, K, M)); None for a case without a capture.
# dram__bytes_read.sum + dram__bytes_write.sum per launch from the committed ncu captures (profiles/): the M = 8192
# cases that can be a step's longest (pair kernels, weight-stationary at K 1024), the per-tile kernel at M 125
NCU_TRAFFIC = {(1, 4096, 1024, 8192): 9_068_032 + 18_014_208, (2, 4096, 1024, 8192): 9_599_232 + 15_053_568,
               (1, 1024, 4096, 8192): 34_213_632 + 245_504, (2, 1024, 4096, 8192): 34_738_688 + 207_360,
               (1, 4096, 1024, 125): 738_816}


def ops(m, n, k, parts=1):
    return 2 * m * n * k * parts


def alg_bytes(wbits, n, k, m, parts=1, out_bytes=2):
    """Algorithmic bytes of one GEMM: packed weights + activations (+ scales, fp16 output for `full`)."""
    wa = n * k * wbits // 8 + parts * m * k
    return wa, wa + 4 * parts * m + 4 * n + out_bytes * m * n


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---- clocks ------------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self, busy_mhz: float = 500.0) -> dict:
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        loaded = [r for r in rows if r[0] >= busy_mhz] or rows
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded)}


# ---- the CPU side (reference arm and cpu_baseline) --------------------------------------------------------------
WORKLOAD = ("BASELINE config 1: M sweep {1,16,125,512,2048,8192} x (N,K) in {(4096,1024),(1024,4096)} x "
            "{1-bit, 2-bit} weights, 1 INT8 part, fp16 out")


def _cpu_work(cases, seed=0):
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import kea_oracle as oracle

    rng = np.random.default_rng(seed)
    work = []
    for wbits, n, k, m in cases:
        if wbits == 1:
            codes = oracle.pack_signs(rng.choice(np.array([-1, 1], dtype=np.int8), size=(n, k)))
        else:
            codes = oracle.pack_ternary(rng.choice(np.array([-1, 0, 1], dtype=np.int8), size=(n, k), p=[.3, .4, .3]))
        q = rng.integers(-127, 128, size=(1, m, k), dtype=np.int8)
        qs = rng.uniform(0.005, 0.02, size=(1, m)).astype(np.float32)
        alpha = rng.uniform(0.01, 0.05, size=n).astype(np.float16).astype(np.float32)
        work.append((codes, wbits, n, k, q, qs, alpha))
    return oracle, work


def cpu_sample(threads: int, min_seconds: float = 10.0, max_seconds: float = 30.0, repeats: int | None = None):
    """Times the reference's CPU algorithm on the host cores over the GPU arm's whole workload (the 24 GEMMs of the
    config-1 sweep; one pass = one step): unpack the export codes, exact integer GEMM through FP32 BLAS (exact: every
    partial sum is an integer below 2^24), the comb<1> epilogue in FP32, FP16 output - the strong CPU restatement
    (oracle.gemm_blas) in PyTorch's multi-threaded CPU kernels on `threads` threads.
    Returns (TOPS, seconds, passes, ops per pass)."""
    import torch

    torch.set_num_threads(threads)
    oracle, work = _cpu_work(CASES)
    total_ops = sum(ops(q.shape[1], n, k) for _, _, n, k, q, _, _ in work)

    def one_pass():
        for codes, wbits, n, k, q, qs, alpha in work:
            oracle.gemm_blas(codes, wbits, q, qs, alpha)

    one_pass()  # warm-up
    passes, t0 = 0, time.perf_counter()
    while True:
        one_pass()
        passes += 1
        elapsed = time.perf_counter() - t0
        if repeats is not None and passes >= repeats:
            break
        if repeats is None and (elapsed >= min_seconds or elapsed + elapsed / passes > max_seconds):
            break
    return total_ops * passes / elapsed / 1e12, elapsed, passes, total_ops


def cpu_baseline_record(tops: float, seconds: float, passes: int, total: int, threads: int) -> dict:
    return {"value": tops, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"the whole config-1 sweep ({len(CASES)} GEMMs, {total / 1e9:.1f} GOP per pass, {passes} passes, "
                      f"{seconds:.1f} s): unpack the export codes, exact integer GEMM through FP32 BLAS, FP32 comb<1> "
                      "epilogue, fp16 out (oracle.gemm_blas: PyTorch CPU kernels)"}


def cpu_literal_sample(threads: int, seconds: float = 5.0) -> dict:
    """The reference test's literal oracle (unpack, then an integer triple loop with the FP32 epilogue; the C
    restatement in oracle/, `threads` threads) on the M <= 16 cases of the sweep: context for the strong baseline."""
    oracle, work = _cpu_work([c for c in CASES if c[3] <= 16], seed=1)
    total = sum(ops(q.shape[1], n, k) for _, _, n, k, q, _, _ in work)
    passes, t0 = 0, time.perf_counter()
    while passes == 0 or time.perf_counter() - t0 < seconds:
        for codes, wbits, n, k, q, qs, alpha in work:
            w, status = oracle.unpack_c(codes, wbits, n, k)
            oracle.gemm(q, qs, w, alpha, threads=threads)
        passes += 1
    elapsed = time.perf_counter() - t0
    return {"value": total * passes / elapsed / 1e12, "unit": UNIT, "cores": threads,
            "sample": f"M <= 16 cases of the sweep ({total / 1e9:.2f} GOP per pass, {passes} passes, {elapsed:.1f} s): "
                      "unpack + integer triple loop + FP32 epilogue (oracle/kea_oracle.c)"}


def cpu_clip_sample() -> dict:
    """The clip's low-bit GEMM chain on the host cores through the reference's CPU algorithm: 24 layers x 8 GEMMs at
    M = 125 (config 2's shapes), each unpack + exact integer GEMM (FP32 BLAS) + FP32 epilogue + fp16 out
    (oracle.gemm_blas, PyTorch CPU kernels on every host thread)."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    shapes = [(4096, 1024), (1024, 4096), (3072, 1024), (1024, 1024), (2048, 1024), (1024, 1024), (4096, 1024),
              (1024, 4096)]
    oracle, work = _cpu_work([(1, n, k, 125) for n, k in shapes * 24], seed=1)
    t0 = time.perf_counter()
    for codes, wbits, n, k, q, qs, alpha in work:
        oracle.gemm_blas(codes, wbits, q, qs, alpha)
    seconds = time.perf_counter() - t0
    return {"ms_per_clip": seconds * 1e3, "cores": threads, "kind": "port",
            "sample": f"all 24 layers ({len(work)} GEMMs at M = 125: unpack + exact integer GEMM through FP32 BLAS + "
                      f"FP32 epilogue + fp16 out, oracle.gemm_blas), {seconds:.2f} s"}


def reference_arm(args) -> None:
    """The reference's CPU algorithm on the host cores, on the GPU arm's own workload and metric: each step one pass
    over the whole config-1 sweep (the strong FP32-BLAS restatement, every host thread)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cpu_sample(threads, repeats=max(1, args.warmup))
    tops, seconds, passes, total = cpu_sample(threads, repeats=max(1, args.steps))
    base = cpu_baseline_record(tops, seconds, passes, total, threads)
    line = {"impl": "reference", "metric": METRIC, "value": tops, "unit": UNIT, "n_gpus": args.gpus,
            "steps": passes, "warmup": args.warmup, "ms_per_step": seconds * 1e3 / passes,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "gemms_per_step": len(CASES), "gop_per_step": total / 1e9,
                       "parallelism": "host cores"},
            "cpu_baseline": base,
            "e2e": {"value": tops, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- the GPU side -----------------------------------------------------------------------------------------------
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--clip-batch", type=int, default=256, help="clips in the config-3 batch (sharded over ranks)")
    ap.add_argument("--no-clip", action="store_true", help="skip the clip workloads (shorter profiling runs)")
    ap.add_argument("--kea-t-clips", type=int, default=1024,
                    help="clips in the config-4 batch (2-bit, two parts, 2-30 s; 0 skips it)")
    ap.add_argument("--case", default=None, metavar="WBITS,N,K,M",
                    help="profiling mode: launch one GEMM case W + K times (rotating cold weights), print its timing")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.case:
        profile_case(args)
        return

    import torch
    import torch.distributed as dist

    from kea_kernels import _lib, formats, lowbit
    from kea_kernels.binary import bits, configs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    pdl = not args.no_pdl
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    def random_codes(wbits, n, k):
        if wbits == 1:
            signs = torch.where(torch.rand(n, k, device=dev, generator=gen) < 0.5, -1, 1).to(torch.int8)
            return bits.pack_signs(signs)
        u = torch.rand(n, k, device=dev, generator=gen)
        return formats.pack_ternary(torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8))

    def random_panels(wbits, n, k, count):
        pb = _lib.panel_bytes(wbits, n, k)
        out = torch.empty(count, pb, dtype=torch.uint8, device=dev)
        base = [lowbit.prepare_panels(random_codes(wbits, n, k), wbits, n, k) for _ in range(min(count, 8))]
        for i in range(count):   # distinct storage per set (the bytes of sets >= 8 repeat, the addresses do not)
            out[i].copy_(base[i % len(base)])
        return out

    # ---- buffers of the step graphs ----
    combos = sorted({(w, n, k) for w, n, k, _ in CASES})
    alphas = {c: (torch.rand(c[1], device=dev, generator=gen) * 0.04 + 0.01).half().float() for c in combos}
    weights = {c: random_panels(*c, POOL) for c in combos}
    acts, outs = {}, {}
    for case in CASES:
        wbits, n, k, m = case
        acts[case] = (torch.randint(-127, 128, (POOL, 1, m, k), dtype=torch.int8, device=dev, generator=gen),
                      torch.rand(POOL, 1, m, device=dev, generator=gen) * 0.015 + 0.005)
        outs[case] = torch.empty(m, n, device=dev, dtype=torch.float16)

    def launch(case, j, *, y=None, q=None, qs=None):
        wbits, n, k, m = case
        qq, ss = acts[case]
        lowbit.gemm(qq[j] if q is None else q, ss[j] if qs is None else qs, k, m, weights[(wbits, n, k)][j], wbits,
                    n, k, alphas[(wbits, n, k)], None, outs[case] if y is None else y, parts=1, pdl=pdl)

    # one-time set-up on this device happens outside any capture
    for case in CASES:
        launch(case, 0)
    torch.cuda.synchronize()
    if _lib.read_device_error():
        raise RuntimeError("device error word set during set-up")

    stream = torch.cuda.Stream(device=dev)
    graphs = []
    with torch.cuda.stream(stream):
        for j in range(POOL):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for case in CASES:
                    launch(case, j)
            graphs.append(g)
    torch.cuda.synchronize()
    step_ops = sum(ops(m, n, k) for _, n, k, m in CASES)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    hbm_peak, bf16_peak, peak_kind = measured_peaks()
    sampler = ClockSampler(local)
    with sampler:
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                graphs[i % POOL].replay()
            burn_until = time.perf_counter() + 1.0      # >= 1 s of load before timing, so clocks settle / sample
            i = 0
            while time.perf_counter() < burn_until:
                graphs[i % POOL].replay()
                i += 1
                if i % 20 == 0:
                    stream.synchronize()
            stream.synchronize()
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(args.steps):
                graphs[i % POOL].replay()
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        value = world * step_ops * args.steps / (ms / 1e3) / 1e12

        # ---- per-case device timing (cold: distinct weights sweep >= 4 x L2; rank 0 reports) ----
        per_case = []
        int8_peak, int8_kind = None, None
        ref_table = None
        if rank == 0:
            per_case = time_cases(torch, lowbit, _lib, configs, dev, stream, random_panels, alphas, pdl)
            int8_peak, int8_kind = int8_peak_tops(torch, dev)
            ref_table = reference_table(torch, lowbit, _lib, dev, stream, random_panels, pdl)
    clocks = sampler.summary()

    # ---- e2e through the C-ABI call with host buffers ----
    e2e = e2e_rate(torch, lowbit, dev, weights, alphas, args, world, dist if world > 1 else None, local)

    # ---- the clip workloads: one 10 s clip (config 2) and a sharded batch of 256 clips (config 3) ----
    del graphs, weights, acts, outs
    torch.cuda.empty_cache()
    clip = None if args.no_clip else clip_workloads(torch, dev, stream, rank, world, dist if world > 1 else None,
                                                     local, pdl, hbm_peak, args.clip_batch)
    if clip is not None and args.kea_t_clips > 0:
        clip["config4"] = kea_t_batch(torch, dev, stream, world, dist if world > 1 else None, local, pdl,
                                      args.kea_t_clips)

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return

    # dominant kernel of the step: the case with the largest share of the step's device time
    share = max(per_case, key=lambda c: c["us"])
    tensor_peak = int8_peak if int8_peak else 2 * bf16_peak
    if share["m"] >= 2048:
        achieved = ops(share["m"], share["n"], share["k"]) / (share["us"] * 1e-6) / 1e12
        roofline = {"bound": "tensor", "achieved": achieved, "peak": tensor_peak, "unit": "TFLOP/s",
                    "frac": achieved / tensor_peak,
                    "traffic": NCU_TRAFFIC.get((share["wbits"], share["n"], share["k"], share["m"])),
                    "kernel": (f"lowbit_gemm_pair_ws_kernel<{share['wbits']}>" if share["k"] <= 1024 else
                               f"lowbit_gemm_pair_kernel<{share['wbits']}, 1>") + f" M={share['m']} N={share['n']} K={share['k']}",
                    "peak_kind": int8_kind or f"2 x bf16 ({peak_kind})",
                    "note": "INT8 ops/s; peak = dense INT8 measured with torch._int_mm 8192^3 on this GPU"}
    else:
        achieved = share["gbs_full"]
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                    "frac": achieved / hbm_peak,
                    "traffic": NCU_TRAFFIC.get((share["wbits"], share["n"], share["k"], share["m"])),
                    "kernel": f"lowbit_gemm_kernel<{share['wbits']}>",
                    "peak_kind": peak_kind}
    small = [c for c in per_case if c["m"] == 125]
    roofline_small = [{"case": f"w{c['wbits']} N={c['n']} K={c['k']} M=125", "bound": "hbm",
                       "achieved_gbs_wa": c["gbs_wa"], "achieved_gbs_full": c["gbs_full"], "peak": hbm_peak,
                       "frac_wa": c["gbs_wa"] / hbm_peak, "frac_full": c["gbs_full"] / hbm_peak,
                       "us_cold": c["us"], "us_hot": c.get("us_hot")} for c in small]

    cpu = None
    if world == 1:
        threads = os.cpu_count() or 1
        cpu = cpu_baseline_record(*cpu_sample(threads), threads)
        cpu["literal_oracle"] = cpu_literal_sample(threads)

    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "gemms_per_step": len(CASES), "gop_per_step": step_ops / 1e9,
                       "l2": "inputs larger than L2: rotating pools of weights/activations, ~220 MB written per step",
                       "parallelism": f"replicas x{world}", "pdl": pdl},
            "roofline": roofline, "roofline_small_m": roofline_small, "cpu_baseline": cpu, "e2e": e2e,
            "clocks": clocks, "gpu_launches": len(CASES) * args.steps, "cases": per_case,
            "int8_peak_tops": int8_peak, "int8_peak_kind": int8_kind, "reference_x3_table": ref_table,
            "clip": clip}
    print(json.dumps(line), flush=True)


def clip_workloads(torch, dev, stream, rank, world, dist, local, pdl, hbm_peak, batch_clips):
    """one synthetic 10 s clip (log-mel N(0, 1) [1, 128, 1000]) through the random-init 24-layer
    1-bit FastConformer encoder and the TDT joint's greedy labels, replayed as one CUDA graph: ms per clip, cold (L2
    flushed before every replay; the encoder's 72 MB of panels would otherwise stay in the 126 MB L2) and hot, and
    end to end with the mel copied in from pinned host memory and the labels copied out. The low-bit path alone (the
    192 quantize + GEMM pairs, captured on their own) gives the clip's HBM roofline: panel + scale bytes / time.
    `batch_clips` clips sharded over the ranks (whole clips, balanced by frames), each rank runs
    its shard as one batch (M = clips x 125 per GEMM) and the labels and timings are gathered with NCCL."""
    from kea_kernels import batch as B
    from kea_kernels import encoder as E

    gen = torch.Generator(device=dev).manual_seed(77)
    enc = E.FastConformerEncoder(device=dev, wbits=1, parts=1, pdl=pdl, seed=5)
    joint = E.TDTJoint(device=dev)
    out = {}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        mel = torch.randn(1, 128, 1000, device=dev, generator=gen)
        for _ in range(3):
            labels = joint.greedy(enc(mel))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            labels = joint.greedy(enc(mel))
        # the low-bit path alone, same shapes and order
        xs = {k: torch.randn(1, 125, k, device=dev, generator=gen) for k in (1024, 4096)}
        for layer in enc.layers:
            for name in E.LAYER_LINEARS:
                layer.lin[name](xs[layer.lin[name].in_features])
        gl = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gl, stream=stream):
            for layer in enc.layers:
                for name in E.LAYER_LINEARS:
                    layer.lin[name](xs[layer.lin[name].in_features])
        stream.synchronize()

        def timed(graph, reps, cold, pre=None, post=None):
            evs = []
            for i in range(reps + 3):
                if cold:
                    flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                if pre:
                    pre()
                graph.replay()
                if post:
                    post()
                e1.record(stream)
                if i >= 3:
                    evs.append((e0, e1))
            stream.synchronize()
            return statistics.median(a.elapsed_time(b) for a, b in evs)

        clip_cold = timed(g, 20, True)
        clip_hot = timed(g, 20, False)
        lowbit_cold = timed(gl, 20, True)
        lowbit_hot = timed(gl, 20, False)
        host_mel = torch.randn(1, 128, 1000).pin_memory()
        host_lab = torch.empty(1, 125, dtype=torch.int32).pin_memory()
        clip_e2e = timed(g, 20, True, pre=lambda: mel.copy_(host_mel, non_blocking=True),
                         post=lambda: host_lab.copy_(labels, non_blocking=True))
    # HBM bytes a clip must stream: the panels and per-channel constants (the 125-frame activations stay in L2)
    panel_bytes = sum(layer.lin[n].panels.numel() + 8 * layer.lin[n].out_features
                      for layer in enc.layers for n in E.LAYER_LINEARS)
    gops = sum(2 * 125 * layer.lin[n].out_features * layer.lin[n].in_features
               for layer in enc.layers for n in E.LAYER_LINEARS) / 1e9
    out["config2"] = {
        "workload": "BASELINE config 2: one synthetic 10 s clip, log-mel N(0,1) [1,128,1000] -> 125 frames, "
                    "random-init 24-layer 1-bit FastConformer (d 1024, 8 heads, FF 4096, conv 9) + TDT joint greedy",
        "ms_per_clip": clip_cold, "ms_per_clip_hot": clip_hot, "ms_per_clip_e2e": clip_e2e,
        "e2e_bytes": {"h2d": host_mel.numel() * 4, "d2h": host_lab.numel() * 4},
        "lowbit_ms": lowbit_cold, "lowbit_ms_hot": lowbit_hot, "lowbit_gemms": 192, "lowbit_launches": 384,
        "lowbit_gop": gops, "lowbit_tops": gops / lowbit_cold,
        "hbm": {"bytes": panel_bytes, "achieved_gbs": panel_bytes / (lowbit_cold * 1e-3) / 1e9, "peak": hbm_peak,
                "frac": panel_bytes / (lowbit_cold * 1e-3) / 1e9 / hbm_peak, "peak_kind": "measured"},
        "l2": "flushed (256 MB written) before every timed replay; hot = back-to-back replays"}
    del g, gl
    torch.cuda.empty_cache()
    if world == 1:
        out["config2"]["cpu_baseline"] = cpu_clip_sample()

    # ---- config 3: the batch, sharded ----
    n_clips = batch_clips
    frames = [125] * n_clips
    mine = B.shard(frames, world)[rank]
    mels = torch.randn(len(mine), 128, 1000, device=dev, generator=gen) if mine else None
    state = {}

    def process(indices):
        if not indices:
            return [], 0.0
        with torch.cuda.stream(stream):
            for _ in range(2):
                lab = joint.greedy(enc(mels))
            gb = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gb, stream=stream):
                lab = joint.greedy(enc(mels))
            gb.replay()
            stream.synchronize()
            ms = timed(gb, 5, False)
        state["graph"] = gb
        return [lab[j] for j in range(len(indices))], ms / 1e3

    if dist is not None:
        dist.barrier(device_ids=[local])
    res = B.run_batch(frames, process, device=dev)
    state.clear()
    t = max(res.seconds)
    m_total = 125 * n_clips
    gop = sum(2 * m_total * layer.lin[n].out_features * layer.lin[n].in_features
              for layer in enc.layers for n in E.LAYER_LINEARS) / 1e9
    out["config3"] = {
        "workload": f"BASELINE config 3: {n_clips} synthetic 10 s clips (M = {m_total} frames per GEMM over the job), "
                    f"sharded over {world} GPU(s) as whole clips; labels and timings gathered with NCCL",
        "clips_per_s": n_clips / t, "frames_per_s": m_total / t, "ms_per_batch": t * 1e3,
        "per_rank_ms": [s * 1e3 for s in res.seconds], "per_rank_frames": res.frames,
        "lowbit_gop": gop, "encoder_lowbit_tops": gop / t / 1e3,
        "labels_gathered": len(res.tokens), "timing": "CUDA events on each rank's stream, max over ranks"}
    return out


KEA_T_FRAMES_CAP = 32000   # padded encoder frames per forward (bounds the subsampling activations to ~10 GB)
# Forward planning (kea_kernels.batch.plan): a forward's cost modelled as a fixed floor plus a cost per padded encoder
# frame, both fitted on B200 to this workload's length-bucket runs (13 forwards / 218k padded frames in 1156 ms on one
# GPU, 12 / 27k in 205 ms per rank on eight); a rank's clips are grouped into padded forwards at the least modelled cost.
KEA_T_FORWARD_US = 6000.0
KEA_T_FRAME_US = 5.0


def kea_t_batch(torch, dev, stream, world, dist, local, pdl, n_clips):
    """a Kea-T-shaped encoder (the same 24-layer FastConformer, 2-bit ternary weights, two
    residual INT8 parts: Kea-T's default x2 mode) over `n_clips` synthetic clips whose lengths are uniform in
    2-30 s (log-mel at 100 frames/s, N(0, 1)). Whole clips are sharded over the ranks by frame count; each rank groups
    its clips into forwards by `batch.plan` (least modelled cost, at most KEA_T_FRAMES_CAP padded frames each) and
    pads each forward to its longest clip (masked as attention keys and before the depthwise convolution). One untimed pass fills the per-length position-projection cache; the timed pass is bracketed by CUDA
    events on the rank's stream, labels and timings gathered with NCCL, max over ranks."""
    from kea_kernels import batch as B
    from kea_kernels import encoder as E

    g = torch.Generator().manual_seed(2024)
    mel_frames = [int(v) for v in (200 + torch.rand(n_clips, generator=g) * 2800).long()]   # 2-30 s at 100 frames/s
    enc = E.FastConformerEncoder(device=dev, wbits=2, parts=2, pdl=pdl, seed=9)
    joint = E.TDTJoint(device=dev)
    enc_frames = [enc.frames(t) for t in mel_frames]
    dgen = torch.Generator(device=dev).manual_seed(4242)

    n_forwards = [0]

    def process(indices):
        if not indices:
            return [], 0.0
        fr = [enc_frames[i] for i in indices]
        work = []
        for group in B.plan(fr, KEA_T_FRAMES_CAP, KEA_T_FORWARD_US, KEA_T_FRAME_US):
            sub = [indices[j] for j in group]                       # longest first
            t_mel = max(mel_frames[i] for i in sub)
            mel = torch.zeros(len(sub), 128, t_mel, device=dev)
            for j, i in enumerate(sub):
                mel[j, :, :mel_frames[i]].normal_(generator=dgen)
            lengths = torch.tensor([enc_frames[i] for i in sub], device=dev)
            work.append((sub, mel, lengths))
        n_forwards[0] = len(work)
        labels = {}
        with torch.cuda.stream(stream):
            for sub, mel, lengths in work:                          # untimed: position cache, allocator
                joint.greedy(enc(mel, lengths))
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            outs = [joint.greedy(enc(mel, lengths)) for _, mel, lengths in work]
            e1.record(stream)
            stream.synchronize()
        for (sub, _, _), lab in zip(work, outs):
            for j, i in enumerate(sub):
                labels[i] = lab[j, :enc_frames[i]]
        return [labels[i] for i in indices], e0.elapsed_time(e1) / 1e3

    if dist is not None:
        dist.barrier(device_ids=[local])
    res = B.run_batch(enc_frames, process, device=dev)
    t = max(res.seconds)
    total = sum(enc_frames)
    ops = sum(2 * layer.lin[n].out_features * layer.lin[n].in_features * enc.parts
              for layer in enc.layers for n in E.LAYER_LINEARS) * total / 1e9
    return {"workload": f"BASELINE config 4: {n_clips} synthetic clips, lengths U[2, 30] s ({total} encoder frames, "
                        f"{min(enc_frames)}-{max(enc_frames)} per clip), Kea-T-shaped random-init encoder (2-bit "
                        f"ternary, x2 residual parts), sharded over {world} GPU(s) by frames, grouped into padded "
                        f"forwards of <= {KEA_T_FRAMES_CAP} frames at least modelled cost ({KEA_T_FORWARD_US:.0f} us "
                        f"per forward + {KEA_T_FRAME_US} us per padded frame); labels and timings gathered with NCCL",
            "forwards_rank0": n_forwards[0],
            "clips_per_s": n_clips / t, "frames_per_s": total / t, "ms_per_batch": t * 1e3,
            "per_rank_ms": [v * 1e3 for v in res.seconds], "per_rank_frames": res.frames,
            "lowbit_gop_unpadded": ops, "encoder_lowbit_tops_unpadded": ops / t / 1e3,
            "labels_gathered": len(res.tokens), "timing": "CUDA events on each rank's stream, max over ranks"}


# The reference's own per-GEMM times (RTX 5090, b1_dot with three residual INT8 parts, FP32 output, hot / cold):
# the TUNED_M table comments of src/kea_kernels/binary/configs.py:17-36, keyed by (N, K, M).
REFERENCE_X3_US = {
    (1024, 1024, 38): (2.88, 2.92), (1024, 1024, 126): (3.53, 3.55), (1024, 1024, 256): (4.93, 5.01),
    (1024, 1024, 368): (6.13, 6.34), (1024, 4096, 38): (5.14, 5.23), (1024, 4096, 126): (9.09, 9.20),
    (1024, 4096, 256): (15.21, 15.45), (1024, 4096, 368): (20.84, 21.17), (2048, 1024, 38): (3.52, None),
    (2048, 1024, 126): (4.90, None), (2048, 1024, 256): (7.58, None), (2048, 1024, 368): (10.42, None),
    (3072, 1024, 38): (3.53, None), (3072, 1024, 126): (6.33, None), (3072, 1024, 256): (10.52, None),
    (3072, 1024, 368): (13.31, None), (4096, 1024, 38): (4.31, 4.36), (4096, 1024, 126): (7.52, 7.63),
    (4096, 1024, 256): (13.09, 13.30), (4096, 1024, 368): (19.24, 19.53)}


def reference_table(torch, lowbit, _lib, dev, stream, random_panels, pdl):
    """The reference's published b1_dot x3 shapes on this GPU: 1-bit weights, three INT8 parts, FP32 output, timed
    hot (one weight set, as the reference's "hot") and cold (a graph of launches over >= 4 x L2 of weight sets)."""
    rows = []
    pools = {}
    for (n, k, m), (ref_hot, ref_cold) in REFERENCE_X3_US.items():
        if (n, k) not in pools:
            pools[(n, k)] = random_panels(1, n, k, max(1, min(1024, COLD_BYTES // _lib.panel_bytes(1, n, k))))
        pool = pools[(n, k)]
        alpha = torch.rand(n, device=dev) * 0.02 + 0.001
        q = torch.randint(-127, 128, (3, m, k), dtype=torch.int8, device=dev)
        qs = torch.rand(3, m, device=dev) * 0.01 + 0.001
        y = torch.empty(m, n, device=dev, dtype=torch.float32)
        launches = min(len(pool), 256)

        def timed(hot):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    for i in range(launches):
                        lowbit.gemm(q, qs, k, m, pool[0 if hot else i % len(pool)], 1, n, k, alpha, None, y, parts=3,
                                    pdl=pdl)
                g.replay()
                stream.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
                stream.synchronize()
            return e0.elapsed_time(e1) * 1e3 / launches

        hot, cold = timed(True), timed(False)
        rows.append({"n": n, "k": k, "m": m, "ref_us_hot": ref_hot, "ref_us_cold": ref_cold, "us_hot": hot,
                     "us_cold": cold, "speedup_hot": ref_hot / hot})
    del pools
    geo = math.exp(sum(math.log(r["speedup_hot"]) for r in rows) / len(rows))
    return {"what": "the reference's published b1_dot x3 times (RTX 5090, src/kea_kernels/binary/configs.py:17-36) "
                    "against this GPU on the same arithmetic (1-bit, 3 INT8 parts, FP32 out)",
            "geomean_speedup_hot": geo, "rows": rows}


def time_cases(torch, lowbit, _lib, configs, dev, stream, random_panels, alphas, pdl):
    """Average device time per launch of each case: a CUDA graph of launches that each read a different weight
    set (cold: the sets span COLD_BYTES >= 4 x L2), timed with CUDA events; small-M cases are also timed hot."""
    out = []
    cold_pools = {}
    for wbits, n, k, m in CASES:
        key = (wbits, n, k)
        pb = _lib.panel_bytes(wbits, n, k)
        if key not in cold_pools:
            cold_pools[key] = random_panels(wbits, n, k, max(1, min(1024, COLD_BYTES // pb)))
        pool = cold_pools[key]
        launches = len(pool) if m <= 512 else 24
        nq = 8
        q = torch.randint(-127, 128, (nq, 1, m, k), dtype=torch.int8, device=dev)
        qs = torch.rand(nq, 1, m, device=dev) * 0.015 + 0.005
        y = torch.empty(m, n, device=dev, dtype=torch.float16)

        def run(i, hot=False):
            lowbit.gemm(q[i % nq], qs[i % nq], k, m, pool[0 if hot else i % len(pool)], wbits, n, k, alphas[key],
                        None, y, parts=1, pdl=pdl)

        def timed(hot):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    for i in range(launches):
                        run(i, hot)
                g.replay()
                stream.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
                stream.synchronize()
            return e0.elapsed_time(e1) * 1e3 / launches

        us = timed(False)
        wa, full = alg_bytes(wbits, n, k, m)
        c = configs.choose(m, n, k, wbits, 1)
        rec = {"wbits": wbits, "n": n, "k": k, "m": m, "us": us, "tops": ops(m, n, k) / us / 1e6,
               "gbs_wa": wa / us / 1e3, "gbs_full": full / us / 1e3, "config": c.label(), "launches": launches}
        if m <= 512:
            rec["us_hot"] = timed(True)
        out.append(rec)
        del q, qs, y
    return out


def profile_case(args) -> None:
    """One case, W + K plain launches on the current stream, each on a different weight set (>= 4 x L2 of weights
    rotate unless the set is larger) and activation set; prints the average of the last K launches (CUDA events).
    This is the command the kernel's ncu captures run (`-s W -c 1` selects one cold launch)."""
    import torch

    from kea_kernels import _lib, formats, lowbit
    from kea_kernels.binary import bits, configs

    wbits, n, k, m = (int(v) for v in args.case.split(","))
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(99)
    sets = max(1, min(64, (4 * L2_BYTES) // max(1, _lib.panel_bytes(wbits, n, k))))
    panels = []
    for _ in range(min(sets, 8)):
        if wbits == 1:
            codes = bits.pack_signs(torch.where(torch.rand(n, k, device=dev, generator=gen) < 0.5, -1, 1).to(torch.int8))
        else:
            u = torch.rand(n, k, device=dev, generator=gen)
            codes = formats.pack_ternary(torch.where(u < 0.3, -1, torch.where(u < 0.7, 0, 1)).to(torch.int8))
        panels.append(lowbit.prepare_panels(codes, wbits, n, k))
    panels = [panels[i % len(panels)].clone() for i in range(sets)]
    nq = 2 if m * k * 4 > L2_BYTES else 4
    q = torch.randint(-127, 128, (nq, 1, m, k), dtype=torch.int8, device=dev, generator=gen)
    qs = torch.rand(nq, 1, m, device=dev, generator=gen) * 0.015 + 0.005
    alpha = (torch.rand(n, device=dev, generator=gen) * 0.04 + 0.01).half().float()
    y = torch.empty(m, n, device=dev, dtype=torch.float16)
    torch.cuda.synchronize()

    def run(i):
        lowbit.gemm(q[i % nq], qs[i % nq], k, m, panels[i % sets], wbits, n, k, alpha, None, y, parts=1)

    for i in range(args.warmup):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        run(args.warmup + i)
    e1.record()
    torch.cuda.synchronize()
    if _lib.read_device_error():
        raise RuntimeError("device error word set")
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    wa, full = alg_bytes(wbits, n, k, m)
    print(json.dumps({"case": {"wbits": wbits, "n": n, "k": k, "m": m}, "config": configs.choose(m, n, k, wbits).label(),
                      "us_per_launch": us, "tops": ops(m, n, k) / us / 1e6, "alg_bytes_wa": wa,
                      "alg_bytes_full": full, "weight_sets": sets}), flush=True)


def int8_peak_tops(torch, dev):
    """Dense INT8 tensor rate of this GPU from torch._int_mm at 8192^3 (best of 10)."""
    try:
        a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device=dev)
        b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device=dev)
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = None
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        return 2 * 8192 ** 3 / (best / 1e3) / 1e12, "measured: torch._int_mm 8192^3, best of 10"
    except Exception as exc:  # noqa: BLE001
        return None, f"unavailable ({type(exc).__name__})"


def e2e_rate(torch, lowbit, dev, weights, alphas, args, world, dist, local):
    """The sweep through the C-ABI call with host buffers: per GEMM, pinned host -> device copy of the INT8
    activations and scales, the call, and a device -> pinned host copy of the fp16 output, all timed."""
    host_q = {c: torch.randint(-127, 128, (1, c[3], c[2]), dtype=torch.int8).pin_memory() for c in CASES}
    host_s = {c: (torch.rand(1, c[3]) * 0.015 + 0.005).pin_memory() for c in CASES}
    host_y = {c: torch.empty(c[3], c[1], dtype=torch.float16).pin_memory() for c in CASES}
    dq = {c: torch.empty_like(host_q[c], device=dev) for c in CASES}
    ds = {c: torch.empty_like(host_s[c], device=dev) for c in CASES}
    dy = {c: torch.empty(c[3], c[1], dtype=torch.float16, device=dev) for c in CASES}
    h2d = sum(host_q[c].numel() + 4 * host_s[c].numel() for c in CASES)
    d2h = sum(2 * host_y[c].numel() for c in CASES)

    def step(j):
        for c in CASES:
            wbits, n, k, m = c
            dq[c].copy_(host_q[c], non_blocking=True)
            ds[c].copy_(host_s[c], non_blocking=True)
            lowbit.gemm(dq[c], ds[c], k, m, weights[(wbits, n, k)][j % POOL], wbits, n, k, alphas[(wbits, n, k)],
                        None, dy[c], parts=1)
            host_y[c].copy_(dy[c], non_blocking=True)

    steps = max(3, min(args.steps, 50))
    for j in range(args.warmup):
        step(j)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier(device_ids=[local])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for j in range(steps):
        step(j)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_ops = sum(ops(m, n, k) for _, n, k, m in CASES)
    return {"value": world * step_ops * steps / (ms / 1e3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": ms / steps,
            "path": "kea_lowbit_gemm via ctypes (kea_kernels.lowbit.gemm), pinned host buffers"}


if __name__ == "__main__":
    main()
