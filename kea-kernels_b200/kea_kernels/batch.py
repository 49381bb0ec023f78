"""Clip-batch scheduling across the GPUs of one node, and the gather of per-clip results.

kea-kernels transcribes one clip at a time (batch 1). Here a batch of independent clips is sharded over R ranks (one
process per GPU): every rank runs the whole encoder on its clips, and the only collective is the gather of results
after the batch (NCCL on GPUs, gloo in the CPU tests). Nothing here touches the GEMM.

  * `buckets(frames, edges)`   - clip indices grouped by length bucket, longest first inside a bucket;
  * `plan(frames, cap, ...)`   - clips grouped into padded forwards at the least modelled cost (a fixed cost per
                                 forward + a cost per padded frame), at most `cap` padded frames per forward;
  * `shard(frames, world)`     - whole clips dealt to ranks, balanced by frame count (longest-processing-time
                                 greedy; deterministic);
  * `pack(rows)`               - varlen packing: per-clip [T_i, D] feature rows -> one [sum T_i, D] matrix + offsets,
                                 so every GEMM of the encoder sees M = sum T_i with no padding rows;
  * `gather(...)`              - all_gather of padded int32 token rows, lengths and per-rank timings, returned in
                                 the batch's original clip order on every rank.

A rank that fails raises on its own process; the others see the failure as an error from their next collective
(the process group's timeout bounds the wait), never as a hang.
"""
from __future__ import annotations

import dataclasses
import time
from typing import Callable, Sequence

import torch
import torch.distributed as dist
from torch import Tensor


def buckets(frames: Sequence[int], edges: Sequence[int]) -> list[list[int]]:
    """Clip indices per length bucket: bucket b holds clips with edges[b-1] < frames <= edges[b] (the last bucket
    takes everything longer), longest first, ties by index."""
    edges = sorted(int(e) for e in edges)
    out: list[list[int]] = [[] for _ in range(len(edges) + 1)]
    for i, f in enumerate(frames):
        if f < 0:
            raise ValueError(f"clip {i}: negative frame count {f}")
        b = 0
        while b < len(edges) and f > edges[b]:
            b += 1
        out[b].append(i)
    for lst in out:
        lst.sort(key=lambda i: (-frames[i], i))
    return out


def plan(frames: Sequence[int], cap: int, forward_cost: float, frame_cost: float) -> list[list[int]]:
    """Groups clips into padded forwards: each group is padded to its longest clip, so it costs
    `forward_cost + frame_cost * len(group) * longest` and holds at most `cap` padded frames (a single clip longer
    than `cap` goes alone). Exact minimum of the summed cost over all groupings: an optimal grouping takes clips
    contiguous in length order, so a dynamic programme over the clips sorted longest first (ties by index) finds it.
    A large `forward_cost` against `frame_cost` merges few-clip length ranges into one forward; a small one keeps
    lengths apart. Returns the groups longest first, each longest first."""
    if cap < 1:
        raise ValueError("cap must be >= 1")
    if forward_cost < 0 or frame_cost < 0:
        raise ValueError("costs must be >= 0")
    for i, f in enumerate(frames):
        if f < 0:
            raise ValueError(f"clip {i}: negative frame count {f}")
    order = sorted(range(len(frames)), key=lambda i: (-frames[i], i))
    lens = [int(frames[i]) for i in order]
    n = len(order)
    best = [0.0] + [float("inf")] * n       # best[j]: least cost of the first j clips in `order`
    start = [0] * (n + 1)
    for j in range(1, n + 1):
        for i in range(j - 1, -1, -1):      # group order[i:j], padded to lens[i]; grows as i falls
            padded = (j - i) * lens[i]
            if padded > cap and i < j - 1:
                break
            c = best[i] + forward_cost + frame_cost * padded
            if c < best[j]:
                best[j], start[j] = c, i
    groups = []
    j = n
    while j > 0:
        groups.append(order[start[j]:j])
        j = start[j]
    return groups[::-1]


def shard(frames: Sequence[int], world: int) -> list[list[int]]:
    """Assigns whole clips to `world` ranks, balancing total frames: clips in decreasing length each go to the rank
    with the fewest frames so far (ties: the lower rank). Every rank's list is in increasing clip index."""
    if world < 1:
        raise ValueError("world must be >= 1")
    load = [0] * world
    ranks: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(frames)), key=lambda i: (-frames[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        ranks[r].append(i)
        load[r] += int(frames[i])
    for lst in ranks:
        lst.sort()
    return ranks


def pack(rows: Sequence[Tensor]) -> tuple[Tensor, Tensor]:
    """[T_i, D] tensors -> (packed [sum T_i, D], offsets int64 [n + 1]); offsets[i] is clip i's first row."""
    if not rows:
        raise ValueError("nothing to pack")
    d = rows[0].shape[-1]
    for r in rows:
        if r.dim() != 2 or r.shape[1] != d:
            raise ValueError("every clip must be [T_i, D] with one D")
    lengths = torch.tensor([r.shape[0] for r in rows], dtype=torch.int64)
    offsets = torch.zeros(len(rows) + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(lengths, 0)
    return torch.cat(list(rows), 0), offsets


def unpack(packed: Tensor, offsets: Tensor) -> list[Tensor]:
    return [packed[int(offsets[i]):int(offsets[i + 1])] for i in range(offsets.numel() - 1)]


@dataclasses.dataclass
class Gathered:
    tokens: list[Tensor]        # int32 [len_i] per clip, in the batch's clip order
    seconds: list[float]        # each rank's device / wall time for its shard
    frames: list[int]           # each rank's frame count


def gather(indices: Sequence[int], tokens: Sequence[Tensor], seconds: float, frames: int, n_clips: int,
           device: torch.device, group=None) -> Gathered:
    """All ranks exchange their clips' results. `indices[j]` is the batch index of this rank's clip j and
    `tokens[j]` its int32 result row. Collectives, in the same order on every rank: all_gather of
    (clip count, longest row), then of the padded [max_count, max_len] rows, their lengths and indices, then of the
    timing record. Without an initialised process group (one process) it is the identity."""
    if len(indices) != len(tokens):
        raise ValueError("one token row per clip")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        order = sorted(range(len(indices)), key=lambda j: indices[j])
        if sorted(indices) != list(range(n_clips)):
            raise ValueError("a single rank must hold every clip")
        return Gathered([tokens[j].to(torch.int32).cpu() for j in order], [float(seconds)], [int(frames)])

    head = torch.tensor([len(indices), max((t.numel() for t in tokens), default=0)], dtype=torch.int64, device=device)
    heads = [torch.empty_like(head) for _ in range(world)]
    dist.all_gather(heads, head, group=group)
    heads = torch.stack(heads).cpu()
    max_count, max_len = int(heads[:, 0].max()), max(1, int(heads[:, 1].max()))

    rows = torch.zeros(max_count, max_len, dtype=torch.int32, device=device)
    meta = torch.full((max_count, 2), -1, dtype=torch.int64, device=device)   # (batch index, length)
    for j, (i, t) in enumerate(zip(indices, tokens)):
        rows[j, :t.numel()] = t.to(device=device, dtype=torch.int32)
        meta[j, 0], meta[j, 1] = int(i), t.numel()
    all_rows = [torch.empty_like(rows) for _ in range(world)]
    all_meta = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(all_rows, rows, group=group)
    dist.all_gather(all_meta, meta, group=group)
    timing = torch.tensor([float(seconds), float(frames)], dtype=torch.float64, device=device)
    all_timing = [torch.empty_like(timing) for _ in range(world)]
    dist.all_gather(all_timing, timing, group=group)

    out: list[Tensor | None] = [None] * n_clips
    for r in range(world):
        rr, mm = all_rows[r].cpu(), all_meta[r].cpu()
        for j in range(int(heads[r, 0])):
            i, n = int(mm[j, 0]), int(mm[j, 1])
            if not 0 <= i < n_clips or out[i] is not None:
                raise RuntimeError(f"gather: clip index {i} from rank {r} is out of range or duplicated")
            out[i] = rr[j, :n].clone()
    missing = [i for i, t in enumerate(out) if t is None]
    if missing:
        raise RuntimeError(f"gather: no rank returned clips {missing[:8]}")
    tim = torch.stack(all_timing).cpu()
    return Gathered(out, [float(v) for v in tim[:, 0]], [int(v) for v in tim[:, 1]])  # type: ignore[arg-type]


def run_batch(frames: Sequence[int], process: Callable[[list[int]], tuple[list[Tensor], float]], *,
              device: torch.device, group=None) -> Gathered:
    """Shards the batch's clips over the ranks, runs `process(my_clip_indices) -> (token rows, seconds)` on this
    rank's shard and gathers everything. `seconds` is the rank's own measurement (CUDA events around its device
    work); the caller takes the max over ranks from the result."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    mine = shard(frames, world)[rank]
    t0 = time.perf_counter()
    tokens, seconds = process(mine)
    if seconds is None:
        seconds = time.perf_counter() - t0
    return gather(mine, tokens, seconds, sum(int(frames[i]) for i in mine), len(frames), device, group)
