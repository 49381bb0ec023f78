"""CPU: the clip-batch scheduler and the result gather (kea_kernels.batch), including two-rank runs on the gloo
backend: shard balance, gather order, and a failing rank that the other rank sees as an error, not a hang."""
from __future__ import annotations

import multiprocessing as mp
import os
import random
import socket
import sys
import time
import traceback

import pytest
import torch

from conftest import ROOT
from kea_kernels import batch


def test_shard_assigns_every_clip_once_and_balances_frames():
    rng = random.Random(0)
    frames = [rng.randint(25, 375) for _ in range(257)]
    for world in (1, 2, 4, 8):
        ranks = batch.shard(frames, world)
        flat = sorted(i for r in ranks for i in r)
        assert flat == list(range(len(frames)))
        loads = [sum(frames[i] for i in r) for r in ranks]
        assert max(loads) - min(loads) <= max(frames)          # greedy LPT bound
        assert all(r == sorted(r) for r in ranks)
        assert ranks == batch.shard(frames, world)             # deterministic
    assert batch.shard([], 4) == [[], [], [], []]
    with pytest.raises(ValueError):
        batch.shard([1], 0)


def test_buckets_group_by_length():
    frames = [10, 300, 125, 125, 40, 900]
    b = batch.buckets(frames, [50, 200, 400])
    assert b == [[4, 0], [2, 3], [1], [5]]
    with pytest.raises(ValueError):
        batch.buckets([-1], [10])


def _set_partitions(items):
    if not items:
        yield []
        return
    for p in _set_partitions(items[1:]):
        for k in range(len(p)):
            yield p[:k] + [[items[0]] + p[k]] + p[k + 1:]
        yield [[items[0]]] + p


def _plan_cost(groups, frames, cap, forward_cost, frame_cost):
    total = 0.0
    for g in groups:
        padded = len(g) * max(frames[i] for i in g)
        if padded > cap and len(g) > 1:
            return float("inf")
        total += forward_cost + frame_cost * padded
    return total


def test_plan_is_the_least_cost_grouping():
    """The planner's grouping costs no more than the best of all set partitions (brute force, up to 6 clips)."""
    rng = random.Random(7)
    for _ in range(150):
        frames = [rng.randint(0, 60) for _ in range(rng.randint(0, 6))]
        cap, fc, pc = rng.randint(1, 200), rng.choice([0, 1, 5, 30, 100]), rng.choice([0, 0.1, 1, 3])
        groups = batch.plan(frames, cap, fc, pc)
        assert sorted(i for g in groups for i in g) == list(range(len(frames)))
        for g in groups:
            assert [frames[i] for i in g] == sorted((frames[i] for i in g), reverse=True)
        best = min(_plan_cost(p, frames, cap, fc, pc) for p in _set_partitions(list(range(len(frames)))))
        assert _plan_cost(groups, frames, cap, fc, pc) == pytest.approx(best)


def test_plan_merges_or_splits_by_cost():
    frames = [100] * 4 + [60] * 4
    assert batch.plan(frames, 10_000, 1.0, 1.0) == [[0, 1, 2, 3], [4, 5, 6, 7]]      # no padding when forwards are cheap
    assert batch.plan(frames, 10_000, 1e6, 1.0) == [list(range(8))]                   # one forward when they are dear
    assert batch.plan(frames, 250, 1e6, 1.0) == [[0, 1], [2, 3], [4, 5, 6, 7]]        # at most 250 padded frames
    assert batch.plan([500, 10], 100, 1.0, 1.0) == [[0], [1]]                         # a clip over the cap goes alone
    assert batch.plan([], 100, 1.0, 1.0) == []
    for bad in ((lambda: batch.plan([1], 0, 1, 1)), (lambda: batch.plan([-1], 9, 1, 1)),
                (lambda: batch.plan([1], 9, -1, 1))):
        with pytest.raises(ValueError):
            bad()


def test_pack_round_trip():
    rows = [torch.randn(t, 8) for t in (3, 0, 5, 1)]
    packed, off = batch.pack(rows)
    assert packed.shape == (9, 8) and off.tolist() == [0, 3, 3, 8, 9]
    for a, b in zip(rows, batch.unpack(packed, off)):
        assert torch.equal(a, b)
    with pytest.raises(ValueError):
        batch.pack([torch.zeros(2, 3), torch.zeros(2, 4)])


def test_single_process_gather_is_identity():
    toks = [torch.tensor([3, 1], dtype=torch.int32), torch.tensor([7], dtype=torch.int32)]
    g = batch.gather([1, 0], toks, 0.5, 3, 2, torch.device("cpu"))
    assert [t.tolist() for t in g.tokens] == [[7], [3, 1]] and g.seconds == [0.5]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens_for(i: int) -> torch.Tensor:
    return torch.arange(i % 5, dtype=torch.int32) * 10 + i     # clip i: i % 5 tokens (some clips have none)


def _rank_main(rank: int, world: int, port: int, mode: str, frames: list, out_q) -> None:
    sys.path.insert(0, str(ROOT / "kea-kernels_b200"))
    from datetime import timedelta

    import torch.distributed as dist

    from kea_kernels import batch as B
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the gather")

        def process(mine):
            return [_tokens_for(i) for i in mine], 0.01 * (rank + 1)

        g = B.run_batch(frames, process, device=torch.device("cpu"))
        out_q.put((rank, "ok", [t.tolist() for t in g.tokens], g.seconds, g.frames))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        out_q.put((rank, "error", f"{type(exc).__name__}: {exc}", traceback.format_exc()[-400:], None))


def _run_ranks(world: int, mode: str, frames: list, limit: float = 90.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, frames, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + limit
    while len(results) < world and time.time() < deadline:
        try:
            r = q.get(timeout=1.0)
            results[r[0]] = r
        except Exception:  # noqa: BLE001 - queue.Empty
            pass
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
        if p.is_alive():
            p.kill()
            p.join()
    return results


def test_two_rank_gather_returns_clips_in_batch_order():
    frames = [125, 300, 25, 125, 250, 90, 375, 40, 10]
    res = _run_ranks(2, "ok", frames)
    assert set(res) == {0, 1}, res
    expected = [_tokens_for(i).tolist() for i in range(len(frames))]
    shards = batch.shard(frames, 2)
    for r in (0, 1):
        rank, status, toks, seconds, fr = res[r]
        assert status == "ok", res[r]
        assert toks == expected
        assert seconds == pytest.approx([0.01, 0.02])
        assert fr == [sum(frames[i] for i in s) for s in shards]


def test_failing_rank_ends_the_other_ranks_collective_with_an_error():
    t0 = time.time()
    res = _run_ranks(2, "fail", [10, 20, 30, 40])
    assert time.time() - t0 < 90
    assert res[1][1] == "error" and "rank 1 failed" in res[1][2]
    assert res[0][1] == "error", res[0]          # its gather raised (peer gone or timeout), it did not hang
