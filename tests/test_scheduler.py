"""Lane scheduling policy on the host (no GPU): grouping and longest-first order
(crates/qwen3tts/src/engine.rs:835-863), tail shedding in quanta of 8
(crates/qwen3tts/src/talker.rs:1002-1017), and the data-parallel split of groups over ranks."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwen3tts.talker import (SHED_QUANTUM, Segment, plan_groups, shard_groups, shard_segments,
                             shed_widths, synthetic_segments)


def test_synthetic_segments_log_uniform():
    segs = synthetic_segments(5000, seed=1)
    f = np.array([s.frames for s in segs])
    assert f.min() >= 40 and f.max() <= 1200
    # log-uniform: the median sits near the geometric mean of the bounds
    assert abs(np.median(f) - np.sqrt(40 * 1200)) < 25


def test_groups_longest_first_stable_and_bounded():
    segs = [Segment(i, 157 if i % 3 else 100, f, f) for i, f in
            enumerate([5, 9, 9, 1, 7, 9, 2, 8, 8, 3, 6, 4, 9, 1, 5])]
    groups = plan_groups(segs, max_lanes=4)
    assert all(len(g) <= 4 for g in groups)
    seen = [s.index for g in groups for s in g]
    assert sorted(seen) == list(range(len(segs)))
    for g in groups:
        assert len({s.prompt_len for s in g}) == 1
        keys = [(-s.weight, s.index) for s in g]
        assert keys == sorted(keys)  # longest first, ties by index
    # runs are cut from one sorted list per prompt width
    g157 = [s for g in groups for s in g if s.prompt_len == 157]
    assert [(-s.weight, s.index) for s in g157] == sorted((-s.weight, s.index) for s in g157)


def simulate(frames, quantum):
    """Brute force: each step, live = smallest multiple of quantum covering the last unfinished
    lane (never growing)."""
    live, step, out = len(frames), 0, []
    while any(f > step for f in frames[:live]):
        last = max(i for i in range(live) if frames[i] > step) + 1
        live = min(live, -(-last // quantum) * quantum)
        out.append(live)
        step += 1
    return out


@pytest.mark.parametrize("seed", range(5))
def test_shed_widths_match_simulation(seed):
    rng = np.random.default_rng(seed)
    frames = sorted(rng.integers(1, 60, int(rng.integers(1, 50))).tolist(), reverse=True)
    w = shed_widths(frames)
    assert w == simulate(frames, SHED_QUANTUM)
    assert len(w) == max(frames)
    assert sum(frames) <= sum(w)  # lane-steps cover every frame
    assert all(x % SHED_QUANTUM == 0 or x == len(frames) for x in w)


def test_shard_groups_lpt_balanced_and_deterministic():
    segs = synthetic_segments(2000, seed=3)
    groups = plan_groups(segs, 48)
    for world in (1, 2, 4, 8):
        shards = shard_groups(groups, world)
        assert shard_groups(groups, world) == shards
        idx = sorted(s.index for sh in shards for g in sh for s in g)
        assert idx == list(range(2000))
        loads = [sum(max(s.frames for s in g) * len(g) for g in sh) for sh in shards]
        assert max(loads) - min(loads) <= max(max(s.frames for s in g) * len(g) for g in groups)


def test_shard_segments_lpt_balanced_and_deterministic():
    # single segments by frames: every segment once, deterministic, and loads within one
    # segment of each other (LPT's bound for items assigned longest first)
    segs = synthetic_segments(2000, seed=3)
    longest = max(s.frames for s in segs)
    for world in (1, 2, 3, 4, 8):
        shards = shard_segments(segs, world)
        assert shard_segments(segs, world) == shards
        assert sorted(s.index for sh in shards for s in sh) == list(range(2000))
        loads = [sum(s.frames for s in sh) for sh in shards]
        assert max(loads) - min(loads) <= longest
        # each rank's queue is its own longest-first grouping
        for sh in shards:
            groups = plan_groups(sh, 48)
            assert sorted(s.index for g in groups for s in g) == sorted(s.index for s in sh)
    # at the document sample's sizes the frame loads are within 0.5% (whole groups: 15-52%)
    for world in (2, 4, 8):
        loads = [sum(s.frames for s in sh)
                 for sh in shard_segments(synthetic_segments(96 * world, seed=0), world)]
        assert max(loads) / (sum(loads) / world) < 1.005


def _rank_main(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    segs = synthetic_segments(300, seed=7)
    mine = shard_groups(plan_groups(segs, 48), world)[rank]
    idx = torch.tensor(sorted(s.index for g in mine for s in g) + [-1] * 300)[:300]
    gathered = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(gathered, idx)
    if rank == 0:
        allidx = sorted(int(v) for t in gathered for v in t.tolist() if v >= 0)
        out.put(allidx)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_shards_cover_every_segment_once():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    got = out.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == list(range(300))
