"""The talker's lane scheduler on B200: groups, longest-first order, tail shedding, and the
data-parallel split of a document's segments over GPUs.

Mirrors crates/qwen3tts/src/engine.rs:831-863 (group segments by prompt length, sort each group
longest-first with an index tie-break, cut it into runs of at most `max_lanes`) and
crates/qwen3tts/src/talker.rs:947-1017 (each step every live lane emits a frame; a lane that
reaches its end is done; the finished tail is shed, the live width rounded up to a multiple of
SHED_QUANTUM). Device-side differences, by design:

  * the KV cache is paged (`PagedKv`), so each lane has its own position and a finished lane's
    pages go back to the pool; with `refill=True` its slot is reused at once by the next queued
    segment (interior refill), which the reference's contiguous cache cannot do;
  * the step for each live width is a CUDA graph captured once and replayed, and the host
    decides lane completion from the segment targets without reading the device every step.

Random-init weights never emit the end code, so a segment's end is its drawn target length
(the synthetic lane sweep: log-uniform in [40, 1200] frames), i.e. the end code is forced there.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

SHED_QUANTUM = 8      # crates/qwen3tts/src/talker.rs:92
MAX_BATCH = 48        # crates/qwen3tts/src/engine.rs:95


@dataclass
class Segment:
    index: int
    prompt_len: int
    frames: int          # frames this segment runs for (its end code is forced there)
    weight: int = 0      # the sort key: the reference sorts by character count


def synthetic_segments(n: int, seed: int = 0, lo: int = 40, hi: int = 1200,
                       prompt_len: int = 157) -> list[Segment]:
    """The synthetic sweep and document: target lengths log-uniform in [lo, hi] frames, one prompt width
    (157, the reference ICL width recorded in fixtures/qwen3tts/oracle.json)."""
    rng = np.random.default_rng(seed)
    f = np.exp(rng.uniform(math.log(lo), math.log(hi), n)).astype(int)
    return [Segment(i, prompt_len, int(f[i]), int(f[i])) for i in range(n)]


def plan_groups(segments: list[Segment], max_lanes: int = MAX_BATCH) -> list[list[Segment]]:
    """Groups of equal prompt length, each sorted longest-first (stable, index tie-break) and
    cut into runs of at most `max_lanes` (crates/qwen3tts/src/engine.rs:835-863)."""
    by_shape: dict[int, list[Segment]] = {}
    for s in segments:
        by_shape.setdefault(s.prompt_len, []).append(s)
    shapes = sorted(by_shape.values(), key=lambda g: g[0].index)
    groups: list[list[Segment]] = []
    for g in shapes:
        g = sorted(g, key=lambda s: (-s.weight, s.index))
        for i in range(0, len(g), max_lanes):
            groups.append(g[i:i + max_lanes])
    return groups


def group_cost(group: list[Segment]) -> int:
    """Steps a group runs for under tail shedding: its longest lane."""
    return max(s.frames for s in group)


def shard_groups(groups: list[list[Segment]], world: int) -> list[list[list[Segment]]]:
    """Longest-processing-time-first assignment of groups to `world` GPUs: each group, most
    expensive first, goes to the least-loaded GPU (ties to the lowest rank). Deterministic,
    so every rank computes the same split without talking to the others."""
    shards: list[list[list[Segment]]] = [[] for _ in range(world)]
    load = [0] * world
    for g in sorted(groups, key=lambda g: (-group_cost(g) * len(g), g[0].index)):
        r = min(range(world), key=lambda i: (load[i], i))
        shards[r].append(g)
        load[r] += group_cost(g) * len(g)
    return shards


def shard_segments(segments: list[Segment], world: int) -> list[list[Segment]]:
    """Longest-processing-time-first assignment of single segments to `world` GPUs by frame
    count (each segment, longest first, to the least-loaded GPU, ties to the lowest rank), for
    ranks that decode with interior refill: a refilling talker's time follows its frames, not
    its groups, and whole groups are too coarse a unit when a rank holds only a few of them.
    Deterministic, so every rank computes the same split without talking to the others. Each
    rank then plans its own groups (plan_groups) over its segments."""
    shards: list[list[Segment]] = [[] for _ in range(world)]
    load = [0] * world
    for s in sorted(segments, key=lambda s: (-s.frames, s.index)):
        r = min(range(world), key=lambda i: (load[i], i))
        shards[r].append(s)
        load[r] += s.frames
    return shards


def shed_widths(frames: list[int], quantum: int = SHED_QUANTUM) -> list[int]:
    """Live width at each step of a group whose lanes run `frames[i]` steps, with the finished
    tail shed (crates/qwen3tts/src/talker.rs:1002-1017). Lanes arrive longest-first, so the
    width only shrinks."""
    widths = []
    n = len(frames)
    live = n
    step = 0
    while True:
        needed = live
        while needed > 0 and frames[needed - 1] <= step:
            needed -= 1
        if needed == 0:
            break
        target = -(-needed // quantum) * quantum
        if target < live:
            live = target
        widths.append(live)
        step += 1
    return widths


@dataclass
class GroupStats:
    frames: int = 0
    steps: int = 0
    lane_steps: int = 0
    graphs: int = 0
    seconds: float = 0.0

    @property
    def useful(self) -> float:
        return self.frames / max(1, self.lane_steps)


class Talker:
    """Runs groups of segments through a `Stack` on one GPU.

    The pool holds `max_lanes` lanes of `capacity` positions. Each live width gets one captured
    graph (built on first use); a step is one replay. `refill=True` admits queued segments into
    finished lanes (their own prompt positions, fresh pages) instead of only shedding the tail.
    """

    def __init__(self, stack, max_lanes: int, capacity: int, block_size: int = 32):
        import torch
        from .stack import PagedKv
        self.torch = torch
        self.stack = stack
        self.geo = stack.geo
        self.max_lanes = max_lanes
        self.capacity = capacity
        per_lane = -(-capacity // block_size)
        self.kv = PagedKv(self.geo, max_lanes, max_lanes * per_lane, block_size, per_lane,
                          stack.device)
        dev = stack.device
        self.codes = torch.zeros(max_lanes, max(1, self.geo.codebooks), dtype=torch.int32,
                                 device=dev)
        self.x0 = torch.zeros(max_lanes, self.geo.dim, device=dev)
        # the step's feedback input, owned here so a reused lane slot can be restarted
        self.x_next = torch.zeros(max(max_lanes, 1), self.geo.dim, device=dev)
        stack.set_feedback(self.x_next)
        self.stream = torch.cuda.Stream(dev)
        self.graphs: dict[int, object] = {}

    def _graph(self, width: int):
        g = self.graphs.get(width)
        if g is None:
            with self.torch.cuda.stream(self.stream):
                g = self.stack.capture(self.kv, None, lanes=width, codes=self.codes,
                                       max_span=self.capacity)
            self.graphs[width] = g
        return g

    def _admit(self, lane: int, seg: Segment, gen) -> None:
        need = seg.prompt_len + seg.frames + 1
        if need > self.capacity:
            raise ValueError(f"segment {seg.index} needs {need} positions, capacity {self.capacity}")
        self.kv.admit(lane, need, seg.prompt_len)
        # The prompt's K/V stand in for prefill (not on this path): seeded values at the lane's
        # prompt positions, and a seeded input row for its first step.
        self.x0[lane].normal_(generator=gen)

    def run(self, queue: list[Segment], refill: bool = False, seed: int = 0) -> GroupStats:
        """Decodes every segment of `queue` (in group order: longest-first) through groups of at
        most `max_lanes` lanes. Every device operation, the page admissions included, is ordered
        on this talker's stream, so the host never waits for the device inside the loop."""
        torch = self.torch
        gen = torch.Generator(device=self.stack.device).manual_seed(seed)
        st = GroupStats()
        pending = list(queue)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            start.record(self.stream)
            while pending:
                lanes: list[Segment | None] = []
                while pending and len(lanes) < self.max_lanes:
                    seg = pending.pop(0)
                    self._admit(len(lanes), seg, gen)
                    lanes.append(seg)
                emitted = [0] * len(lanes)
                # first step from the seeded rows; later steps feed back the code embeddings
                self.stack.decode_step(self.kv, self.x0, lanes=len(lanes), codes=self.codes,
                                       max_span=self.capacity)
                live = len(lanes)
                while True:
                    for i in range(live):
                        if lanes[i] is not None and emitted[i] < lanes[i].frames:
                            emitted[i] += 1
                            st.frames += 1
                    st.lane_steps += live
                    st.steps += 1
                    for i in range(live):  # lanes whose last frame was this step
                        if lanes[i] is not None and emitted[i] >= lanes[i].frames:
                            self.kv.release(i)
                            if refill and pending:
                                seg = pending.pop(0)
                                self._admit(i, seg, gen)
                                self.x_next[i].copy_(self.x0[i])  # restart the slot's input
                                lanes[i] = seg
                                emitted[i] = 0
                            else:
                                lanes[i] = None
                    needed = live
                    while needed > 0 and lanes[needed - 1] is None:
                        needed -= 1
                    if needed == 0:
                        break
                    live = min(live, -(-needed // SHED_QUANTUM) * SHED_QUANTUM)
                    self._graph(live).replay()
            end.record(self.stream)
        st.graphs = len(self.graphs)
        self.stream.synchronize()
        st.seconds = start.elapsed_time(end) * 1e-3
        return st
