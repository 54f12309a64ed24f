"""The engine's segment schedule over the text-to-audio pipeline, as crates/qwen3tts/src/
engine.rs:831-1033 runs a request's segments through the talker:

  * segments are grouped by prompt width (groups in order of their first segment), each group
    sorted longest-first by character count with an index tie-break and cut into runs of at
    most `max_batch` lanes (engine.rs:835-863);
  * a run of more than one lane gets per-lane frame budgets: the frames-per-character ratio
    learned from the segments already decoded, times 2, clamped to [24, cap], where cap =
    min(request budget, 512); before 16 segments have been seen every lane gets the cap
    (engine.rs:941-954);
  * if any lane of a batched run reached the cap, the run is redone one segment at a time with
    the full budget rather than shipping truncated audio (engine.rs:976-1011);
  * after each run the ratio is the median (upper middle element) of frames / characters over
    segments of at least 40 characters (engine.rs:1013-1025).

The generation itself is the caller's: `batched(requests)` and `single(request)` return each
request's frames ([n][16] codes), e.g. `Synthesizer.generate` on a pool sized for the batch cap
and on a one-lane pool sized for the full budget.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import Callable, Optional

SEGMENT_MIN_CHARS = 40        # engine.rs:50
SEGMENT_MIN_FRAMES = 24       # engine.rs:55
MAX_BATCH = 48                # engine.rs:95
SEGMENT_BUDGET_SLACK = 2.0    # engine.rs:116
SEGMENT_RATIO_SAMPLE = 16     # engine.rs:129
BATCH_FRAME_CAP = 512         # engine.rs:137
MAX_NEW_TOKENS = 4096         # cfg.rs:124 (talker)


def plan_runs(widths: list[int], chars: list[int], max_batch: int = MAX_BATCH) -> list[list[int]]:
    """Segment indices in runs: equal prompt width, longest-first by characters (stable, index
    tie-break), at most `max_batch` per run (engine.rs:835-863)."""
    by_width: dict[int, list[int]] = {}
    for i, w in enumerate(widths):
        by_width.setdefault(w, []).append(i)
    runs = []
    for g in sorted(by_width.values(), key=lambda g: g[0]):
        g = sorted(g, key=lambda i: (-chars[i], i))
        runs += [g[k:k + max_batch] for k in range(0, len(g), max_batch)]
    return runs


def lane_budgets(chars: list[int], ratio: Optional[float], cap: int) -> list[int]:
    """Frames each lane of a batched run may emit (engine.rs:948-954): chars x ratio x 2,
    truncated, clamped to [24, cap]; the cap for every lane while no ratio is known. (The
    reference's clamp requires cap >= 24; a smaller cap is every lane's budget here.)"""
    if ratio is None:
        return [cap] * len(chars)
    lo = min(SEGMENT_MIN_FRAMES, cap)
    return [min(max(int(c * ratio * SEGMENT_BUDGET_SLACK), lo), cap) for c in chars]


def learned_ratio(seen: list[float]) -> Optional[float]:
    """The median frames-per-character once 16 segments are in (engine.rs:1020-1024)."""
    if len(seen) < SEGMENT_RATIO_SAMPLE:
        return None
    s = sorted(seen)
    return s[len(s) // 2]


@dataclass
class RunLog:
    segments: list[int]   # the batched run's segment indices, longest first
    budgets: list[int]
    rerun: bool


@dataclass
class Engine:
    batched: Callable[[list], list]        # requests -> frames per request (one run)
    single: Callable[[object], list]       # request -> frames (full budget)
    max_batch: int = MAX_BATCH
    budget: int = MAX_NEW_TOKENS
    batch_cap: int = BATCH_FRAME_CAP
    log: list[RunLog] = field(default_factory=list)

    def run(self, requests: list, widths: list[int], chars: list[int]) -> list[list]:
        """Frames per request, in request order. `widths` are the prompts' widths (the grouping
        key), `chars` the segments' character counts (the sort key and the ratio's unit)."""
        if not (len(requests) == len(widths) == len(chars)):
            raise ValueError("requests, widths and chars differ in length")
        budget = max(1, min(self.budget, MAX_NEW_TOKENS))
        out: list = [None] * len(requests)
        seen: list[float] = []
        ratio = None
        for run in plan_runs(widths, chars, self.max_batch):
            frames = None
            if len(run) > 1:
                cap = min(budget, self.batch_cap)
                budgets = lane_budgets([chars[i] for i in run], ratio, cap)
                got = self.batched([dataclasses.replace(requests[i], max_frames=b)
                                    for i, b in zip(run, budgets)])
                rerun = any(len(f) >= cap for f in got)
                self.log.append(RunLog(list(run), budgets, rerun))
                if not rerun:
                    frames = got
            if frames is None:
                frames = [self.single(dataclasses.replace(requests[i], max_frames=budget))
                          for i in run]
            for i, f in zip(run, frames):
                out[i] = f
                if chars[i] >= SEGMENT_MIN_CHARS:
                    seen.append(len(f) / chars[i])
            if len(seen) >= SEGMENT_RATIO_SAMPLE:
                ratio = learned_ratio(seen)
        return out
