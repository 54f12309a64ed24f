"""The engine's segment schedule (crates/qwen3tts/src/engine.rs:831-1033) on CPU: runs by prompt
width, longest-first by characters; per-lane budgets from the learned frames-per-character
ratio; a batched run that reaches the cap redone one segment at a time with the full budget.
Generation is a stand-in that emits a segment's natural number of frames up to its budget."""
from dataclasses import dataclass

import pytest

from qwen3tts.engine import (BATCH_FRAME_CAP, SEGMENT_RATIO_SAMPLE, Engine, learned_ratio,
                             lane_budgets, plan_runs)


@dataclass
class Req:
    key: int
    natural: int       # frames the talker would emit before its end code
    max_frames: int = 4096


def fake(req):
    return [[req.key] * 16 for _ in range(min(req.natural, req.max_frames))]


def test_plan_runs_groups_by_width_longest_first():
    widths = [10, 12, 10, 10, 12, 10]
    chars = [5, 9, 7, 7, 3, 2]
    assert plan_runs(widths, chars, max_batch=2) == [[2, 3], [0, 5], [1, 4]]
    assert plan_runs(widths, chars, max_batch=48) == [[2, 3, 0, 5], [1, 4]]


def test_lane_budgets_and_ratio():
    assert lane_budgets([10, 200], None, 512) == [512, 512]
    # 10 * 1.3 * 2 = 26; 200 * 1.3 * 2 = 520 -> cap; 3 * 1.3 * 2 = 7.8 -> 24
    assert lane_budgets([10, 200, 3], 1.3, 512) == [26, 512, 24]
    assert lane_budgets([7], 1.0, 16) == [16]  # a cap below 24 is every lane's budget
    assert learned_ratio([1.0] * (SEGMENT_RATIO_SAMPLE - 1)) is None
    seen = [float(i) for i in range(16)]
    assert learned_ratio(seen) == 8.0          # the upper middle element


def test_engine_budgets_and_rerun():
    # 20 segments of one width: the first run of 16 has no ratio (cap budgets); the next runs
    # are budgeted at chars x ratio x 2
    chars = [100 + 5 * i for i in range(20)]
    natural = [c // 2 for c in chars]        # 0.5 frames per character
    reqs = [Req(i, natural[i]) for i in range(20)]
    batches = []

    def batched(rs):
        batches.append([(r.key, r.max_frames) for r in rs])
        return [fake(r) for r in rs]

    singles = []

    def single(r):
        singles.append((r.key, r.max_frames))
        return fake(r)

    eng = Engine(batched, single, max_batch=16)
    out = eng.run(reqs, [157] * 20, chars)
    assert [len(f) for f in out] == natural
    assert not singles
    first = batches[0]
    assert [k for k, _ in first] == sorted(range(20), key=lambda i: -chars[i])[:16]
    assert all(b == BATCH_FRAME_CAP for _, b in first)
    ratio = learned_ratio([natural[k] / chars[k] for k, _ in first])
    assert [b for _, b in batches[1]] == lane_budgets([chars[k] for k, _ in batches[1]], ratio,
                                                      BATCH_FRAME_CAP)

    # a lane that runs to the cap: the whole run is redone unbatched with the full budget
    reqs = [Req(0, 600), Req(1, 30), Req(2, 40)]
    batches.clear()
    eng = Engine(batched, single, max_batch=48)
    out = eng.run(reqs, [157] * 3, [120, 50, 60])
    assert eng.log[-1].rerun and eng.log[-1].budgets == [512, 512, 512]
    assert eng.log[-1].segments == [0, 2, 1]
    assert singles == [(0, 4096), (2, 4096), (1, 4096)]
    assert [len(f) for f in out] == [600, 30, 40]


def test_engine_single_segment_runs_unbatched():
    singles = []
    eng = Engine(lambda rs: pytest.fail("batched"), lambda r: singles.append(r.key) or fake(r),
                 budget=100)
    out = eng.run([Req(0, 150)], [9], [10])
    assert singles == [0] and len(out[0]) == 100
