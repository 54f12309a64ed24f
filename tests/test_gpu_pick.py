"""The talker's greedy pick rule on a B200 (sample_with_u with greedy on,
crates/qwen3tts/src/talker.rs:154-189, 940, 971-981) against the CPU oracle, bit for bit.

Hand-made logits and histories: ids emitted 1, 2 and 7 times, rows where the runner-up sits one
ulp either side of the leader's penalised value (so one f32 division more or less, or a power of
the penalty instead of the sequence, changes the pick), negative rows (the penalty multiplies),
banned maxima, a young eos and exact ties (the last maximum wins). The pick is integer output:
every row must equal the oracle's, with no tie allowance."""
from collections import Counter

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

VOCAB, EOS, MIN_NEW, PENALTY = 3072, 2150, 2, 1.05
BANNED = [i for i in range(VOCAB - 1024, VOCAB) if i != EOS]


def seq_penalty(x, times):
    p = np.float32(PENALTY)
    for _ in range(times):
        x = np.float32(x / p) if x > 0 else np.float32(x * p)
    return x


def hand_made(seed, rows):
    """Logits, histories and frame counts built so the per-occurrence rule decides."""
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((rows, VOCAB)) * 1.5).astype(np.float32)
    seen = [[] for _ in range(rows)]
    frames = rng.integers(0, 6, rows).astype(np.int32)
    for r in range(rows):
        kind = r % 8
        a, b = (int(i) for i in rng.choice(VOCAB - 1024, 2, replace=False))
        k = (1, 2, 7)[r % 3]
        sign = 1.0 if kind < 4 else -1.0
        top = np.float32(sign * (6.0 + rng.random()))
        logits[r, a] = top
        pen = seq_penalty(top, k)
        # the runner-up one ulp above, at, or below the leader's penalised value
        step = (-1, 0, 1)[(r // 3) % 3]
        runner = np.nextafter(pen, np.float32(np.inf if step > 0 else -np.inf)) if step else pen
        if sign < 0:
            # negative rows: the runner-up must still beat every other id
            logits[r, np.abs(logits[r]) < 20] = np.minimum(logits[r, np.abs(logits[r]) < 20], -30)
            logits[r, a] = top
        logits[r, b] = np.float32(runner)
        seen[r] = [a] * k + [int(i) for i in rng.choice(VOCAB - 1024, 5)]
        rng.shuffle(seen[r])
        if kind == 3:
            # an exact tie between two ids after the penalty: the higher index wins
            c = int(rng.integers(0, VOCAB - 1024))
            logits[r, c] = logits[r, b]
        if kind == 5:
            # a banned id and a young eos above everything
            logits[r, BANNED[r % len(BANNED)]] = 100.0
            logits[r, EOS] = 90.0
            frames[r] = 0
        if kind == 6:
            frames[r] = MIN_NEW  # eos allowed: it wins
            logits[r, EOS] = 95.0
    return logits, seen, frames


def device_rule(seen, frames):
    from qwen3tts import PickState
    rows = len(seen)
    pick = PickState(VOCAB, rows, BANNED, EOS, MIN_NEW, PENALTY)
    counts = np.zeros((rows, VOCAB), np.int16)
    for r, h in enumerate(seen):
        for i, t in Counter(h).items():
            counts[r, i] = t
    pick.counts.copy_(torch.from_numpy(counts))
    pick.frames.copy_(torch.from_numpy(frames))
    return pick


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_pick_rule_bit_exact(tt, orc, seed):
    rows = 96
    logits, seen, frames = hand_made(seed, rows)
    pick = device_rule(seen, frames)
    got = tt.topk.talker_pick(torch.from_numpy(logits).cuda(), pick).cpu().numpy()
    tt.check()
    want, _, _ = orc.talker_pick(logits, BANNED, seen, frames, EOS, MIN_NEW, PENALTY)
    bad = np.flatnonzero(got.astype(np.uint32) != want)
    assert bad.size == 0, [(int(r), int(got[r]), int(want[r])) for r in bad[:8]]
    # the rule decided: a plain argmax (or a once-per-id penalty) picks differently on many rows
    once = [sorted(set(h)) for h in seen]
    want_once, _, _ = orc.talker_pick(logits, BANNED, once, frames, EOS, MIN_NEW, PENALTY)
    assert (want_once != want).sum() >= rows // 8


def test_pick_records_history(tt, orc):
    rows = 32
    logits, seen, frames = hand_made(9, rows)
    pick = device_rule(seen, frames)
    x = torch.from_numpy(logits).cuda()
    for step in range(3):
        got = tt.topk.talker_pick(x, pick, record=True).cpu().numpy()
        want, _, _ = orc.talker_pick(logits, BANNED, seen, frames, EOS, MIN_NEW, PENALTY)
        assert np.array_equal(got.astype(np.uint32), want), step
        for r, c in enumerate(want):
            if int(c) != EOS:
                seen[r].append(int(c))
        frames = frames + 1
    tt.check()
    assert pick.frames.cpu().numpy().tolist() == frames.tolist()
    for r in range(rows):
        assert pick.history(r) == dict(Counter(seen[r])), r
