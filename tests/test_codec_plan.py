"""The codec's chunked-decode plan (crates/qwen3tts/src/codec.rs:581-604), host side."""
import pytest

from qwen3tts.codec import CHUNK_FRAMES, CHUNK_LEFT_CONTEXT, chunk_plan


@pytest.mark.parametrize("n", [1, 24, 299, 300, 301, 324, 325, 326, 900, 1234, 5000])
def test_plan_partitions_and_spans(n):
    plan = chunk_plan(n)
    span = CHUNK_FRAMES + CHUNK_LEFT_CONTEXT
    kept = []
    for w in plan:
        assert 0 <= w.lo <= w.start < w.end <= n
        assert w.hi <= n and w.hi - w.lo <= span
        assert w.drop == w.start - w.lo <= CHUNK_LEFT_CONTEXT
        assert w.end - w.start <= CHUNK_FRAMES
        assert w.drop + (w.end - w.start) <= w.span  # the kept frames lie inside the window
        kept.extend(range(w.start, w.end))
        if n >= span:
            assert w.span == span  # one uniform length, padded on the right
    assert kept == list(range(n))
    if n < span:
        assert len(plan) in (1, 2) and plan[0].span == plan[0].hi - plan[0].lo
