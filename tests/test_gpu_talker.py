"""The lane scheduler driving the decode step on a B200: every segment emits exactly its frames,
the lane-steps match the tail-shedding model, refill reuses finished lanes, and a lane run by
the scheduler computes what direct decode steps compute."""
import numpy as np
import pytest
import torch

from _model import device_stack, make_heads, make_talker

pytestmark = pytest.mark.gpu


def small_stack(orc, layers=2, seed=5):
    g, Ls, final, kc, vc, pos, x = make_talker(orc, 1, layers, 2048, 16, 8, 6144, 8, seed,
                                               codebooks=2, vocab=2048)
    hb, eb = make_heads(orc, seed + 1, g)
    return device_stack(orc, g, Ls, final, hb, eb)


def test_talker_accounts_frames_and_shedding(tt, orc):
    from qwen3tts.talker import Segment, Talker, plan_groups, shed_widths
    stack = small_stack(orc)
    rng = np.random.default_rng(0)
    segs = [Segment(i, 20, int(f), int(f)) for i, f in enumerate(rng.integers(1, 40, 37))]
    groups = plan_groups(segs, max_lanes=16)
    talker = Talker(stack, max_lanes=16, capacity=80)
    queue = [s for g in groups for s in g]
    st = talker.run(queue)
    tt.check()
    assert st.frames == sum(s.frames for s in segs)
    want_lane_steps = sum(sum(shed_widths([s.frames for s in g])) for g in groups)
    assert st.lane_steps == want_lane_steps
    assert st.steps == sum(max(s.frames for s in g) for g in groups)
    assert talker.kv.free_pages() == talker.kv.num_blocks  # every page returned

    st2 = talker.run(queue, refill=True)
    tt.check()
    assert st2.frames == st.frames
    assert st2.steps <= st.steps and st2.useful >= st.useful


def test_talker_lane_matches_direct_steps(tt, orc):
    """One 6-frame segment through the scheduler vs six direct decode steps from the same
    seeded input: identical codes at the last step."""
    from qwen3tts import PagedKv
    from qwen3tts.talker import Segment, Talker
    stack = small_stack(orc, seed=9)
    talker = Talker(stack, max_lanes=8, capacity=64)
    talker.run([Segment(0, 10, 6, 6)], seed=3)
    got = talker.codes[0].clone()
    # direct: same pages layout, same seeded first input
    gen = torch.Generator(device="cuda").manual_seed(3)
    x0 = torch.zeros(8, 2048, device="cuda")
    x0[0].normal_(generator=gen)
    kv = PagedKv(stack.geo, 8, talker.kv.num_blocks, talker.kv.block_size, talker.kv.max_blocks)
    kv.admit(0, 17, 10)
    fb = torch.zeros(8, 2048, device="cuda")
    stack.set_feedback(fb)
    codes = torch.zeros(8, 2, dtype=torch.int32, device="cuda")
    stack.decode_step(kv, x0, lanes=1, codes=codes, max_span=64)
    for _ in range(5):
        stack.decode_step(kv, None, lanes=1, codes=codes, max_span=64)
    torch.cuda.synchronize()
    tt.check()
    assert torch.equal(codes[0], got)
    assert int(kv.positions[0]) == 16
