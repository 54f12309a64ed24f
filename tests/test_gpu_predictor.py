"""The depth predictor (crates/qwen3tts/src/talker.rs:255-550) on a B200 against the CPU oracle's
composition: one frame = the two-position prefill through the projection and the predictor's
stack, 15 greedy depth steps (head i, pick, stack on resized[i][code]) and the embedding sum at
talker width. Bar: every pick equal to the oracle's, except near-ties (device pick within 1e-3
of the row's largest |logit| of the oracle's maximum, at most 2% of picks), which the oracle then
follows; the frame's sum equal to the oracle's for the same picks (rel <= 1e-6)."""
import numpy as np
import pytest
import torch

from _model import dev_f32, device_predictor, make_predictor

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def run_frame(tt, orc, lanes, dim, layers, heads, n_kv, ffn, vocab, steps, embed_dim, seed):
    g, Ls, final, pw, hidden, code0 = make_predictor(orc, lanes, dim, layers, heads, n_kv, ffn,
                                                     vocab, steps, embed_dim, seed)
    p = device_predictor(orc, g, Ls, final, pw)
    kv = p.new_state(lanes)
    codes, total = p.frame(kv, dev_f32(hidden), dev_f32(code0))
    torch.cuda.synchronize()
    tt.check()
    got = codes.cpu().numpy().astype(np.uint32)
    return g, Ls, final, pw, hidden, code0, p, kv, got, total.cpu().numpy()


def check_against_oracle(orc, g, Ls, final, pw, hidden, code0, got, total):
    tol = 1e-3 * 2.0  # picks' logits are O(1): 1e-3 of a max |logit| near 2
    want, want_sum, ties, mism = orc.predictor_frame(hidden, code0, Ls, final, pw, g, forced=got,
                                                     tie_tol=tol)
    assert mism == 0, (mism, got, want)
    assert ties <= max(1, int(0.02 * got.size)), ties
    assert np.array_equal(want, got)
    assert rel(total, want_sum) < 1e-6
    return ties


def test_predictor_small_geometry(tt, orc):
    r = run_frame(tt, orc, lanes=5, dim=256, layers=2, heads=4, n_kv=2, ffn=512, vocab=256,
                  steps=4, embed_dim=384, seed=31)
    g, Ls, final, pw, hidden, code0, p, kv, got, total = r
    check_against_oracle(orc, g, Ls, final, pw, hidden, code0, got, total)
    # the lanes' positions resume after the prefill and advance once per later depth step
    assert kv.positions.cpu().tolist() == [2 + pw.steps - 1] * 5


def test_predictor_reference_geometry(tt, orc):
    """dim 1024, 5 layers, 16/8 heads, ffn 3072, 15 heads of 2048 ids, talker width 2048
    (crates/qwen3tts/src/cfg.rs predictor constants)."""
    r = run_frame(tt, orc, lanes=8, dim=1024, layers=5, heads=16, n_kv=8, ffn=3072, vocab=2048,
                  steps=15, embed_dim=2048, seed=32)
    g, Ls, final, pw, hidden, code0, p, kv, got, total = r
    check_against_oracle(orc, g, Ls, final, pw, hidden, code0, got, total)


def test_predictor_graph_replay_and_frames_restart(tt, orc):
    """A captured frame replays to the eager call's exact outputs; frames restart the positions,
    so a second frame on the same state gives the same result; new inputs give new picks."""
    lanes = 6
    g, Ls, final, pw, hidden, code0 = make_predictor(orc, lanes, 256, 2, 4, 2, 512, 256, 5, 256,
                                                     seed=33)
    p = device_predictor(orc, g, Ls, final, pw)
    kv = p.new_state(lanes)
    h = dev_f32(hidden)
    c0 = dev_f32(code0)
    codes_e, total_e = p.frame(kv, h, c0)
    codes_e2, total_e2 = p.frame(kv, h, c0)
    torch.cuda.synchronize()
    assert torch.equal(codes_e, codes_e2) and torch.equal(total_e, total_e2)
    s = torch.cuda.Stream()
    codes = torch.empty_like(codes_e)
    total = torch.empty_like(total_e)
    with torch.cuda.stream(s):
        graph = p.capture(kv, h, c0, codes, total)
        graph.replay()
    s.synchronize()
    tt.check()
    assert torch.equal(codes, codes_e) and torch.equal(total, total_e)
    h.copy_(torch.from_numpy(-hidden).cuda())
    with torch.cuda.stream(s):
        graph.replay()
    s.synchronize()
    got = codes.cpu().numpy().astype(np.uint32)
    assert not np.array_equal(got, codes_e.cpu().numpy())
    check_against_oracle(orc, g, Ls, final, pw, -hidden, code0, got, total.cpu().numpy())
    del graph


def test_predictor_48_lanes_sum_identity(tt, orc):
    """At the benchmark's 48 lanes (reference geometry): picks in range and the frame's sum equal
    to code0_embed plus the picked rows of the tables, gathered independently here."""
    r = run_frame(tt, orc, lanes=48, dim=1024, layers=5, heads=16, n_kv=8, ffn=3072, vocab=2048,
                  steps=15, embed_dim=2048, seed=34)
    g, Ls, final, pw, hidden, code0, p, kv, got, total = r
    assert got.max() < 2048
    tables = orc.f16_value(pw.tables)
    acc = np.zeros_like(code0)
    for i in range(pw.steps):
        acc = acc + tables[i][got[:, i].astype(np.int64)]
    assert rel(total, code0 + acc) < 1e-6
    # the first lanes against the oracle too
    check_against_oracle(orc, g, Ls, final, pw, hidden[:4], code0[:4], got[:4], total[:4])


def test_predictor_paged_and_rejects_bad_shapes(tt, orc):
    """Pages of 8 positions, two per lane (the prefill's paired rows share both); then a state
    without room for steps + 1 positions and more lanes than the context holds are refused."""
    from ttsnn import _lib
    g, Ls, final, pw, hidden, code0 = make_predictor(orc, 3, 256, 1, 4, 2, 512, 128, 9, 256,
                                                     seed=35)
    p = device_predictor(orc, g, Ls, final, pw)
    kv = p.new_state(3, block_size=8)
    assert kv.max_blocks == 2
    codes, total = p.frame(kv, dev_f32(hidden), dev_f32(code0))
    torch.cuda.synchronize()
    tt.check()
    check_against_oracle(orc, g, Ls, final, pw, hidden, code0,
                         codes.cpu().numpy().astype(np.uint32), total.cpu().numpy())
    too_small = p.new_state(3, block_size=8)
    too_small.max_blocks = 1  # 8 positions < steps + 1
    with pytest.raises(_lib.TtsError) as e:
        p.frame(too_small, dev_f32(hidden), dev_f32(code0))
    assert e.value.status == 2
    many = torch.zeros(257, 256, device="cuda")
    with pytest.raises(_lib.TtsError) as e:
        p.frame(kv, many, many)
    assert e.value.status == 2


def test_predictor_top_k_sampling(tt, orc):
    """depth_on_device (talker.rs:478-515): the 15 picks drawn from each head's top 50 at
    temperature 0.9 with the caller's draws [steps, lanes]; against the oracle's host sampler
    on the same draws. The oracle follows a differing pick when the draw lies within 1e-4 of
    its interval's edge or when its logit is within 2e-3 of the oracle pick's (two near-equal
    candidates swapped in the walk's order); at most 5% of the picks."""
    lanes = 8
    g, Ls, final, pw, hidden, code0 = make_predictor(orc, lanes, 1024, 5, 16, 8, 3072, 2048, 15,
                                                     2048, seed=36)
    p = device_predictor(orc, g, Ls, final, pw)
    kv = p.new_state(lanes)
    draws = np.random.default_rng(37).random((15, lanes)).astype(np.float32)
    d = dev_f32(draws)
    p.set_sampling(d, 50, 0.9)
    codes, total = p.frame(kv, dev_f32(hidden), dev_f32(code0))
    torch.cuda.synchronize()
    tt.check()
    got = codes.cpu().numpy().astype(np.uint32)
    want, want_sum, ties, mism = orc.predictor_frame(hidden, code0, Ls, final, pw, g, forced=got,
                                                     tie_tol=1e-4, draws=draws, top_k=50,
                                                     temperature=0.9, logit_tol=2e-3)
    assert mism == 0, (got, want)
    assert ties <= 6
    assert rel(total.cpu().numpy(), want_sum) < 1e-6
    greedy, _ = orc.predictor_frame(hidden, code0, Ls, final, pw, g)[:2]
    assert not np.array_equal(got, greedy)  # sampling, not the argmax
    # back to greedy
    p.set_sampling(None)
    codes2, _ = p.frame(kv, dev_f32(hidden), dev_f32(code0))
    torch.cuda.synchronize()
    g2 = codes2.cpu().numpy().astype(np.uint32)
    _, _, _, mism2 = orc.predictor_frame(hidden, code0, Ls, final, pw, g, forced=g2, tie_tol=2e-3)
    assert mism2 == 0
