"""Text ids to audio through the whole pipeline (crates/qwen3tts/src/talker.rs:683-1073,
codec.rs:544-604) on a B200 with small seeded models: prompts built (x-vector and in-context),
prefilled together as decode rows, then frames from the talker loop until the end code or the
frame budget, and the codec's chunked decode. Each lane's recorded frames are checked against
the oracle run on the same prompt: its prefill as position-by-position decode steps, then the
oracle talker loop (picks equal except near-ties, which the oracle follows)."""
import numpy as np
import pytest
import torch

from _model import dev_f16, dev_f32, device_predictor, device_stack, make_heads, make_predictor, make_talker

pytestmark = pytest.mark.gpu


def _models(orc):
    from qwen3tts.codec_ref import Codec
    from qwen3tts.prompt import PromptBuilder, TextProjection
    rng = np.random.default_rng(81)
    dim = 256
    g, Ls, final, _, _, _, _ = make_talker(orc, 1, 2, dim, 4, 2, 512, 8, 81, codebooks=1,
                                           vocab=3072, lengths=[0])
    head, embed = make_heads(orc, 82, g)
    talker = device_stack(orc, g, Ls, final, head, embed, rope_len=512)
    pg, pLs, pfinal, pw, _, _ = make_predictor(orc, 1, dim, 1, 4, 2, 512, 2048, 15, dim, 83)
    pred = device_predictor(orc, pg, pLs, pfinal, pw)
    table = (rng.standard_normal((151_936, 64)) * 0.5).astype(np.float32)
    text = TextProjection(lambda ids: torch.from_numpy(table[ids]),
                          dev_f16(orc.f16_bits(rng.standard_normal((256, 64)) * 0.1)),
                          dev_f32(rng.standard_normal(256) * 0.1),
                          dev_f16(orc.f16_bits(rng.standard_normal((256, 256)) * 0.06)),
                          dev_f32(rng.standard_normal(256) * 0.1))
    builder = PromptBuilder(text, dev_f16(embed[0]).float(), dev_f16(pw.tables))
    small = dict(latent=256, tf_dim=128, tf_layers=1, tf_heads=2, tf_ffn=256, decoder_dim=128,
                 rates=(2, 2, 2, 2), codebook=2048, inner=64, codebook_dim=128)
    codec = Codec.from_weights(Codec.synthetic_weights(seed=5, **small).__getitem__,
                               rates=small["rates"])
    return rng, dim, g, Ls, final, head, embed, talker, pg, pLs, pfinal, pw, pred, builder, codec


def test_text_to_audio(tt, orc):
    from qwen3tts import reference_pick
    from qwen3tts.frames import CODEC_EOS, MIN_NEW_TOKENS, REPETITION_PENALTY
    from qwen3tts.pipeline import Request, Synthesizer
    (rng, dim, g, Ls, final, head, embed, talker, pg, pLs, pfinal, pw, pred, builder,
     codec) = _models(orc)
    synth = Synthesizer(talker, pred, builder, reference_pick(lanes=8), codec, max_lanes=8,
                        capacity=256)
    reqs = [Request([100, 200, 300, 400], spk=torch.randn(dim, device="cuda") * 0.05, max_frames=5),
            Request([7, 8], ref_text=[11, 12, 13],
                    ref_codes=[list(rng.integers(0, 2048, 16)) for _ in range(2)], max_frames=4),
            Request([5], language=2070, max_frames=3)]
    frames = synth.generate(reqs)
    torch.cuda.synchronize()
    tt.check()
    assert [len(f) <= r.max_frames for f, r in zip(frames, reqs)] == [True] * 3
    assert all(len(fr) == 16 for f in frames for fr in f)

    # the oracle on each lane's prompt
    banned = [i for i in range(2048, 3072) if i != CODEC_EOS]
    pad = builder.text([151_671])[0].cpu().numpy()
    cos, sin = orc.rope_table(300, 128, g.rope_base)
    for r, got in zip(reqs, frames):
        prompt, trailing, _ = builder.build(r.text, r.ref_text, r.ref_codes, r.spk, r.language)
        P = prompt.cpu().numpy()
        cap = P.shape[0] + 8
        kc = [np.zeros((1, g.n_kv, cap, 128), np.uint16) for _ in Ls]
        vc = [np.zeros((1, g.n_kv, cap, 128), np.uint16) for _ in Ls]
        for t in range(P.shape[0] - 1):
            orc.decode_step(P[t:t + 1], Ls, final, kc, vc, np.array([t], np.int32), cos, sin, g)
        st = orc.TalkerState(kc, vc, np.array([P.shape[0] - 1], np.int32), [[]],
                             np.zeros(1, np.int64), P[-1:].copy())
        rows = np.broadcast_to(pad, (1, max(trailing.shape[0], 1), dim)).copy()
        rows[0, :trailing.shape[0]] = trailing.cpu().numpy()
        for f in got:
            c0, codes, ties, mism = orc.talker_frame(
                st, Ls, final, g, head, embed[0], banned, CODEC_EOS, MIN_NEW_TOKENS,
                REPETITION_PENALTY, pLs, pfinal, pw, pg, rows, pad,
                forced0=np.array([f[0]], np.uint32), forced=np.array([f[1:]], np.uint32),
                tie_tol=2e-3)
            assert mism == 0 and ties <= 1
    wav = synth.decode(frames[0])
    torch.cuda.synchronize()
    assert wav.shape[0] == len(frames[0]) * 64 and torch.isfinite(wav).all()

    # the voice clip's last 25 frames decoded ahead and dropped (engine.rs:1119-1135): equal to
    # decoding clip + frames and cutting the clip's samples, and not the cold decode
    clip = [list(rng.integers(0, 2048, 16)) for _ in range(40)]
    warm = synth.decode(frames[0], context=clip)
    both = synth.decode(clip[-25:] + frames[0])
    torch.cuda.synchronize()
    assert warm.shape == wav.shape and torch.equal(warm, both[25 * 64:])
    assert not torch.equal(warm, wav)
    # the whole document once, cut per request at exact frame boundaries
    pieces = synth.decode_document(frames, context=clip)
    joined = synth.decode([fr for f in frames for fr in f], context=clip)
    torch.cuda.synchronize()
    assert [p.shape[0] for p in pieces] == [len(f) * 64 for f in frames]
    assert torch.equal(torch.cat(pieces), joined)


def test_engine_over_the_pipeline(tt, orc):
    """The engine's schedule (crates/qwen3tts/src/engine.rs:919-1011) over two synthesizers: a
    batched pool sized for the batch cap and a one-lane pool for the full budget. A run whose
    lanes reach the cap is redone one segment at a time; every segment's frames then equal the
    one-lane pool's own output for it."""
    from qwen3tts import reference_pick
    from qwen3tts.engine import Engine
    from qwen3tts.pipeline import Request, Synthesizer
    (rng, dim, g, Ls, final, head, embed, talker, pg, pLs, pfinal, pw, pred, builder,
     codec) = _models(orc)
    batched = Synthesizer(talker, pred, builder, reference_pick(lanes=8), max_lanes=8,
                          capacity=128)
    single = Synthesizer(talker, pred, builder, reference_pick(lanes=1), max_lanes=1,
                         capacity=128)
    spk = torch.randn(dim, device="cuda") * 0.05
    reqs = [Request([100 + i, 200, 300 + 7 * i][: 1 + i % 3], spk=spk) for i in range(4)]
    widths = [builder.build(r.text, spk=r.spk)[0].shape[0] for r in reqs]
    chars = [50, 80, 20, 80]
    eng = Engine(batched.generate, lambda r: single.generate([r])[0], budget=7, batch_cap=5)
    out = eng.run(reqs, widths, chars)
    torch.cuda.synchronize()
    tt.check()
    import dataclasses
    assert eng.log and all(lg.budgets == [5] * len(lg.segments) for lg in eng.log)
    for lg in eng.log:
        if lg.rerun:  # some lane reached the cap: each segment redone with the full budget
            for i in lg.segments:
                assert single.generate([dataclasses.replace(reqs[i], max_frames=7)])[0] == out[i]
        else:         # every lane ended below the cap: the batched run's own frames
            again = batched.generate([dataclasses.replace(reqs[i], max_frames=5)
                                      for i in lg.segments])
            assert again == [out[i] for i in lg.segments]
            assert all(len(out[i]) < 5 for i in lg.segments)
    assert all(1 <= len(f) <= 7 for f in out)
