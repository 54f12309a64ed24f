"""The codec conv stack on a B200 against the CPU oracle: the reference's ResidualUnit and
DecoderBlock (crates/qwen3tts/src/codec.rs:199-260), config[1]'s snake residual block at full
size (SNR >= 30 dB on sampled windows), and chunked batch decoding."""
import numpy as np
import pytest
import torch

from _model import dev_f32

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def snr_db(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return 10 * np.log10((want ** 2).sum() / max(((got - want) ** 2).sum(), 1e-300))


def f16(orc, a):
    return orc.f16_value(orc.f16_bits(a))


def test_residual_unit_and_decoder_block(tt, orc):
    from qwen3tts.codec import Conv, DecoderBlock, ResidualUnit, SnakeBeta, TransConv
    rng = np.random.default_rng(1)
    cin, c, s, length = 128, 64, 4, 200

    def snake(ch):
        la = rng.uniform(-0.5, 0.5, ch).astype(np.float32)
        lb = rng.uniform(-0.5, 0.5, ch).astype(np.float32)
        return la, lb, SnakeBeta(dev_f32(la), dev_f32(lb))

    def fold(la, lb):
        return np.exp(la).astype(np.float32), (1.0 / (np.exp(lb) + 1e-9)).astype(np.float32)

    la0, lb0, act = snake(cin)
    wt = f16(orc, rng.standard_normal((cin, c, 2 * s), dtype=np.float32) / np.sqrt(2 * cin))
    bt = rng.standard_normal(c, dtype=np.float32) * 0.1
    up = TransConv(dev_f32(wt), dev_f32(bt), s)
    units, ref_units = [], []
    for d in (1, 3, 9):
        la1, lb1, a1 = snake(c)
        la2, lb2, a2 = snake(c)
        w1 = f16(orc, rng.standard_normal((c, c, 7), dtype=np.float32) / np.sqrt(7 * c))
        w2 = f16(orc, rng.standard_normal((c, c, 1), dtype=np.float32) / np.sqrt(c))
        b1 = rng.standard_normal(c, dtype=np.float32) * 0.1
        b2 = rng.standard_normal(c, dtype=np.float32) * 0.1
        units.append(ResidualUnit(a1, Conv(dev_f32(w1), dev_f32(b1), d), a2,
                                  Conv(dev_f32(w2), dev_f32(b2), 1)))
        ref_units.append((fold(la1, lb1), w1, b1, d, fold(la2, lb2), w2, b2))
    block = DecoderBlock(act, up, units)
    x = f16(orc, rng.standard_normal((1, length, cin), dtype=np.float32))
    got = block(dev_f32(x).half()).float().cpu().numpy()

    # oracle: snake -> transposed conv as reversed taps -> three units, f32 throughout
    import ttsnn.nlc as nlc
    tap = nlc.transpose_tap_weight(torch.from_numpy(wt), s).numpy()
    tb = nlc.transpose_bias(torch.from_numpy(bt), s).numpy()
    h = orc.conv1d_nlc(x, tap, tb, 1, snake=fold(la0, lb0)).reshape(1, length * s, c)
    for (sn1, w1, b1, d, sn2, w2, b2) in ref_units:
        y = orc.conv1d_nlc(h, np.ascontiguousarray(w1.transpose(2, 1, 0)), b1, d, snake=sn1)
        h = orc.conv1d_nlc(y, np.ascontiguousarray(w2.transpose(2, 1, 0)), b2, 1, snake=sn2, res=h)
    tt.check()
    assert got.shape == h.shape
    # f16 activations between convs (the reference's WAV_DTYPE is f32): SNR bar
    assert snr_db(got, h) >= 30.0, snr_db(got, h)


def test_config1_block_full_size_snr(tt, orc):
    """[8, 512, 24000] through the three snake-conv-residual steps; checked on windows against
    the oracle run on each window plus the receptive field (3 * 27 rows per side)."""
    from qwen3tts.codec import SnakeBlock
    gen = torch.Generator(device="cuda").manual_seed(0)
    blk = SnakeBlock(512, gen, "cuda")
    x = torch.randn(8, 24000, 512, generator=gen, device="cuda").half()
    y = blk(x).float()
    tt.check()
    halo = 3 * 27
    convs = []
    for conv, act in blk.convs:
        w_tap = conv.w.float().permute(1, 2, 0).cpu().numpy()  # [cout, k, cin] -> [k, cin, cout]
        convs.append((np.ascontiguousarray(w_tap), conv.bias.cpu().numpy(),
                      act.alpha.cpu().numpy(), act.brecip.cpu().numpy()))
    rng = np.random.default_rng(0)
    worst = 1e9
    for b, start in [(0, 0), (7, 24000 - 256)] + [(int(rng.integers(8)), int(rng.integers(0, 23700)))
                                                  for _ in range(4)]:
        lo, hi = max(0, start - halo), min(24000, start + 256 + halo)
        xw = x[b:b + 1, lo:hi].float().cpu().numpy()
        # the same zero padding at the true edges; interior window edges are far enough away
        want = orc.snake_residual_block(xw, convs)
        # the GPU rounds each conv's output to f16; the oracle stays f32
        got = y[b:b + 1, start:start + 256].cpu().numpy()
        ref = want[:, start - lo:start - lo + 256]
        worst = min(worst, snr_db(got, ref))
    assert worst >= 30.0, worst


def test_wave_stack_matches_oracle(tt, orc):
    """The whole synthetic decoder (2 x2 + x8/x5/x4/x3 upsamplers, 12 snake blocks, output conv)
    on two frames against the oracle composition; this also checks the stack's buffer reuse."""
    from qwen3tts.codec import SAMPLES_PER_FRAME, WaveStack
    ws = WaveStack("cuda", seed=0)
    gen = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(2, 2, 1024, generator=gen, device="cuda").half()
    got = ws.raw(x)[..., 0].float().cpu().numpy()
    wav = ws(x)
    tt.check()
    want = oracle_wave(orc, ws, x.float().cpu().numpy())[..., 0]
    assert got.shape == (2, 2 * SAMPLES_PER_FRAME)
    assert snr_db(got, want) >= 30.0, snr_db(got, want)
    assert wav.shape == (2, 2 * SAMPLES_PER_FRAME) and float(wav.abs().max()) <= 1.0


def test_chunked_document_decode_matches_whole(tt):
    """Chunk windows decoded as one batch give, on every kept frame of an interior window,
    exactly the samples of decoding the whole document at once: the left context and right
    lookahead cover the stack's receptive field, and each output row sums in a fixed order."""
    from qwen3tts.codec import SAMPLES_PER_FRAME, WaveStack, chunk_plan, gather_windows, stitch
    ws = WaveStack("cuda", seed=3)
    gen = torch.Generator(device="cuda").manual_seed(4)
    n, right = 700, 8
    frames = torch.randn(n, 1024, generator=gen, device="cuda").half()
    plan = chunk_plan(n, right=right)
    assert len(plan) == 3 and all(w.span == plan[0].span for w in plan)
    whole = ws(frames[None])[0]
    batch = ws(gather_windows(frames, plan))
    doc = stitch(batch, plan, SAMPLES_PER_FRAME)
    tt.check()
    assert doc.shape == whole.shape == (n * SAMPLES_PER_FRAME,)
    exact = [w for w in plan if w.end + right <= n]
    assert len(exact) == 2
    for w in exact:
        lo, hi = w.start * SAMPLES_PER_FRAME, w.end * SAMPLES_PER_FRAME
        assert torch.equal(doc[lo:hi], whole[lo:hi]), (w, (doc[lo:hi] - whole[lo:hi]).abs().max())


def _tap(conv) -> np.ndarray:
    """A conv module's device weight [cout, k, cin] as the oracle's tap-major [k, cin, cout]."""
    return np.ascontiguousarray(conv.w.float().permute(1, 2, 0).cpu().numpy())


def _np(t):
    return None if t is None else t.float().cpu().numpy()


def oracle_wave(orc, ws, x, trace=False):
    """WaveStack.raw on the CPU oracle, f32 throughout (the GPU keeps f16 between convs)."""
    mags = []
    h = x
    b = h.shape[0]

    def up(h, m, snake=None):
        length = h.shape[1]
        y = orc.conv1d_nlc(h, _tap(m), _np(m.bias), 1, m.m - 1,
                           snake=None if snake is None else (_np(snake.alpha), _np(snake.brecip)))
        return y.reshape(b, length * m.stride, m.cout)

    for m in ws.pre:
        h = up(h, m)
        mags.append(("pre", h.shape, float(np.abs(h).max())))
    for act, m, blocks in ws.stages:
        h = up(h, m, act)
        for blk in blocks:
            for conv, a in blk.convs:
                h = orc.conv1d_nlc(h, _tap(conv), _np(conv.bias), conv.dilation, conv.pad_left,
                                   snake=(_np(a.alpha), _np(a.brecip)), res=h)
        mags.append(("stage", h.shape, float(np.abs(h).max())))
    y = orc.conv1d_nlc(h, _tap(ws.out), _np(ws.out.bias), 1, ws.out.pad_left,
                       snake=(_np(ws.out_act.alpha), _np(ws.out_act.brecip)))
    return (y, mags) if trace else y
