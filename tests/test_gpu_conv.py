"""The codec's channels-last conv (implicit GEMM on tcgen05, SnakeBeta on load, bias and
residual in the epilogue) on a B200 against the CPU oracle. Inputs are rounded to f16 first
(the kernel's I/O type); the output is f16, so the bar is max relative error <= 2e-3 per conv
and an SNR >= 30 dB for the config[1] block."""
import numpy as np
import pytest
import torch

from _model import dev_f16, dev_f32

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def snr_db(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return 10 * np.log10((want ** 2).sum() / max(((got - want) ** 2).sum(), 1e-300))


def case(rng, orc, b, length, cin, cout, k):
    x = orc.f16_value(orc.f16_bits(rng.standard_normal((b, length, cin), dtype=np.float32)))
    w = orc.f16_value(orc.f16_bits(rng.standard_normal((k, cin, cout), dtype=np.float32) / np.sqrt(k * cin)))
    bias = (rng.standard_normal(cout, dtype=np.float32) * 0.1)
    return x, w, bias


# (b, len, cin, cout, k, dil, pad) — crates/tts-nn/src/nlc.rs:367-372 shapes where the kernel's
# channel rules allow (cin % 64), lengths not a multiple of the 128-row tile, "same" and causal;
# 256- and 512-channel outputs run on CTA pairs, 64-channel multiples on the TMA epilogue
@pytest.mark.parametrize("b,length,cin,cout,k,dil,pad", [
    (1, 300, 64, 64, 7, 1, 6), (1, 4200, 128, 96, 7, 9, 54), (1, 4096, 64, 96, 7, 1, 6),
    (1, 5000, 128, 192, 7, 3, 18), (1, 4097, 64, 96, 1, 1, 0), (2, 1000, 256, 256, 7, 3, 9),
    (3, 777, 512, 512, 7, 9, 27), (1, 130, 64, 1024, 3, 1, 2),
    # CTA pairs with few rows: 512 channels shorter than one CTA's 128 positions (the odd CTA
    # has no live row), and 256-channel tiles short enough for one sub-tile per CTA
    (1, 50, 64, 512, 3, 1, 2), (2, 200, 128, 256, 7, 1, 6)])
def test_conv_plain(tt, orc, b, length, cin, cout, k, dil, pad):
    rng = np.random.default_rng(length + cin)
    x, w, bias = case(rng, orc, b, length, cin, cout, k)
    want = orc.conv1d_nlc(x, w, bias, dil, pad)
    got = tt.nlc.conv1d(dev_f32(x), tt.nlc.device_weight(dev_f32(w)), dev_f32(bias), dil, pad)
    torch.cuda.synchronize()
    tt.check()
    assert rel(got.float().cpu().numpy(), want) < 2e-3


@pytest.mark.parametrize("length,c,k,dil", [(5000, 64, 1, 1), (4100, 192 + 64, 7, 3), (2000, 512, 7, 9)])
def test_snake_conv_residual(tt, orc, length, c, k, dil):
    # crates/tts-nn/src/nlc.rs:263-288: fused == snake -> causal conv -> + res
    rng = np.random.default_rng(length)
    x, w, bias = case(rng, orc, 1, length, c, c, k)
    res = orc.f16_value(orc.f16_bits(rng.standard_normal((1, length, c), dtype=np.float32)))
    alpha = rng.uniform(0.5, 2.0, c).astype(np.float32)
    brecip = rng.uniform(0.2, 1.5, c).astype(np.float32)
    want = orc.conv1d_nlc(x, w, bias, dil, None, snake=(alpha, brecip), res=res)
    got = tt.nlc.snake_conv_residual(dev_f32(x).half(), dev_f32(w), dev_f32(bias), dil,
                                     (dev_f32(alpha), dev_f32(brecip)), dev_f32(res).half())
    tt.check()
    assert rel(got.float().cpu().numpy(), want) < 2e-3


@pytest.mark.parametrize("cin,cout,length,stride,mult", [(64, 64, 300, 8, 2), (128, 64, 257, 5, 2),
                                                         (64, 32, 100, 4, 1), (64, 64, 90, 3, 2)])
def test_transposed_conv_as_reversed_taps(tt, orc, cin, cout, length, stride, mult):
    # crates/tts-nn/src/nlc.rs:164-174: the upsampling conv as one causal conv over the
    # reversed tap groups, output phases interleaved on the channel axis
    rng = np.random.default_rng(stride * 100 + length)
    x = orc.f16_value(orc.f16_bits(rng.standard_normal((1, length, cin), dtype=np.float32)))
    w = rng.standard_normal((cin, cout, mult * stride), dtype=np.float32) * 0.05
    bias = rng.standard_normal(cout, dtype=np.float32) * 0.1
    tap = tt.nlc.transpose_tap_weight(torch.from_numpy(w), stride).numpy()
    tap = orc.f16_value(orc.f16_bits(tap))
    tb = tt.nlc.transpose_bias(torch.from_numpy(bias), stride).numpy()
    want = orc.conv1d_nlc(x, tap, tb, 1).reshape(1, length * stride, cout)
    y = tt.nlc.conv1d(dev_f32(x), tt.nlc.device_weight(dev_f32(tap)), dev_f32(tb), 1, mult - 1)
    got = y.reshape(1, length * stride, cout)
    tt.check()
    assert rel(got.float().cpu().numpy(), want) < 2e-3


def test_conv_declines_unsupported(tt):
    x = torch.zeros(1, 100, 96, dtype=torch.float16, device="cuda")
    w = torch.zeros(64, 7, 96, dtype=torch.float16, device="cuda")
    with pytest.raises(tt.TtsError) as e:
        tt.nlc.conv1d(x, w, None, 1, 6)
    assert "cin" in str(e.value)
