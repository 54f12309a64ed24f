"""The codec decoder at the reference's structure (crates/qwen3tts/src/codec.rs:320-424) on a
B200: built from checkpoint-named tensors (seeded random, no checkpoint here) at reduced widths
whose last three stages are not multiples of 64 (run zero-padded), its waveform stack against
the oracle's unpadded composition on the same latent (SNR >= 30 dB: f16 between convs); and at
the reference's full shape, a 40-frame decode: 76800 samples, finite, inside the clamp."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(latent=256, tf_dim=128, tf_layers=2, tf_heads=2, tf_ffn=256, decoder_dim=128,
             rates=(2, 2, 2, 2), codebook=64, inner=64, codebook_dim=128)


def snr_db(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(10 * np.log10((want ** 2).sum() / max(((got - want) ** 2).sum(), 1e-30)))


def oracle_back(orc, w, latent, rates):
    """Head conv, decoder blocks and output conv on the oracle, unpadded, f32 throughout."""
    import ttsnn.nlc as nlc
    n = lambda k: w[k].float().cpu().numpy()
    f16 = lambda a: orc.f16_value(orc.f16_bits(a))
    tap = lambda a: np.ascontiguousarray(f16(a).transpose(2, 1, 0))
    fold = lambda p: (np.exp(n(f"{p}.alpha")).astype(np.float32),
                      (1.0 / (np.exp(n(f"{p}.beta")) + 1e-9)).astype(np.float32))
    h = orc.conv1d_nlc(latent, tap(n("decoder.decoder.0.conv.weight")),
                       n("decoder.decoder.0.conv.bias"), 1)
    for j, r in enumerate(rates):
        p = f"decoder.decoder.{j + 1}.block"
        wt = f16(n(f"{p}.1.conv.weight"))
        cout = wt.shape[1]
        t = nlc.transpose_tap_weight(torch.from_numpy(wt), r).numpy()
        tb = nlc.transpose_bias(torch.from_numpy(n(f"{p}.1.conv.bias")), r).numpy()
        length = h.shape[1]
        h = orc.conv1d_nlc(h, t, tb, 1, wt.shape[2] // r - 1, snake=fold(f"{p}.0"))
        h = h.reshape(1, length * r, cout)
        for u, d in enumerate((1, 3, 9)):
            q = f"{p}.{u + 2}"
            y = orc.conv1d_nlc(h, tap(n(f"{q}.conv1.conv.weight")), n(f"{q}.conv1.conv.bias"), d,
                               snake=fold(f"{q}.act1"))
            h = orc.conv1d_nlc(y, tap(n(f"{q}.conv2.conv.weight")), n(f"{q}.conv2.conv.bias"), 1,
                               snake=fold(f"{q}.act2"), res=h)
    last = len(rates) + 1
    y = orc.conv1d_nlc(h, tap(n(f"decoder.decoder.{last + 1}.conv.weight")),
                       n(f"decoder.decoder.{last + 1}.conv.bias"), 1,
                       snake=fold(f"decoder.decoder.{last}"))
    return np.clip(y[0, :, 0], -1, 1)


def test_padded_stages_match_unpadded_oracle(tt, orc):
    from qwen3tts.codec_ref import Codec
    w = Codec.synthetic_weights(seed=3, **SMALL)
    codec = Codec.from_weights(w.__getitem__, rates=SMALL["rates"])
    codes = torch.randint(0, SMALL["codebook"], (24, 16), dtype=torch.int32, device="cuda")
    wav, latent, h = codec(codes, trace=True)
    torch.cuda.synchronize()
    tt.check()
    assert wav.shape == (24 * 4 * 16,)
    # padded channels stay exactly zero through the last stages
    assert h.shape[-1] == 64 and float(h[..., 8:].abs().max()) == 0.0
    want = oracle_back(orc, w, latent.half().float().cpu().numpy(), SMALL["rates"])
    assert snr_db(wav.cpu().numpy(), want) >= 30


def test_reference_shape_decode(tt):
    from qwen3tts.codec_ref import Codec, SAMPLES_PER_FRAME
    codec = Codec.from_weights(Codec.synthetic_weights(seed=4).__getitem__)
    codes = torch.randint(0, 2048, (40, 16), dtype=torch.int32, device="cuda")
    wav = codec(codes)
    torch.cuda.synchronize()
    tt.check()
    assert SAMPLES_PER_FRAME == 1920 and wav.shape == (40 * 1920,)
    assert torch.isfinite(wav).all() and float(wav.abs().max()) <= 1.0
    assert float(wav.abs().mean()) > 0
