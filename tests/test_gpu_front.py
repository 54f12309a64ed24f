"""The codec decoder's front (crates/qwen3tts/src/codec.rs:161-196, 245-317, 403-424) on a
B200: each new row op against its oracle restatement (LayerNorm, GELU epilogue, depthwise
conv, RoPE, windowed causal attention, RVQ lookups), then the composed front (split RVQ,
pre-conv, pre-transformer with LayerScale and a sliding window, two x2 upsamplers with
ConvNeXt) against the oracle composition of the same ops, at reduced widths. Bars: row ops
rel <= 1e-5 (f32 both sides; 2e-3 where the device writes f16), the front's output SNR >= 30
dB (f16 activations between stages, as the codec stack)."""
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
    return float(10 * np.log10((want ** 2).sum() / max(((got - want) ** 2).sum(), 1e-30)))


def f16v(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def test_row_ops(tt, orc):
    rng = np.random.default_rng(71)
    x = rng.standard_normal((37, 256)).astype(np.float32) * 3 + 1
    w = rng.uniform(0.5, 1.5, 256).astype(np.float32)
    b = rng.standard_normal(256).astype(np.float32) * 0.1
    got = tt.layer_norm(dev_f32(x), dev_f32(w), dev_f32(b), 1e-6)
    assert rel(got.cpu().numpy(), orc.layer_norm(x, w, b, 1e-6)) < 1e-5
    y = rng.standard_normal((37, 256)).astype(np.float32) * 2
    sc = rng.uniform(0, 0.1, 256).astype(np.float32)
    got = tt.bias_act(dev_f32(y), dev_f32(b), gelu=True, scale=dev_f32(sc), res=dev_f32(x))
    want = x + sc * orc.gelu_exact(y + b)
    assert rel(got.cpu().numpy(), want) < 1e-5
    got16 = tt.bias_act(dev_f32(y), dev_f32(b), gelu=True, out_f16=True)
    assert rel(got16.float().cpu().numpy(), orc.gelu_exact(y + b)) < 2e-3
    xs = rng.standard_normal((2, 50, 64)).astype(np.float32)
    dw = rng.standard_normal((64, 1, 7)).astype(np.float32) * 0.3
    db = rng.standard_normal(64).astype(np.float32)
    got = tt.nlc.depthwise(dev_f32(xs), dev_f32(dw), dev_f32(db))
    assert rel(got.cpu().numpy(), orc.depthwise(xs, dw[:, 0], db)) < 1e-5
    cos, sin = orc.rope_table(64, 64, 1e4)
    qkv = rng.standard_normal((40, 3 * 4 * 64)).astype(np.float32)
    d = dev_f32(qkv)
    tt.rope_rows(d, 0, 4, 64, dev_f32(cos), dev_f32(sin))
    tt.rope_rows(d, 256, 4, 64, dev_f32(cos), dev_f32(sin))
    want = orc.rope_rows(orc.rope_rows(qkv, 0, 4, 64, cos, sin), 256, 4, 64, cos, sin)
    assert rel(d.cpu().numpy(), want) < 1e-6
    for window in (0, 8, 72):
        got = tt.window_attention(d, 4, 64, window, 0.125, out_f16=False)
        assert rel(got.cpu().numpy(), orc.window_attention(want, 4, 64, window, 0.125)) < 1e-5
    codes = rng.integers(0, 50, (33, 16)).astype(np.int32)
    tables = rng.standard_normal((15, 50, 64)).astype(np.float32)
    from qwen3tts.codec_front import rvq_gather
    got = rvq_gather(torch.from_numpy(codes).cuda(), 1, dev_f32(tables))
    assert rel(got.cpu().numpy(), orc.rvq_gather(codes, 1, tables)) < 1e-6
    tt.check()


# ---- the composed front at reduced widths
C_IN, C_Q, LAT, D, H, HD, FFN, WIN = 64, 128, 256, 128, 4, 64, 256, 8


def make_front(rng):
    r = lambda *s, sc=0.05: (rng.standard_normal(s) * sc).astype(np.float32)
    p = {"cb_sem": r(1, 64, C_IN, sc=1.0), "cb_ac": r(15, 64, C_IN, sc=0.3),
         "op_sem": r(C_Q, C_IN, sc=0.1), "op_ac": r(C_Q, C_IN, sc=0.1),
         "pre_conv_w": r(LAT, C_Q, 3), "pre_conv_b": r(LAT),
         "pre_in_w": r(D, LAT), "pre_in_b": r(D), "pre_out_w": r(LAT, D), "pre_out_b": r(LAT),
         "norm": rng.uniform(0.8, 1.2, D).astype(np.float32), "layers": []}
    for _ in range(2):
        p["layers"].append({"an": rng.uniform(0.8, 1.2, D).astype(np.float32),
                            "fn": rng.uniform(0.8, 1.2, D).astype(np.float32),
                            "q": r(H * HD, D, sc=0.1), "k": r(H * HD, D, sc=0.1),
                            "v": r(H * HD, D, sc=0.1), "o": r(D, H * HD, sc=0.1),
                            "gate": r(FFN, D, sc=0.1), "up": r(FFN, D, sc=0.1),
                            "down": r(D, FFN, sc=0.1),
                            "as": rng.uniform(0.05, 0.2, D).astype(np.float32),
                            "ms": rng.uniform(0.05, 0.2, D).astype(np.float32)})
    p["ups"] = []
    for _ in range(2):
        p["ups"].append({"tw": r(LAT, LAT, 2), "tb": r(LAT), "dw": r(LAT, 1, 7, sc=0.3),
                         "db": r(LAT), "nw": rng.uniform(0.8, 1.2, LAT).astype(np.float32),
                         "nb": r(LAT), "w1": r(4 * LAT, LAT), "b1": r(4 * LAT),
                         "w2": r(LAT, 4 * LAT), "b2": r(LAT), "g": r(LAT, sc=0.5)})
    return p


def device_front(p):
    import ttsnn
    from qwen3tts.codec import Conv, TransConv
    from qwen3tts.codec_front import CodecFront, ConvNext, PreTransformer, Rvq, TfLayer
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    layers = [TfLayer(T(l["an"]), T(l["fn"]),
                      ttsnn.Proj(T(np.concatenate([l["q"], l["k"], l["v"]]))),
                      ttsnn.Proj(T(l["o"])),
                      ttsnn.Proj(ttsnn.interleave_gate_up(T(l["gate"]).half(), T(l["up"]).half())),
                      ttsnn.Proj(T(l["down"])), T(l["as"]), T(l["ms"])) for l in p["layers"]]
    tf = PreTransformer(layers, T(p["norm"]), heads=H, head_dim=HD, window=WIN)
    ups = [(TransConv(T(u["tw"]), T(u["tb"]), 2),
            ConvNext(T(u["dw"]), T(u["db"]), T(u["nw"]), T(u["nb"]), T(u["w1"]), T(u["b1"]),
                     T(u["w2"]), T(u["b2"]), T(u["g"]))) for u in p["ups"]]
    return CodecFront(Rvq(T(p["cb_sem"]), T(p["op_sem"]), 0), Rvq(T(p["cb_ac"]), T(p["op_ac"]), 1),
                      Conv(T(p["pre_conv_w"]), T(p["pre_conv_b"])), ttsnn.Proj(T(p["pre_in_w"])),
                      T(p["pre_in_b"]), tf, ttsnn.Proj(T(p["pre_out_w"])), T(p["pre_out_b"]), ups)


def oracle_front(orc, p, codes):
    bits = lambda w: orc.f16_bits(w)
    q = (orc.proj(orc.rvq_gather(codes, 0, p["cb_sem"]), bits(p["op_sem"]))
         + orc.proj(orc.rvq_gather(codes, 1, p["cb_ac"]), bits(p["op_ac"])))
    # pre_conv: causal k3 on f16 activations, f16 out
    w_tap = np.ascontiguousarray(orc.f16_value(bits(p["pre_conv_w"])).transpose(2, 1, 0))
    h = f16v(orc.conv1d_nlc(f16v(q)[None], w_tap, p["pre_conv_b"], 1, 2)[0])
    x = orc.proj(h, bits(p["pre_in_w"])) + p["pre_in_b"]
    cos, sin = orc.rope_table(len(codes) + 4, HD, 1e4)
    for l in p["layers"]:
        xn = orc.rms_norm(x, l["an"], 1e-5)
        qkv = orc.proj(xn, bits(np.concatenate([l["q"], l["k"], l["v"]])))
        qkv = orc.rope_rows(orc.rope_rows(qkv, 0, H, HD, cos, sin), H * HD, H, HD, cos, sin)
        a = f16v(orc.window_attention(qkv, H, HD, WIN, 1.0 / 8))
        x = x + l["as"] * orc.proj(a, bits(l["o"]))
        xn = orc.rms_norm(x, l["fn"], 1e-5)
        act = f16v(orc.swiglu(orc.proj(xn, bits(l["gate"])), orc.proj(xn, bits(l["up"]))))
        x = x + l["ms"] * orc.proj(act, bits(l["down"]))
    t = orc.rms_norm(x, p["norm"], 1e-5)
    h = orc.proj(t, bits(p["pre_out_w"])) + p["pre_out_b"]
    lat = h[None]
    for u in p["ups"]:
        xin = f16v(lat)
        w = orc.f16_value(bits(u["tw"]))  # [in, out, 2]
        y = np.einsum("bli,iop->blpo", xin, w) + u["tb"][None, None, None, :]
        y = f16v(y.reshape(1, -1, LAT))
        hdw = orc.depthwise(y, u["dw"][:, 0], u["db"])
        hn = orc.layer_norm(hdw, u["nw"], u["nb"], 1e-6)[0]
        g = f16v(orc.gelu_exact(orc.proj(hn, bits(u["w1"])) + u["b1"]))
        lat = (y[0] + u["g"] * (orc.proj(g, bits(u["w2"])) + u["b2"]))[None]
    return q, h, lat


def test_front_matches_oracle(tt, orc):
    rng = np.random.default_rng(72)
    p = make_front(rng)
    front = device_front(p)
    codes = rng.integers(0, 64, (40, 16)).astype(np.int32)
    q, h, lat = front(torch.from_numpy(codes).cuda(), trace=True)
    torch.cuda.synchronize()
    tt.check()
    wq, wh, wlat = oracle_front(orc, p, codes)
    assert rel(q.cpu().numpy(), wq) < 1e-5
    assert snr_db(h.cpu().numpy(), wh) >= 30
    assert lat.shape == (1, 160, LAT)
    assert snr_db(lat.float().cpu().numpy(), wlat) >= 30
