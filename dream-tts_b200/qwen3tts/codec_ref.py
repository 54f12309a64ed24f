"""The codec decoder at the reference's shape (crates/qwen3tts/src/codec.rs:320-424): codes
[T, 16] -> 24 kHz waveform [T * 1920], clamped to [-1, 1]. The front (codec_front.py) gives the
[4 T, 1024] latent; then the head conv (k7, 1024 -> 1536), four decoder blocks (SnakeBeta,
transposed conv x8 / x5 / x4 / x3, three residual units at dilations 1, 3, 9; 1536 -> 768 ->
384 -> 192 -> 96 channels), SnakeBeta and the output conv (k7, 96 -> 1).

The conv kernel takes input widths in multiples of 64, so a stage whose width is not one (the
last block's 96 channels) runs zero-padded to the next multiple: the padded output channels
have zero weights and bias, so they stay exactly zero through the snakes (snake(0) = 0), the
residual adds and the next convs, and the real channels are computed as without padding. The
output conv is padded to 32 output channels; channel 0 is the waveform.

Weights come by the reference's checkpoint names (`from_weights`, with any `get(name)`), or
seeded random-init at the same shapes (`synthetic`).
"""
from __future__ import annotations

import math

import torch

import ttsnn

from .codec import Conv, DecoderBlock, ResidualUnit, SnakeBeta, TransConv
from .codec_front import CodecFront, ConvNext, PreTransformer, Rvq, TfLayer

# crates/qwen3tts/src/cfg.rs (codec)
QUANTIZERS, SEMANTIC, CODEBOOK, INNER, CODEBOOK_DIM = 16, 1, 2048, 256, 512
LATENT, TF_DIM, TF_LAYERS, TF_HEADS, TF_HD, TF_FFN, WINDOW = 1024, 512, 8, 16, 64, 1024, 72
DECODER_DIM, RATES, DILATIONS = 1536, (8, 5, 4, 3), (1, 3, 9)
SAMPLES_PER_FRAME = 2 * 2 * 8 * 5 * 4 * 3


def _pad64(c: int) -> int:
    return -(-c // 64) * 64


def _pad(t: torch.Tensor, dims: dict) -> torch.Tensor:
    """Zero-pad dimensions {axis: new size} of t."""
    shape = list(t.shape)
    for ax, n in dims.items():
        shape[ax] = n
    out = torch.zeros(shape, dtype=t.dtype, device=t.device)
    out[tuple(slice(0, s) for s in t.shape)] = t
    return out


def _snake(get, prefix: str, width: int) -> SnakeBeta:
    a = get(f"{prefix}.alpha").float().flatten()
    b = get(f"{prefix}.beta").float().flatten()
    if width > a.numel():  # padded channels: alpha = beta = 1 (log 0); their inputs are zero
        a = _pad(a, {0: width})
        b = _pad(b, {0: width})
    return SnakeBeta(a, b)


class Codec:
    def __init__(self, front: CodecFront, head: Conv, blocks: list[DecoderBlock],
                 out_act: SnakeBeta, out_conv: Conv):
        self.front, self.head, self.blocks = front, head, blocks
        self.out_act, self.out_conv = out_act, out_conv

    @classmethod
    def from_weights(cls, get, device="cuda", widths=None, rates=RATES) -> "Codec":
        """The reference's loader (codec.rs:320-395): `get(name)` returns a checkpoint tensor
        (folded codebooks are built here: embedding_sum / cluster_usage.clamp(1e-5))."""
        g = lambda n: get(n).to(device)

        def rvq(prefix, layers, q0):
            books = []
            for i in range(layers):
                p = f"{prefix}.vq.layers.{i}._codebook"
                usage = g(f"{p}.cluster_usage").float().clamp(min=1e-5)
                books.append(g(f"{p}.embedding_sum").float() / usage[:, None])
            return Rvq(torch.stack(books), g(f"{prefix}.output_proj.weight").float(), q0)

        semantic = rvq("decoder.quantizer.rvq_first", SEMANTIC, 0)
        acoustic = rvq("decoder.quantizer.rvq_rest", QUANTIZERS - SEMANTIC, SEMANTIC)
        pre_conv = Conv(g("decoder.pre_conv.conv.weight"), g("decoder.pre_conv.conv.bias"), 1)
        t = "decoder.pre_transformer"
        layers = []
        n_layers = 0
        while True:
            p = f"{t}.layers.{n_layers}"
            try:
                g(f"{p}.input_layernorm.weight")
            except Exception:
                break
            a = f"{p}.self_attn"
            layers.append(TfLayer(
                g(f"{p}.input_layernorm.weight").float(), g(f"{p}.post_attention_layernorm.weight").float(),
                ttsnn.Proj(torch.cat([g(f"{a}.q_proj.weight"), g(f"{a}.k_proj.weight"),
                                      g(f"{a}.v_proj.weight")])),
                ttsnn.Proj(g(f"{a}.o_proj.weight")),
                ttsnn.Proj(ttsnn.interleave_gate_up(g(f"{p}.mlp.gate_proj.weight").half(),
                                                    g(f"{p}.mlp.up_proj.weight").half())),
                ttsnn.Proj(g(f"{p}.mlp.down_proj.weight")),
                g(f"{p}.self_attn_layer_scale.scale").float(),
                g(f"{p}.mlp_layer_scale.scale").float()))
            n_layers += 1
        hd = TF_HD
        heads = layers[0].wqkv.n // (3 * hd)
        tf = PreTransformer(layers, g(f"{t}.norm.weight"), heads=heads, head_dim=hd,
                            window=WINDOW)
        ups = []
        i = 0
        while True:
            p = f"decoder.upsample.{i}"
            try:
                w0 = g(f"{p}.0.conv.weight")
            except Exception:
                break
            c = f"{p}.1"
            ups.append((TransConv(w0, g(f"{p}.0.conv.bias"), 2),
                        ConvNext(g(f"{c}.dwconv.conv.weight"), g(f"{c}.dwconv.conv.bias"),
                                 g(f"{c}.norm.weight"), g(f"{c}.norm.bias"),
                                 g(f"{c}.pwconv1.weight"), g(f"{c}.pwconv1.bias"),
                                 g(f"{c}.pwconv2.weight"), g(f"{c}.pwconv2.bias"),
                                 g(f"{c}.gamma"))))
            i += 1
        front = CodecFront(semantic, acoustic, pre_conv, ttsnn.Proj(g(f"{t}.input_proj.weight")),
                           g(f"{t}.input_proj.bias"), tf, ttsnn.Proj(g(f"{t}.output_proj.weight")),
                           g(f"{t}.output_proj.bias"), ups)
        head = Conv(g("decoder.decoder.0.conv.weight"), g("decoder.decoder.0.conv.bias"), 1)
        blocks = []
        cin = head.cout
        for j, r in enumerate(rates):
            p = f"decoder.decoder.{j + 1}.block"
            w_up = g(f"{p}.1.conv.weight")  # [in, out, 2r]
            cout = w_up.shape[1]
            cin_p, cout_p = cin if j == 0 else _pad64(cin), _pad64(cout)
            up = TransConv(_pad(w_up.float(), {0: cin_p, 1: cout_p}),
                           _pad(g(f"{p}.1.conv.bias").float(), {0: cout_p}), r)
            units = []
            for u, d in enumerate(DILATIONS):
                q = f"{p}.{u + 2}"
                c1 = _pad(g(f"{q}.conv1.conv.weight").float(), {0: cout_p, 1: cout_p})
                c2 = _pad(g(f"{q}.conv2.conv.weight").float(), {0: cout_p, 1: cout_p})
                units.append(ResidualUnit(
                    _snake(g, f"{q}.act1", cout_p),
                    Conv(c1, _pad(g(f"{q}.conv1.conv.bias").float(), {0: cout_p}), d),
                    _snake(g, f"{q}.act2", cout_p),
                    Conv(c2, _pad(g(f"{q}.conv2.conv.bias").float(), {0: cout_p}), 1)))
            blocks.append(DecoderBlock(_snake(g, f"{p}.0", cin_p), up, units))
            cin = cout
        last = len(rates) + 1
        cin_p = _pad64(cin)
        out_act = _snake(g, f"decoder.decoder.{last}", cin_p)
        w_out = _pad(g(f"decoder.decoder.{last + 1}.conv.weight").float(), {0: 32, 1: cin_p})
        b_out = _pad(g(f"decoder.decoder.{last + 1}.conv.bias").float(), {0: 32})
        return cls(front, head, blocks, out_act, Conv(w_out, b_out, 1))

    @staticmethod
    def synthetic_weights(seed: int = 0, device="cuda", latent=LATENT, tf_dim=TF_DIM,
                          tf_layers=TF_LAYERS, tf_heads=TF_HEADS, tf_ffn=TF_FFN,
                          decoder_dim=DECODER_DIM, rates=RATES, codebook=CODEBOOK,
                          inner=INNER, codebook_dim=CODEBOOK_DIM) -> dict:
        """Seeded random tensors with the checkpoint's names and shapes, scaled so activations
        stay O(1) through the stack (no checkpoint exists in this image)."""
        gen = torch.Generator(device=device).manual_seed(seed)
        w = {}

        def r(name, *shape, scale=None, fan=None):
            s = scale if scale is not None else 1.0 / math.sqrt(fan or shape[-1])
            w[name] = torch.randn(*shape, generator=gen, device=device) * s

        def ones(name, n, jitter=0.1):
            w[name] = 1.0 + (torch.rand(n, generator=gen, device=device) - 0.5) * 2 * jitter

        for prefix, layers in (("decoder.quantizer.rvq_first", SEMANTIC),
                               ("decoder.quantizer.rvq_rest", QUANTIZERS - SEMANTIC)):
            for i in range(layers):
                p = f"{prefix}.vq.layers.{i}._codebook"
                r(f"{p}.embedding_sum", codebook, inner, scale=1.0 / math.sqrt(layers))
                w[f"{p}.cluster_usage"] = torch.rand(codebook, generator=gen, device=device) + 0.5
            r(f"{prefix}.output_proj.weight", codebook_dim, inner, 1)
        r("decoder.pre_conv.conv.weight", latent, codebook_dim, 3, fan=codebook_dim * 3)
        r("decoder.pre_conv.conv.bias", latent, scale=0.02)
        t = "decoder.pre_transformer"
        r(f"{t}.input_proj.weight", tf_dim, latent)
        r(f"{t}.input_proj.bias", tf_dim, scale=0.02)
        r(f"{t}.output_proj.weight", latent, tf_dim)
        r(f"{t}.output_proj.bias", latent, scale=0.02)
        ones(f"{t}.norm.weight", tf_dim)
        hw = tf_heads * TF_HD
        for i in range(tf_layers):
            p = f"{t}.layers.{i}"
            for n in ("q", "k", "v"):
                r(f"{p}.self_attn.{n}_proj.weight", hw, tf_dim)
            r(f"{p}.self_attn.o_proj.weight", tf_dim, hw)
            r(f"{p}.mlp.gate_proj.weight", tf_ffn, tf_dim)
            r(f"{p}.mlp.up_proj.weight", tf_ffn, tf_dim)
            r(f"{p}.mlp.down_proj.weight", tf_dim, tf_ffn)
            ones(f"{p}.input_layernorm.weight", tf_dim)
            ones(f"{p}.post_attention_layernorm.weight", tf_dim)
            w[f"{p}.self_attn_layer_scale.scale"] = torch.full((tf_dim,), 0.01, device=device)
            w[f"{p}.mlp_layer_scale.scale"] = torch.full((tf_dim,), 0.01, device=device)
        for i in range(2):
            p = f"decoder.upsample.{i}"
            r(f"{p}.0.conv.weight", latent, latent, 2, fan=latent)
            r(f"{p}.0.conv.bias", latent, scale=0.02)
            c = f"{p}.1"
            r(f"{c}.dwconv.conv.weight", latent, 1, 7, fan=7)
            r(f"{c}.dwconv.conv.bias", latent, scale=0.02)
            ones(f"{c}.norm.weight", latent)
            r(f"{c}.norm.bias", latent, scale=0.02)
            r(f"{c}.pwconv1.weight", 4 * latent, latent)
            r(f"{c}.pwconv1.bias", 4 * latent, scale=0.02)
            r(f"{c}.pwconv2.weight", latent, 4 * latent)
            r(f"{c}.pwconv2.bias", latent, scale=0.02)
            w[f"{c}.gamma"] = torch.full((latent,), 0.1, device=device)
        r("decoder.decoder.0.conv.weight", decoder_dim, latent, 7, fan=latent * 7)
        r("decoder.decoder.0.conv.bias", decoder_dim, scale=0.02)
        cin = decoder_dim
        for j, rate in enumerate(rates):
            p = f"decoder.decoder.{j + 1}.block"
            cout = cin // 2
            for a in ("alpha", "beta"):
                w[f"{p}.0.{a}"] = (torch.rand(cin, generator=gen, device=device) - 0.5) * 0.4
            r(f"{p}.1.conv.weight", cin, cout, 2 * rate, fan=cin * 2)
            r(f"{p}.1.conv.bias", cout, scale=0.02)
            for u in range(3):
                q = f"{p}.{u + 2}"
                for n in ("act1", "act2"):
                    for a in ("alpha", "beta"):
                        w[f"{q}.{n}.{a}"] = (torch.rand(cout, generator=gen, device=device) - 0.5) * 0.4
                r(f"{q}.conv1.conv.weight", cout, cout, 7, fan=cout * 7 * 4)
                r(f"{q}.conv1.conv.bias", cout, scale=0.01)
                r(f"{q}.conv2.conv.weight", cout, cout, 1, fan=cout * 4)
                r(f"{q}.conv2.conv.bias", cout, scale=0.01)
            cin = cout
        last = len(rates) + 1
        for a in ("alpha", "beta"):
            w[f"decoder.decoder.{last}.{a}"] = (torch.rand(cin, generator=gen, device=device) - 0.5) * 0.4
        r(f"decoder.decoder.{last + 1}.conv.weight", 1, cin, 7, fan=cin * 7 * 4)
        w[f"decoder.decoder.{last + 1}.conv.bias"] = torch.zeros(1, device=device)
        return w

    def __call__(self, codes: torch.Tensor, trace: bool = False):
        """Codec::forward (codec.rs:403-424): codes [T, 16] -> waveform f32 [T * 1920]."""
        latent = self.front(codes)
        h = self.head(latent.half())
        for blk in self.blocks:
            h = blk(h)
        y = self.out_conv(h, snake=self.out_act)
        wav = y[0, :, 0].float().clamp(-1.0, 1.0)
        return (wav, latent, h) if trace else wav
