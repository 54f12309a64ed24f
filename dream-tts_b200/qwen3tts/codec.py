"""The codec decoder's conv stack on B200 (crates/qwen3tts/src/codec.rs), channels-last f16
activations with f32 accumulation, every convolution on the tcgen05 implicit-GEMM kernel.

Modules mirror the reference's: `SnakeBeta` (codec.rs:55-73), `Conv` (:85-120), `TransConv`
(:124-159, the transposed conv as one causal conv over reversed tap groups), `ResidualUnit`
(:199-230), `DecoderBlock` (:232-260), and `chunk_plan`, the chunked decode with left context and
uniform right-padded spans (:581-604). Beyond the reference, both SnakeBeta activations of a
residual unit and the block activation before the upsampling conv are applied inside the conv's
operand load, and a whole document's chunks decode as one batch (the conv's batch axis).

Synthetic benchmark workloads: `SnakeBlock` is the codec residual block (three k7 convs,
dilations 1/3/9, 'same' padding, Snake with 1/alpha, each `x + conv(snake(x))`), and
`WaveStack` is the synthetic document's decoder (x8, x5, x4, x3 transposed convs 1024->512->256->128->64,
three config[1] blocks after each), preceded by the reference's two x2 upsamplers at 1024
channels so one 12.5 Hz frame becomes 1920 samples at 24 kHz.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ttsnn import nlc

CHUNK_FRAMES = 300        # crates/qwen3tts/src/cfg.rs:281
CHUNK_LEFT_CONTEXT = 25   # crates/qwen3tts/src/cfg.rs:282
SAMPLES_PER_FRAME = 1920  # crates/qwen3tts/src/cfg.rs:14-15 (2*2 * 8*5*4*3)


@dataclass
class Window:
    start: int   # first frame kept
    end: int     # one past the last frame kept
    lo: int      # first frame fed (start minus the left context)
    hi: int      # one past the last real frame fed
    span: int    # frames fed after right padding (repeating the last frame)
    drop: int    # leading frames of output discarded (the context)


def chunk_plan(n: int, chunk: int = CHUNK_FRAMES, ctx: int = CHUNK_LEFT_CONTEXT,
               right: int = 0) -> list[Window]:
    """The reference's chunked decode (crates/qwen3tts/src/codec.rs:581-604): chunks of
    `chunk` frames, each fed with up to `ctx` frames of left context; when the document is at
    least one span long every window is padded on the right to the same span by repeating its
    last frame (the reference decoder is causal, so frames after the kept ones cannot change
    them). `right` > 0 adds that many frames of right context for a decoder that looks ahead
    (`WaveStack`'s 'same'-padded blocks); the reference's plan is `right=0`."""
    span = chunk + ctx + right
    out = []
    start = 0
    while start < n:
        end = min(start + chunk, n)
        lo = max(0, start - ctx)
        hi = min(lo + span, n)
        out.append(Window(start, end, lo, hi, span if n >= span else hi - lo, start - lo))
        start = end
    return out


def gather_windows(frames: torch.Tensor, plan: list[Window]) -> torch.Tensor:
    """[n, C] per-frame inputs -> [windows, span, C], padding each window by repeating its last
    real frame. All windows of a plan have one span (or the plan has one window)."""
    span = plan[0].span
    rows = []
    for w in plan:
        idx = torch.arange(w.lo, w.lo + span, device=frames.device).clamp(max=w.hi - 1)
        rows.append(frames.index_select(0, idx))
    return torch.stack(rows, 0)


def stitch(out: torch.Tensor, plan: list[Window], per_frame: int) -> torch.Tensor:
    """[windows, span * per_frame, ...] decoded windows -> the document's kept samples."""
    pieces = [out[i, w.drop * per_frame:(w.drop + w.end - w.start) * per_frame]
              for i, w in enumerate(plan)]
    return torch.cat(pieces, 0)


class SnakeBeta:
    """x + brecip * sin^2(alpha * x) with the reference's load-time folds:
    alpha = exp(log_alpha), brecip = 1 / (exp(log_beta) + 1e-9) (codec.rs:61-68)."""

    def __init__(self, log_alpha: torch.Tensor, log_beta: torch.Tensor):
        self.alpha = log_alpha.float().exp().contiguous()
        self.brecip = (1.0 / (log_beta.float().exp() + 1e-9)).contiguous()

    @classmethod
    def snake(cls, alpha: torch.Tensor) -> "SnakeBeta":
        """Plain Snake, x + sin^2(alpha x) / alpha, as the synthetic residual block uses it."""
        s = cls.__new__(cls)
        s.alpha = alpha.float().contiguous()
        s.brecip = (1.0 / alpha.float()).contiguous()
        return s

    def pair(self):
        return self.alpha, self.brecip


class Conv:
    """Conv1d over channels-last [b, L, cin] from torch's [out, in, k] weight; causal by default
    (pad_left = (k-1)*d, codec.rs:85-120), 'same' with pad_left = (k-1)*d/2."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, dilation: int = 1,
                 pad_left: int | None = None):
        self.cout, self.cin, self.k = weight.shape
        self.w = nlc.device_weight(nlc.tap_weight(weight.float()))
        self.bias = None if bias is None else bias.float().contiguous()
        self.dilation = dilation
        self.pad_left = (self.k - 1) * dilation if pad_left is None else pad_left

    def __call__(self, x, snake: SnakeBeta | None = None, res=None, out=None):
        return nlc.conv1d(x, self.w, self.bias, self.dilation, self.pad_left,
                          snake=None if snake is None else snake.pair(), res=res, out=out)


class TransConv:
    """Transposed conv, stride s, kernel m*s, as one causal conv over m reversed tap groups that
    emits the s output phases interleaved on the channel axis, then a free reshape
    (crates/tts-nn/src/nlc.rs:141-183; codec.rs:124-159). Weight is torch's [in, out, k]."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor, stride: int):
        cin, cout, k = weight.shape
        self.stride, self.cout, self.m = stride, cout, k // stride
        tap = nlc.transpose_tap_weight(weight.float(), stride)  # [m, cin, s*cout]
        self.w = nlc.device_weight(tap)
        self.bias = nlc.transpose_bias(bias.float(), stride).contiguous()

    def __call__(self, x, snake: SnakeBeta | None = None):
        b, length, _ = x.shape
        y = nlc.conv1d(x, self.w, self.bias, 1, self.m - 1,
                       snake=None if snake is None else snake.pair())
        return y.reshape(b, length * self.stride, self.cout)


class ResidualUnit:
    """SnakeBeta, k7 dilated conv, SnakeBeta, k1 conv, residual (codec.rs:199-230); both
    activations run inside the convs' operand loads."""

    def __init__(self, act1, conv1: Conv, act2, conv2: Conv):
        self.act1, self.conv1, self.act2, self.conv2 = act1, conv1, act2, conv2

    def __call__(self, x):
        h = self.conv1(x, snake=self.act1)
        return self.conv2(h, snake=self.act2, res=x)


class DecoderBlock:
    """SnakeBeta, upsampling TransConv, three residual units at dilations 1, 3, 9
    (codec.rs:232-260)."""

    def __init__(self, act, up: TransConv, units: list[ResidualUnit]):
        self.act, self.up, self.units = act, up, units

    def __call__(self, x):
        h = self.up(x, snake=self.act)
        for u in self.units:
            h = u(h)
        return h


class SnakeBlock:
    """The synthetic codec residual block: for dilation 1, 3, 9, x = x + conv_k7(snake(x)) with 'same' padding;
    each step is one conv launch with the snake on load and the residual in the epilogue."""

    def __init__(self, channels: int, gen: torch.Generator, device, std: float = 0.02):
        self.convs = []
        for d in (1, 3, 9):
            w = torch.randn(channels, channels, 7, generator=gen, device=device) * std
            alpha = torch.exp(torch.rand(channels, generator=gen, device=device) * 2 - 1)
            self.convs.append((Conv(w, torch.zeros(channels, device=device), d, 3 * d),
                               SnakeBeta.snake(alpha)))

    def __call__(self, x, spare=None):
        """`spare`: two buffers shaped like x, neither aliasing it (a conv reads its input's
        halo while other CTAs write the output). Returns spare[0]."""
        s0, s1 = spare if spare is not None else (torch.empty_like(x), torch.empty_like(x))
        (c0, a0), (c1, a1), (c2, a2) = self.convs
        c0(x, snake=a0, res=x, out=s0)
        c1(s0, snake=a1, res=s0, out=s1)
        c2(s1, snake=a2, res=s1, out=s0)
        return s0


class WaveStack:
    """The synthetic document decoder: two x2 upsamplers at 1024 channels (the reference's, for
    24 kHz), then x8, x5, x4, x3 transposed convs (kernel 2 * stride) 1024 -> 512 -> 256 -> 128
    -> 64, three `SnakeBlock`s after each, a final Snake and k7 conv to one channel, clamped to
    [-1, 1]. Random-init (no checkpoint in this image); the upsampler and output weights are
    scaled (0.3 / sqrt(fan-in), 0.05 / sqrt(fan-in)) so activations stay within f16 range through
    the 36 snake convs and the waveform mostly inside the clamp. Input: [b, frames, 1024]."""

    RATES = (8, 5, 4, 3)
    WIDTHS = (1024, 512, 256, 128, 64)

    def __init__(self, device, seed: int = 0, blocks: int = 3):
        gen = torch.Generator(device=device).manual_seed(seed)

        def tconv(cin, cout, s):
            w = torch.randn(cin, cout, 2 * s, generator=gen, device=device) * (0.3 / math.sqrt(2 * cin))
            return TransConv(w, torch.zeros(cout, device=device), s)

        self.pre = [tconv(1024, 1024, 2), tconv(1024, 1024, 2)]
        self.stages = []
        for s, cin, cout in zip(self.RATES, self.WIDTHS[:-1], self.WIDTHS[1:]):
            act = SnakeBeta.snake(torch.exp(torch.rand(cin, generator=gen, device=device) * 2 - 1))
            self.stages.append((act, tconv(cin, cout, s),
                                [SnakeBlock(cout, gen, device) for _ in range(blocks)]))
        self.out_act = SnakeBeta.snake(torch.exp(torch.rand(64, generator=gen, device=device) * 2 - 1))
        w = torch.zeros(32, 64, 7, device=device)  # one real output channel, padded to 32
        w[0] = torch.randn(64, 7, generator=gen, device=device) * (0.05 / math.sqrt(64 * 7))
        self.out = Conv(w, torch.zeros(32, device=device), 1)

    def flops_per_frame(self) -> float:
        f = 0.0
        t = 1
        for _ in self.pre:
            f += 2 * 1024 * 1024 * 2 * t * 2  # m=1 tap, 2 phases per input frame
            t *= 2
        for (act, up, blocks), cin, cout, s in zip(self.stages, self.WIDTHS[:-1], self.WIDTHS[1:],
                                                   self.RATES):
            f += 2 * t * cin * cout * s * 2      # 2 tap groups, s phases
            t *= s
            f += len(blocks) * 3 * 2 * t * cout * cout * 7
        f += 2 * t * 64 * 32 * 7
        return f

    def raw(self, x):
        """The stack up to the final conv, unclamped: [b, frames * 1920, 32] f16 whose
        channel 0 is the waveform."""
        h = x
        for up in self.pre:
            h = up(h)
        for act, up, blocks in self.stages:
            h = up(h, snake=act)
            spare = (torch.empty_like(h), torch.empty_like(h))
            for blk in blocks:
                out = blk(h, spare)
                spare = (h, spare[1])
                h = out
        return self.out(h, snake=self.out_act)

    def __call__(self, x):
        """[b, frames, 1024] f16 latents -> [b, frames * 1920] f16 samples in [-1, 1]."""
        return self.raw(x)[..., 0].clamp_(-1.0, 1.0)
