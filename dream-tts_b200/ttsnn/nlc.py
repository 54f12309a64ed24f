"""Channels-last convolutions (crates/tts-nn/src/nlc.rs, nlcconv.rs) on the tcgen05
implicit-GEMM kernel. Weight helpers follow the reference's layouts; `device_weight` turns
the reference's tap-major `[k, in, out]` into the kernel's `[out, k, in]`."""
from __future__ import annotations

import torch

from . import _lib as L
from ._ctx import ctx_of, ptr, stream


def tap_weight(w: torch.Tensor) -> torch.Tensor:
    """torch `[out, in, k]` -> tap-major `[k, in, out]` (nlc.rs:30-33)."""
    return w.permute(2, 1, 0).contiguous()


def device_weight(w_tap: torch.Tensor) -> torch.Tensor:
    """Tap-major `[k, in, out]` -> `[out, k, in]` f16, K-major per output channel."""
    return w_tap.permute(2, 0, 1).to(torch.float16).contiguous()


def transpose_weights(w: torch.Tensor, stride: int) -> list[torch.Tensor]:
    """Transposed-conv weight `[in, out, k]` -> one `[in, out * stride]` matrix per tap group
    (nlc.rs:141-162)."""
    cin, out, k = w.shape
    if k % stride:
        raise ValueError(f"polyphase form needs kernel divisible by stride, got k={k} stride={stride}")
    t = w.permute(0, 2, 1).contiguous()  # [in, k, out]
    return [t[:, i * stride:(i + 1) * stride, :].reshape(cin, stride * out)
            for i in range(k // stride)]


def transpose_tap_weight(w: torch.Tensor, stride: int) -> torch.Tensor:
    """The transposed conv as a causal conv: tap groups reversed, `[m, in, out * stride]`
    (nlc.rs:164-174)."""
    taps = transpose_weights(w, stride)
    return torch.stack(taps[::-1], 0).contiguous()


def transpose_bias(b: torch.Tensor, stride: int) -> torch.Tensor:
    """Bias repeated over the `stride` interleaved output phases (nlc.rs:176-183)."""
    return b.reshape(1, -1).expand(stride, -1).reshape(-1).contiguous()


def conv1d(x: torch.Tensor, w_dev: torch.Tensor, bias: torch.Tensor | None, dilation: int,
           pad_left: int, snake: tuple[torch.Tensor, torch.Tensor] | None = None,
           res: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """`x [b, L, cin]` f16 * `w_dev [cout, k, cin]` f16 -> `[b, L, cout]` f16 with f32
    accumulation; rows outside [0, L) read as zero; optional SnakeBeta on load and residual."""
    b, length, cin = x.shape
    cout, k, wcin = w_dev.shape
    if wcin != cin:
        raise ValueError(f"conv input width {cin} != weight {wcin}")
    xh = x.to(torch.float16).contiguous()
    y = out if out is not None else torch.empty(b, length, cout, device=x.device,
                                                dtype=torch.float16)
    bi = None if bias is None else bias.to(torch.float32).contiguous()
    a = br = None
    if snake is not None:
        a = snake[0].to(torch.float32).contiguous()
        br = snake[1].to(torch.float32).contiguous()
    r = None if res is None else res.to(torch.float16).contiguous()
    L.call("tts_conv1d_nlc", ctx_of(xh), ptr(xh), b, length, cin, ptr(w_dev), cout, k,
           int(dilation), int(pad_left), ptr(bi), ptr(a), ptr(br), ptr(r), ptr(y), stream())
    return y


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None,
                  dilation: int) -> torch.Tensor:
    """Causal conv over `[b, L, C_in]` with a tap-major weight `[k, in, out]` (nlc.rs:70-132).
    Returns x's dtype; the kernel computes in f16 with f32 accumulation."""
    k = w.shape[0]
    y = conv1d(x, device_weight(w), bias, dilation, (k - 1) * dilation)
    return y if x.dtype == torch.float16 else y.to(x.dtype)


def snake_conv_residual(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, dilation: int,
                        snake: tuple[torch.Tensor, torch.Tensor],
                        res: torch.Tensor) -> torch.Tensor | None:
    """`res + causal_conv1d(snake(x))` in one launch (nlc.rs:40-68); None when the shapes are
    outside the kernel, for the caller to compose."""
    b, length, cin = x.shape
    k, _, cout = w.shape
    if cin % 64 or cout % 32 or tuple(res.shape) != (b, length, cout):
        return None
    y = conv1d(x, device_weight(w), bias, dilation, (k - 1) * dilation, snake=snake, res=res)
    return y if x.dtype == torch.float16 else y.to(x.dtype)


def depthwise(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """`nlc::depthwise` (crates/tts-nn/src/nlc.rs:232-256): causal per-channel conv over
    [b, L, C] with torch's [C, 1, k] taps, f32."""
    xf = x.to(torch.float32).contiguous()
    b, L_, C_ = xf.shape
    k = w.shape[-1]
    taps = w.reshape(C_, k).to(torch.float32).contiguous()
    bb = None if bias is None else bias.to(torch.float32).contiguous()
    y = torch.empty_like(xf)
    L.call("tts_depthwise_conv", ctx_of(xf), ptr(xf), b, L_, C_, ptr(taps), k, ptr(bb), ptr(y),
           stream())
    return y
