"""Fused elementwise ops (crates/tts-nn/src/fused.rs): SwiGLU's tail and SnakeBeta."""
from __future__ import annotations

import torch

from ._ctx import ctx_of, ptr, stream
from . import _lib as L


def swiglu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """`silu(gate) * up` (fused.rs:289-386), f32."""
    if gate.shape != up.shape:
        raise ValueError("swiglu_mul: shapes differ")
    g = gate.to(torch.float32).contiguous()
    u = up.to(torch.float32).contiguous()
    y = torch.empty_like(g)
    L.call("tts_swiglu_mul", ctx_of(g), ptr(g), ptr(u), g.numel(), ptr(y), 0, stream())
    return y


def snake_beta_nlc(x: torch.Tensor, alpha: torch.Tensor, beta_recip: torch.Tensor) -> torch.Tensor:
    """`x + beta_recip * sin^2(alpha * x)` channels-last, f32 math, f16 or f32 I/O
    (fused.rs:526-663). alpha and beta_recip are the load-time folds exp(alpha) and
    1/(exp(beta) + 1e-9) (crates/qwen3tts/src/codec.rs:61-68)."""
    c = x.shape[-1]
    if alpha.numel() != c or beta_recip.numel() != c:
        raise ValueError("snake_beta_nlc: per-channel parameters must match the last dim")
    xc = x.contiguous()
    half = xc.dtype == torch.float16
    if not half:
        xc = xc.to(torch.float32)
    y = torch.empty_like(xc)
    a = alpha.to(torch.float32).contiguous()
    br = beta_recip.to(torch.float32).contiguous()
    L.call("tts_snake_beta_nlc", ctx_of(xc), ptr(xc), 1 if half else 0, ptr(a), ptr(br),
           xc.numel() // c, c, ptr(y), 1 if half else 0, stream())
    return y
