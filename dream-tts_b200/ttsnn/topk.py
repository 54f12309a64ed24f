"""Device-side code picking (crates/tts-nn/src/topk.rs; greedy path of
crates/qwen3tts/src/talker.rs:154-189)."""
from __future__ import annotations

import torch

from . import _lib as L
from ._ctx import ctx_of, ptr, stream


def argmax(logits: torch.Tensor, banned: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy pick per row over `[rows, n]` f32 with banned ids at -inf; ties go to the
    highest index, as Rust's `max_by` keeps the last maximum."""
    x = logits.to(torch.float32).contiguous()
    rows, n = x.reshape(-1, x.shape[-1]).shape
    out = torch.empty(rows, dtype=torch.int32, device=x.device)
    b = None
    if banned is not None:
        b = banned.to(torch.uint8).contiguous()
        if b.numel() != n:
            raise ValueError("argmax: banned mask must cover every id")
    L.call("tts_argmax", ctx_of(x), ptr(x), rows, n, ptr(b), ptr(out), stream())
    return out
