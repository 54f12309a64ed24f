"""Device-side code picking: greedy (crates/qwen3tts/src/talker.rs:154-189) and top-k sampling
with caller-supplied draws (crates/tts-nn/src/topk.rs)."""
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


def talker_pick(logits: torch.Tensor, rule, record: bool = False) -> torch.Tensor:
    """sample_with_u's greedy branch (crates/qwen3tts/src/talker.rs:154-189) on `[rows, vocab]`
    f32 under a pick rule (`rule.c`, a PickRule; counts and frames indexed by row): banned ids
    and a young eos at -inf, each id's logit penalised once per time the row emitted it, the
    last of equal maxima. With `record`, the picks join the rows' histories (talker.rs:984-996)."""
    x = logits.to(torch.float32).contiguous()
    rows, n = x.shape
    out = torch.empty(rows, dtype=torch.int32, device=x.device)
    L.call("tts_talker_pick", ctx_of(x), ptr(x), rows, n, rule.c, 1 if record else 0, ptr(out),
           stream())
    return out


MAX_N = 4096
MAX_K = 64


def sample(logits: torch.Tensor, draws: torch.Tensor, k: int, temperature: float) -> torch.Tensor:
    """One index per row of `logits` `[rows, n]` drawn from its top `k` at `temperature` with
    `draws[row]` in `[0, 1)` (crates/tts-nn/src/topk.rs:98-107): no nucleus cut, no penalty."""
    x = logits.to(torch.float32).contiguous()
    rows, n = x.shape
    d = draws.to(torch.float32).contiguous()
    if d.numel() != rows:
        raise L.TtsError(1, f"topk_sample: {d.numel()} draws for {rows} rows")
    out = torch.empty(rows, dtype=torch.int32, device=x.device)
    L.call("tts_topk_sample", ctx_of(x), ptr(x), rows, n, ptr(d), int(k), float(temperature),
           ptr(out), stream())
    return out
