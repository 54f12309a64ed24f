"""Decode attention reading the KV cache in place (crates/tts-nn/src/attn.rs)."""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from ._ctx import ctx_of, ptr, stream
from .qkrope import contiguous_cache


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, span: int,
                     window_start: int) -> torch.Tensor:
    """`q [b, n_kv, gqa, 128]` f32 (scale folded in) over caches `[b, n_kv, cap, 128]` f16:
    softmax over positions `[window_start, span)` (attn.rs:22-73). Returns f32 like q."""
    b, n_kv, gqa, hd = q.shape
    cap = k.shape[2]
    if span > cap:
        raise ValueError(f"span {span} exceeds capacity {cap}")
    if k.dtype != torch.float16:
        raise L.TtsError(2, "decode_attention: the cache must be f16")
    kv, table = contiguous_cache(k, v)
    spans = torch.full((b,), span, dtype=torch.int32, device=q.device)
    window = span - window_start if window_start > 0 else 0
    qc = q.to(torch.float32).contiguous()
    out = torch.empty(b, n_kv, gqa, hd, device=q.device, dtype=torch.float32)
    L.call("tts_decode_attention", ctx_of(qc), ptr(qc), b, gqa, C.byref(kv), ptr(spans),
           span, window, ptr(out), 0, stream())
    return out


def decode_attention_paged(q: torch.Tensor, kv: L.KvCache, spans: torch.Tensor, max_span: int,
                           window: int = 0, out_f16: bool = True) -> torch.Tensor:
    """Paged form: per-lane spans; q `[lanes, n_kv * gqa, 128]`."""
    lanes, heads, hd = q.shape
    gqa = heads // kv.n_kv
    out = torch.empty(lanes, heads * hd, device=q.device,
                      dtype=torch.float16 if out_f16 else torch.float32)
    L.call("tts_decode_attention", ctx_of(q), ptr(q), lanes, gqa, C.byref(kv), ptr(spans),
           int(max_span), int(window), ptr(out), 1 if out_f16 else 0, stream())
    return out
