"""QK-norm, RoPE and the KV-cache write in one launch (crates/tts-nn/src/qkrope.rs)."""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from ._ctx import ctx_of, ptr, stream


def eligible(qkv: torch.Tensor, k_cache: torch.Tensor, head_dim: int) -> bool:
    """Shapes the kernel takes (qkrope.rs:11-18): f32 activations, f16 cache, head_dim 128."""
    return (qkv.is_cuda and qkv.dtype == torch.float32 and k_cache.dtype == torch.float16
            and head_dim == 128)


def contiguous_cache(k_cache: torch.Tensor, v_cache: torch.Tensor) -> tuple[L.KvCache, torch.Tensor]:
    """The reference's per-lane cache `[b, n_kv, cap, 128]` as a paged cache: one page of
    `cap` positions per lane, page i = lane i of the (possibly narrowed) view."""
    b, n_kv, cap, hd = k_cache.shape
    for c in (k_cache, v_cache):
        if not c.is_contiguous():
            raise ValueError("qk_rope: cache must be contiguous")
    table = torch.arange(b, dtype=torch.int32, device=k_cache.device).reshape(b, 1)
    kv = L.KvCache(k_cache.data_ptr(), v_cache.data_ptr(), table.data_ptr(), 1, cap, b, n_kv, hd)
    return kv, table


def apply(qkv: torch.Tensor, norms: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
          k_cache: torch.Tensor, v_cache: torch.Tensor, heads: int, start, eps: float,
          f32_kv: bool = False) -> tuple[torch.Tensor, None]:
    """`qkv [b, 1, (heads + 2 n_kv) * 128]` f32 -> q `[b, heads, 1, 128]`; k and v are written
    as f16 into the caches `[b, n_kv, cap, 128]` at position `start` (qkrope.rs:26-69).
    `start` may also be an int32 tensor `[b]` of per-lane positions (lanes of different lengths
    in one step, which the paged decode step does; the reference uses one start per call).

    Decode only (t == 1): prefill's multi-position form is not on this path.
    """
    b, t, width = qkv.shape
    _, n_kv, cap, hd = k_cache.shape
    if t != 1:
        raise L.TtsError(2, "qk_rope: only t == 1 (a decode step) is supported")
    if f32_kv:
        raise L.TtsError(2, "qk_rope: the f32 k/v side outputs are prefill-only")
    if isinstance(start, torch.Tensor):
        pos = start.to(device=qkv.device, dtype=torch.int32).contiguous()
        if pos.numel() != b:
            raise ValueError("qk_rope: one position per lane")
        end = int(pos.max().item()) + t
    else:
        pos = torch.full((b,), int(start), dtype=torch.int32, device=qkv.device)
        end = int(start) + t
    if end > cap:
        raise ValueError(f"qk_rope: {end} positions exceed {cap}")
    if width != (heads + 2 * n_kv) * hd:
        raise ValueError("qk_rope: qkv width does not match heads and cache")
    x = qkv.reshape(b, width).contiguous()
    kv, table = contiguous_cache(k_cache, v_cache)
    q = torch.empty(b, heads, hd, device=qkv.device, dtype=torch.float32)
    nm = norms.to(torch.float32).contiguous()
    L.call("tts_qk_rope_append", ctx_of(x), ptr(x), b, heads, ptr(nm), ptr(cos.contiguous()),
           ptr(sin.contiguous()), cos.shape[0], ptr(pos), C.byref(kv), float(eps), ptr(q),
           stream())
    return q.reshape(b, heads, 1, hd), None
