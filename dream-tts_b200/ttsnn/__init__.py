"""tts-nn on B200: the operator surface crates/qwen3tts calls, backed by sm_100a kernels.

Names, argument meanings and error behaviour follow the reference crate `tts-nn`
(crates/tts-nn/src/lib.rs and its op modules); tensors are torch CUDA tensors, and every op
runs through the C ABI of libtts_cuda.so (include/tts_cuda.h). Nothing here computes on the
CPU: a shape the kernels do not take raises TtsError(UNSUPPORTED_SHAPE).
"""
from __future__ import annotations

import math

import torch

from . import _lib as L
from ._ctx import check, ctx, ctx_of, launch_count, ptr, stream
from ._lib import TtsError
from . import attn, fused, nlc, qkrope, topk  # noqa: F401  (submodules mirror tts-nn's)

__all__ = ["Proj", "pack_weight", "interleave_gate_up", "rms_norm", "rope_table_f32", "abs_and_rel", "TtsError", "check", "ctx",
           "launch_count", "attn", "fused", "nlc", "qkrope", "topk"]


class Proj:
    """`Proj::Half` (crates/tts-nn/src/lib.rs:388-401, 510-533): f16 weight, f32 in and out.

    The weight stays in the checkpoint's `[out, in]` layout, which is the K-major operand the
    tcgen05 GEMM wants (the reference transposes to `[in, out]` at load instead,
    lib.rs:473-489). `forward` casts x to f16 (lib.rs:517) and accumulates in f32, like the
    reference's skinny kernel (skinny.rs:155-165).
    """

    def __init__(self, w_out_in: torch.Tensor, packed: bool = True):
        if w_out_in.dim() != 2:
            raise ValueError("Proj: weight must be [out, in]")
        w = w_out_in.to(torch.float16).contiguous()
        self.n, self.k = w.shape
        # packed: each 128 x 64 tile the GEMM streams is one contiguous block (pack_weight)
        self.packed = packed and self.n % 128 == 0 and self.k % 64 == 0
        self.w = pack_weight(w) if self.packed else w

    @classmethod
    def from_tensor(cls, t: torch.Tensor, device: torch.device | None = None) -> "Proj":
        return cls(t.to(device or t.device))

    def forward(self, x: torch.Tensor, epilogue: int = L.EPI_F32,
                out: torch.Tensor | None = None) -> torch.Tensor:
        if x.shape[-1] != self.k:
            raise ValueError(f"Proj: input width {x.shape[-1]} != {self.k}")
        lead = x.shape[:-1]
        rows = math.prod(lead) if lead else 1
        h = x.to(torch.float16).reshape(rows, self.k).contiguous()
        if epilogue == L.EPI_F32:
            y = out if out is not None else torch.empty(rows, self.n, device=x.device,
                                                        dtype=torch.float32)
        elif epilogue == L.EPI_F16:
            y = out if out is not None else torch.empty(rows, self.n, device=x.device,
                                                        dtype=torch.float16)
        elif epilogue == L.EPI_RESIDUAL_F32:
            if out is None:
                raise ValueError("Proj: the residual epilogue needs `out` (the residual stream)")
            y = out
        elif epilogue == L.EPI_SWIGLU_F16:
            y = out if out is not None else torch.empty(rows, self.n // 2, device=x.device,
                                                        dtype=torch.float16)
        else:
            raise ValueError("Proj: unknown epilogue")
        L.call("tts_proj_forward_packed" if self.packed else "tts_proj_forward", ctx_of(x),
               ptr(h), rows, self.k, ptr(self.w), self.n, epilogue, ptr(y), 0, stream())
        return y.reshape(*lead, y.shape[-1]) if epilogue != L.EPI_RESIDUAL_F32 else y

    __call__ = forward

    def forward_rows(self, x: torch.Tensor, epilogue: int = L.EPI_F32,
                     out: torch.Tensor | None = None) -> torch.Tensor:
        """The projection shaped for many token rows (tts_proj_forward_rows): x [rows, k] with
        any rows; epilogue f32, residual (into `out`) or SwiGLU; n % 256 == 0."""
        if not self.packed:
            raise ValueError("Proj.forward_rows: needs a packed weight")
        h = x.to(torch.float16).reshape(-1, self.k).contiguous()
        rows = h.shape[0]
        if epilogue == L.EPI_F32:
            y = out if out is not None else torch.empty(rows, self.n, device=x.device)
        elif epilogue == L.EPI_RESIDUAL_F32:
            if out is None:
                raise ValueError("Proj: the residual epilogue needs `out` (the residual stream)")
            y = out
        elif epilogue == L.EPI_SWIGLU_F16:
            y = out if out is not None else torch.empty(rows, self.n // 2, device=x.device,
                                                        dtype=torch.float16)
        else:
            raise ValueError("Proj.forward_rows: epilogue must be f32, residual or SwiGLU")
        L.call("tts_proj_forward_rows", ctx_of(x), ptr(h), rows, self.k, ptr(self.w), self.n,
               epilogue, ptr(y), 0, stream())
        return y


def pack_weight(w: torch.Tensor) -> torch.Tensor:
    """`[n, k]` f16 -> the decode GEMM's streaming layout `[n/128][k/64][128][64]` (returned
    with shape `[n, k]`; only the element order differs). Load-time, like the reference's
    host-side relayout of every projection (crates/tts-nn/src/lib.rs:1252-1298)."""
    src = w.to(torch.float16).contiguous()
    n, k = src.shape
    out = torch.empty_like(src)
    L.call("tts_weight_pack", ctx_of(src), ptr(src), n, k, ptr(out), stream())
    return out


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """`[ffn, dim]` gate and up -> `[2 ffn, dim]` in the SwiGLU epilogue's tile order."""
    ffn, dim = gate.shape
    g = gate.to(torch.float16).contiguous()
    u = up.to(torch.float16).contiguous()
    out = torch.empty(2 * ffn, dim, device=gate.device, dtype=torch.float16)
    L.call("tts_interleave_gate_up", ctx_of(g), ptr(g), ptr(u), ffn, dim, ptr(out), stream())
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             out_f16: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over the last dim in f32 (crates/tts-nn/src/lib.rs:1001-1003)."""
    dim = x.shape[-1]
    xf = x.to(torch.float32).contiguous()
    w = weight.to(torch.float32).contiguous()
    if w.numel() != dim:
        raise ValueError(f"rms_norm: weight has {w.numel()} elements for width {dim}")
    y = torch.empty_like(xf)
    L.call("tts_rms_norm", ctx_of(xf), ptr(xf), ptr(w), xf.numel() // dim, dim, float(eps),
           ptr(y), ptr(out_f16), stream())
    return y


def rope_table_f32(length: int, head_dim: int, base: float,
                   device: torch.device | str = "cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """Half-split RoPE tables `[length, head_dim/2]`, phases in f64 rounded to f32
    (crates/tts-nn/src/lib.rs:1178-1205)."""
    half = head_dim // 2
    i = torch.arange(half, dtype=torch.float64)
    freq = 1.0 / torch.pow(torch.tensor(base, dtype=torch.float64), 2.0 * i / head_dim)
    t = torch.arange(length, dtype=torch.float64)[:, None]
    ph = t * freq[None, :]
    return (torch.cos(ph).to(torch.float32).to(device),
            torch.sin(ph).to(torch.float32).to(device))


def abs_and_rel(a: torch.Tensor, b: torch.Tensor) -> tuple[float, float]:
    """Max abs difference and that difference over b's peak magnitude (lib.rs:1239-1248)."""
    a = a.detach().to(torch.float32).flatten().cpu()
    b = b.detach().to(torch.float32).flatten().cpu()
    d = (a - b).abs().max().item() if a.numel() else 0.0
    s = b.abs().max().item() if b.numel() else 0.0
    return d, (d / s if s > 0 else 0.0)


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, eps: float,
               out_f16: bool = False) -> torch.Tensor:
    """`layer_norm` (crates/tts-nn/src/lib.rs:1006-1035): mean, centred variance, affine."""
    dim = x.shape[-1]
    xf = x.to(torch.float32).contiguous()
    w = weight.to(torch.float32).contiguous()
    b = None if bias is None else bias.to(torch.float32).contiguous()
    y = torch.empty(xf.shape, device=x.device, dtype=torch.float16 if out_f16 else torch.float32)
    L.call("tts_layer_norm", ctx_of(xf), ptr(xf), ptr(w), ptr(b), xf.numel() // dim, dim,
           float(eps), ptr(y), 1 if out_f16 else 0, stream())
    return y


def bias_act(y: torch.Tensor, bias: torch.Tensor | None = None, gelu: bool = False,
             scale: torch.Tensor | None = None, res: torch.Tensor | None = None,
             out_f16: bool = False, silu: bool = False) -> torch.Tensor:
    """A projection's f32 result finished: act(y + bias) (GELU with the exact erf,
    `gelu_exact` lib.rs:1129, or SiLU), times a per-channel `scale`, plus `res`."""
    yf = y.to(torch.float32).contiguous()
    n = yf.shape[-1]
    rows = yf.numel() // n
    out = torch.empty(yf.shape, device=y.device, dtype=torch.float16 if out_f16 else torch.float32)
    f = lambda t: None if t is None else t.to(torch.float32).contiguous()
    b, sc, r = f(bias), f(scale), f(res)
    L.call("tts_bias_act", ctx_of(yf), ptr(yf), rows, n, ptr(b), 2 if silu else (1 if gelu else 0), ptr(sc),
           ptr(r), ptr(out), 1 if out_f16 else 0, stream())
    return out


def gelu_exact(x: torch.Tensor) -> torch.Tensor:
    """`gelu_exact` (crates/tts-nn/src/lib.rs:1129): 0.5 x (1 + erf(x / sqrt 2)), f32."""
    return bias_act(x, gelu=True)


def rope_rows(x: torch.Tensor, col0: int, heads: int, head_dim: int, cos: torch.Tensor,
              sin: torch.Tensor, pos0: int = 0) -> None:
    """Half-split RoPE (candle_nn::rotary_emb::rope) in place on `heads` heads of `head_dim`
    from column `col0` of the f32 rows of x; row t at position pos0 + t."""
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("rope_rows: x must be contiguous f32 [T, ld]")
    T, ld = x.shape
    L.call("tts_rope_rows", ctx_of(x), ptr(x), T, ld, int(col0), int(heads), int(head_dim),
           ptr(cos.contiguous()), ptr(sin.contiguous()), int(pos0), stream())


def window_attention(qkv: torch.Tensor, heads: int, head_dim: int, window: int, scale: float,
                     out_f16: bool = True) -> torch.Tensor:
    """Causal self-attention over one sequence with a sliding window (the prefill branch of
    Stack::forward with causal_window_mask, qwen3.rs:409-444): qkv f32 [T, 3 heads hd]."""
    q = qkv.to(torch.float32).contiguous()
    T = q.shape[0]
    out = torch.empty(T, heads * head_dim, device=q.device,
                      dtype=torch.float16 if out_f16 else torch.float32)
    L.call("tts_window_attention", ctx_of(q), ptr(q), T, int(heads), int(head_dim), int(window),
           float(scale), ptr(out), 1 if out_f16 else 0, stream())
    return out
