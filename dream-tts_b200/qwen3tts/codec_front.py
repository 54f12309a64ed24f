"""The codec decoder's front on B200 (crates/qwen3tts/src/codec.rs:161-196, 245-317, 403-424):
split RVQ dequantisation (1 semantic + 15 acoustic codebooks, summed lookups, 1x1 output
projections), the causal pre-conv, the 8-layer pre-transformer (dim 512, 16 heads of 64, a
72-frame sliding window, LayerScale on both residual branches, no QK-norm), and the two x2
upsampling stages (causal transposed conv + ConvNeXt: depthwise k7, LayerNorm, 4x MLP with
GELU, gamma, residual), giving the [T * 4, 1024] latent the waveform stack takes.

Projections run on the prefill-shaped GEMM for many rows, else the decode GEMM (f16 weights,
f32 accumulate; rows in chunks of 448), the convolutions on the conv kernel, and the row ops
(lookups, RoPE, windowed attention, LayerNorm, depthwise conv, bias/GELU/scale/residual
epilogues) on the kernels of csrc/codec_front.cu.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

import ttsnn
from ttsnn import _lib as L
from ttsnn._ctx import ctx_of, ptr, stream

from .codec import Conv, TransConv

MAX_ROWS = 448  # rows per projection call (the decode GEMM's limit)
# Above this many rows a projection runs on the prefill-shaped GEMM (tokens as the MMA's M, all
# rows in one launch) where its shape allows; below it the decode GEMM streams the weights.
ROWS_GEMM_MIN = 129


def proj_rows(p: ttsnn.Proj, x: torch.Tensor, epilogue: int = L.EPI_F32) -> torch.Tensor:
    """A projection over any number of rows: one prefill-shaped GEMM for many rows (packed
    weight, n a multiple of 256, f32 or SwiGLU output), else the decode GEMM in chunks it takes."""
    rows = x.shape[0]
    if (rows >= ROWS_GEMM_MIN and p.packed and p.n % 256 == 0
            and epilogue in (L.EPI_F32, L.EPI_SWIGLU_F16)):
        return p.forward_rows(x, epilogue)
    outs = [p.forward(x[r:r + MAX_ROWS], epilogue) for r in range(0, rows, MAX_ROWS)]
    return outs[0] if len(outs) == 1 else torch.cat(outs)


def rvq_gather(codes: torch.Tensor, q0: int, tables: torch.Tensor) -> torch.Tensor:
    """Sum of each row's codebook entries for codebooks q0 .. q0 + len(tables) - 1."""
    T, ncodes = codes.shape
    nq, entries, dim = tables.shape
    out = torch.empty(T, dim, device=codes.device)
    L.call("tts_rvq_gather", ctx_of(codes), ptr(codes), T, ncodes, q0, nq, ptr(tables), entries,
           dim, ptr(out), stream())
    return out


class Rvq:
    """One ResidualVectorQuantizer stack's decode path (codec.rs:245-304): codebooks already
    folded (embedding_sum / cluster_usage.clamp(1e-5)) f32 [nq, entries, inner], output
    projection [out, inner] (the 1x1 conv)."""

    def __init__(self, codebooks: torch.Tensor, output_proj: torch.Tensor, q0: int):
        self.tables = codebooks.float().contiguous()
        self.proj = ttsnn.Proj(output_proj.reshape(output_proj.shape[0], -1))
        self.q0 = q0

    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        return proj_rows(self.proj, rvq_gather(codes, self.q0, self.tables))


@dataclass
class TfLayer:
    """A pre-transformer layer (qwen3.rs Layer with layer_scale, no qk_norm, gqa 1)."""
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    wqkv: ttsnn.Proj
    wo: ttsnn.Proj
    gate_up: ttsnn.Proj
    down: ttsnn.Proj
    attn_scale: torch.Tensor
    mlp_scale: torch.Tensor


class PreTransformer:
    """Stack::forward at t > 1 over one chunk (qwen3.rs:294-467 with the codec's geometry:
    dim 512, 16 heads x 64, window 72, eps 1e-5, RoPE base 1e4, LayerScale)."""

    def __init__(self, layers: list[TfLayer], norm: torch.Tensor, heads: int = 16,
                 head_dim: int = 64, window: int = 72, eps: float = 1e-5,
                 rope_base: float = 1e4, max_len: int = 4096):
        self.layers, self.norm = layers, norm.float().contiguous()
        self.heads, self.hd, self.window, self.eps = heads, head_dim, window, eps
        dev = norm.device
        self.cos, self.sin = ttsnn.rope_table_f32(max_len, head_dim, rope_base, dev)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        h = x.float().contiguous()
        H, hd = self.heads, self.hd
        for ly in self.layers:
            xn = ttsnn.rms_norm(h, ly.attn_norm, self.eps)
            qkv = proj_rows(ly.wqkv, xn)
            ttsnn.rope_rows(qkv, 0, H, hd, self.cos, self.sin)
            ttsnn.rope_rows(qkv, H * hd, H, hd, self.cos, self.sin)
            a = ttsnn.window_attention(qkv, H, hd, self.window, 1.0 / hd ** 0.5)
            h = ttsnn.bias_act(proj_rows(ly.wo, a), scale=ly.attn_scale, res=h)
            xn = ttsnn.rms_norm(h, ly.ffn_norm, self.eps)
            act = proj_rows(ly.gate_up, xn, L.EPI_SWIGLU_F16)
            h = ttsnn.bias_act(proj_rows(ly.down, act), scale=ly.mlp_scale, res=h)
        return ttsnn.rms_norm(h, self.norm, self.eps)


class ConvNext:
    """ConvNeXt block (codec.rs:161-196): depthwise k7 causal, LayerNorm (eps 1e-6), pw1 +
    GELU, pw2, gamma, residual; channels-last."""

    def __init__(self, dw_w, dw_b, norm_w, norm_b, pw1_w, pw1_b, pw2_w, pw2_b, gamma):
        self.dw_w, self.dw_b = dw_w.float().contiguous(), dw_b.float().contiguous()
        self.norm_w, self.norm_b = norm_w.float().contiguous(), norm_b.float().contiguous()
        self.pw1, self.pw1_b = ttsnn.Proj(pw1_w), pw1_b.float().contiguous()
        self.pw2, self.pw2_b = ttsnn.Proj(pw2_w), pw2_b.float().contiguous()
        self.gamma = gamma.float().contiguous()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        b, length, c = x.shape
        xf = x.float().contiguous()
        h = ttsnn.nlc.depthwise(xf, self.dw_w, self.dw_b)
        h = ttsnn.layer_norm(h, self.norm_w, self.norm_b, 1e-6).reshape(b * length, c)
        u = ttsnn.bias_act(proj_rows(self.pw1, h), self.pw1_b, gelu=True, out_f16=True)
        y = ttsnn.bias_act(proj_rows(self.pw2, u), self.pw2_b, scale=self.gamma,
                           res=xf.reshape(b * length, c))
        return y.reshape(b, length, c)


class CodecFront:
    """codes [T, 16] -> latent [1, 4 T, 1024] (codec.rs:403-424 up to the head conv)."""

    def __init__(self, semantic: Rvq, acoustic: Rvq, pre_conv: Conv, pre_in: ttsnn.Proj,
                 pre_in_b: torch.Tensor, tf: PreTransformer, pre_out: ttsnn.Proj,
                 pre_out_b: torch.Tensor, upsample: list[tuple[TransConv, ConvNext]]):
        self.semantic, self.acoustic, self.pre_conv = semantic, acoustic, pre_conv
        self.pre_in, self.pre_in_b = pre_in, pre_in_b.float().contiguous()
        self.tf, self.pre_out, self.pre_out_b = tf, pre_out, pre_out_b.float().contiguous()
        self.upsample = upsample

    def __call__(self, codes: torch.Tensor, trace: bool = False):
        codes = codes.to(torch.int32).contiguous()
        q = ttsnn.bias_act(self.semantic.decode(codes), res=self.acoustic.decode(codes))
        h = self.pre_conv(q.half()[None])[0]  # causal k3, 512 -> 1024
        x = ttsnn.bias_act(proj_rows(self.pre_in, h), self.pre_in_b)
        t = self.tf(x)
        h = ttsnn.bias_act(proj_rows(self.pre_out, t), self.pre_out_b)
        latent = h[None]
        for up, nxt in self.upsample:
            latent = nxt(up(latent.half()))
        if trace:
            return q, h, latent
        return latent
