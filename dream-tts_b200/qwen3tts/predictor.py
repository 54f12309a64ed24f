"""The talker's depth predictor on B200 (crates/qwen3tts/src/talker.rs:255-550).

Per talker frame it picks the 15 residual codes: the talker's hidden state and its code-0
embedding, projected to the predictor's width, prefill a 5-layer decoder stack of its own; then
per residual codebook i the stack's last hidden goes through head i, the greedy pick's row of
`resized[i]` (the codebook table already projected, talker.rs:268-273) is the next input, and
the frame ends with the sum of the picked codes' table rows at talker width plus the code-0
embedding (gather_sum, talker.rs:528-550), the talker's next input.

The whole frame is one native call (tts_predictor_frame) or one CUDA graph: the two-position
prefill runs as one stack step over paired rows sharing a lane's page, and each depth step is a
stack step whose heads are head i and whose feedback is a row of resized[i].
"""
from __future__ import annotations

import ctypes as C

import torch

import ttsnn
from ttsnn import _lib as L
from ttsnn._ctx import ptr, stream

from .stack import Geometry, Graph, PagedKv, Stack

# crates/qwen3tts/src/cfg.rs: the predictor's shape (dim 1024, 5 layers, 16 q / 8 kv heads of
# 128, ffn 3072, 15 residual codebooks of 2048 ids, talker width 2048, RoPE base 1e6)
PREDICTOR_GEOMETRY = Geometry(dim=1024, layers=5, heads=16, n_kv=8, head_dim=128, ffn=3072,
                              eps=1e-6, rope_base=1e6, rope_len=64, codebooks=1, vocab=2048)
STEPS = 15
EMBED_DIM = 2048


def resize_tables(tables: torch.Tensor, resize: torch.Tensor,
                  bias: torch.Tensor | None) -> torch.Tensor:
    """`resized[i] = tables[i] @ resize^T + bias` in f32 (talker.rs:315-323), computed once at
    load (in f64 here, rounded to f32)."""
    w = resize.to(torch.float64)
    out = tables.to(torch.float64) @ w.T
    if bias is not None:
        out = out + bias.to(torch.float64)
    return out.to(torch.float32).contiguous()


class TextFeed:
    """Each lane's trailing text embeddings f32 [lanes, len, dim] and the pad row f32 [dim]
    (talker.rs:933-937, 1043-1048); `frames` int32 [lanes] on the device counts each lane's
    frames (the pick rule's counter): a frame adds row frames - 1, or the pad row past the end."""

    def __init__(self, rows: torch.Tensor, pad: torch.Tensor, frames: torch.Tensor):
        self.rows = rows.to(torch.float32).contiguous()
        self.pad = pad.to(torch.float32).contiguous()
        self.frames = frames
        self.c = L.TextFeed(self.rows.data_ptr(), self.rows.shape[1], self.pad.data_ptr(),
                            frames.data_ptr())


def _feed(text: "TextFeed | None"):
    return None if text is None else C.byref(text.c)


class Predictor:
    """`Predictor` of talker.rs:255-330 over a `Stack` created with codebooks = 1 and vocab =
    the residual codebook size (its heads unset: the predictor supplies one per depth step)."""

    def __init__(self, stack: Stack, resize: torch.Tensor, resize_bias: torch.Tensor | None,
                 heads: torch.Tensor, tables: torch.Tensor, resized: torch.Tensor | None = None):
        g = stack.geo
        if g.codebooks != 1:
            raise ValueError("the predictor's stack needs codebooks = 1")
        self.stack = stack
        self.steps, vocab, self.embed_dim = tables.shape
        if vocab != g.vocab or heads.shape != (self.steps * vocab, g.dim):
            raise ValueError("heads must be [steps * vocab, dim] and tables [steps, vocab, embed]")
        dev = stack.device
        self.resize = resize.to(dev, torch.float16).contiguous()
        self.resize_bias = (None if resize_bias is None
                            else resize_bias.to(dev, torch.float32).contiguous())
        self.heads = ttsnn.pack_weight(heads.to(dev, torch.float16).contiguous())
        self.tables = tables.to(dev, torch.float16).contiguous()
        self.resized = (resize_tables(self.tables, self.resize, self.resize_bias)
                        if resized is None else resized.to(dev, torch.float32).contiguous())
        w = L.PredictorWeights(self.resize.data_ptr(), ptr(self.resize_bias),
                               self.heads.data_ptr(), self.resized.data_ptr(),
                               self.tables.data_ptr(), self.steps, self.embed_dim)
        h = C.c_void_p()
        L.call("tts_predictor_create", stack.handle, C.byref(w), C.byref(h))
        self.handle = h

    def set_sampling(self, draws: torch.Tensor | None, top_k: int = 50,
                     temperature: float = 0.9) -> None:
        """Top-k sampling of the depth picks with draws f32 [steps, lanes] (refilled by the
        caller before each frame; step-major as the reference draws them), or greedy (None).
        The defaults are the reference's sub-talker settings (cfg.rs: top_k 50, temperature
        0.9, top_p 1)."""
        self._draws = draws
        if draws is None:
            L.call("tts_predictor_set_sampling", self.handle, None, 0, 0, 0.0)
            return
        if draws.dtype != torch.float32 or not draws.is_contiguous() or draws.shape[0] != self.steps:
            raise ValueError("draws must be contiguous f32 [steps, lanes]")
        L.call("tts_predictor_set_sampling", self.handle, ptr(draws), draws.shape[1], int(top_k),
               float(temperature))

    def new_state(self, lanes: int, block_size: int = 16) -> PagedKv:
        """KV pages for `lanes` lanes of one frame: steps + 1 positions each, one page per lane
        (the reference's `new_state(b)` with capacity CODE_GROUPS + 2, talker.rs:291-298)."""
        per_lane = -(-(self.steps + 1) // block_size)
        kv = PagedKv(self.stack.geo, lanes, lanes * per_lane, block_size, per_lane,
                     device=self.stack.device)
        for lane in range(lanes):
            kv.admit(lane, self.steps + 1)
        return kv

    def frame(self, kv: PagedKv, hidden: torch.Tensor, code0_embed: torch.Tensor,
              codes: torch.Tensor | None = None, total: torch.Tensor | None = None,
              text: "TextFeed | None" = None):
        """One frame for kv.lanes lanes: hidden, code0_embed f32 [lanes, embed_dim] -> codes
        int32 [lanes, steps] and the talker's next-input sum f32 [lanes, embed_dim] (plus each
        lane's text row when `text` is given)."""
        n = hidden.shape[0]
        if codes is None:
            codes = torch.empty(n, self.steps, dtype=torch.int32, device=hidden.device)
        if total is None:
            total = torch.empty(n, self.embed_dim, dtype=torch.float32, device=hidden.device)
        st = kv.state(n, self.steps + 1)
        L.call("tts_predictor_frame", self.handle, C.byref(st), ptr(hidden), ptr(code0_embed),
               _feed(text), ptr(codes), ptr(total), stream())
        return codes, total

    def capture(self, kv: PagedKv, hidden: torch.Tensor, code0_embed: torch.Tensor,
                codes: torch.Tensor, total: torch.Tensor, text: "TextFeed | None" = None) -> Graph:
        """The frame as one CUDA graph on the current (non-default) stream."""
        st = kv.state(hidden.shape[0], self.steps + 1)
        g = C.c_void_p()
        L.call("tts_predictor_graph_capture", self.handle, C.byref(st), ptr(hidden),
               ptr(code0_embed), _feed(text), ptr(codes), ptr(total), stream(), C.byref(g))
        return Graph(g, [kv, hidden, code0_embed, codes, total, text])

    def weight_bytes(self) -> int:
        """Bytes a frame streams from HBM for weights: the stack and one head per depth step
        (each step reads the whole stack once)."""
        return (self.stack.weight_bytes() * self.steps
                + self.heads.numel() * 2 + self.resize.numel() * 2 * 2)

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                L.load().tts_predictor_destroy(self.handle)
                self.handle = None
        except Exception:
            pass
