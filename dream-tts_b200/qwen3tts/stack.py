"""The qwen3 decoder stack and its decode-time state on B200.

Mirrors crates/qwen3tts/src/qwen3.rs: `Geometry`, `Stack` (layer weights, final norm, RoPE
tables) and `State` (the KV cache and how many positions each lane holds). The cache is paged:
K and V pools of fixed-size pages shared by every lane of a group, a block table per lane, and
a position per lane, all device-resident, so lanes of different lengths step together and a
finished lane gives its pages back without touching the others (the reference's contiguous
per-batch cache can only narrow a finished tail, qwen3.rs:198-211).

The decode step itself runs in native code (libtts_cuda.so, tts_stack_decode_step); this
module owns the tensors and hands pointers across the C ABI.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

import ttsnn
from ttsnn import _lib as L
from ttsnn._ctx import ctx, ptr, stream


@dataclass
class Geometry:
    """Layer shape (crates/qwen3tts/src/qwen3.rs:15-39) plus the talker's codebook heads."""
    dim: int = 2048
    layers: int = 28
    heads: int = 16
    n_kv: int = 8
    head_dim: int = 128
    ffn: int = 6144
    eps: float = 1e-6
    rope_base: float = 1e6
    rope_len: int = 4096
    codebooks: int = 16
    vocab: int = 2048

    @property
    def gqa(self) -> int:
        return self.heads // self.n_kv

    def c_struct(self) -> L.StackGeometry:
        return L.StackGeometry(self.dim, self.layers, self.heads, self.n_kv, self.head_dim,
                               self.ffn, self.eps, self.rope_base, self.rope_len,
                               self.codebooks, self.vocab)


@dataclass
class LayerTensors:
    """One layer on the device, in the layout the kernels take (qwen3.rs:61-119 does the same
    folding at load: q/k/v concatenated, 1/sqrt(head_dim) folded into the q norm). Projection
    weights are packed (`ttsnn.pack_weight`); build from plain `[out, in]` tensors with
    `from_plain` or from checkpoint tensors with `load`."""
    attn_norm: torch.Tensor  # f32 [dim]
    ffn_norm: torch.Tensor   # f32 [dim]
    wqkv: torch.Tensor       # f16 [(heads + 2 n_kv) * hd, dim]
    qk_norms: torch.Tensor   # f32 [2, hd]
    wo: torch.Tensor         # f16 [dim, heads * hd]
    w_gate_up: torch.Tensor  # f16 [2 ffn, dim], tile-interleaved
    w_down: torch.Tensor     # f16 [dim, ffn]

    @classmethod
    def from_plain(cls, attn_norm, ffn_norm, wqkv, qk_norms, wo, w_gate_up, w_down) -> "LayerTensors":
        """From plain `[out, in]` f16 projections (gate/up already interleaved)."""
        return cls(attn_norm.to(torch.float32).contiguous(), ffn_norm.to(torch.float32).contiguous(),
                   ttsnn.pack_weight(wqkv), qk_norms.to(torch.float32).contiguous(),
                   ttsnn.pack_weight(wo), ttsnn.pack_weight(w_gate_up), ttsnn.pack_weight(w_down))

    @classmethod
    def load(cls, q_proj, k_proj, v_proj, o_proj, gate, up, down, attn_norm, ffn_norm, q_norm,
             k_norm, head_dim: int = 128) -> "LayerTensors":
        """From checkpoint-layout tensors ([out, in] projections), as Layer::load does."""
        dev = q_proj.device
        wqkv = torch.cat([q_proj, k_proj, v_proj], 0).to(torch.float16).contiguous()
        qn = q_norm.to(torch.float32) * (1.0 / head_dim ** 0.5)
        return cls.from_plain(attn_norm.to(dev), ffn_norm.to(dev), wqkv,
                              torch.stack([qn, k_norm.to(torch.float32)]).to(dev),
                              o_proj.to(torch.float16), ttsnn.interleave_gate_up(gate, up),
                              down.to(torch.float16))


class PagedKv:
    """KV pages for one group of lanes: pools f16 [layers][num_blocks][n_kv][block_size][128],
    block table int32 [lanes][max_blocks], positions int32 [lanes] (each lane's cached length).
    The buffers are torch tensors; the page bookkeeping (free list, per-lane pages, reference
    counts of shared prefix pages, table rows and positions) is the native pool's
    (tts_kv_pool_*), the same allocator a host engine binds through the C ABI. Admissions are
    ordered on the current stream."""

    def __init__(self, geo: Geometry, lanes: int, num_blocks: int, block_size: int,
                 max_blocks: int, device: torch.device | str = "cuda"):
        self.geo = geo
        self.lanes = lanes
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.max_blocks = max_blocks
        shape = (geo.layers, num_blocks, geo.n_kv, block_size, geo.head_dim)
        self.k = torch.zeros(shape, dtype=torch.float16, device=device)
        self.v = torch.zeros(shape, dtype=torch.float16, device=device)
        self.table = torch.zeros(lanes, max_blocks, dtype=torch.int32, device=device)
        self.positions = torch.zeros(lanes, dtype=torch.int32, device=device)
        desc = L.KvPoolDesc(geo.layers, geo.n_kv, geo.head_dim, block_size, num_blocks, lanes,
                            max_blocks, self.k.data_ptr(), self.v.data_ptr(),
                            self.table.data_ptr(), self.positions.data_ptr())
        h = C.c_void_p()
        dev = self.k.device.index if self.k.device.index is not None else torch.cuda.current_device()
        L.call("tts_kv_pool_create", ctx(dev), C.byref(desc), C.byref(h))
        self.handle = h

    def admit(self, lane: int, capacity: int, length: int = 0) -> list[int]:
        """Give `lane` pages for `capacity` positions; it holds `length` of them already."""
        L.call("tts_kv_pool_admit", self.handle, int(lane), int(capacity), int(length), stream())
        return self.pages(lane)

    def admit_pages(self, lane: int, pages, length: int = 0) -> None:
        """Admit `lane` with the given free pages (block-table order)."""
        arr = (C.c_int * len(pages))(*[int(p) for p in pages])
        L.call("tts_kv_pool_admit_pages", self.handle, int(lane), arr, len(pages), int(length),
               stream())

    def share_prefix(self, src: int, lane: int, length: int, capacity: int) -> list[int]:
        """Admit `lane` with the first `length` cached positions of lane `src` (the shared
        prompt prefix every lane of a group starts from, which the reference broadcast-copies
        into each lane, crates/qwen3tts/src/qwen3.rs:261-284): its full pages are shared
        through the block table, only a partly filled last page is copied, and fresh pages
        cover the rest of `capacity`. `src` must hold at least `length` positions."""
        L.call("tts_kv_pool_share_prefix", self.handle, int(src), int(lane), int(length),
               int(capacity), stream())
        return self.pages(lane)

    def release(self, lane: int) -> None:
        L.call("tts_kv_pool_release", self.handle, int(lane))

    def pages(self, lane: int) -> list[int]:
        n = C.c_int(0)
        buf = (C.c_int * self.max_blocks)()
        L.call("tts_kv_pool_lane_pages", self.handle, int(lane), buf, self.max_blocks, C.byref(n))
        return list(buf[:n.value])

    def page_refs(self, page: int) -> int:
        return int(L.load().tts_kv_pool_page_refs(self.handle, int(page)))

    def free_pages(self) -> int:
        return int(L.load().tts_kv_pool_free_pages(self.handle))

    def state(self, lanes: int | None = None, max_span: int | None = None) -> L.DecodeState:
        n = self.lanes if lanes is None else lanes
        ms = max_span if max_span is not None else self.max_blocks * self.block_size
        return L.DecodeState(n, self.positions.data_ptr(), self.table.data_ptr(),
                             self.max_blocks, self.block_size, self.num_blocks,
                             self.k.data_ptr(), self.v.data_ptr(), ms)

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                L.load().tts_kv_pool_destroy(self.handle)
                self.handle = None
        except Exception:
            pass


class PickState:
    """The talker's greedy pick rule on the device (talker.rs:154-189, 940, 971-981): `banned`
    ids never picked, `eos` banned while a lane has fewer than `min_new` frames, and each id's
    logit divided (positive) or multiplied (negative) by `penalty` once per time the lane has
    emitted it. The per-id emission counts u16 [lanes, vocab] (held as int16) and frame counts
    int32 [lanes] live on the device and are updated by every step; `reset(lane)` clears a lane
    slot for a new segment."""

    def __init__(self, vocab: int, lanes: int, banned, eos: int = -1, min_new: int = 0,
                 penalty: float = 1.0, device: torch.device | str = "cuda"):
        import numpy as np
        if vocab % 32:
            raise ValueError("vocab must be a multiple of 32")
        words = vocab // 32
        bits = np.zeros(words, np.uint32)
        for i in banned:
            bits[int(i) >> 5] |= np.uint32(1 << (int(i) & 31))
        self.vocab, self.eos, self.min_new, self.penalty = vocab, eos, min_new, penalty
        self.ban = torch.from_numpy(bits.view(np.int32)).to(device)
        self.counts = torch.zeros(lanes, vocab, dtype=torch.int16, device=device)
        self.frames = torch.zeros(lanes, dtype=torch.int32, device=device)
        self.c = L.PickRule(self.ban.data_ptr(), self.counts.data_ptr(), self.frames.data_ptr(),
                            float(penalty), int(eos), int(min_new))

    def reset(self, lane: int) -> None:
        self.counts[lane].zero_()
        self.frames[lane] = 0

    def history(self, lane: int) -> dict[int, int]:
        """The lane's emitted ids and how often each was emitted (the reference's `seen` list
        as a multiset)."""
        c = self.counts[lane].to(torch.int32) & 0xFFFF
        nz = torch.nonzero(c).flatten().tolist()
        return {int(i): int(c[i]) for i in nz}


class Graph:
    """A captured decode step, replayed with `replay()` (one tts_graph_launch)."""

    def __init__(self, handle: C.c_void_p, keep: list):
        self.handle = handle
        self._keep = keep

    def replay(self) -> None:
        L.call("tts_graph_launch", self.handle, stream())

    def __del__(self):
        try:
            if self.handle:
                L.load().tts_graph_destroy(self.handle)
                self.handle = None
        except Exception:
            pass


class Stack:
    """`Stack` of crates/qwen3tts/src/qwen3.rs:214-467 with the talker's heads, on B200."""

    def __init__(self, geo: Geometry, layers: list[LayerTensors], final_norm: torch.Tensor,
                 heads: torch.Tensor | None = None, embed: torch.Tensor | None = None):
        if len(layers) != geo.layers:
            raise ValueError(f"{len(layers)} layers for geometry with {geo.layers}")
        self.geo = geo
        self.layers = layers
        self.device = layers[0].wqkv.device
        self.final_norm = final_norm.to(self.device, torch.float32).contiguous()
        # heads `[codebooks * vocab, dim]` plain; packed here for the GEMM
        self.heads = None if heads is None else ttsnn.pack_weight(heads)
        self.embed = None if embed is None else embed.to(torch.float16).contiguous()
        self._ctx = ctx(self.device.index)
        h = C.c_void_p()
        g = geo.c_struct()
        L.call("tts_stack_create", self._ctx, C.byref(g), C.byref(h))
        self.handle = h
        for i, lt in enumerate(layers):
            w = L.LayerWeights(lt.attn_norm.data_ptr(), lt.ffn_norm.data_ptr(),
                               lt.wqkv.data_ptr(), lt.qk_norms.data_ptr(), lt.wo.data_ptr(),
                               lt.w_gate_up.data_ptr(), lt.w_down.data_ptr())
            L.call("tts_stack_set_layer", h, i, C.byref(w))
        L.call("tts_stack_set_head", h, ptr(self.final_norm), ptr(self.heads), ptr(self.embed))

    def set_pick(self, pick: "PickState | None") -> None:
        """Use the talker's pick rule for the codec head (one codebook); None: plain argmax."""
        self._pick = pick
        L.call("tts_stack_set_pick", self.handle, None if pick is None else C.byref(pick.c))

    def set_feedback(self, x_next: torch.Tensor | None) -> None:
        """Use `x_next` ([lanes, dim] f32, caller-owned) as the step's feedback input buffer."""
        self._feedback = x_next
        L.call("tts_stack_set_feedback", self.handle, ptr(x_next))

    def weight_bytes(self) -> int:
        n = 0
        for lt in self.layers:
            n += sum(t.numel() * t.element_size() for t in
                     (lt.wqkv, lt.wo, lt.w_gate_up, lt.w_down))
        if self.heads is not None:
            n += self.heads.numel() * 2
        return n

    def prefill(self, kv: PagedKv, lens, x: torch.Tensor, h_out: torch.Tensor | None = None,
                max_span: int | None = None) -> None:
        """Stack::forward at t > 1: lane i (of the first len(lens)) appends lens[i] rows of `x`
        (f32 [sum(lens), dim], lane after lane) at its next positions, causal over its cached
        and new rows; `h_out` (f32 [sum(lens), dim]) gets every row's final-normed hidden."""
        import numpy as np
        arr = np.ascontiguousarray(np.asarray(lens, dtype=np.int32))
        st = kv.state(len(arr), max_span)
        L.call("tts_stack_prefill", self.handle, C.byref(st),
               arr.ctypes.data_as(C.c_void_p), ptr(x), ptr(h_out), stream())

    def decode_step(self, kv: PagedKv, x: torch.Tensor | None = None, lanes: int | None = None,
                    h_out: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                    codes: torch.Tensor | None = None, max_span: int | None = None) -> None:
        """One step for `lanes` lanes (default all): writes each lane's K/V at its position,
        advances the positions, and fills the optional outputs."""
        st = kv.state(lanes, max_span)
        L.call("tts_stack_decode_step", self.handle, C.byref(st), ptr(x), ptr(h_out),
               ptr(logits), ptr(codes), stream())

    def capture(self, kv: PagedKv, x: torch.Tensor | None = None, lanes: int | None = None,
                h_out: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                codes: torch.Tensor | None = None, max_span: int | None = None) -> Graph:
        """The same step as a CUDA graph on the current (non-default) stream."""
        st = kv.state(lanes, max_span)
        g = C.c_void_p()
        L.call("tts_stack_graph_capture", self.handle, C.byref(st), ptr(x), ptr(h_out),
               ptr(logits), ptr(codes), stream(), C.byref(g))
        return Graph(g, [kv, x, h_out, logits, codes])

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                L.load().tts_stack_destroy(self.handle)
                self.handle = None
        except Exception:
            pass
