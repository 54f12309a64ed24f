"""Talker::generate_batch's decode loop on B200, greedy (crates/qwen3tts/src/talker.rs:903-1073).

One frame per lane per call: the talker's decode step with its codec head (3072 ids) under the
reference's pick rule (the top 1024 ids banned except the end code, the end code banned for the
first MIN_NEW_TOKENS frames, repetition penalty 1.05 on each lane's emitted codes), code 0's
codec_embed row, the depth predictor's 15 residual codes and their embedding sum, and the lane's
trailing text row (or the tts_pad row) added as the next step's input. The whole frame is one
native call (tts_talker_frame) or one CUDA graph per live width.

The loop starts from each lane's last prompt position: its input row sits in the feedback
buffer and its earlier positions in the KV pages (the causal mask makes that the reference's
prefill followed by its first head).
"""
from __future__ import annotations

import ctypes as C

import torch

from ttsnn import _lib as L
from ttsnn._ctx import ptr, stream

from .predictor import Predictor, TextFeed
from .stack import Graph, PagedKv, PickState, Stack

# crates/qwen3tts/src/cfg.rs (talker): vocabulary, end code, first frames without it, penalty
VOCAB = 3072
CODEC_EOS = 2150
MIN_NEW_TOKENS = 2
REPETITION_PENALTY = 1.05
BANNED_TOP = 1024


def reference_pick(vocab: int = VOCAB, lanes: int = 48, eos: int = CODEC_EOS,
                   min_new: int = MIN_NEW_TOKENS, penalty: float = REPETITION_PENALTY,
                   banned_top: int = BANNED_TOP, device="cuda") -> PickState:
    """The talker's rule (talker.rs:940): the top `banned_top` ids banned except eos."""
    banned = [i for i in range(vocab - banned_top, vocab) if i != eos]
    return PickState(vocab, lanes, banned, eos, min_new, penalty, device)


class FrameLoop:
    """The talker stack (one codebook head: codec_head, its table: codec_embed) and the depth
    predictor driven together, a frame per call, for up to `max_lanes` lanes."""

    def __init__(self, talker: Stack, predictor: Predictor, max_lanes: int, capacity: int,
                 pick: PickState, text_rows: torch.Tensor, pad: torch.Tensor,
                 block_size: int = 32):
        g = talker.geo
        if g.codebooks != 1 or talker.heads is None or talker.embed is None:
            raise ValueError("the talker needs one codebook head and its embedding table")
        dev = talker.device
        self.talker, self.predictor = talker, predictor
        self.max_lanes, self.capacity = max_lanes, capacity
        per_lane = -(-capacity // block_size)
        self.kv = PagedKv(g, max_lanes, max_lanes * per_lane, block_size, per_lane, dev)
        self.pkv = predictor.new_state(max_lanes)
        self.pick = pick
        talker.set_pick(pick)
        self.feedback = torch.zeros(max_lanes, g.dim, device=dev)
        talker.set_feedback(self.feedback)
        self.hidden = torch.zeros(max_lanes, g.dim, device=dev)
        self.code0 = torch.zeros(max_lanes, dtype=torch.int32, device=dev)
        self.codes = torch.zeros(max_lanes, predictor.steps, dtype=torch.int32, device=dev)
        self.text = TextFeed(text_rows, pad, pick.frames)
        self.graphs: dict[int, Graph] = {}

    def admit(self, lane: int, prompt_len: int, frames: int, first_input: torch.Tensor) -> None:
        """A segment in lane slot `lane`: `prompt_len - 1` cached positions (the prompt's K/V are
        the caller's), its last prompt row as the first input, room for `frames` frames."""
        self.kv.admit(lane, prompt_len + frames + 1, prompt_len - 1)
        self.pick.reset(lane)
        self.feedback[lane].copy_(first_input)

    def _states(self, lanes: int):
        return (self.kv.state(lanes, self.capacity),
                self.pkv.state(lanes, self.predictor.steps + 1))

    def frame(self, lanes: int) -> None:
        """One frame for lanes [0, lanes): code0 int32 [lanes], codes int32 [lanes, 15]."""
        ts, ps = self._states(lanes)
        L.call("tts_talker_frame", self.talker.handle, C.byref(ts), self.predictor.handle,
               C.byref(ps), C.byref(self.text.c), ptr(self.hidden), ptr(self.code0),
               ptr(self.codes), stream())

    def graph(self, lanes: int) -> Graph:
        """The frame at width `lanes` as a CUDA graph (captured on first use, current stream)."""
        g = self.graphs.get(lanes)
        if g is None:
            ts, ps = self._states(lanes)
            h = C.c_void_p()
            L.call("tts_talker_frame_capture", self.talker.handle, C.byref(ts),
                   self.predictor.handle, C.byref(ps), C.byref(self.text.c), ptr(self.hidden),
                   ptr(self.code0), ptr(self.codes), stream(), C.byref(h))
            g = Graph(h, [self.kv, self.pkv, self.text])
            self.graphs[lanes] = g
        return g
