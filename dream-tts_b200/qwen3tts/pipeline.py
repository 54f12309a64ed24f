"""Text ids to audio on B200, the reference's `Talker::generate_batch` + `Codec::decode` path
(crates/qwen3tts/src/talker.rs:683-1073, codec.rs:544-604) with greedy picks: prompts built per
request, prefilled together (the prompts' rows as decode rows), then one graph replay per frame
for every live lane (talker step, code 0 under the pick rule, the depth predictor, the next
input), the codes read back each frame for the end code as the reference does, the finished
tail shed in quanta of 8, and each request's frames decoded by the codec in the reference's
chunks of 300 frames with 25 of left context.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .codec import chunk_plan, gather_windows
from .frames import CODEC_EOS, FrameLoop
from .prompt import TTS_PAD, PromptBuilder
from .talker import SHED_QUANTUM

# frames of the voice clip decoded ahead of the generated frames (cfg::codec::CHUNK_LEFT_CONTEXT)
CONTEXT_FRAMES = 25


@dataclass
class Request:
    text: list                       # BPE ids of the text to speak
    ref_text: list = field(default_factory=list)   # the voice asset's transcript ids (ICL)
    ref_codes: list = field(default_factory=list)  # its frames, [n][16]
    spk: torch.Tensor | None = None  # x-vector [dim]
    language: object = None          # None, a codec id, or a [dim] vector
    max_frames: int = 1200


class Synthesizer:
    def __init__(self, talker, predictor, prompt: PromptBuilder, pick, codec=None,
                 max_lanes: int = 48, capacity: int = 2048, block_size: int = 32):
        self.talker, self.predictor, self.prompt, self.pick = talker, predictor, prompt, pick
        self.codec = codec
        self.max_lanes, self.capacity, self.block_size = max_lanes, capacity, block_size

    def generate(self, requests: list[Request]) -> list[list[list[int]]]:
        """Frames [n][16] per request, in request order (groups of at most max_lanes lanes)."""
        out = []
        for g0 in range(0, len(requests), self.max_lanes):
            out += self._group(requests[g0:g0 + self.max_lanes])
        return out

    def _group(self, reqs: list[Request]) -> list[list[list[int]]]:
        dev = self.talker.device
        built = [self.prompt.build(r.text, r.ref_text, r.ref_codes, r.spk, r.language) for r in reqs]
        pad = self.prompt.text([TTS_PAD])[0]
        n = len(reqs)
        dim = self.talker.geo.dim
        tlen = max(b[1].shape[0] for b in built)
        rows = pad.expand(self.max_lanes, tlen, dim).clone()
        for i, (_, trailing, _) in enumerate(built):
            rows[i, :trailing.shape[0]] = trailing
        loop = FrameLoop(self.talker, self.predictor, self.max_lanes, self.capacity, self.pick,
                         rows, pad, self.block_size)
        # prompts: every lane's rows but the last prefilled together; the last is the first
        # frame's input (the talker step at that position, then the head)
        for i, ((prompt, _, _), r) in enumerate(zip(built, reqs)):
            need = prompt.shape[0] + r.max_frames + 2
            if need > self.capacity:
                raise ValueError(f"request {i} needs {need} positions, capacity {self.capacity}")
            loop.kv.admit(i, need, 0)
            loop.pick.reset(i)
            loop.feedback[i].copy_(prompt[-1])
        lens = [b[0].shape[0] - 1 for b in built]
        x = torch.cat([b[0][:-1] for b in built]).contiguous()
        if x.shape[0]:
            self.talker.prefill(loop.kv, lens, x, max_span=self.capacity)
        frames: list[list[list[int]]] = [[] for _ in range(n)]
        done = [False] * n
        live = n
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))  # the prefill and the lane setup
        with torch.cuda.stream(stream):
            for _ in range(max(r.max_frames for r in reqs)):
                loop.graph(live).replay()
                c0 = loop.code0[:live].cpu().tolist()
                rest = loop.codes[:live].cpu().tolist()
                for i in range(min(live, n)):
                    if done[i]:
                        continue
                    if c0[i] == CODEC_EOS:
                        done[i] = True
                        continue
                    frames[i].append([c0[i]] + rest[i])
                    if len(frames[i]) >= reqs[i].max_frames:
                        done[i] = True
                needed = n
                while needed > 0 and done[needed - 1]:
                    needed -= 1
                if needed == 0:
                    break
                live = min(live, -(-needed // SHED_QUANTUM) * SHED_QUANTUM)
        stream.synchronize()
        loop.graphs.clear()
        for i in range(n):
            loop.kv.release(i)
        return frames

    def decode(self, frames: list[list[int]], context: list[list[int]] | None = None) -> torch.Tensor:
        """Codec::decode (codec.rs:544-604): chunks of 300 frames with 25 of left context, the
        context's audio dropped; 1920 samples per frame. With `context` (the voice asset's
        ref_codes, which the talker continues), its last 25 frames are decoded ahead of
        `frames` and their audio dropped, as the engine does (engine.rs:1119-1135), so the
        first frames have their real history instead of a cold start."""
        if self.codec is None:
            raise ValueError("no codec")
        ctx = list(context[-CONTEXT_FRAMES:]) if context else []
        codes = torch.tensor(ctx + list(frames), dtype=torch.int32, device=self.talker.device)
        plan = chunk_plan(codes.shape[0])
        wins = gather_windows(codes, plan)
        pieces = []
        for i, w in enumerate(plan):
            wav = self.codec(wins[i, :w.hi - w.lo].contiguous())
            per = wav.shape[0] // (w.hi - w.lo)  # SAMPLES_PER_FRAME at the reference's rates
            pieces.append(wav[w.drop * per:(w.drop + w.end - w.start) * per])
        joined = torch.cat(pieces)
        per = joined.shape[0] // codes.shape[0]
        return joined[len(ctx) * per:]

    def decode_document(self, frames: list[list[list[int]]],
                        context: list[list[int]] | None = None) -> list[torch.Tensor]:
        """The engine's stage 2 (engine.rs:1107-1171): the codec once over every request's
        frames concatenated (each segment gets real history rather than a cold start), the
        voice's context ahead of them and dropped, then the audio cut at exact frame
        boundaries, one piece per request."""
        flat = [fr for f in frames for fr in f]
        wav = self.decode(flat, context)
        per = wav.shape[0] // max(len(flat), 1)
        out, o = [], 0
        for f in frames:
            out.append(wav[o:o + len(f) * per])
            o += len(f) * per
        return out
