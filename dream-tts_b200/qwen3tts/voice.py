"""Voice assets: `voices/<name>/voice.json` + `voice.safetensors` (crates/tts-core/src/voice.rs:
34-140), read through the native safetensors reader, and the request a qwen3tts synthesis builds
from one (crates/qwen3tts/src/engine.rs:714-736): the speaker x-vector `spk_embedding` [1, dim]
f32, the reference clip's frames `ref_codes` [T, 16] and its transcript's ids `ref_text_tokens`
[1, N]. Tensors stay on the host, as the reference keeps them (voice.rs:67-79); the engine moves
the x-vector to the device.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch

from .pipeline import Request
from .weights import Weights


class VoiceError(ValueError):
    pass


@dataclass
class Voice:
    engine: str
    name: str
    text: str = ""
    seconds: float | None = None
    language: str | None = None
    tensors: dict = field(default_factory=dict)

    @classmethod
    def load(cls, path: str) -> "Voice":
        """Voice::load (voice.rs:77-98): the manifest, then every tensor of voice.safetensors
        onto the host."""
        manifest_path = os.path.join(path, "voice.json")
        try:
            with open(manifest_path) as f:
                m = json.load(f)
        except (OSError, json.JSONDecodeError) as e:
            raise VoiceError(f"reading {manifest_path}: {e}") from e
        for key in ("engine", "name"):
            if key not in m:
                raise VoiceError(f"parsing {manifest_path}: missing field `{key}`")
        w = Weights(os.path.join(path, "voice.safetensors"))
        try:
            tensors = {n: w.cpu(n) for n in w.names()}
        finally:
            w.close()
        return cls(engine=m["engine"], name=m["name"], text=m.get("text", "") or "",
                   seconds=m.get("seconds"), language=m.get("language"), tensors=tensors)

    def keys(self) -> list[str]:
        return sorted(self.tensors)

    def get(self, name: str) -> torch.Tensor:
        """Voice::get (voice.rs:100-109), with the reference's error naming what is there."""
        if name not in self.tensors:
            raise VoiceError(f"voice `{self.name}` (engine {self.engine}) has no tensor `{name}`; "
                             f"it has: {', '.join(self.keys())}")
        return self.tensors[name]

    def get_rows_u32(self, name: str) -> list[list[int]]:
        """Voice::get_rows_u32 (voice.rs:122-140): a 2-D tensor as rows of u32."""
        t = self.get(name)
        if t.dim() != 2:
            raise VoiceError(f"tensor `{name}` in voice `{self.name}` is not 2-D")
        return (t.to(torch.int64) & 0xFFFFFFFF).tolist()

    def speaker(self, dim: int, device="cuda") -> torch.Tensor:
        """Talker::speaker (crates/qwen3tts/src/talker.rs:1162-1169): the x-vector as f32 on the
        device, refused when its width is not the talker's."""
        t = self.get("spk_embedding").to(torch.float32)
        if t.numel() != dim:
            raise VoiceError(f"x-vector is {t.numel()}-wide, expected {dim} — 0.6B asset?")
        return t.reshape(dim).to(device)

    def request(self, text: list, dim: int, xvector_only: bool = False, language=None,
                max_frames: int = 1200, device="cuda") -> Request:
        """The synthesis request for `text` in this voice (engine.rs:714-736): the x-vector,
        and unless `xvector_only` (the engine's clone=xvector), the clip's frames and its
        transcript's ids for the in-context prompt. A voice without `ref_codes` or
        `ref_text_tokens` speaks by its x-vector alone, as the reference's unwrap_or_default
        leaves it."""
        spk = self.speaker(dim, device)
        codes = self.get_rows_u32("ref_codes") if "ref_codes" in self.tensors else []
        ref_text = (self.get_rows_u32("ref_text_tokens")[0]
                    if "ref_text_tokens" in self.tensors else [])
        if xvector_only:
            codes, ref_text = [], []
        return Request(list(text), ref_text=ref_text, ref_codes=codes, spk=spk,
                       language=language, max_frames=max_frames)
