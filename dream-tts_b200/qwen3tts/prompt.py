"""The talker's prompt (crates/qwen3tts/src/talker.rs:607-786): the text projection of token ids
and the assembly of the prefill sequence and the trailing text rows, as
`Talker::build_prompt_shared` does. Tokenisation is the caller's (ids in, as the reference's
Talker takes them). Rows are f32 [n, dim] on the device; assembly is a handful of row
concatenations and sums on small tensors at segment start.
"""
from __future__ import annotations

import torch

import ttsnn

from .codec_front import proj_rows

# crates/qwen3tts/src/cfg.rs (talker): special ids of the codec and text vocabularies
CODEC_PAD, CODEC_BOS, CODEC_EOS = 2148, 2149, 2150
CODEC_THINK, CODEC_NOTHINK, CODEC_THINK_BOS, CODEC_THINK_EOS = 2154, 2155, 2156, 2157
TTS_PAD, TTS_BOS, TTS_EOS = 151_671, 151_672, 151_673
IM_START, ASSISTANT, NEWLINE = 151_644, 77_091, 198


class TextProjection:
    """`text_projection` (talker.rs:607-616): text_embedding rows (read from the host as asked,
    `rows(ids)` -> [n, text_dim]) through linear_fc1 + SiLU + linear_fc2, both with bias."""

    def __init__(self, rows, fc1_w, fc1_b, fc2_w, fc2_b, device="cuda"):
        self.rows, self.device = rows, device
        self.fc1, self.fc1_b = ttsnn.Proj(fc1_w.to(device)), fc1_b.to(device).float().contiguous()
        self.fc2, self.fc2_b = ttsnn.Proj(fc2_w.to(device)), fc2_b.to(device).float().contiguous()

    def __call__(self, ids) -> torch.Tensor:
        e = self.rows(list(ids)).to(self.device).float().contiguous()
        h = ttsnn.bias_act(proj_rows(self.fc1, e), self.fc1_b, silu=True)
        return ttsnn.bias_act(proj_rows(self.fc2, h), self.fc2_b)


class PromptBuilder:
    """`build_prompt_shared` (talker.rs:683-786) over the talker's codec_embed [vocab, dim] and
    the predictor's residual tables [15, 2048, dim] (frame_embed, talker.rs:653-659)."""

    def __init__(self, text: TextProjection, codec_embed: torch.Tensor, tables: torch.Tensor):
        self.text = text
        self.codec_embed = codec_embed.float()
        self.tables = tables

    def codec_row(self, i: int) -> torch.Tensor:
        return self.codec_embed[i:i + 1]

    def frame_embed(self, codes) -> torch.Tensor:
        """codec_embed[code 0] + the sum of the residual codes' table rows (gather_sum)."""
        if len(codes) != 16:
            raise ValueError(f"expected 16 codes, got {len(codes)}")
        acc = torch.zeros_like(self.codec_embed[:1])
        for i, c in enumerate(codes[1:]):
            acc = acc + self.tables[i, int(c)].float()[None]
        return self.codec_row(int(codes[0])) + acc

    def build(self, text, ref_text=(), ref_codes=(), spk: torch.Tensor | None = None,
              language=None):
        """-> (prompt [L, dim], trailing [n, dim], shared positions). `language`: None (auto),
        a codec id (a tag), or a [dim] vector."""
        pad = self.text([TTS_PAD])
        bos = self.text([TTS_BOS])
        eos = self.text([TTS_EOS])
        codec = []
        if language is None:
            codec += [self.codec_row(CODEC_NOTHINK), self.codec_row(CODEC_THINK_BOS)]
        else:
            row = (self.codec_row(int(language)) if isinstance(language, int)
                   else language.reshape(1, -1).float().to(self.codec_embed.device))
            codec += [self.codec_row(CODEC_THINK), self.codec_row(CODEC_THINK_BOS), row]
        codec.append(self.codec_row(CODEC_THINK_EOS))
        if spk is not None:
            codec.append(spk.reshape(1, -1).float().to(self.codec_embed.device))
        codec += [self.codec_row(CODEC_PAD), self.codec_row(CODEC_BOS)]
        codec = torch.cat(codec)
        n = codec.shape[0]
        text_side = torch.cat([pad] * (n - 2) + [bos])
        prefix = text_side + codec[:n - 1]
        role = self.text([IM_START, ASSISTANT, NEWLINE])
        shared = role.shape[0] + prefix.shape[0]
        parts = [role, prefix]
        if len(ref_codes) and len(ref_text):
            # in-context: ref transcript + text + eos summed with codec_bos + the ref frames
            text_embed = torch.cat([self.text(list(ref_text) + list(text)), eos])
            codec_embed = torch.cat([self.codec_row(CODEC_BOS)] +
                                    [self.frame_embed(f) for f in ref_codes])
            tl, cl = text_embed.shape[0], codec_embed.shape[0]
            shared += min(len(ref_text), cl)
            if tl > cl:
                parts.append(text_embed[:cl] + codec_embed)
                trailing = text_embed[cl:]
            else:
                parts.append(torch.cat([text_embed] + [pad] * (cl - tl)) + codec_embed)
                trailing = pad
        else:
            if not len(text):
                raise ValueError("no text to speak")
            parts.append(self.text(list(text[:1])) + codec[n - 1:])
            trailing = torch.cat([self.text(list(text[1:])), eos]) if len(text) > 1 else eos
        return torch.cat(parts).contiguous(), trailing.contiguous(), shared
