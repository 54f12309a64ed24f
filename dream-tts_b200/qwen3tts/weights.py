"""Checkpoint loading (crates/tts-nn/src/lib.rs:153-373; crates/qwen3tts/src/qwen3.rs:61-119,
229-250; talker.rs:276-330, 575-605): a memory-mapped safetensors file read by the native
reader, and the load-time work that turns checkpoint tensors into the device layouts the
kernels take (q/k/v concatenated, 1/sqrt(head_dim) folded into the q norm, gate/up tile
interleave, weight packing, weight-norm folds, the predictor's resized tables).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ttsnn import _lib as L

from .predictor import PREDICTOR_GEOMETRY, Predictor
from .stack import Geometry, LayerTensors, Stack

# crates/qwen3tts/src/cfg.rs (talker): the talker stack's shape, its codec vocabulary
TALKER_GEOMETRY = Geometry(dim=2048, layers=28, heads=16, n_kv=8, head_dim=128, ffn=6144,
                           eps=1e-6, rope_base=1e6, rope_len=4096, codebooks=1, vocab=3072)

_NP = {L_dt: t for L_dt, t in ((0, np.float32), (1, np.float16), (3, np.int32), (4, np.int64),
                               (5, np.uint8), (6, np.float64), (7, np.int8), (8, np.int16),
                               (9, np.bool_))}


class Weights:
    """A safetensors checkpoint, memory-mapped (the reference's `Weights`). `cpu(name)` is the
    tensor on the host in its on-disk dtype (a copy of the mapped bytes), `get(name)` the same
    as f32 on a device."""

    def __init__(self, path: str):
        lib = L.load()
        h = C.c_void_p()
        L.call("tts_safetensors_open", path.encode(), C.byref(h))
        self.handle = h
        self.path = path
        n = lib.tts_safetensors_count(h)
        v = L.TensorView()
        self._names = []
        for i in range(n):
            L.call("tts_safetensors_at", h, i, C.byref(v))
            self._names.append(v.name.decode())

    def names(self) -> list[str]:
        return list(self._names)

    def has(self, name: str) -> bool:
        v = L.TensorView()
        return L.load().tts_safetensors_find(self.handle, name.encode(), C.byref(v)) == 0

    def __len__(self) -> int:
        return len(self._names)

    def cpu(self, name: str) -> torch.Tensor:
        v = L.TensorView()
        L.call("tts_safetensors_find", self.handle, name.encode(), C.byref(v))
        shape = tuple(int(v.shape[d]) for d in range(v.ndim))
        raw = np.ctypeslib.as_array((C.c_uint8 * v.nbytes).from_address(v.data)) if v.nbytes else \
            np.zeros(0, np.uint8)
        if v.dtype == 2:  # bf16: the bits as int16, reinterpreted
            t = torch.from_numpy(raw.copy().view(np.int16)).view(torch.bfloat16)
        elif v.dtype in _NP:
            t = torch.from_numpy(raw.copy().view(_NP[v.dtype]))
        else:
            raise L.TtsError(2, f"{name}: unsupported dtype")
        return t.reshape(shape)

    def get(self, name: str, device="cuda", dtype=torch.float32) -> torch.Tensor:
        return self.cpu(name).to(dtype).to(device)

    def weight_norm(self, prefix: str, device="cuda") -> torch.Tensor:
        """`get_weight_norm` (lib.rs:323-331, 367-373): `{prefix}.weight` if present, else
        g * v / |v| (norm over everything but the output dim) from the parametrization."""
        if self.has(f"{prefix}.weight"):
            return self.get(f"{prefix}.weight", device)
        g = self.cpu(f"{prefix}.parametrizations.weight.original0").to(torch.float32)
        v = self.cpu(f"{prefix}.parametrizations.weight.original1").to(torch.float32)
        flat = v.reshape(v.shape[0], -1)
        w = flat * (g.reshape(-1, 1) / flat.pow(2).sum(1, keepdim=True).sqrt())
        return w.reshape(v.shape).to(device)

    def close(self) -> None:
        if getattr(self, "handle", None):
            L.load().tts_safetensors_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load_layer(w: Weights, prefix: str, geo: Geometry, device) -> LayerTensors:
    """`Layer::load` (qwen3.rs:61-119): q/k/v concatenated on the host, the q norm scaled by
    1/sqrt(head_dim), f16 projections packed for the kernels."""
    a = f"{prefix}.self_attn"
    return LayerTensors.load(
        w.cpu(f"{a}.q_proj.weight").to(device), w.cpu(f"{a}.k_proj.weight").to(device),
        w.cpu(f"{a}.v_proj.weight").to(device), w.cpu(f"{a}.o_proj.weight").to(device),
        w.cpu(f"{prefix}.mlp.gate_proj.weight").to(device),
        w.cpu(f"{prefix}.mlp.up_proj.weight").to(device),
        w.cpu(f"{prefix}.mlp.down_proj.weight").to(device),
        w.get(f"{prefix}.input_layernorm.weight", device),
        w.get(f"{prefix}.post_attention_layernorm.weight", device),
        w.get(f"{a}.q_norm.weight", device), w.get(f"{a}.k_norm.weight", device),
        head_dim=geo.head_dim)


def load_stack(w: Weights, prefix: str, geo: Geometry, device="cuda", heads: str | None = None,
               embed: str | None = None) -> Stack:
    """`Stack::load` (qwen3.rs:229-250): layers `{prefix}layers.{i}`, final `{prefix}norm`;
    optionally one codebook head and its embedding table (the talker's codec_head and
    codec_embedding)."""
    layers = [load_layer(w, f"{prefix}layers.{i}", geo, device) for i in range(geo.layers)]
    h = None if heads is None else w.cpu(heads).to(device).half()
    e = None if embed is None else w.cpu(embed).to(device).half()[None]
    return Stack(geo, layers, w.get(f"{prefix}norm.weight", device), h, e)


def load_talker(w: Weights, device="cuda", geo: Geometry = TALKER_GEOMETRY) -> Stack:
    """The talker of talker.rs:575-605: `talker.model.` stack with `talker.codec_head` and
    `talker.model.codec_embedding` as its one codebook head and table."""
    return load_stack(w, "talker.model.", geo, device, heads="talker.codec_head.weight",
                      embed="talker.model.codec_embedding.weight")


def load_predictor(w: Weights, device="cuda", geo: Geometry = PREDICTOR_GEOMETRY,
                   steps: int = 15) -> Predictor:
    """`Predictor::load` (talker.rs:276-330): its stack at `talker.code_predictor.model.`, the
    15 heads `lm_head.{i}`, the tables `codec_embedding.{i}` and small_to_mtp_projection;
    `resized` computed at load in f32 as the reference does."""
    stack = load_stack(w, "talker.code_predictor.model.", geo, device)
    p = "talker.code_predictor"
    heads = torch.cat([w.cpu(f"{p}.lm_head.{i}.weight") for i in range(steps)]).to(device)
    tables = torch.stack([w.cpu(f"{p}.model.codec_embedding.{i}.weight")
                          for i in range(steps)]).to(device)
    return Predictor(stack, w.cpu(f"{p}.small_to_mtp_projection.weight").to(device),
                     w.get(f"{p}.small_to_mtp_projection.bias", device), heads, tables)


def load_codec(w: Weights, device="cuda"):
    """`Codec::load` (codec.rs:320-395): the whole decoder from its checkpoint names (folded
    codebooks, pre-transformer, upsamplers, waveform stack)."""
    from .codec_ref import Codec
    return Codec.from_weights(w.cpu, device)
