"""Per-device contexts and small helpers shared by the op modules."""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

MAX_LANES = 448
_ctx: dict[int, C.c_void_p] = {}


def ctx(device: int | None = None) -> C.c_void_p:
    """The library context of `device` (created on first use, with scratch for 448 lanes)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    if dev not in _ctx:
        p = C.c_void_p()
        L.call("tts_ctx_create", dev, MAX_LANES, C.byref(p))
        _ctx[dev] = p
    return _ctx[dev]


def ctx_of(t: torch.Tensor) -> C.c_void_p:
    if not t.is_cuda:
        raise ValueError("tts-nn (B200): tensors must live on a CUDA device; there is no CPU path")
    return ctx(t.device.index)


def stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t: torch.Tensor | None) -> C.c_void_p:
    return C.c_void_p(0 if t is None else t.data_ptr())


def check(device: int | None = None) -> None:
    """Synchronises and raises if a kernel's bounded wait gave up since the last check."""
    L.call("tts_ctx_check", ctx(device), stream())


def launch_count(reset: bool = False) -> int:
    return int(L.load().tts_launch_count(1 if reset else 0))
