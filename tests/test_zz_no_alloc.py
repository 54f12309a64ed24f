"""tts_decode_attention_static — decode attention for callers that cannot allocate device memory
(a real-time audio thread, where cudaMalloc can stall the whole device, or a host engine that
owns all device memory in its own arena). Its scratch lives in a fixed device array inside the
library. Checked through the C ABI against the context-based tts_decode_attention on two calls
in a row, within the attention tests' tolerance. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LANES, N_KV, GQA, BS = 12, 8, 2, 32


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def paged_inputs(seed, spans):
    rng = np.random.default_rng(seed)
    per = 36  # 36 pages of 32 positions = 1152 >= every span
    nb = LANES * per + 7
    table = rng.permutation(nb)[:LANES * per].reshape(LANES, per).astype(np.int32)
    k = torch.randn(nb, N_KV, BS, 128, device="cuda").half()
    v = torch.randn(nb, N_KV, BS, 128, device="cuda").half()
    q = torch.randn(LANES, N_KV * GQA, 128, device="cuda") * 0.1
    t = torch.from_numpy(table).cuda()
    s = torch.tensor(spans, dtype=torch.int32, device="cuda")
    return q, k, v, t, s, per, nb


def test_static_scratch_matches_context_entry_point(tt):
    from ttsnn import _lib as L
    lib = L.load()
    torch.cuda.set_device(0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    ctx = tt.ctx(0)
    max_span = 1100
    # two calls in a row with different spans: multi-chunk lanes use the partials and counters
    for call, spans in enumerate(([1, 31, 256, 257, 600, 1100, 5, 64, 999, 300, 512, 700],
                                  [1100, 2, 700, 33, 1024, 255, 129, 900, 1, 513, 64, 1099])):
        q, k, v, t, s, per, nb = paged_inputs(100 + call, spans)
        kv = L.KvCache(k.data_ptr(), v.data_ptr(), t.data_ptr(), per, BS, nb, N_KV, 128)
        want = torch.empty(LANES, N_KV * GQA * 128, device="cuda")
        got = torch.full_like(want, float("nan"))
        rc = lib.tts_decode_attention(ctx, C.c_void_p(q.data_ptr()), LANES, GQA, C.byref(kv),
                                      C.c_void_p(s.data_ptr()), max_span, 0,
                                      C.c_void_p(want.data_ptr()), 0, stream)
        assert rc == 0, L.last_error()
        rc = lib.tts_decode_attention_static(C.c_void_p(q.data_ptr()), LANES, GQA, C.byref(kv),
                                             C.c_void_p(s.data_ptr()), max_span, 0,
                                             C.c_void_p(got.data_ptr()), 0, stream)
        assert rc == 0, L.last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), f"call {call}: output not fully written"
        assert rel(got.cpu().numpy(), want.cpu().numpy()) < 1e-5, f"call {call}"


def test_static_scratch_rejects_oversize(tt):
    from ttsnn import _lib as L
    lib = L.load()
    q, k, v, t, s, per, nb = paged_inputs(7, [1] * LANES)
    kv = L.KvCache(k.data_ptr(), v.data_ptr(), t.data_ptr(), per, BS, nb, N_KV, 128)
    out = torch.empty(512, N_KV * GQA * 128, device="cuda")
    # 512 lanes x 8 kv heads x 32 chunks x 2 x 520 B is far beyond the 4 MiB of partials
    rc = lib.tts_decode_attention_static(C.c_void_p(q.data_ptr()), 512, GQA, C.byref(kv),
                                         C.c_void_p(s.data_ptr()), 8192, 0,
                                         C.c_void_p(out.data_ptr()), 0, None)
    assert rc == 2
    assert "limit" in L.last_error()
