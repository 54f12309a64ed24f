"""The prefill-shaped projection (tts_proj_forward_rows: token rows as the MMA's M, 256 weight
rows per tile, the whole K per tile) against the CPU oracle on the same seeded inputs: plain f32
out, the residual epilogue and SwiGLU, at row counts that are not multiples of the 128-row tile
and up to several thousand rows (the prefill's 48 x 157 prompt rows). Tolerances as for the
decode projection: f16 inputs, f32 accumulation on both sides."""
import numpy as np
import pytest
import torch

from _model import dev_f16, dev_f32

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def np_(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("rows,k,n", [(1, 256, 256), (77, 512, 1024), (300, 2048, 256),
                                      (1000, 1024, 2048), (7536, 2048, 4096)])
def test_proj_rows_f32(tt, orc, rows, k, n):
    rng = np.random.default_rng(rows + k + n)
    x = rng.standard_normal((rows, k), dtype=np.float32)
    w = orc.f16_bits(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
    P = tt.Proj(dev_f16(w))
    got = P.forward_rows(dev_f32(x))
    torch.cuda.synchronize()
    tt.check()
    sel = np.unique(np.r_[0, rows - 1, rng.integers(0, rows, 64)])  # the oracle on sampled rows
    want = orc.proj(x[sel], w)
    assert got.shape == (rows, n) and rel(np_(got)[sel], want) < 1e-4, (rows, k, n)


def test_proj_rows_residual_and_swiglu(tt, orc):
    from ttsnn import _lib as L
    rng = np.random.default_rng(5)
    rows, k = 613, 1024
    x = rng.standard_normal((rows, k), dtype=np.float32)
    w = orc.f16_bits(rng.standard_normal((512, k), dtype=np.float32) * 0.02)
    h0 = rng.standard_normal((rows, 512), dtype=np.float32)
    h = dev_f32(h0)
    tt.Proj(dev_f16(w)).forward_rows(dev_f32(x), L.EPI_RESIDUAL_F32, out=h)
    torch.cuda.synchronize()
    assert rel(np_(h), h0 + orc.proj(x, w)) < 1e-5
    g = orc.f16_bits(rng.standard_normal((768, k), dtype=np.float32) * 0.02)
    u = orc.f16_bits(rng.standard_normal((768, k), dtype=np.float32) * 0.02)
    gu = tt.interleave_gate_up(dev_f16(g), dev_f16(u))
    act = tt.Proj(gu).forward_rows(dev_f32(x), L.EPI_SWIGLU_F16)
    torch.cuda.synchronize()
    tt.check()
    want = orc.swiglu(orc.proj(x, g), orc.proj(x, u))
    assert act.shape == (rows, 768) and rel(np_(act), want) < 2e-3
    # the decode projection gives the same rows (same f16 operands, f32 accumulation)
    dec = tt.Proj(gu).forward(dev_f32(x[:48]), L.EPI_SWIGLU_F16)
    assert rel(np_(act)[:48], np_(dec)) < 2e-3


def test_proj_rows_declines_unsupported(tt):
    from ttsnn import _lib as L
    P = tt.Proj(torch.zeros(384, 64, dtype=torch.float16, device="cuda"))  # n % 256 != 0
    with pytest.raises(L.TtsError):
        P.forward_rows(torch.zeros(10, 64, device="cuda"))
