"""Per-operator parity on a B200: each C-ABI op against the CPU oracle on the same seeded
inputs. Shapes follow the reference's own tests (cited per test). Tolerances are stated per
test; the bar for f16 ops is max relative error <= 2e-2."""
import numpy as np
import pytest
import torch

from _model import dev_f16, dev_f32

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    s = np.abs(b).max()
    return float(np.abs(a - b).max() / s) if s > 0 else float(np.abs(a - b).max())


def np_(t):
    return t.detach().float().cpu().numpy()


# crates/tts-nn/src/skinny.rs:181-189 shapes, plus the lane counts of the sweep (1..384)
SHAPES = [(48, 2048, 4096), (48, 2048, 6144), (48, 6144, 2048), (48, 1024, 3072), (40, 3072, 1024),
          (32, 1024, 2048), (8, 1024, 4096), (1, 2048, 2048), (128, 2048, 2048), (256, 1024, 1024),
          (384, 2048, 1024), (17, 512, 384)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_proj_f32(tt, orc, m, k, n):
    rng = np.random.default_rng(m * 7 + k + n)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = orc.f16_bits(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
    want = orc.proj(x, w)
    got = tt.Proj(dev_f16(w)).forward(dev_f32(x))
    torch.cuda.synchronize()
    tt.check()
    # f16 inputs, f32 accumulation on both sides: only the summation order differs
    assert rel(np_(got), want) < 1e-4, (m, k, n)


def test_proj_epilogues(tt, orc):
    from ttsnn import _lib as L
    rng = np.random.default_rng(11)
    m, k, n = 48, 2048, 1024
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = orc.f16_bits(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
    want = orc.proj(x, w)
    P = tt.Proj(dev_f16(w))
    y16 = P.forward(dev_f32(x), L.EPI_F16)
    assert y16.dtype == torch.float16 and rel(np_(y16), want) < 2e-3
    h0 = rng.standard_normal((m, n), dtype=np.float32)
    h = dev_f32(h0)
    P.forward(dev_f32(x), L.EPI_RESIDUAL_F32, out=h)
    assert rel(np_(h), h0 + want) < 1e-5
    # SwiGLU: gate/up interleaved per 128-row tile
    g = orc.f16_bits(rng.standard_normal((512, k), dtype=np.float32) * 0.02)
    u = orc.f16_bits(rng.standard_normal((512, k), dtype=np.float32) * 0.02)
    gu = tt.interleave_gate_up(dev_f16(g), dev_f16(u))
    act = tt.Proj(gu).forward(dev_f32(x), L.EPI_SWIGLU_F16)
    want_act = orc.swiglu(orc.proj(x, g), orc.proj(x, u))
    assert act.shape == (m, 512) and rel(np_(act), want_act) < 2e-3
    tt.check()


def test_proj_declines_unsupported(tt):
    P = tt.Proj(torch.zeros(100, 64, dtype=torch.float16, device="cuda"))
    with pytest.raises(tt.TtsError) as e:
        P.forward(torch.zeros(4, 64, device="cuda"))
    assert "n must be" in str(e.value)


def test_rms_norm(tt, orc):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((48, 2048), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    got = tt.rms_norm(dev_f32(x), dev_f32(w), 1e-6)
    assert rel(np_(got), orc.rms_norm(x, w, 1e-6)) < 1e-6


@pytest.mark.parametrize("b,start,off", [(8, 37, 2), (4, 0, 1), (48, 1000, 0)])
def test_qk_rope_lane_window(tt, orc, b, start, off):
    # crates/tts-nn/src/qkrope.rs:191-260: a lane window of a larger cache; nothing outside it
    # is written.
    heads, n_kv, cap, eps = 16, 8, 1100, 1e-6
    rng = np.random.default_rng(b + start)
    cos, sin = orc.rope_table(cap, 128, 1e6)
    norms = rng.uniform(0.5, 1.5, (2, 128)).astype(np.float32)
    qkv = rng.standard_normal((b, (heads + 2 * n_kv) * 128), dtype=np.float32)
    kc = torch.zeros(b + 3, n_kv, cap, 128, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    q, _ = tt.qkrope.apply(dev_f32(qkv).reshape(b, 1, -1), dev_f32(norms), dev_f32(cos), dev_f32(sin),
                           kc[off:off + b], vc[off:off + b], heads, start, eps)
    wq, wk, wv = orc.qk_rope(qkv, norms, cos, sin, np.full(b, start, np.int32), heads, n_kv, eps)
    assert rel(np_(q).reshape(b, heads, 128), wq) < 1e-5
    assert rel(np_(kc[off:off + b, :, start]), wk) < 1e-3
    assert rel(np_(vc[off:off + b, :, start]), wv) < 1e-3
    outside = kc[:off].abs().sum() + kc[off + b:].abs().sum() + vc[:off].abs().sum() + vc[off + b:].abs().sum()
    assert outside.item() == 0.0
    assert kc[off:off + b, :, :start].abs().sum().item() == 0.0
    tt.check()


def test_qk_rope_config0_per_row_positions(tt, orc):
    """Benchmark config[0]'s RoPE: X [48, 2048] ~N(0, 1) seed 0 viewed as 16 heads x 128,
    theta 1e6, one position per row drawn from U{0..1023}, through the reference's op on this
    path (qkrope::apply: per-head RMSNorm with eps 1e-6, half-split RoPE from the f64-built f32
    table, K/V appended at each row's own position; qkrope.rs:26-69, qwen3.rs:358-394)."""
    heads, n_kv, cap, eps = 16, 8, 1024, 1e-6
    rng = np.random.default_rng(0)
    x = rng.standard_normal((48, 2048), dtype=np.float32)
    kv_part = rng.standard_normal((48, 2 * n_kv * 128), dtype=np.float32)
    qkv = np.concatenate([x, kv_part], axis=1)
    pos = rng.integers(0, 1024, 48).astype(np.int32)
    norms = rng.uniform(0.5, 1.5, (2, 128)).astype(np.float32)
    cos, sin = orc.rope_table(cap, 128, 1e6)
    kc = torch.zeros(48, n_kv, cap, 128, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    q, _ = tt.qkrope.apply(dev_f32(qkv).reshape(48, 1, -1), dev_f32(norms), dev_f32(cos),
                           dev_f32(sin), kc, vc, heads, torch.from_numpy(pos), eps)
    wq, wk, wv = orc.qk_rope(qkv, norms, cos, sin, pos, heads, n_kv, eps)
    assert rel(np_(q).reshape(48, heads, 128), wq) < 1e-5
    lanes = np.arange(48)
    assert rel(np_(kc)[lanes, :, pos], wk) < 1e-3
    assert rel(np_(vc)[lanes, :, pos], wv) < 1e-3
    # nothing but each row's own position is written
    written = (kc != 0).any(dim=3).any(dim=1).cpu().numpy()
    assert np.array_equal(np.flatnonzero(written.reshape(-1)), np.sort(lanes * cap + pos))
    tt.check()


@pytest.mark.parametrize("b,n_kv,gqa,cap,span,wstart",
                         [(48, 8, 2, 400, 250, 0), (40, 8, 2, 17, 3, 0), (8, 8, 2, 300, 211, 90),
                          (4, 8, 1, 64, 33, 0), (6, 8, 2, 2100, 2050, 0)])
def test_decode_attention_ref_shapes(tt, orc, b, n_kv, gqa, cap, span, wstart):
    # crates/tts-nn/src/attn.rs:402-433 shapes (+ one multi-chunk span); reference bound 1e-5
    rng = np.random.default_rng(span)
    q = rng.standard_normal((b, n_kv, gqa, 128), dtype=np.float32) * 0.1
    kb = orc.f16_bits(rng.standard_normal((b, n_kv, cap, 128), dtype=np.float32))
    vb = orc.f16_bits(rng.standard_normal((b, n_kv, cap, 128), dtype=np.float32))
    want = orc.decode_attention(q, kb, vb, span, wstart)
    got = tt.attn.decode_attention(dev_f32(q), dev_f16(kb), dev_f16(vb), span, wstart)
    assert rel(np_(got), want) < 1e-5
    tt.check()


def test_decode_attention_paged_ragged(tt, orc):
    """Per-lane spans (1..1100) over shuffled pages; one call serves every lane."""
    from ttsnn import _lib as L
    lanes, n_kv, gqa, bs = 24, 8, 2, 32
    rng = np.random.default_rng(5)
    spans = np.concatenate([[1, 2, 31, 32, 33, 256, 257, 1100], rng.integers(1, 1100, lanes - 8)]).astype(np.int32)
    cap = 1120
    per = cap // bs
    q = rng.standard_normal((lanes, n_kv * gqa, 128), dtype=np.float32) * 0.1
    kb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    vb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    nb = lanes * per + 5
    order = rng.permutation(nb)
    table = order[:lanes * per].reshape(lanes, per).astype(np.int32)
    def pages(c):
        p = c.reshape(lanes, n_kv, per, bs, 128).transpose(0, 2, 1, 3, 4).reshape(-1, n_kv, bs, 128)
        host = np.zeros((nb, n_kv, bs, 128), np.uint16)
        host[table.reshape(-1)] = p
        return dev_f16(host)
    kp, vp = pages(kb), pages(vb)
    tdev = torch.from_numpy(table).cuda()
    kv = L.KvCache(kp.data_ptr(), vp.data_ptr(), tdev.data_ptr(), per, bs, nb, n_kv, 128)
    got = tt.attn.decode_attention_paged(dev_f32(q), kv, torch.from_numpy(spans).cuda(), 1100,
                                         out_f16=False)
    want = orc.decode_attention(q.reshape(lanes, n_kv, gqa, 128), kb, vb, spans, 0)
    assert rel(np_(got), want.reshape(lanes, -1)) < 1e-5
    tt.check()


def test_swiglu_snake_argmax(tt, orc):
    rng = np.random.default_rng(9)
    g = rng.standard_normal(48 * 6144, dtype=np.float32) * 3
    u = rng.standard_normal(48 * 6144, dtype=np.float32)
    assert rel(np_(tt.fused.swiglu_mul(dev_f32(g), dev_f32(u))), orc.swiglu(g, u)) < 1e-6
    x = rng.standard_normal((4000, 512), dtype=np.float32)
    a = np.exp(rng.uniform(-1, 1, 512)).astype(np.float32)
    br = (1.0 / a).astype(np.float32)
    want = orc.snake_beta(x, a, br)
    assert rel(np_(tt.fused.snake_beta_nlc(dev_f32(x), dev_f32(a), dev_f32(br))), want) < 1e-6
    x16 = orc.f16_value(orc.f16_bits(x))
    got16 = tt.fused.snake_beta_nlc(dev_f32(x16).half(), dev_f32(a), dev_f32(br))
    assert got16.dtype == torch.float16 and rel(np_(got16), orc.snake_beta(x16, a, br)) < 2e-3
    logits = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 1.0, 5.0, 5.0]], np.float32)
    assert tt.topk.argmax(dev_f32(logits)).tolist() == [2, 3]
    banned = torch.tensor([0, 0, 1, 1], dtype=torch.uint8, device="cuda")
    assert tt.topk.argmax(dev_f32(logits), banned).tolist() == [1, 0]
    big = rng.standard_normal((48, 3072), dtype=np.float32)
    mask = np.zeros(3072, np.uint8)
    mask[2048:] = 1
    mask[2150] = 0
    assert np.array_equal(tt.topk.argmax(dev_f32(big), torch.from_numpy(mask).cuda()).cpu().numpy(),
                          orc.argmax(big, mask).astype(np.int32))


def _paged(rng, kb, vb, bs, spare=5):
    """Contiguous `[lanes, n_kv, cap, 128]` f16 bits -> shuffled pages + block table."""
    lanes, n_kv, cap, _ = kb.shape
    per = cap // bs
    nb = lanes * per + spare
    table = rng.permutation(nb)[:lanes * per].reshape(lanes, per).astype(np.int32)

    def pages(c):
        p = c.reshape(lanes, n_kv, per, bs, 128).transpose(0, 2, 1, 3, 4).reshape(-1, n_kv, bs, 128)
        host = np.zeros((nb, n_kv, bs, 128), np.uint16)
        host[table.reshape(-1)] = p
        return dev_f16(host)
    return pages(kb), pages(vb), table, nb


@pytest.mark.parametrize("bs,n_kv,gqa,window", [(8, 8, 2, 0), (16, 4, 4, 0), (64, 2, 8, 0),
                                                (128, 8, 1, 0), (32, 8, 2, 300), (16, 8, 2, 129)])
def test_decode_attention_paged_geometries(tt, orc, bs, n_kv, gqa, window):
    """Page sizes 8..128 (one TMA box per page run), gqa 1..8, sliding windows whose start
    falls mid-chunk; per-lane spans cross chunk and page edges."""
    from ttsnn import _lib as L
    rng = np.random.default_rng(bs * 10 + gqa + window)
    lanes, cap = 20, 1152
    spans = np.concatenate([[1, 7, 8, 127, 128, 129, 640, 1152],
                            rng.integers(1, cap + 1, lanes - 8)]).astype(np.int32)
    q = rng.standard_normal((lanes, n_kv * gqa, 128), dtype=np.float32) * 0.1
    kb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    vb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    kp, vp, table, nb = _paged(rng, kb, vb, bs)
    tdev = torch.from_numpy(table).cuda()
    kv = L.KvCache(kp.data_ptr(), vp.data_ptr(), tdev.data_ptr(), cap // bs, bs, nb, n_kv, 128)
    got = tt.attn.decode_attention_paged(dev_f32(q), kv, torch.from_numpy(spans).cuda(), cap,
                                         window=window, out_f16=False)
    wstart = np.where((window > 0) & (spans > window), spans - window, 0).astype(np.int32)
    want = orc.decode_attention(q.reshape(lanes, n_kv, gqa, 128), kb, vb, spans, wstart)
    assert rel(np_(got), want.reshape(lanes, -1)) < 1e-5
    tt.check()


def test_decode_attention_pages_outside_pool(tt, orc):
    """Block-table entries outside [0, num_blocks) read as zero rows and are reported as
    out-of-range device data (not as a timeout); the other lanes are unaffected."""
    from ttsnn import _lib as L
    rng = np.random.default_rng(77)
    lanes, n_kv, gqa, cap, bs = 6, 8, 2, 512, 32
    spans = np.array([512, 300, 64, 511, 129, 33], np.int32)
    q = rng.standard_normal((lanes, n_kv * gqa, 128), dtype=np.float32) * 0.1
    kb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    vb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    kp, vp, table, nb = _paged(rng, kb, vb, bs)
    bad = [(0, 3, -1), (1, 0, nb), (3, 15, nb + 7)]  # (lane, page, entry)
    kz, vz = kb.copy(), vb.copy()
    for lane, page, entry in bad:
        table[lane, page] = entry
        kz[lane, :, page * bs:(page + 1) * bs] = 0
        vz[lane, :, page * bs:(page + 1) * bs] = 0
    tdev = torch.from_numpy(table).cuda()
    kv = L.KvCache(kp.data_ptr(), vp.data_ptr(), tdev.data_ptr(), cap // bs, bs, nb, n_kv, 128)
    got = tt.attn.decode_attention_paged(dev_f32(q), kv, torch.from_numpy(spans).cuda(), cap,
                                         out_f16=False)
    with pytest.raises(tt.TtsError) as e:
        tt.check()
    assert e.value.status == 1  # TTS_ERR_INVALID_ARG: bad device data, not a timeout
    assert "out of range" in str(e.value)
    want = orc.decode_attention(q.reshape(lanes, n_kv, gqa, 128), kz, vz, spans, 0)
    assert rel(np_(got), want.reshape(lanes, -1)) < 1e-5
    tt.check()  # the flag was cleared by the previous check


def test_decode_attention_rejects_unaligned_pages(tt):
    from ttsnn import _lib as L
    kp = torch.zeros(4, 8, 12, 128, dtype=torch.float16, device="cuda")
    table = torch.zeros(2, 2, dtype=torch.int32, device="cuda")
    kv = L.KvCache(kp.data_ptr(), kp.data_ptr(), table.data_ptr(), 2, 12, 4, 8, 128)
    q = torch.zeros(2, 16, 128, device="cuda")
    with pytest.raises(tt.TtsError) as e:
        tt.attn.decode_attention_paged(q, kv, torch.full((2,), 20, dtype=torch.int32, device="cuda"), 100)
    assert "multiple of 8" in str(e.value)


@pytest.mark.parametrize("bs,n_kv,gqa,window", [(12, 8, 2, 0), (16, 8, 1, 0), (8, 4, 4, 0),
                                                (5, 2, 8, 0), (16, 8, 2, 9), (64, 8, 2, 0)])
def test_decode_attention_short_spans(tt, orc, bs, n_kv, gqa, window):
    """max_span <= 64 takes the CUDA-core kernel: any page size (the tensor-core kernel's
    multiple-of-8 rule does not apply), gqa 1..8, windows, per-lane spans 1..64, and one page
    outside the pool read as zeros and reported."""
    from ttsnn import _lib as L
    rng = np.random.default_rng(bs * 100 + gqa * 10 + window)
    lanes, cap = 14, -(-64 // bs) * bs
    spans = np.concatenate([[1, 2, 16, 17, 63, 64], rng.integers(1, 65, lanes - 6)]).astype(np.int32)
    q = rng.standard_normal((lanes, n_kv * gqa, 128), dtype=np.float32) * 0.1
    kb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    vb = orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
    kp, vp, table, nb = _paged(rng, kb, vb, bs)
    kz, vz = kb.copy(), vb.copy()
    last = (int(spans[4]) - 1) // bs  # lane 4 (span 63): its last page is outside the pool
    table[4, last] = nb + 3
    kz[4, :, last * bs:(last + 1) * bs] = 0
    vz[4, :, last * bs:(last + 1) * bs] = 0
    tdev = torch.from_numpy(table).cuda()
    kv = L.KvCache(kp.data_ptr(), vp.data_ptr(), tdev.data_ptr(), cap // bs, bs, nb, n_kv, 128)
    got = tt.attn.decode_attention_paged(dev_f32(q), kv, torch.from_numpy(spans).cuda(), 64,
                                         window=window, out_f16=False)
    with pytest.raises(tt.TtsError) as e:
        tt.check()
    assert e.value.status == 1
    wstart = np.where((window > 0) & (spans > window), spans - window, 0).astype(np.int32)
    want = orc.decode_attention(q.reshape(lanes, n_kv, gqa, 128), kz, vz, spans, wstart)
    assert rel(np_(got), want.reshape(lanes, -1)) < 1e-5
    got16 = tt.attn.decode_attention_paged(dev_f32(q), kv, torch.from_numpy(spans).cuda(), 64,
                                           window=window, out_f16=True)
    assert rel(np_(got16.float()), want.reshape(lanes, -1)) < 2e-3
    with pytest.raises(tt.TtsError):
        tt.check()


@pytest.mark.parametrize("rows,n,k,temp", [(64, 2048, 50, 0.9), (32, 3072, 64, 1.3),
                                           (16, 4096, 1, 0.9), (40, 100, 7, 0.0)])
def test_topk_sample(tt, orc, rows, n, k, temp):
    """tts_topk_sample against the host sampler's restatement on the same logits and draws:
    equal picks, ties (logits quantised to a few levels) broken by the lower index."""
    rng = np.random.default_rng(n + k)
    logits = rng.standard_normal((rows, n)).astype(np.float32) * 2
    logits[: rows // 2] = np.round(logits[: rows // 2] * 2) / 2  # many exact ties
    draws = rng.random(rows).astype(np.float32)
    draws[0] = 0.0
    draws[1] = 0.99999
    got = tt.topk.sample(dev_f32(logits), dev_f32(draws), k, temp)
    want = orc.topk_sample(logits, draws, k, temp)
    assert np.array_equal(np_(got).astype(np.uint32), want)
    tt.check()


def test_topk_sample_limits(tt):
    x = torch.zeros(2, 5000, device="cuda")
    d = torch.zeros(2, device="cuda")
    with pytest.raises(tt.TtsError) as e:
        tt.topk.sample(x, d, 10, 1.0)
    assert e.value.status == 2
    with pytest.raises(tt.TtsError):
        tt.topk.sample(x[:, :100], d, 65, 1.0)
