"""Prefill (Stack::forward at t > 1, crates/qwen3tts/src/qwen3.rs:294-467) and shared prompt
prefixes (the reference's broadcast copy of a shared prefix into every lane, qwen3.rs:261-284)
on a B200 against the CPU oracle's restatement of the reference's prefill branch (qwen3.rs:
415-444, the CPU arm): projections through matmul_2d with f16 results, the new positions
attending over their own f32 K/V concatenated after the f16 cache prefix. The device attends
over its f16 pages for both (its projections keep f32 results). Bar: every row's hidden and the
written K/V within 2e-2, positions advanced; prefill over two chunks of rows (more rows than a
call takes at once); 48 lanes x 157 positions at the talker's widths, then more rows on top of
the prefilled prefix; shared pages read by several lanes, only the partly filled one copied."""
import numpy as np
import pytest
import torch

from _model import dev_f32, device_stack, gather_pages, make_talker

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def oracle_prefill(orc, g, Ls, final, kc, vc, lane, start, rows, cos, sin):
    """The lane's rows through the reference's prefill branch (views keep the caches in
    place); a single row takes the decode branch (t == 1), CPU arm both."""
    ks = [a[lane:lane + 1] for a in kc]
    vs = [a[lane:lane + 1] for a in vc]
    if rows.shape[0] == 1:
        return orc.decode_step(rows, Ls, final, ks, vs, np.array([start], np.int32), cos, sin,
                               g, round_f16=True)
    return orc.prefill(rows[None], Ls, final, ks, vs, start, cos, sin, g)[0]


def setup(orc, tt, lanes, cap, bs, seed):
    from qwen3tts import PagedKv
    g, Ls, final, kc, vc, pos, x = make_talker(orc, lanes, 2, 256, 4, 2, 512, cap, seed,
                                               lengths=[0] * lanes)
    for a in kc + vc:
        a[:] = 0
    stack = device_stack(orc, g, Ls, final)
    per = cap // bs
    kv = PagedKv(stack.geo, lanes, lanes * per + 4, bs, per)
    cos, sin = orc.rope_table(cap + 8, 128, g.rope_base)
    return g, Ls, final, kc, vc, stack, kv, cos, sin


def test_prefill_matches_reference_prefill(tt, orc):
    """Three lanes: one already holding 10 positions; 590 new rows in all (two chunks)."""
    lanes, cap, bs = 3, 384, 32
    g, Ls, final, kc, vc, stack, kv, cos, sin = setup(orc, tt, lanes, cap, bs, 51)
    rng = np.random.default_rng(52)
    start = [0, 10, 0]
    lens = [300, 250, 40]
    for i in range(lanes):
        kv.admit(i, cap, 0)
    # lane 1's first 10 positions: prefilled first, on their own
    pre = rng.standard_normal((10, g.dim), dtype=np.float32)
    stack.prefill(kv, [0, 10, 0], dev_f32(pre), max_span=cap)
    oracle_prefill(orc, g, Ls, final, kc, vc, 1, 0, pre, cos, sin)
    rows = [rng.standard_normal((n, g.dim), dtype=np.float32) for n in lens]
    x = np.concatenate(rows)
    h = torch.empty(x.shape[0], g.dim, device="cuda")
    stack.prefill(kv, lens, dev_f32(x), h_out=h, max_span=cap)
    torch.cuda.synchronize()
    tt.check()
    got = h.cpu().numpy()
    r0 = 0
    for i in range(lanes):
        want = oracle_prefill(orc, g, Ls, final, kc, vc, i, start[i], rows[i], cos, sin)
        assert rel(got[r0:r0 + lens[i]], want) < 2e-2, i
        r0 += lens[i]
    assert kv.positions.cpu().tolist() == [start[i] + lens[i] for i in range(lanes)]
    table = kv.table.cpu().numpy()
    for li in range(g.layers):
        gk = gather_pages(kv.k[li], table, lanes, g.n_kv, cap, bs)
        for i in range(lanes):
            n = start[i] + lens[i]
            assert rel(orc.f16_value(gk[i, :, :n]), orc.f16_value(kc[li][i, :, :n])) < 2e-2
    # a decode step continues from the prefilled state
    xs = rng.standard_normal((lanes, g.dim), dtype=np.float32)
    hs = torch.empty(lanes, g.dim, device="cuda")
    stack.decode_step(kv, dev_f32(xs), h_out=hs, max_span=cap)
    want = orc.decode_step(xs, Ls, final, kc, vc, np.array([start[i] + lens[i] for i in range(lanes)],
                                                           np.int32), cos, sin, g, round_f16=True)
    torch.cuda.synchronize()
    assert rel(hs.cpu().numpy(), want) < 2e-2


def test_prefill_48_lanes_157_positions_talker_widths(tt, orc):
    """The reference's ICL prompt width (157, fixtures/qwen3tts/oracle.json) at 48 lanes on the
    config[2] talker's widths (2048, 16/8 heads, 6144; 2 layers), then 5 more rows per lane on
    top of the 157 cached positions (the branch that concatenates the f16 prefix)."""
    from qwen3tts import PagedKv
    lanes, cap, bs, width = 48, 192, 32, 157
    g, Ls, final, kc, vc, pos, x = make_talker(orc, lanes, 2, 2048, 16, 8, 6144, cap, 71,
                                               lengths=[0] * lanes, fast_kv=True)
    for a in kc + vc:
        a[:] = 0
    stack = device_stack(orc, g, Ls, final)
    kv = PagedKv(stack.geo, lanes, lanes * (cap // bs) + 4, bs, cap // bs)
    for i in range(lanes):
        kv.admit(i, cap, 0)
    cos, sin = orc.rope_table(cap + 8, 128, g.rope_base)
    rng = np.random.default_rng(72)
    for start, t in ((0, width), (width, 5)):
        rows = rng.standard_normal((lanes, t, g.dim), dtype=np.float32)
        h = torch.empty(lanes * t, g.dim, device="cuda")
        stack.prefill(kv, [t] * lanes, dev_f32(rows.reshape(-1, g.dim)), h_out=h, max_span=cap)
        torch.cuda.synchronize()
        tt.check()
        want = orc.prefill(rows, Ls, final, kc, vc, start, cos, sin, g)
        r = rel(h.cpu().numpy(), want.reshape(-1, g.dim))
        print(f"prefill start {start}, {t} rows x {lanes} lanes: hidden rel {r:.2e}")
        assert r < 2e-2, start
    assert kv.positions.cpu().tolist() == [width + 5] * lanes
    table = kv.table.cpu().numpy()
    for li in range(g.layers):
        gk = gather_pages(kv.k[li], table, lanes, g.n_kv, width + 5, bs)
        assert rel(orc.f16_value(gk), orc.f16_value(kc[li][:, :, :width + 5])) < 2e-2


@pytest.mark.parametrize("cap,lens,start", [(192, [150, 100, 70, 31], [0, 20, 0, 5]),
                                             (128, [100, 64, 3, 120], [0, 7, 0, 0])])
def test_prefill_short_prompts(tt, orc, cap, lens, start):
    """Short prompts with lanes that already hold positions, through the layer-major prefill:
    every row's hidden and the written K/V against the reference's prefill, as above."""
    lanes, bs = len(lens), 32
    g, Ls, final, kc, vc, stack, kv, cos, sin = setup(orc, tt, lanes, cap, bs, 61 + cap)
    rng = np.random.default_rng(62 + cap)
    for i in range(lanes):
        kv.admit(i, cap, 0)
    pre = [rng.standard_normal((start[i], g.dim), dtype=np.float32) for i in range(lanes)]
    stack.prefill(kv, start, dev_f32(np.concatenate(pre)), max_span=cap)
    for i in range(lanes):
        if start[i]:
            oracle_prefill(orc, g, Ls, final, kc, vc, i, 0, pre[i], cos, sin)
    rows = [rng.standard_normal((n, g.dim), dtype=np.float32) for n in lens]
    x = dev_f32(np.concatenate(rows))
    h = torch.empty(x.shape[0], g.dim, device="cuda")
    stack.prefill(kv, lens, x, h_out=h, max_span=cap)
    torch.cuda.synchronize()
    tt.check()
    got = h.cpu().numpy()
    r0 = 0
    for i in range(lanes):
        want = oracle_prefill(orc, g, Ls, final, kc, vc, i, start[i], rows[i], cos, sin)
        assert rel(got[r0:r0 + lens[i]], want) < 2e-2, i
        r0 += lens[i]
    table = kv.table.cpu().numpy()
    for li in range(g.layers):
        gk = gather_pages(kv.k[li], table, lanes, g.n_kv, cap, bs)
        for i in range(lanes):
            n = start[i] + lens[i]
            assert rel(orc.f16_value(gk[i, :, :n]), orc.f16_value(kc[li][i, :, :n])) < 2e-2


def test_shared_prefix(tt, orc):
    """Lane 0 prefills a 45-position prefix; lanes 1 and 2 share its first page through the
    block table and copy the partly filled second one, then append their own rows: each lane
    matches the oracle lane that prefilled the whole prefix itself."""
    lanes, cap, bs = 3, 128, 32
    g, Ls, final, kc, vc, stack, kv, cos, sin = setup(orc, tt, lanes, cap, bs, 53)
    rng = np.random.default_rng(54)
    prefix = rng.standard_normal((45, g.dim), dtype=np.float32)
    kv.admit(0, cap, 0)
    stack.prefill(kv, [45], dev_f32(prefix), max_span=cap)
    for i in (1, 2):
        pages = kv.share_prefix(0, i, 45, cap)
        assert pages[0] == int(kv.table[0, 0]) and pages[1] != int(kv.table[0, 1])
    free_before = kv.free_pages()
    own = [rng.standard_normal((n, g.dim), dtype=np.float32) for n in (5, 20, 7)]
    h = torch.empty(32, g.dim, device="cuda")
    stack.prefill(kv, [5, 20, 7], dev_f32(np.concatenate(own)), h_out=h, max_span=cap)
    torch.cuda.synchronize()
    tt.check()
    got = h.cpu().numpy()
    r0 = 0
    for i in range(lanes):
        oracle_prefill(orc, g, Ls, final, kc, vc, i, 0, prefix, cos, sin)
        want = oracle_prefill(orc, g, Ls, final, kc, vc, i, 45, own[i], cos, sin)
        assert rel(got[r0:r0 + len(own[i])], want) < 2e-2, i
        r0 += len(own[i])
    assert kv.positions.cpu().tolist() == [50, 65, 52]
    # the shared page is freed only when its last lane lets it go
    shared = int(kv.table[0, 0])
    kv.release(0)
    kv.release(1)
    assert kv.page_refs(shared) == 1
    kv.release(2)
    assert kv.page_refs(shared) == 0 and kv.free_pages() > free_before
