"""The talker decode step (Stack::forward at t == 1 + codebook heads + greedy pick) on a B200
against the CPU oracle's composition of the reference's ops (crates/qwen3tts/src/qwen3.rs:
294-467). Bar: hidden and logits max relative error <= 2e-2 (f16 weights, f32 accumulate),
greedy code agreement >= 99.5%, K/V written at each lane's position, positions advanced.

Two arms of the reference are restated: the Metal arm (skinny matmul, f32 projection outputs)
and the CPU arm BASELINE names as the parity target (`--no-default-features`: every Proj goes
through matmul_2d, whose f16 result is cast back to f32, crates/tts-nn/src/lib.rs:519-528). The
device keeps f32 projection outputs; the full config[2] step is checked against both arms. In the
CPU arm the logits are f16 values, so exact ties are common: a device pick that lands on an id
whose f16 logit equals the row's maximum is a tie under the last-max rule, counted and
reported, not a disagreement."""
import numpy as np
import pytest
import torch

from _model import (dev_f32, device_stack, gather_pages, make_heads, make_talker,
                    paged_from_contiguous)

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def run_case(tt, orc, lanes, layers, dim, heads, n_kv, ffn, lengths, codebooks, vocab, bs, seed,
             fast_kv=False, cpu_arm=False):
    cap = int(max(lengths)) + 2
    g, Ls, final, kc, vc, pos, x = make_talker(orc, lanes, layers, dim, heads, n_kv, ffn, cap, seed,
                                               codebooks=codebooks, vocab=vocab, lengths=lengths,
                                               fast_kv=fast_kv)
    hb, eb = make_heads(orc, seed + 1, g)
    stack = device_stack(orc, g, Ls, final, hb, eb)
    kv, table = paged_from_contiguous(stack.geo, kc, vc, pos, bs, seed + 2)
    cos, sin = orc.rope_table(cap + 8, 128, g.rope_base)

    h_out = torch.empty(lanes, dim, device="cuda")
    logits = torch.empty(lanes, codebooks * vocab, device="cuda")
    codes = torch.empty(lanes, codebooks, dtype=torch.int32, device="cuda")
    stack.decode_step(kv, dev_f32(x), h_out=h_out, logits=logits, codes=codes, max_span=cap)
    torch.cuda.synchronize()
    tt.check()

    out = {}
    if cpu_arm:
        # the CPU arm first: each arm writes this step's K/V at the lanes' positions before its
        # attention reads them, so the Metal arm below runs on its own K/V
        ch = orc.decode_step(x, Ls, final, kc, vc, pos, cos, sin, g, round_f16=True)
        cl, cc = orc.heads_pick(ch, hb, g, round_f16=True)
        out.update(cpu_h=ch, cpu_logits=cl, cpu_codes=cc)
    want_h = orc.decode_step(x, Ls, final, kc, vc, pos, cos, sin, g)
    want_logits, want_codes = orc.heads_pick(want_h, hb, g)
    out.update(stack=stack, kv=kv, table=table, g=g, kc=kc, vc=vc, pos=pos, h=h_out,
               logits=logits, codes=codes, want_h=want_h, want_logits=want_logits,
               want_codes=want_codes, eb=eb)
    return out


def agreement_with_f16_ties(codes, logits16, g):
    """Greedy agreement against f16-rounded logits: a pick agrees when its f16 logit equals its
    row's maximum (the oracle's last-max pick, or another id of an exact tie). Returns
    (agreement, exact agreements, tie agreements) as fractions of all picks."""
    b = codes.shape[0]
    l = logits16.reshape(b, g.codebooks, g.vocab)
    mx = l.max(axis=2)
    got = np.take_along_axis(l, codes.astype(np.int64)[:, :, None], axis=2)[:, :, 0]
    last = np.array([[int(np.flatnonzero(l[i, q] == mx[i, q])[-1]) for q in range(g.codebooks)]
                     for i in range(b)])
    exact = codes == last
    tie = (got == mx) & ~exact
    return float((exact | tie).mean()), float(exact.mean()), float(tie.mean())


def check_case(orc, r, lanes, bs):
    assert rel(r["h"].cpu().numpy(), r["want_h"]) < 2e-2
    assert rel(r["logits"].cpu().numpy(), r["want_logits"]) < 2e-2
    agree = (r["codes"].cpu().numpy() == r["want_codes"].astype(np.int32)).mean()
    assert agree >= 0.995, agree
    assert np.array_equal(r["kv"].positions.cpu().numpy(), r["pos"] + 1)
    g = r["g"]
    for li in (0, g.layers - 1):
        got_k = gather_pages(r["kv"].k[li], r["table"], lanes, g.n_kv, int(r["pos"].max()) + 1, bs)
        lane = np.arange(lanes)
        gk = orc.f16_value(got_k[lane, :, r["pos"]])
        wk = orc.f16_value(r["kc"][li][lane, :, r["pos"]])
        assert rel(gk, wk) < 2e-2
    return agree


def test_step_small_long_spans(tt, orc):
    """2 layers at the talker's real widths; spans 1..1100 cover multi-chunk attention."""
    lengths = [0, 1, 63, 64, 255, 256, 700, 1099]
    r = run_case(tt, orc, 8, 2, 2048, 16, 8, 6144, lengths, 4, 2048, 16, 21)
    check_case(orc, r, 8, 16)


def test_step_graph_replay_matches_eager(tt, orc):
    lengths = list(np.random.default_rng(3).integers(64, 400, 16))
    r = run_case(tt, orc, 16, 2, 2048, 16, 8, 6144, lengths, 2, 2048, 32, 31)
    stack, kv = r["stack"], r["kv"]
    snap = (kv.k.clone(), kv.v.clone(), kv.positions.clone())

    def restore():
        kv.k.copy_(snap[0]); kv.v.copy_(snap[1]); kv.positions.copy_(snap[2])

    # x = None continues from the sum of the picked codes' embedding rows
    hA = torch.empty(16, 2048, device="cuda")
    stack.decode_step(kv, None, h_out=hA, max_span=1024)
    restore()
    x_next = dev_f32(orc.embed_sum(r["codes"].cpu().numpy(), r["eb"]))
    hB = torch.empty_like(hA)
    stack.decode_step(kv, x_next, h_out=hB, max_span=1024)
    torch.cuda.synchronize()
    assert rel(hA.cpu().numpy(), hB.cpu().numpy()) < 1e-6

    # a captured graph replays the eager step exactly (same kernels, deterministic reductions)
    restore()
    h1 = torch.empty_like(hA)
    c1 = torch.empty(16, 2, dtype=torch.int32, device="cuda")
    stack.decode_step(kv, x_next, h_out=h1, codes=c1, max_span=1024)
    restore()
    h2 = torch.empty_like(hA)
    c2 = torch.empty_like(c1)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        graph = stack.capture(kv, x_next, h_out=h2, codes=c2, max_span=1024)
        graph.replay()
    s.synchronize()
    tt.check()
    assert torch.equal(h1, h2) and torch.equal(c1, c2)
    assert torch.equal(kv.positions, snap[2] + 1)


def test_step_config2_48_lanes_28_layers(tt, orc):
    """Benchmark config[2] exactly as bench.py runs it: 28 layers, 48 lanes, 16 heads x 2048,
    KV lengths U[64, 1024] seed 0 in 32-position pages; against both reference arms."""
    lengths = np.random.default_rng(0).integers(64, 1025, 48)
    r = run_case(tt, orc, 48, 28, 2048, 16, 8, 6144, lengths, 16, 2048, 32, 41, fast_kv=True,
                 cpu_arm=True)
    agree = check_case(orc, r, 48, 32)
    g = r["g"]
    h = r["h"].cpu().numpy()
    logits = r["logits"].cpu().numpy()
    codes = r["codes"].cpu().numpy()
    cpu_h, cpu_l = rel(h, r["cpu_h"]), rel(logits, r["cpu_logits"])
    cpu_agree, cpu_exact, cpu_ties = agreement_with_f16_ties(codes, r["cpu_logits"], g)
    print(f"config[2] Metal arm: hidden rel {rel(h, r['want_h']):.2e}, logits rel "
          f"{rel(logits, r['want_logits']):.2e}, greedy agreement {agree:.4f}; CPU arm: hidden "
          f"rel {cpu_h:.2e}, logits rel {cpu_l:.2e}, greedy agreement {cpu_agree:.4f} "
          f"({cpu_exact:.4f} exact, {cpu_ties:.4f} on f16 ties)")
    assert cpu_h < 2e-2 and cpu_l < 2e-2
    assert cpu_agree >= 0.995, cpu_agree
