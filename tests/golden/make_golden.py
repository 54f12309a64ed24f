"""Writes tests/golden/oracle_ops.npz: seeded inputs and the CPU oracle's outputs for each of
its operators (projection, RMSNorm, RoPE table, QK-norm + RoPE, decode attention, SwiGLU,
SnakeBeta, conv1d, argmax with bans, top-k sampling). The inputs are stored, not regenerated,
so the file pins the oracle's results against regressions on any machine:

    python tests/golden/make_golden.py

Run it only when the oracle's arithmetic is meant to change; tests/test_golden.py recomputes
every case from the stored inputs and compares."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle as orc  # noqa: E402


def cases() -> dict:
    rng = np.random.default_rng(2024)
    out = {}
    # projection: x f32, W f16 [n, k] (tts-nn Proj::Half, f32 accumulate)
    x = rng.standard_normal((6, 192), dtype=np.float32)
    w = orc.f16_bits(rng.standard_normal((256, 192), dtype=np.float32) * 0.02)
    out.update(proj_x=x, proj_w=w, proj_y=orc.proj(x, w), proj_y16=orc.proj(x, w, True))
    # RMSNorm, eps 1e-6
    x = rng.standard_normal((6, 256), dtype=np.float32) * 3
    g = rng.uniform(0.5, 1.5, 256).astype(np.float32)
    out.update(rms_x=x, rms_w=g, rms_y=orc.rms_norm(x, g, 1e-6))
    # RoPE table (f64 -> f32), theta 1e6, head_dim 128
    c, s = orc.rope_table(64, 128, 1e6)
    out.update(rope_cos=c, rope_sin=s)
    # QK-norm + RoPE: 4 lanes, 4 q heads, 2 kv heads
    qkv = rng.standard_normal((4, 8 * 128), dtype=np.float32)
    norms = rng.uniform(0.8, 1.2, (2, 128)).astype(np.float32)
    pos = np.array([0, 5, 31, 63], np.int32)
    q, k, v = orc.qk_rope(qkv, norms, c, s, pos, 4, 2, 1e-6)
    out.update(qkr_qkv=qkv, qkr_norms=norms, qkr_pos=pos, qkr_q=q, qkr_k=k, qkr_v=v)
    # decode attention: 2 lanes, 2 kv heads x gqa 2, cache 32, spans 32 and 17 (window start 4)
    qa = rng.standard_normal((2, 2, 2, 128), dtype=np.float32) * 0.1
    kc = orc.f16_bits(rng.standard_normal((2, 2, 32, 128), dtype=np.float32))
    vc = orc.f16_bits(rng.standard_normal((2, 2, 32, 128), dtype=np.float32))
    span = np.array([32, 17], np.int32)
    ws = np.array([0, 4], np.int32)
    out.update(att_q=qa, att_k=kc, att_v=vc, att_span=span, att_ws=ws,
               att_o=orc.decode_attention(qa, kc, vc, span, ws))
    # SwiGLU and SnakeBeta
    gg = rng.standard_normal((4, 256), dtype=np.float32) * 2
    uu = rng.standard_normal((4, 256), dtype=np.float32)
    out.update(swi_g=gg, swi_u=uu, swi_y=orc.swiglu(gg, uu))
    xs = rng.standard_normal((3, 64), dtype=np.float32)
    alpha = np.exp(rng.uniform(-1, 1, 64)).astype(np.float32)
    brecip = (1.0 / alpha).astype(np.float32)
    out.update(snk_x=xs, snk_a=alpha, snk_b=brecip, snk_y=orc.snake_beta(xs, alpha, brecip))
    # conv1d (channels-last), k 5, dilation 2, "same" padding, snake on load, bias, residual
    xc = rng.standard_normal((1, 40, 32), dtype=np.float32)
    wt = (rng.standard_normal((5, 32, 32), dtype=np.float32) * 0.05).astype(np.float32)
    bias = rng.standard_normal(32, dtype=np.float32) * 0.1
    ac = np.exp(rng.uniform(-1, 1, 32)).astype(np.float32)
    bc = (1.0 / ac).astype(np.float32)
    res = rng.standard_normal((1, 40, 32), dtype=np.float32)
    out.update(cnv_x=xc, cnv_w=wt, cnv_b=bias, cnv_a=ac, cnv_r=bc, cnv_res=res,
               cnv_y=orc.conv1d_nlc(xc, wt, bias, 2, 4, (ac, bc), res))
    # greedy argmax (ties: the last maximum wins; banned ids never win)
    lg = rng.standard_normal((4, 300), dtype=np.float32)
    lg[1, 17] = lg[1, 250] = 9.0
    banned = np.zeros(300, np.uint8)
    banned[[3, 250, 299]] = 1
    out.update(arg_logits=lg, arg_banned=banned, arg_codes=orc.argmax(lg),
               arg_codes_banned=orc.argmax(lg, banned))
    # top-k sampling with given draws
    lt = rng.standard_normal((5, 200), dtype=np.float32) * 2
    draws = rng.uniform(0, 1, 5).astype(np.float32)
    out.update(tk_logits=lt, tk_draws=draws, tk_codes=orc.topk_sample(lt, draws, 20, 0.9))
    return out


if __name__ == "__main__":
    path = os.path.join(HERE, "oracle_ops.npz")
    np.savez_compressed(path, **cases())
    print(path, os.path.getsize(path), "bytes")
