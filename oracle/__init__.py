"""CPU oracle for the qwen3tts hot path — TEST INFRASTRUCTURE ONLY.

Python face of oracle/oracle.c (a plain-C restatement of the reference's CPU arithmetic) plus
the compositions the reference builds from those ops: the decoder layer's decode step
(crates/qwen3tts/src/qwen3.rs:294-467), the greedy head pick, and the codec residual block.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this package; the
product library never links or calls it.

PARITY UNPINNED: the reference ships no golden vectors for these ops and cannot be built or
run here (Rust, no toolchain, no checkpoint). The restatement is cross-checked against
independent PyTorch-CPU formulas and the structural identities of the reference's own tests
(tests/test_oracle.py); tests/golden/ pins it against regressions.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
_lib = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def build() -> str:
    src = os.path.join(HERE, "oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB)
        L.orc_proj.argtypes = [u16p, u16p, f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_rms_norm.argtypes = [f32p, f32p, f32p, C.c_int64, C.c_int, C.c_float]
        L.orc_rope_table.argtypes = [C.c_int, C.c_int, C.c_double, f32p, f32p]
        L.orc_qk_rope.argtypes = [f32p, f32p, f32p, f32p, i32p, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_float, f32p, f32p, f32p]
        L.orc_decode_attention.argtypes = [f32p, u16p, u16p, i32p, i32p, C.c_int, C.c_int,
                                           C.c_int, C.c_int, C.c_int, f32p]
        L.orc_swiglu.argtypes = [f32p, f32p, f32p, C.c_int64]
        L.orc_snake_beta.argtypes = [f32p, f32p, f32p, f32p, C.c_int64, C.c_int]
        L.orc_conv1d_nlc.argtypes = [f32p, f32p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     f32p] + [C.c_int] * 7
        L.orc_argmax.argtypes = [f32p, C.c_void_p, u32p, C.c_int, C.c_int]
        L.orc_num_threads.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def threads() -> int:
    return lib().orc_num_threads()


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


# ---------------------------------------------------------------- f16 helpers
def f16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> IEEE binary16 bit patterns (round to nearest even)."""
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16))


def f16_value(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


# ---------------------------------------------------------------- ops (oracle.c)
def proj(x_f32: np.ndarray, w_bits: np.ndarray, round_f16: bool = False) -> np.ndarray:
    """Proj::Half: f16(x) . W^T with W `[n, k]` f16 bits; f32 accumulate."""
    lead = x_f32.shape[:-1]
    k = x_f32.shape[-1]
    n = w_bits.shape[0]
    xb = f16_bits(x_f32.reshape(-1, k))
    y = np.empty((xb.shape[0], n), np.float32)
    lib().orc_proj(xb, _c(w_bits, np.uint16), y, xb.shape[0], k, n, 1 if round_f16 else 0)
    return y.reshape(*lead, n)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_rms_norm(x, _c(w), y, x.size // x.shape[-1], x.shape[-1], float(eps))
    return y


def rope_table(length: int, hd: int, base: float) -> tuple[np.ndarray, np.ndarray]:
    c = np.empty((length, hd // 2), np.float32)
    s = np.empty((length, hd // 2), np.float32)
    lib().orc_rope_table(int(length), int(hd), float(base), c, s)
    return c, s


def qk_rope(qkv: np.ndarray, norms: np.ndarray, cos: np.ndarray, sin: np.ndarray,
            pos: np.ndarray, heads: int, n_kv: int, eps: float, hd: int = 128):
    b = qkv.shape[0]
    q = np.empty((b, heads, hd), np.float32)
    k = np.empty((b, n_kv, hd), np.float32)
    v = np.empty((b, n_kv, hd), np.float32)
    lib().orc_qk_rope(_c(qkv), _c(norms), _c(cos), _c(sin), _c(pos, np.int32), b, heads, n_kv,
                      hd, float(eps), q, k, v)
    return q, k, v


def decode_attention(q: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, span, wstart):
    """q `[b, n_kv, gqa, hd]` f32; caches `[b, n_kv, cap, hd]` f16 bits; span/wstart per lane."""
    b, n_kv, gqa, hd = q.shape
    cap = k_bits.shape[2]
    sp = np.broadcast_to(np.asarray(span, np.int32), (b,)).copy()
    ws = np.broadcast_to(np.asarray(wstart, np.int32), (b,)).copy()
    out = np.empty_like(_c(q))
    lib().orc_decode_attention(_c(q), _c(k_bits, np.uint16), _c(v_bits, np.uint16), sp, ws, b,
                               n_kv, gqa, hd, cap, out)
    return out


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = _c(g)
    y = np.empty_like(g)
    lib().orc_swiglu(g, _c(u), y, g.size)
    return y


def snake_beta(x: np.ndarray, alpha: np.ndarray, brecip: np.ndarray) -> np.ndarray:
    x = _c(x)
    y = np.empty_like(x)
    c = x.shape[-1]
    lib().orc_snake_beta(x, _c(alpha), _c(brecip), y, x.size // c, c)
    return y


def _vp(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def conv1d_nlc(x: np.ndarray, w_tap: np.ndarray, bias=None, dilation: int = 1,
               pad_left: int | None = None, snake=None, res=None) -> np.ndarray:
    """x `[b, L, cin]`, w_tap `[k, cin, cout]`; pad_left defaults to causal (k-1)*dilation."""
    b, length, cin = x.shape
    k, _, cout = w_tap.shape
    if pad_left is None:
        pad_left = (k - 1) * dilation
    x = _c(x)
    w = _c(w_tap)
    keep = [None if a is None else _c(a) for a in
            (bias, None if snake is None else snake[0], None if snake is None else snake[1], res)]
    y = np.empty((b, length, cout), np.float32)
    lib().orc_conv1d_nlc(x, w, *[_vp(a) for a in keep], y, b, length, cin, cout, k,
                         int(dilation), int(pad_left))
    return y


def argmax(logits: np.ndarray, banned: np.ndarray | None = None) -> np.ndarray:
    x = _c(logits)
    n = x.shape[-1]
    rows = x.size // n
    out = np.empty(rows, np.uint32)
    bb = None if banned is None else _c(banned, np.uint8)
    lib().orc_argmax(x, _vp(bb), out, rows, n)
    return out.reshape(x.shape[:-1])


# ---------------------------------------------------------------- compositions
@dataclass
class Geometry:
    dim: int = 2048
    layers: int = 28
    heads: int = 16
    n_kv: int = 8
    head_dim: int = 128
    ffn: int = 6144
    eps: float = 1e-6
    rope_base: float = 1e6
    codebooks: int = 16
    vocab: int = 2048


@dataclass
class Layer:
    """One decoder layer's weights as the reference holds them after load (qwen3.rs:61-119):
    projection weights f16 bits `[out, in]`, norms f32, qk_norms `[2, hd]` with the q weight
    already scaled by 1/sqrt(hd) (qwen3.rs:82-87)."""
    attn_norm: np.ndarray
    ffn_norm: np.ndarray
    wqkv: np.ndarray
    qk_norms: np.ndarray
    wo: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray


def synthetic_layer(rng: np.random.Generator, g: Geometry) -> Layer:
    """Seeded random-init layer with the distributions the benchmark configs name: projections
    ~N(0, 0.02) as f16, norm weights near 1, 1/sqrt(head_dim) folded into the q norm."""
    dim, hd = g.dim, g.head_dim
    nq = (g.heads + 2 * g.n_kv) * hd

    def w(n, k):
        return f16_bits(rng.standard_normal((n, k), dtype=np.float32) * 0.02)

    qn = rng.uniform(0.8, 1.2, hd).astype(np.float32) / np.sqrt(hd)
    kn = rng.uniform(0.8, 1.2, hd).astype(np.float32)
    return Layer(attn_norm=rng.uniform(0.8, 1.2, dim).astype(np.float32),
                 ffn_norm=rng.uniform(0.8, 1.2, dim).astype(np.float32),
                 wqkv=w(nq, dim), qk_norms=np.stack([qn, kn]).astype(np.float32),
                 wo=w(dim, g.heads * hd), gate=w(g.ffn, dim), up=w(g.ffn, dim),
                 down=w(dim, g.ffn))


def decode_step(x: np.ndarray, layers: list[Layer], final_norm: np.ndarray, kcache: list,
                vcache: list, pos: np.ndarray, cos: np.ndarray, sin: np.ndarray, g: Geometry,
                round_f16: bool = False) -> np.ndarray:
    """Stack::forward at t == 1 (crates/qwen3tts/src/qwen3.rs:294-467), composed CPU form
    (:358-394), with a per-lane position. kcache/vcache: per layer `[b, n_kv, cap, hd]` f16
    bits, updated in place at each lane's position. Returns the final-normed hidden f32."""
    b = x.shape[0]
    gqa = g.heads // g.n_kv
    h = _c(x).copy()
    pos = np.asarray(pos, np.int32)
    lanes = np.arange(b)
    for li, L in enumerate(layers):
        normed = rms_norm(h, L.attn_norm, g.eps)
        qkv = proj(normed, L.wqkv, round_f16)
        q, k, v = qk_rope(qkv, L.qk_norms, cos, sin, pos, g.heads, g.n_kv, g.eps, g.head_dim)
        kcache[li][lanes, :, pos, :] = f16_bits(k)
        vcache[li][lanes, :, pos, :] = f16_bits(v)
        att = decode_attention(q.reshape(b, g.n_kv, gqa, g.head_dim), kcache[li], vcache[li],
                               pos + 1, 0)
        h = h + proj(att.reshape(b, g.heads * g.head_dim), L.wo, round_f16)
        normed = rms_norm(h, L.ffn_norm, g.eps)
        tail = swiglu(proj(normed, L.gate, round_f16), proj(normed, L.up, round_f16))
        h = h + proj(tail, L.down, round_f16)
    return rms_norm(h, final_norm, g.eps)


def proj_rows(x_f32: np.ndarray, w_bits: np.ndarray, round_f16: bool = True) -> np.ndarray:
    """`matmul_2d(f16(x), W^T)` for many rows (crates/tts-nn/src/lib.rs:438-459, 516-528): f16
    operands, f32 accumulation (a BLAS sgemm here; the `gemm` crate's accumulation order is not
    pinned), the result rounded to f16 and cast back to f32 when `round_f16`, as the CPU arm
    and every projection of more than 48 rows leave it."""
    xf = f16_value(f16_bits(x_f32.reshape(-1, x_f32.shape[-1])))
    y = xf @ f16_value(w_bits).T
    if round_f16:
        y = f16_value(f16_bits(y))
    return y.astype(np.float32).reshape(*x_f32.shape[:-1], w_bits.shape[0])


def prefill(x: np.ndarray, layers: list[Layer], final_norm: np.ndarray, kcache: list,
            vcache: list, start: int, cos: np.ndarray, sin: np.ndarray, g: Geometry,
            round_f16: bool = True) -> np.ndarray:
    """Stack::forward at t > 1 for one group of lanes sharing `start` (crates/qwen3tts/src/
    qwen3.rs:294-467, the prefill branch :415-444), the CPU arm by default:
      * every projection through matmul_2d with an f16 result (`round_f16`);
      * QK-norm and RoPE per row at position start + i (qwen3.rs:358-394), K and V written to
        the f16 caches, and kept at f32 as the new positions' `fresh` k/v;
      * attention of the new rows over the cached prefix [0, start) read back from f16 and
        concatenated with the fresh f32 k/v, scores q.K^T in f32, the causal mask (column >
        row -> -inf, causal_window_mask), softmax_last_dim, probs.V.
    x f32 [b, t, dim]; caches per layer [b, n_kv, cap, hd] f16 bits, written in place at
    [start, start + t). Returns every row's final-normed hidden [b, t, dim]."""
    b, t, dim = x.shape
    gqa = g.heads // g.n_kv
    hd = g.head_dim
    h = _c(x).reshape(b * t, dim).copy()
    pos = np.tile(np.arange(start, start + t, dtype=np.int32), b)
    span = start + t
    mask = np.where(np.arange(span)[None, :] > (start + np.arange(t))[:, None], -np.inf,
                    0.0).astype(np.float32)  # [t, span]
    for li, L in enumerate(layers):
        normed = rms_norm(h, L.attn_norm, g.eps)
        qkv = proj_rows(normed, L.wqkv, round_f16)
        q, k, v = qk_rope(qkv, L.qk_norms, cos, sin, pos, g.heads, g.n_kv, g.eps, hd)
        q = q.reshape(b, t, g.n_kv, gqa, hd)
        k = k.reshape(b, t, g.n_kv, hd)
        v = v.reshape(b, t, g.n_kv, hd)
        kcache[li][:, :, start:span] = f16_bits(k.transpose(0, 2, 1, 3))
        vcache[li][:, :, start:span] = f16_bits(v.transpose(0, 2, 1, 3))
        att = np.empty((b, t, g.n_kv, gqa, hd), np.float32)
        for lane in range(b):
            for kh in range(g.n_kv):
                k_all = np.concatenate([f16_value(kcache[li][lane, kh, :start]), k[lane, :, kh]])
                v_all = np.concatenate([f16_value(vcache[li][lane, kh, :start]), v[lane, :, kh]])
                for j in range(gqa):
                    sc = q[lane, :, kh, j] @ k_all.T + mask  # [t, span]
                    sc = sc - sc.max(axis=1, keepdims=True)
                    e = np.exp(sc)
                    p = e / e.sum(axis=1, keepdims=True)
                    att[lane, :, kh, j] = p @ v_all
        h = h + proj_rows(att.reshape(b * t, g.heads * hd), L.wo, round_f16)
        normed = rms_norm(h, L.ffn_norm, g.eps)
        tail = swiglu(proj_rows(normed, L.gate, round_f16), proj_rows(normed, L.up, round_f16))
        h = h + proj_rows(tail, L.down, round_f16)
    return rms_norm(h, final_norm, g.eps).reshape(b, t, dim)


def heads_pick(hidden: np.ndarray, heads_bits: np.ndarray, g: Geometry, round_f16: bool = False):
    """Codebook heads `[codebooks * vocab, dim]` f16 and the greedy pick per head. With
    `round_f16` the logits are rounded to f16 as the CPU arm's `matmul_2d(..).to_dtype(f32)`
    leaves them (crates/tts-nn/src/lib.rs:519-528), which makes exact ties common."""
    logits = proj(hidden, heads_bits, round_f16)
    b = hidden.shape[0]
    codes = argmax(logits.reshape(b, g.codebooks, g.vocab))
    return logits, codes


def embed_sum(codes: np.ndarray, embed_bits: np.ndarray) -> np.ndarray:
    """Sum over codebooks of each picked code's embedding row (talker.rs:528-550)."""
    cb = embed_bits.shape[0]
    rows = [f16_value(embed_bits[q][codes[:, q]]) for q in range(cb)]
    out = np.zeros_like(rows[0])
    for r in rows:
        out = out + r
    return out


def snake_residual_block(x: np.ndarray, convs, dilations=(1, 3, 9), same: bool = True):
    """The config's codec residual block, channels-last: for each dilation,
    x = x + conv_d(snake_d(x)) with k = 7 ("same" padding when `same`, else causal).
    convs: list of (w_tap [k, c, c], bias [c], alpha [c], brecip [c])."""
    for (w, bias, alpha, brecip), d in zip(convs, dilations):
        k = w.shape[0]
        pad = (k - 1) * d // 2 if same else (k - 1) * d
        x = conv1d_nlc(x, w, bias, d, pad, snake=(alpha, brecip), res=x)
    return x


# ---------------------------------------------------------------- depth predictor
@dataclass
class PredictorWeights:
    """The code predictor's own weights besides its stack (talker.rs:255-330): the talker-to-
    predictor projection (small_to_mtp_projection, with bias), one head per residual codebook,
    the residual codebooks' tables at talker width, and `resized` = each table through the
    projection, precomputed at load (talker.rs:268-273, 315-323)."""
    resize: np.ndarray       # f16 bits [dim, embed_dim]
    resize_bias: np.ndarray  # f32 [dim]
    heads: np.ndarray        # f16 bits [steps * vocab, dim]
    tables: np.ndarray       # f16 bits [steps, vocab, embed_dim]
    resized: np.ndarray      # f32 [steps, vocab, dim]

    @property
    def steps(self) -> int:
        return self.tables.shape[0]


def linear(x: np.ndarray, w_bits: np.ndarray, bias: np.ndarray | None) -> np.ndarray:
    """`Linear::forward` in f32 (an f32 weight, f32 inputs, plus bias), computed in f64 and
    rounded once to f32."""
    y = np.asarray(x, np.float64) @ f16_value(w_bits).astype(np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y.astype(np.float32)


def resize_tables(tables_bits: np.ndarray, resize_bits: np.ndarray, bias) -> np.ndarray:
    """talker.rs:315-323: `resized[i] = host.forward(tables[i])`, f32, bias folded in."""
    return np.stack([linear(f16_value(t), resize_bits, bias) for t in tables_bits])


def synthetic_predictor(rng: np.random.Generator, g: Geometry, steps: int,
                        embed_dim: int) -> PredictorWeights:
    """Seeded random-init predictor weights: projections and tables ~N(0, 0.02) as f16, bias
    ~N(0, 0.02)."""
    def w(*shape):
        return f16_bits(rng.standard_normal(shape, dtype=np.float32) * 0.02)

    resize = w(g.dim, embed_dim)
    bias = (rng.standard_normal(g.dim, dtype=np.float32) * 0.02).astype(np.float32)
    heads = w(steps * g.vocab, g.dim)
    tables = w(steps, g.vocab, embed_dim)
    return PredictorWeights(resize, bias, heads, tables, resize_tables(tables, resize, bias))


def topk_interval(logits: np.ndarray, k: int, temperature: float, pick: int):
    """Where `pick` sits in the host sampler's walk over one row: (lo, hi) of the scaled draw
    u * renorm that selects it, or None when it is not among the k best."""
    t = np.float32(temperature if temperature > 0 else 1.0)
    l = np.asarray(logits, np.float32)
    order = sorted(range(l.shape[0]), key=lambda i: (-float(l[i]), i))[:k]
    if pick not in order:
        return None
    p = np.exp((l[order].astype(np.float64) - float(l[order[0]])) / float(t))
    c = np.concatenate([[0.0], np.cumsum(p / p.sum())])
    j = order.index(pick)
    return c[j], c[j + 1]


def predictor_frame(hidden: np.ndarray, code0_embed: np.ndarray, layers: list[Layer],
                    final_norm: np.ndarray, pw: PredictorWeights, g: Geometry,
                    forced: np.ndarray | None = None, tie_tol: float = 0.0,
                    draws: np.ndarray | None = None, top_k: int = 50,
                    temperature: float = 0.9, logit_tol: float = 0.0):
    """Predictor::frame_batch with greedy picks (talker.rs:407-468) and gather_sum (:528-550).

    hidden, code0_embed f32 [b, embed_dim]. The two-position prefill (talker.rs:416-420) is run
    as decode steps at positions 0 and 1, which the causal mask makes the same computation. Each
    depth step: head i on the last hidden, the greedy pick, then (before the last) the stack on
    resized[i][code]. Returns (codes u32 [b, steps], sum f32 [b, embed_dim], ties, mismatches).

    `forced` (u32 [b, steps], e.g. the device's picks) is followed wherever its logit is within
    `tie_tol` of the maximum: a near-tie resolved the other way by a different but equally valid
    accumulation order, which the chain then continues from. Picks outside that band count in
    `mismatches` and the oracle keeps its own.

    With `draws` (f32 [steps, b]) the picks are the host sampler's top-k draws instead
    (depth_on_device, talker.rs:478-515); a forced pick is then followed when the scaled draw
    lies within `tie_tol` of its interval of the walk, or when its logit is within `logit_tol`
    of the oracle pick's (two near-equal candidates whose order in the walk, and so whose
    intervals, another accumulation order swaps)."""
    b = hidden.shape[0]
    steps = pw.steps
    cap = steps + 2
    cos, sin = rope_table(cap, g.head_dim, g.rope_base)
    kc = [np.zeros((b, g.n_kv, cap, g.head_dim), np.uint16) for _ in layers]
    vc = [np.zeros((b, g.n_kv, cap, g.head_dim), np.uint16) for _ in layers]
    x0 = linear(hidden, pw.resize, pw.resize_bias)
    x1 = linear(code0_embed, pw.resize, pw.resize_bias)
    decode_step(x0, layers, final_norm, kc, vc, np.zeros(b, np.int32), cos, sin, g)
    h = decode_step(x1, layers, final_norm, kc, vc, np.ones(b, np.int32), cos, sin, g)
    codes = np.zeros((b, steps), np.uint32)
    ties = mismatches = 0
    for i in range(steps):
        logits = proj(h, pw.heads[i * g.vocab:(i + 1) * g.vocab])
        pick = argmax(logits) if draws is None else topk_sample(logits, draws[i], top_k,
                                                                 temperature)
        if forced is not None:
            for lane in range(b):
                f = int(forced[lane, i])
                if f == int(pick[lane]):
                    continue
                if draws is None:
                    near = 0 <= f < g.vocab and logits[lane, f] >= logits[lane, pick[lane]] - tie_tol
                else:
                    iv = topk_interval(logits[lane], top_k, temperature, f)
                    u = float(draws[i][lane])
                    o = int(pick[lane])
                    near = iv is not None and (iv[0] - tie_tol <= u <= iv[1] + tie_tol or
                                               abs(float(logits[lane, f] - logits[lane, o]))
                                               <= logit_tol)
                if near:
                    pick[lane] = f
                    ties += 1
                else:
                    mismatches += 1
        codes[:, i] = pick
        if i + 1 < steps:
            x = pw.resized[i][pick.astype(np.int64)]
            h = decode_step(x, layers, final_norm, kc, vc, np.full(b, 2 + i, np.int32), cos, sin, g)
    rows = [f16_value(pw.tables[i][codes[:, i].astype(np.int64)]) for i in range(steps)]
    acc = np.zeros_like(rows[0])
    for r in rows:
        acc = acc + r
    return codes, np.asarray(code0_embed, np.float32) + acc, ties, mismatches


# ---------------------------------------------------------------- the talker's frame
def penalize(x: np.float32, times: int, penalty: np.float32) -> np.float32:
    """The repetition penalty of sample_with_u (crates/qwen3tts/src/talker.rs:167-179) applied
    for `times` occurrences of one id in the history: each occurrence, while the logit is finite,
    divides it by the penalty if positive, else multiplies it, one f32 operation at a time."""
    for _ in range(times):
        if not np.isfinite(x):
            break
        x = np.float32(x / penalty) if x > 0 else np.float32(x * penalty)
    return x


def talker_pick(logits: np.ndarray, banned, seen: list, frames: np.ndarray, eos: int,
                min_new: int, penalty: float, forced: np.ndarray | None = None,
                tie_tol: float = 0.0):
    """sample_with_u with greedy on (crates/qwen3tts/src/talker.rs:154-189) for each row: banned
    ids (and eos while the row has fewer than `min_new` frames, :971-981) to -inf, then the
    repetition penalty once per entry of the row's history `seen[r]` (a list of emitted ids with
    repeats, as `seen[lane].push(c)` builds it, :987), then the last of equal maxima. `forced`
    picks within `tie_tol` of the row's maximum are followed (near-ties resolved the other way
    by a different accumulation order). Returns (picks, ties, mismatches)."""
    b, n = logits.shape
    picks = np.zeros(b, np.uint32)
    ties = mismatches = 0
    pen = np.float32(penalty)
    for r in range(b):
        l = logits[r].astype(np.float32).copy()
        for i in banned:
            l[i] = -np.inf
        if frames[r] < min_new and 0 <= eos < n:
            l[eos] = -np.inf
        if penalty != 1.0:
            # every occurrence of an id acts on that id's logit alone, so the entries can be
            # grouped by id without changing any result
            times: dict[int, int] = {}
            for i in seen[r]:
                if 0 <= int(i) < n:
                    times[int(i)] = times.get(int(i), 0) + 1
            for i, t in times.items():
                l[i] = penalize(l[i], t, pen)
        best = int(np.flatnonzero(l == l.max())[-1])
        if forced is not None and int(forced[r]) != best:
            f = int(forced[r])
            if 0 <= f < n and np.isfinite(l[f]) and l[f] >= l[best] - tie_tol:
                best = f
                ties += 1
            else:
                mismatches += 1
        picks[r] = best
    return picks, ties, mismatches


@dataclass
class TalkerState:
    """One group's talker-side state: per-layer caches [b, n_kv, cap, hd] f16 bits, positions,
    the pick rule's history (per lane, the emitted ids with repeats) and frame counts, and the
    next input rows."""
    kc: list
    vc: list
    pos: np.ndarray
    seen: list
    frames: np.ndarray
    x: np.ndarray


def talker_frame(st: TalkerState, layers: list[Layer], final_norm: np.ndarray, g: Geometry,
                 codec_head: np.ndarray, codec_embed: np.ndarray, banned, eos: int,
                 min_new: int, penalty: float, p_layers: list[Layer], p_final: np.ndarray,
                 pw: PredictorWeights, pg: Geometry, text_rows: np.ndarray, pad: np.ndarray,
                 forced0=None, forced=None, tie_tol: float = 0.0,
                 tie_tol0: float | None = None, stats: dict | None = None):
    """One iteration of Talker::generate_batch with greedy picks (talker.rs:953-1057), started
    from the step that feeds the talker stack: Stack::forward on `st.x` at each lane's
    position, codec head, pick, code 0's codec_embed row, the predictor's frame on the hidden
    state and that row, then the sum plus the lane's text row (trailing row frames - 1, else the
    pad row) as the next input. `tie_tol0` (default `tie_tol`) is the near-tie band of code 0's
    pick, `tie_tol` the predictor's; `stats` (optional) receives the code-0 and predictor tie
    counts separately. Updates `st`; returns (code0, codes, ties, mismatches)."""
    cap = st.kc[0].shape[2]
    cos, sin = rope_table(cap + 1, g.head_dim, g.rope_base)
    h = decode_step(st.x, layers, final_norm, st.kc, st.vc, st.pos, cos, sin, g)
    st.pos = st.pos + 1
    logits = proj(h, codec_head)
    code0, t0, m0 = talker_pick(logits, banned, st.seen, st.frames, eos, min_new, penalty,
                                forced0, tie_tol if tie_tol0 is None else tie_tol0)
    for r, c in enumerate(code0):
        if int(c) != eos:
            st.seen[r].append(int(c))
    st.frames = st.frames + 1
    code0_embed = f16_value(codec_embed[code0.astype(np.int64)])
    codes, total, t1, m1 = predictor_frame(h, code0_embed, p_layers, p_final, pw, pg, forced,
                                           tie_tol)
    if stats is not None:
        stats["ties0"] = stats.get("ties0", 0) + t0
        stats["ties_predictor"] = stats.get("ties_predictor", 0) + t1
    length = text_rows.shape[1]
    for r in range(total.shape[0]):
        t = int(st.frames[r]) - 1
        total[r] = total[r] + (text_rows[r, t] if 0 <= t < length else pad)
    st.x = total
    return code0, codes, t0 + t1, m0 + m1


# ---------------------------------------------------------------- top-k sampling
def topk_sample(logits: np.ndarray, draws: np.ndarray, k: int, temperature: float) -> np.ndarray:
    """The host sampler at top_p = 1 and no penalty (crates/qwen3tts/src/talker.rs:189-236,
    the form crates/tts-nn/src/topk.rs:122-142 tests the device kernel against): the k best ids
    (value descending, index ascending on ties), p_j = exp((l_j - max) / t) in f32 normalised
    by their sequential sum, u = draw * (sum of the normalised p), walked down in order."""
    t = np.float32(temperature if temperature > 0 else 1.0)
    out = np.zeros(logits.shape[0], np.uint32)
    for r in range(logits.shape[0]):
        l = np.asarray(logits[r], np.float32)
        order = sorted(range(l.shape[0]), key=lambda i: (-float(l[i]), i))[:k]
        mx = l[order[0]]
        p = [np.float32(np.exp(np.float32((l[i] - mx) / t))) for i in order]
        total = np.float32(0)
        for q in p:
            total = np.float32(total + q)
        p = [np.float32(q / total) for q in p]
        renorm = np.float32(0)
        for q in p:
            renorm = np.float32(renorm + q)
        u = np.float32(np.float32(draws[r]) * renorm)
        pick = order[k - 1]
        for j, q in enumerate(p):
            u = np.float32(u - q)
            if u <= 0:
                pick = order[j]
                break
        out[r] = pick
    return out


# ---------------------------------------------------------------- codec front (numpy)
def layer_norm(x: np.ndarray, w: np.ndarray, b, eps: float) -> np.ndarray:
    """layer_norm_plain + affine (crates/tts-nn/src/lib.rs:1006-1035), f64 then f32."""
    x = np.asarray(x, np.float64)
    mean = x.mean(-1, keepdims=True)
    c = x - mean
    var = (c * c).mean(-1, keepdims=True)
    y = c / np.sqrt(var + eps) * np.asarray(w, np.float64)
    if b is not None:
        y = y + np.asarray(b, np.float64)
    return y.astype(np.float32)


def gelu_exact(x: np.ndarray) -> np.ndarray:
    """0.5 x (1 + erf(x / sqrt 2)) (lib.rs:1129)."""
    from scipy.special import erf
    x = np.asarray(x, np.float64)
    return (0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))).astype(np.float32)


def depthwise(x: np.ndarray, w: np.ndarray, bias) -> np.ndarray:
    """nlc::depthwise (crates/tts-nn/src/nlc.rs:232-256): x [b, L, C], w [C, k], causal."""
    b, L, C = x.shape
    k = w.shape[1]
    xp = np.concatenate([np.zeros((b, k - 1, C), np.float64), np.asarray(x, np.float64)], 1)
    y = sum(xp[:, t:t + L] * np.asarray(w[:, t], np.float64) for t in range(k))
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y.astype(np.float32)


def rope_rows(x: np.ndarray, col0: int, heads: int, hd: int, cos: np.ndarray,
              sin: np.ndarray, pos0: int = 0) -> np.ndarray:
    """Half-split rotate_half RoPE (candle_nn::rotary_emb::rope) on heads of x [T, ld]."""
    y = np.asarray(x, np.float32).copy()
    T = y.shape[0]
    half = hd // 2
    c = cos[pos0:pos0 + T][:, None, :]
    s = sin[pos0:pos0 + T][:, None, :]
    blk = y[:, col0:col0 + heads * hd].reshape(T, heads, hd)
    a, b = blk[..., :half].copy(), blk[..., half:].copy()
    blk[..., :half] = a * c - b * s
    blk[..., half:] = b * c + a * s
    y[:, col0:col0 + heads * hd] = blk.reshape(T, heads * hd)
    return y


def window_attention(qkv: np.ndarray, heads: int, hd: int, window: int, scale: float):
    """The prefill branch of Stack::forward (qwen3.rs:409-444) with causal_window_mask
    (lib.rs:1210-1225) for one sequence, gqa 1: qkv [T, 3 heads hd] f32, in f64."""
    T = qkv.shape[0]
    q = qkv[:, :heads * hd].reshape(T, heads, hd).astype(np.float64)
    k = qkv[:, heads * hd:2 * heads * hd].reshape(T, heads, hd).astype(np.float64)
    v = qkv[:, 2 * heads * hd:].reshape(T, heads, hd).astype(np.float64)
    s = np.einsum("thd,jhd->htj", q, k) * scale
    rows = np.arange(T)[:, None]
    cols = np.arange(T)[None, :]
    lo = rows + 1 - window if window > 0 else np.zeros_like(rows)
    mask = (cols > rows) | (cols < lo)
    s = np.where(mask[None], -np.inf, s)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    o = np.einsum("htj,jhd->thd", p, v)
    return o.reshape(T, heads * hd).astype(np.float32)


def rvq_gather(codes: np.ndarray, q0: int, tables: np.ndarray) -> np.ndarray:
    """Rvq::decode's lookups (codec.rs:285-299): sum over the stack's codebooks, in order."""
    nq = tables.shape[0]
    out = np.zeros((codes.shape[0], tables.shape[2]), np.float32)
    for q in range(nq):
        out = out + tables[q][codes[:, q0 + q].astype(np.int64)]
    return out
