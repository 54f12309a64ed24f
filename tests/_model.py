"""Seeded synthetic talker weights and decode state shared by the oracle and GPU tests.

Benchmark config[2]: random-init f16 projection weights ~N(0, 0.02), norm weights near 1,
KV caches prefilled ~N(0, 1), lane lengths per test. No checkpoint exists in this image.
"""
from __future__ import annotations

import numpy as np


def make_layer(orc, rng, g):
    return orc.synthetic_layer(rng, g)


def normal_f16_table(rng, shape):
    """~N(0, 1) f16 bits drawn from a seeded table of 65,536 normal values: the same
    distribution as drawing each element, fast enough for the benchmark's multi-GB caches."""
    import oracle
    table = oracle.f16_bits(rng.standard_normal(65536, dtype=np.float32))
    n = int(np.prod(shape))
    return table[np.frombuffer(rng.bytes(2 * n), np.uint16)].reshape(shape)


def make_talker(orc, lanes, layers, dim, heads, n_kv, ffn, cap, seed, codebooks=0, vocab=0,
                lengths=None, fast_kv=False):
    rng = np.random.default_rng(seed)
    g = orc.Geometry(dim=dim, layers=layers, heads=heads, n_kv=n_kv, ffn=ffn,
                     codebooks=codebooks, vocab=vocab)
    Ls = [make_layer(orc, rng, g) for _ in range(layers)]
    final = rng.uniform(0.8, 1.2, dim).astype(np.float32)
    if fast_kv:
        kc = [normal_f16_table(rng, (lanes, n_kv, cap, 128)) for _ in range(layers)]
        vc = [normal_f16_table(rng, (lanes, n_kv, cap, 128)) for _ in range(layers)]
    else:
        kc = [orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
              for _ in range(layers)]
        vc = [orc.f16_bits(rng.standard_normal((lanes, n_kv, cap, 128), dtype=np.float32))
              for _ in range(layers)]
    if lengths is None:
        pos = rng.integers(cap // 2, cap - 1, lanes).astype(np.int32)
    else:
        pos = np.asarray(lengths, np.int32)
    x = rng.standard_normal((lanes, dim), dtype=np.float32)
    return g, Ls, final, kc, vc, pos, x


def make_heads(orc, seed, g):
    rng = np.random.default_rng(seed)
    heads = orc.f16_bits(rng.standard_normal((g.codebooks * g.vocab, g.dim), dtype=np.float32) * 0.02)
    embed = orc.f16_bits(rng.standard_normal((g.codebooks, g.vocab, g.dim), dtype=np.float32) * 0.02)
    return heads, embed


# ---------------------------------------------------------------- device transfer (GPU tests)
def dev_f16(bits, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.float16).to(device)


def dev_f32(a, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


def device_stack(orc, g, layers, final, heads=None, embed=None, rope_len=4096):
    import torch
    from qwen3tts import Geometry, LayerTensors, Stack
    import ttsnn
    geo = Geometry(dim=g.dim, layers=g.layers, heads=g.heads, n_kv=g.n_kv, head_dim=g.head_dim,
                   ffn=g.ffn, eps=g.eps, rope_base=g.rope_base, rope_len=rope_len,
                   codebooks=g.codebooks if heads is not None else 0,
                   vocab=g.vocab if heads is not None else 0)
    lts = []
    for L in layers:
        lts.append(LayerTensors.from_plain(dev_f32(L.attn_norm), dev_f32(L.ffn_norm), dev_f16(L.wqkv),
                                           dev_f32(L.qk_norms), dev_f16(L.wo),
                                           ttsnn.interleave_gate_up(dev_f16(L.gate), dev_f16(L.up)),
                                           dev_f16(L.down)))
    return Stack(geo, lts, dev_f32(final), None if heads is None else dev_f16(heads),
                 None if embed is None else dev_f16(embed))


def paged_from_contiguous(geo, kc, vc, pos, block_size, seed, spare_blocks=3, capacity=None):
    """Scatter the oracle's contiguous caches [lanes, n_kv, cap, 128] (per layer) into pages,
    with the lanes' pages drawn in a shuffled order so the block table is exercised."""
    import torch
    from qwen3tts import PagedKv
    lanes, n_kv, cap, hd = kc[0].shape
    cap_use = capacity or cap
    per_lane = -(-cap_use // block_size)
    num_blocks = lanes * per_lane + spare_blocks
    kv = PagedKv(geo, lanes, num_blocks, block_size, per_lane)
    rng = np.random.default_rng(seed)
    order = rng.permutation(num_blocks)
    table = order[:lanes * per_lane].reshape(lanes, per_lane).astype(np.int32)
    for i in range(lanes):
        kv.admit_pages(i, table[i].tolist(), int(pos[i]))
    for li in range(len(kc)):
        for src, pool in ((kc[li], kv.k), (vc[li], kv.v)):
            padded = np.zeros((lanes, n_kv, per_lane * block_size, hd), np.uint16)
            padded[:, :, :min(cap, per_lane * block_size)] = src[:, :, :per_lane * block_size]
            pages = padded.reshape(lanes, n_kv, per_lane, block_size, hd).transpose(0, 2, 1, 3, 4)
            host = np.zeros((num_blocks, n_kv, block_size, hd), np.uint16)
            host[table.reshape(-1)] = pages.reshape(lanes * per_lane, n_kv, block_size, hd)
            pool[li].copy_(dev_f16(host))
    return kv, table


def gather_pages(kv_pool_layer, table, lanes, n_kv, length, block_size):
    """Pages back to the contiguous [lanes, n_kv, length, 128] layout (f16 bits)."""
    pool = kv_pool_layer.cpu().view(__import__("torch").int16).numpy().view(np.uint16)
    per_lane = table.shape[1]
    out = pool[table.reshape(-1)].reshape(lanes, per_lane, n_kv, block_size, 128)
    out = out.transpose(0, 2, 1, 3, 4).reshape(lanes, n_kv, per_lane * block_size, 128)
    return out[:, :, :length]


# ---------------------------------------------------------------- depth predictor
def make_predictor(orc, lanes, dim, layers, heads, n_kv, ffn, vocab, steps, embed_dim, seed):
    """Seeded predictor weights and one frame's inputs: the talker's normed hidden ~N(0, 1) and
    its code-0 embedding (an f16 table row ~N(0, 0.02))."""
    rng = np.random.default_rng(seed)
    g = orc.Geometry(dim=dim, layers=layers, heads=heads, n_kv=n_kv, ffn=ffn, codebooks=1,
                     vocab=vocab)
    Ls = [make_layer(orc, rng, g) for _ in range(layers)]
    final = rng.uniform(0.8, 1.2, dim).astype(np.float32)
    pw = orc.synthetic_predictor(rng, g, steps, embed_dim)
    hidden = rng.standard_normal((lanes, embed_dim), dtype=np.float32)
    code0 = orc.f16_value(orc.f16_bits(rng.standard_normal((lanes, embed_dim), dtype=np.float32)
                                       * 0.02))
    return g, Ls, final, pw, hidden, code0


def device_predictor(orc, g, layers, final, pw):
    """The predictor on the device: its stack (codebooks 1, heads supplied per depth step) and
    weights, with the oracle's f32 resized tables."""
    from qwen3tts import Geometry, LayerTensors, Predictor, Stack
    import ttsnn
    geo = Geometry(dim=g.dim, layers=g.layers, heads=g.heads, n_kv=g.n_kv, head_dim=g.head_dim,
                   ffn=g.ffn, eps=g.eps, rope_base=g.rope_base, rope_len=64, codebooks=1,
                   vocab=g.vocab)
    lts = [LayerTensors.from_plain(dev_f32(L.attn_norm), dev_f32(L.ffn_norm), dev_f16(L.wqkv),
                                   dev_f32(L.qk_norms), dev_f16(L.wo),
                                   ttsnn.interleave_gate_up(dev_f16(L.gate), dev_f16(L.up)),
                                   dev_f16(L.down)) for L in layers]
    stack = Stack(geo, lts, dev_f32(final))
    return Predictor(stack, dev_f16(pw.resize), dev_f32(pw.resize_bias), dev_f16(pw.heads),
                     dev_f16(pw.tables), dev_f32(pw.resized))
