"""Loading a checkpoint by the reference's tensor names (crates/qwen3tts/src/qwen3.rs:61-119,
229-250; talker.rs:276-330, 575-605) on a B200: a small bf16 checkpoint with the talker's and
the predictor's names is written here, loaded through the safetensors reader into a talker
stack (codec head + codec_embedding) and a predictor, and run against the oracle built from
the same tensors."""
import numpy as np
import pytest
import torch

from _model import dev_f32
from test_weights import write_safetensors

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def bf16(rng, *shape, scale=0.02, offset=0.0):
    t = (torch.from_numpy(rng.standard_normal(shape).astype(np.float32)) * scale + offset)
    return t.to(torch.bfloat16)


def layer_tensors(rng, prefix, dim, heads, n_kv, ffn, hd=128):
    a = f"{prefix}.self_attn"
    return {f"{a}.q_proj.weight": bf16(rng, heads * hd, dim),
            f"{a}.k_proj.weight": bf16(rng, n_kv * hd, dim),
            f"{a}.v_proj.weight": bf16(rng, n_kv * hd, dim),
            f"{a}.o_proj.weight": bf16(rng, dim, heads * hd),
            f"{a}.q_norm.weight": bf16(rng, hd, scale=0.1, offset=1.0),
            f"{a}.k_norm.weight": bf16(rng, hd, scale=0.1, offset=1.0),
            f"{prefix}.mlp.gate_proj.weight": bf16(rng, ffn, dim),
            f"{prefix}.mlp.up_proj.weight": bf16(rng, ffn, dim),
            f"{prefix}.mlp.down_proj.weight": bf16(rng, dim, ffn),
            f"{prefix}.input_layernorm.weight": bf16(rng, dim, scale=0.1, offset=1.0),
            f"{prefix}.post_attention_layernorm.weight": bf16(rng, dim, scale=0.1, offset=1.0)}


def oracle_layer(orc, t, prefix, hd=128):
    f16 = lambda x: orc.f16_bits(x.float().numpy())
    f32 = lambda x: x.float().numpy()
    a = f"{prefix}.self_attn"
    qn = (t[f"{a}.q_norm.weight"].to(torch.float32) * (1.0 / hd ** 0.5)).numpy()
    return orc.Layer(attn_norm=f32(t[f"{prefix}.input_layernorm.weight"]),
                     ffn_norm=f32(t[f"{prefix}.post_attention_layernorm.weight"]),
                     wqkv=np.concatenate([f16(t[f"{a}.q_proj.weight"]), f16(t[f"{a}.k_proj.weight"]),
                                          f16(t[f"{a}.v_proj.weight"])]),
                     qk_norms=np.stack([qn, f32(t[f"{a}.k_norm.weight"])]).astype(np.float32),
                     wo=f16(t[f"{a}.o_proj.weight"]), gate=f16(t[f"{prefix}.mlp.gate_proj.weight"]),
                     up=f16(t[f"{prefix}.mlp.up_proj.weight"]),
                     down=f16(t[f"{prefix}.mlp.down_proj.weight"]))


def test_load_talker_and_predictor(tt, orc, tmp_path):
    from qwen3tts import Geometry, PagedKv
    from qwen3tts.weights import Weights, load_predictor, load_talker
    rng = np.random.default_rng(61)
    dim, vocab, steps, pvocab = 256, 384, 3, 128
    t = {}
    for i in range(2):
        t.update(layer_tensors(rng, f"talker.model.layers.{i}", dim, 4, 2, 512))
    t["talker.model.norm.weight"] = bf16(rng, dim, scale=0.1, offset=1.0)
    t["talker.codec_head.weight"] = bf16(rng, vocab, dim)
    t["talker.model.codec_embedding.weight"] = bf16(rng, vocab, dim)
    t.update(layer_tensors(rng, "talker.code_predictor.model.layers.0", dim, 4, 2, 512))
    t["talker.code_predictor.model.norm.weight"] = bf16(rng, dim, scale=0.1, offset=1.0)
    for i in range(steps):
        t[f"talker.code_predictor.lm_head.{i}.weight"] = bf16(rng, pvocab, dim)
        t[f"talker.code_predictor.model.codec_embedding.{i}.weight"] = bf16(rng, pvocab, dim)
    t["talker.code_predictor.small_to_mtp_projection.weight"] = bf16(rng, dim, dim)
    t["talker.code_predictor.small_to_mtp_projection.bias"] = bf16(rng, dim)
    path = str(tmp_path / "model.safetensors")
    write_safetensors(path, {k: ("BF16", v.view(torch.int16).numpy()) for k, v in t.items()})

    w = Weights(path)
    tg = Geometry(dim=dim, layers=2, heads=4, n_kv=2, ffn=512, rope_len=256, codebooks=1,
                  vocab=vocab)
    talker = load_talker(w, geo=tg)
    pg = Geometry(dim=dim, layers=1, heads=4, n_kv=2, ffn=512, rope_len=64, codebooks=1,
                  vocab=pvocab)
    pred = load_predictor(w, geo=pg, steps=steps)

    # the talker: one decode step from fresh lanes at position 0
    lanes = 4
    g = orc.Geometry(dim=dim, layers=2, heads=4, n_kv=2, ffn=512, codebooks=1, vocab=vocab)
    Ls = [oracle_layer(orc, t, f"talker.model.layers.{i}") for i in range(2)]
    final = t["talker.model.norm.weight"].float().numpy()
    kv = PagedKv(talker.geo, lanes, lanes * 2, 32, 2)
    for i in range(lanes):
        kv.admit(i, 64, 0)
    x = rng.standard_normal((lanes, dim)).astype(np.float32)
    h = torch.empty(lanes, dim, device="cuda")
    logits = torch.empty(lanes, vocab, device="cuda")
    talker.decode_step(kv, dev_f32(x), h_out=h, logits=logits, max_span=64)
    torch.cuda.synchronize()
    tt.check()
    cos, sin = orc.rope_table(64, 128, g.rope_base)
    kc = [np.zeros((lanes, 2, 64, 128), np.uint16) for _ in range(2)]
    vc = [np.zeros((lanes, 2, 64, 128), np.uint16) for _ in range(2)]
    want_h = orc.decode_step(x, Ls, final, kc, vc, np.zeros(lanes, np.int32), cos, sin, g)
    assert rel(h.cpu().numpy(), want_h) < 2e-2
    head = orc.f16_bits(t["talker.codec_head.weight"].float().numpy())
    assert rel(logits.cpu().numpy(), orc.proj(want_h, head)) < 2e-2

    # the predictor: one frame against the oracle's, from the loaded tensors
    pLs = [oracle_layer(orc, t, "talker.code_predictor.model.layers.0")]
    pfinal = t["talker.code_predictor.model.norm.weight"].float().numpy()
    f16 = lambda k: orc.f16_bits(t[k].float().numpy())
    tables = np.stack([f16(f"talker.code_predictor.model.codec_embedding.{i}.weight")
                       for i in range(steps)])
    resize = f16("talker.code_predictor.small_to_mtp_projection.weight")
    bias = t["talker.code_predictor.small_to_mtp_projection.bias"].float().numpy()
    heads = np.concatenate([f16(f"talker.code_predictor.lm_head.{i}.weight") for i in range(steps)])
    pw = orc.PredictorWeights(resize, bias, heads, tables, orc.resize_tables(tables, resize, bias))
    pog = orc.Geometry(dim=dim, layers=1, heads=4, n_kv=2, ffn=512, codebooks=1, vocab=pvocab)
    hidden = rng.standard_normal((lanes, dim)).astype(np.float32)
    code0 = orc.f16_value(orc.f16_bits(rng.standard_normal((lanes, dim)).astype(np.float32) * 0.02))
    pkv = pred.new_state(lanes)
    codes, total = pred.frame(pkv, dev_f32(hidden), dev_f32(code0))
    torch.cuda.synchronize()
    tt.check()
    got = codes.cpu().numpy().astype(np.uint32)
    want, want_sum, ties, mism = orc.predictor_frame(hidden, code0, pLs, pfinal, pw, pog,
                                                     forced=got, tie_tol=2e-3)
    assert mism == 0 and ties <= 1
    assert rel(total.cpu().numpy(), want_sum) < 1e-6
    w.close()
