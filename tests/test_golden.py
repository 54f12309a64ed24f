"""The CPU oracle against its committed golden fixtures (tests/golden/oracle_ops.npz, written by
tests/golden/make_golden.py from stored seeded inputs): every operator recomputed from the
stored inputs must reproduce the stored outputs, bit-exact for integer results (argmax, top-k
picks) and within 1e-6 relative for floating point (the same C code; only a compiler's
contraction choices may move the last bit). This pins the oracle that every GPU parity test
compares against: a change to its arithmetic shows up here first."""
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "oracle_ops.npz"))


def close(a, b, tol=1e-6):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)) <= tol


def test_projection_and_norms(orc, gold):
    g = gold
    assert close(orc.proj(g["proj_x"], g["proj_w"]), g["proj_y"])
    assert close(orc.proj(g["proj_x"], g["proj_w"], True), g["proj_y16"])
    assert close(orc.rms_norm(g["rms_x"], g["rms_w"], 1e-6), g["rms_y"])
    c, s = orc.rope_table(64, 128, 1e6)
    assert np.array_equal(c, g["rope_cos"]) and np.array_equal(s, g["rope_sin"])


def test_qk_rope_and_attention(orc, gold):
    g = gold
    q, k, v = orc.qk_rope(g["qkr_qkv"], g["qkr_norms"], g["rope_cos"], g["rope_sin"],
                          g["qkr_pos"], 4, 2, 1e-6)
    assert close(q, g["qkr_q"]) and close(k, g["qkr_k"]) and close(v, g["qkr_v"])
    o = orc.decode_attention(g["att_q"], g["att_k"], g["att_v"], g["att_span"], g["att_ws"])
    assert close(o, g["att_o"])


def test_activations_and_conv(orc, gold):
    g = gold
    assert close(orc.swiglu(g["swi_g"], g["swi_u"]), g["swi_y"])
    assert close(orc.snake_beta(g["snk_x"], g["snk_a"], g["snk_b"]), g["snk_y"])
    y = orc.conv1d_nlc(g["cnv_x"], g["cnv_w"], g["cnv_b"], 2, 4, (g["cnv_a"], g["cnv_r"]),
                       g["cnv_res"])
    assert close(y, g["cnv_y"])


def test_picks(orc, gold):
    g = gold
    assert np.array_equal(orc.argmax(g["arg_logits"]), g["arg_codes"])
    assert np.array_equal(orc.argmax(g["arg_logits"], g["arg_banned"]), g["arg_codes_banned"])
    # the tie at ids 17 and 250 of row 1: the last maximum wins, and a banned one never does
    assert g["arg_codes"][1] == 250 and g["arg_codes_banned"][1] == 17
    assert np.array_equal(orc.topk_sample(g["tk_logits"], g["tk_draws"], 20, 0.9), g["tk_codes"])
