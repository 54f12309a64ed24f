"""The safetensors reader (crates/tts-nn/src/lib.rs:153-373's Weights over a mapped file) on
files written here in the format's layout: names, dtypes, shapes and bytes round-trip, the
metadata block is skipped, broken files are refused with the file and entry named, and the
weight-norm fold matches its definition (lib.rs:367-373). No GPU."""
import json
import os
import struct

import numpy as np
import pytest
import torch


def write_safetensors(path, tensors, metadata=None, order=None):
    """tensors: name -> (dtype string, numpy array of the bytes' dtype)."""
    header = {}
    blobs = []
    off = 0
    for name in (order or sorted(tensors)):
        dt, arr = tensors[name]
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata is not None:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


@pytest.fixture(scope="module")
def lib():
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "dream-tts_b200"))
    import build
    build.build()
    from qwen3tts import weights
    return weights


def test_round_trip(lib, tmp_path):
    rng = np.random.default_rng(0)
    f32 = rng.standard_normal((3, 5)).astype(np.float32)
    f16 = rng.standard_normal((4, 8)).astype(np.float16)
    bf = torch.randn(6, 2).to(torch.bfloat16)
    i64 = np.arange(7, dtype=np.int64)
    scalar = np.array(3.5, np.float32)
    p = str(tmp_path / "m.safetensors")
    write_safetensors(p, {"a.weight": ("F32", f32), 'b"q': ("F16", f16),
                          "c": ("BF16", bf.view(torch.int16).numpy()), "ids": ("I64", i64),
                          "s": ("F32", scalar)},
                      metadata={"format": "pt", "nested": {"x": [1, 2.5, True, None]}})
    w = lib.Weights(p)
    assert sorted(w.names()) == sorted(["a.weight", 'b"q', "c", "ids", "s"])
    assert w.has("a.weight") and not w.has("nope")
    assert np.array_equal(w.cpu("a.weight").numpy(), f32)
    assert np.array_equal(w.cpu('b"q').numpy(), f16)
    assert torch.equal(w.cpu("c"), bf)
    assert np.array_equal(w.cpu("ids").numpy(), i64)
    assert w.cpu("s").shape == () and float(w.cpu("s")) == 3.5
    assert w.get('b"q', device="cpu").dtype == torch.float32
    with pytest.raises(Exception, match="missing tensor nope"):
        w.cpu("nope")
    w.close()


def test_refuses_broken_files(lib, tmp_path):
    from ttsnn import _lib as L
    good = {"x": ("F32", np.zeros((2, 2), np.float32))}
    p = str(tmp_path / "ok.safetensors")
    write_safetensors(p, good)
    raw = open(p, "rb").read()
    cases = {
        "short": raw[:5],
        "truncated": raw[:-4],                                   # data_offsets past the end
        "header_len": struct.pack("<Q", 1 << 40) + raw[8:],
        "not_json": struct.pack("<Q", 8) + b"[1,2]   ",
    }
    for name, data in cases.items():
        q = str(tmp_path / f"{name}.safetensors")
        open(q, "wb").write(data)
        with pytest.raises(L.TtsError) as e:
            lib.Weights(q)
        assert e.value.status == 1 and name + ".safetensors" in str(e.value), name
    # shape and byte count disagree
    q = str(tmp_path / "size.safetensors")
    write_safetensors(q, {"x": ("F32", np.zeros(3, np.float32))})
    b = bytearray(open(q, "rb").read())
    b = b.replace(b'"shape": [3]', b'"shape": [4]')
    open(q, "wb").write(bytes(b))
    with pytest.raises(L.TtsError, match="does not match its shape"):
        lib.Weights(q)
    with pytest.raises(L.TtsError):
        lib.Weights(str(tmp_path / "absent.safetensors"))


def test_weight_norm_fold(lib, tmp_path):
    rng = np.random.default_rng(1)
    g = rng.uniform(0.5, 2, (6, 1, 1)).astype(np.float32)
    v = rng.standard_normal((6, 4, 3)).astype(np.float32)
    p = str(tmp_path / "wn.safetensors")
    write_safetensors(p, {"conv.parametrizations.weight.original0": ("F32", g),
                          "conv.parametrizations.weight.original1": ("F32", v),
                          "plain.weight": ("F32", v)})
    w = lib.Weights(p)
    got = w.weight_norm("conv", device="cpu").numpy()
    want = g * v / np.sqrt((v.reshape(6, -1) ** 2).sum(1)).reshape(6, 1, 1)
    assert np.allclose(got, want, rtol=1e-6)
    assert np.array_equal(w.weight_norm("plain", device="cpu").numpy(), v)
