"""Voice assets (crates/tts-core/src/voice.rs; crates/qwen3tts/src/engine.rs:714-736) read from
their files through the native safetensors reader, on the CPU: the manifest's fields, the three
tensors a qwen3tts request takes, the x-vector width check, clone=xvector, and the reference's
error messages for a missing tensor or manifest."""
import json
import os

import numpy as np
import pytest
import torch

REF_VOICE = "/root/reference/voices/male-qwen3tts"


def write_voice(d, spk_dim=2048, frames=7, text_ids=5, with_codes=True):
    from safetensors.numpy import save_file
    os.makedirs(d, exist_ok=True)
    rng = np.random.default_rng(3)
    tensors = {"spk_embedding": rng.standard_normal((1, spk_dim)).astype(np.float32)}
    if with_codes:
        tensors["ref_codes"] = rng.integers(0, 2048, (frames, 16)).astype(np.int32)
        tensors["ref_text_tokens"] = rng.integers(0, 151000, (1, text_ids)).astype(np.int32)
    save_file(tensors, os.path.join(d, "voice.safetensors"))
    with open(os.path.join(d, "voice.json"), "w") as f:
        json.dump({"engine": "qwen3tts", "name": "synthetic", "text": "hello there",
                   "seconds": 1.5, "notes": None, "language": "english"}, f)
    return tensors


def test_voice_asset_round_trip(tmp_path):
    from qwen3tts.voice import Voice
    t = write_voice(str(tmp_path / "v"))
    v = Voice.load(str(tmp_path / "v"))
    assert (v.engine, v.name, v.text, v.seconds, v.language) == \
        ("qwen3tts", "synthetic", "hello there", 1.5, "english")
    assert v.keys() == ["ref_codes", "ref_text_tokens", "spk_embedding"]
    assert v.get_rows_u32("ref_codes") == t["ref_codes"].tolist()
    r = v.request([1, 2, 3], 2048, device="cpu", max_frames=9)
    assert r.text == [1, 2, 3] and r.max_frames == 9
    assert r.ref_codes == t["ref_codes"].tolist()
    assert r.ref_text == t["ref_text_tokens"][0].tolist()
    assert torch.equal(r.spk, torch.from_numpy(t["spk_embedding"][0]))
    x = v.request([1], 2048, xvector_only=True, device="cpu")
    assert x.ref_codes == [] and x.ref_text == [] and x.spk is not None


def test_voice_asset_refusals(tmp_path):
    from qwen3tts.voice import Voice, VoiceError
    write_voice(str(tmp_path / "narrow"), spk_dim=1024)
    v = Voice.load(str(tmp_path / "narrow"))
    with pytest.raises(VoiceError, match="1024-wide, expected 2048"):
        v.speaker(2048, device="cpu")
    with pytest.raises(VoiceError, match="has no tensor `nope`; it has: ref_codes"):
        v.get("nope")
    write_voice(str(tmp_path / "bare"), with_codes=False)
    r = Voice.load(str(tmp_path / "bare")).request([4], 2048, device="cpu")
    assert r.ref_codes == [] and r.ref_text == []
    with pytest.raises(VoiceError, match="reading"):
        Voice.load(str(tmp_path / "missing"))


@pytest.mark.skipif(not os.path.isdir(REF_VOICE), reason="the reference's voice assets are absent")
def test_reference_voice_asset_reads():
    """One of the reference's own voice assets (read in place, where it exists)."""
    from qwen3tts.voice import Voice
    v = Voice.load(REF_VOICE)
    assert v.engine == "qwen3tts" and v.name == "male-qwen3tts"
    codes = v.get_rows_u32("ref_codes")
    meta = json.load(open(os.path.join(REF_VOICE, "voice.json")))
    assert len(codes) == meta["frames"] and all(len(r) == meta["codebooks"] for r in codes)
    assert all(0 <= c < 2048 for r in codes for c in r)
    assert v.speaker(meta["enc_dim"], device="cpu").shape == (2048,)
    assert len(v.get_rows_u32("ref_text_tokens")[0]) > 0
