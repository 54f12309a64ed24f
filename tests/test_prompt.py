"""The talker's prompt assembly (crates/qwen3tts/src/talker.rs:683-786) on the host with a fake
text projection whose rows encode their ids, so every position of the prompt can be read
back: role rows, the codec-tag prefix summed with the pad/bos text rows, the first text row on
codec_bos (x-vector path) or the in-context block (ICL path), the trailing rows and the shared
count. No GPU."""
import pytest
import torch


def setup():
    from qwen3tts import prompt as P
    dim = 4

    class FakeText:
        def __call__(self, ids):
            return torch.tensor([[float(i), 0.0, 0.0, 1.0] for i in ids])

    codec = torch.zeros(3072, dim)
    codec[:, 1] = torch.arange(3072, dtype=torch.float32)
    tables = torch.zeros(15, 2048, dim)
    tables[:, :, 2] = 1.0  # each residual code's row adds 1 to column 2
    return P, P.PromptBuilder(FakeText(), codec, tables)


def test_xvector_prompt_layout():
    P, b = setup()
    spk = torch.tensor([0.0, 0.0, 0.0, 5.0])
    prompt, trailing, shared = b.build([11, 12, 13], spk=spk)
    # role: im_start, assistant, newline
    assert prompt[:3, 0].tolist() == [P.IM_START, P.ASSISTANT, P.NEWLINE]
    # prefix: pads (+ the last bos) over nothink, think_bos, think_eos, spk, pad
    codec_ids = [P.CODEC_NOTHINK, P.CODEC_THINK_BOS, P.CODEC_THINK_EOS, None, P.CODEC_PAD]
    text_ids = [P.TTS_PAD] * 4 + [P.TTS_BOS]
    for j, (c, t) in enumerate(zip(codec_ids, text_ids)):
        row = prompt[3 + j]
        assert row[0] == t
        if c is None:
            assert row[1] == 0 and row[3] == 1 + 5  # the x-vector row
        else:
            assert row[1] == c
    # the first text token rides on codec_bos
    assert prompt[8, 0] == 11 and prompt[8, 1] == P.CODEC_BOS
    assert prompt.shape[0] == 9 and shared == 8
    assert trailing[:, 0].tolist() == [12, 13, P.TTS_EOS]


def test_icl_prompt_layout():
    P, b = setup()
    ref_codes = [[5] + [7] * 15, [6] + [8] * 15]
    prompt, trailing, shared = b.build([21, 22, 23], ref_text=[31, 32], ref_codes=ref_codes,
                                       language=2050)
    # prefix with a language tag: think, think_bos, tag, think_eos, pad (then bos consumed)
    assert prompt[3:8, 1].tolist() == [P.CODEC_THINK, P.CODEC_THINK_BOS, 2050,
                                       P.CODEC_THINK_EOS, P.CODEC_PAD]
    # ICL block: text (ref + target + eos) summed with codec_bos + the two frames
    blk = prompt[8:]
    assert blk.shape[0] == 3  # the codec side: bos + 2 frames
    assert blk[:, 0].tolist() == [31, 32, 21]
    assert blk[:, 1].tolist() == [P.CODEC_BOS, 5, 6]
    assert blk[1:, 2].tolist() == [15.0, 15.0]  # fifteen residual rows each
    assert trailing[:, 0].tolist() == [22, 23, P.TTS_EOS]
    assert shared == 3 + 5 + 2
    # a longer codec side pads the text with tts_pad and trails the pad row alone
    prompt, trailing, _ = b.build([21], ref_text=[31], ref_codes=ref_codes * 2)
    assert prompt[-5:, 0].tolist() == [31, 21, P.TTS_EOS, P.TTS_PAD, P.TTS_PAD]
    assert trailing[:, 0].tolist() == [P.TTS_PAD]
    with pytest.raises(ValueError):
        b.build([])
