"""CPU: s2k_build_prompt against a restatement of s2::build_prompt
(src/s2_prompt.cpp:5-103) in plain Python, with a toy tokenizer (the real
one needs the model's tokenizer.json): text-only and voice-clone prompts,
with and without a speaker tag in the transcript, and a reference clip
without its transcript (ignored, as in the reference)."""
from __future__ import annotations

import numpy as np
import pytest

import s2k

IM_END, VOICE, SEM0 = 151645, 151673, 151552
SPECIAL = {"<|im_start|>system": [151644, 9125], "<|im_start|>user": [151644, 882],
           "<|im_start|>assistant": [151644, 77091], "<|speaker:0|>": [151669]}


def toy_encode(text: str) -> list:
    if text in SPECIAL:
        return list(SPECIAL[text])
    return [1000 + (ord(ch) % 5000) for ch in text]


def build_prompt_py(text, prompt_text, codes, ncb):
    """src/s2_prompt.cpp:5-103 restated."""
    nl = [198]
    has_ref = codes is not None and codes.shape[1] > 0 and prompt_text != ""
    pre, post = [], []
    if has_ref:
        pre += toy_encode("<|im_start|>system") + nl
        pre += toy_encode("convert the provided text to speech reference to the following:\n\nText:\n")
        if "<|speaker:" not in prompt_text:
            pre += toy_encode("<|speaker:0|>")
        pre += toy_encode(prompt_text) + toy_encode("\n\nSpeech:\n")
        post += [IM_END] + nl
    else:
        post += toy_encode("<|im_start|>system") + nl + toy_encode("convert the provided text to speech")
        post += [IM_END] + nl
    post += toy_encode("<|im_start|>user") + nl + toy_encode(text) + [IM_END] + nl
    post += toy_encode("<|im_start|>assistant") + nl + [VOICE]
    T = codes.shape[1] if has_ref else 0
    grid = np.zeros((ncb + 1, len(pre) + T + len(post)), np.int32)
    grid[0, : len(pre)] = pre
    if has_ref:
        grid[0, len(pre): len(pre) + T] = codes[0] + SEM0
        grid[1:, len(pre): len(pre) + T] = codes
    grid[0, len(pre) + T:] = post
    return grid


@pytest.mark.parametrize("case", ["text_only", "clone", "clone_speaker_tag", "codes_without_transcript"])
def test_build_prompt_matches_reference_restatement(case):
    ncb = 10
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 4096, (ncb, 37)).astype(np.int32)
    text = "Hello there, this is a test."
    if case == "text_only":
        args = ("", None)
    elif case == "clone":
        args = ("the reference transcript", codes)
    elif case == "clone_speaker_tag":
        args = ("<|speaker:1|>a tagged transcript", codes)
    else:
        args = ("", codes)
    got = s2k.build_prompt(toy_encode, text, args[0], args[1], ncb, IM_END, VOICE, SEM0)
    want = build_prompt_py(text, args[0], args[1], ncb)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def test_build_prompt_encoder_failure():
    def bad(text):
        raise ValueError("no tokenizer")
    with pytest.raises(s2k.S2KError) as e:
        s2k.build_prompt(bad, "x")
    assert e.value.status == -1
