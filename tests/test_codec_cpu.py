"""CPU checks of the codec decode oracle (the restatement of
AudioCodec::decode, src/s2_codec.cpp:1297-1447) and of the window algebra of
its two callers (decode_codes_windowed, src/s2_pipeline.cpp:198-289; the
streaming decode_window_and_emit, :1034-1141).  No GPU."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import synthetic


@pytest.fixture(scope="module")
def small():
    ch = synthetic.codec_preset("small")
    co = oracle.CodecOracle(ch)
    co.load_tensors(synthetic.make_codec(ch, seed=5))
    yield ch, co
    co.close()


def test_decode_length_and_range(small):
    ch, co = small
    codes = synthetic.codec_codes(ch, 20, seed=1)
    a = co.decode(codes)
    assert a.shape == (20 * ch.samples_per_frame,)
    assert co.samples_per_frame() == ch.samples_per_frame == 48
    assert np.isfinite(a).all() and np.abs(a).max() < 1.0
    assert a.std() > 0.05  # the synthetic weights keep the tanh out of saturation


def test_decode_is_causal(small):
    """Every stage is causal (left-padded convolutions, transposed
    convolutions cropped on the right, a causal / windowed attention mask), so
    a prefix of the codes decodes to the same samples, bit for bit."""
    ch, co = small
    codes = synthetic.codec_codes(ch, 24, seed=2)
    full = co.decode(codes)
    for n in (1, 7, 13):
        pre = co.decode(codes[:, :n])
        assert np.array_equal(pre, full[: n * ch.samples_per_frame]), n


def test_codes_are_clamped(small):
    """sanitize_decode_codes (src/s2_codec.cpp:1160-1188): out-of-range codes
    decode as the nearest valid code."""
    ch, co = small
    codes = synthetic.codec_codes(ch, 10, seed=3)
    wild = codes.copy()
    wild[0, 2] = -5
    wild[0, 5] = ch.quantizer_semantic_codebook_size + 100
    wild[2, 7] = ch.quantizer_residual_codebook_size
    clamped = wild.copy()
    clamped[0] = np.clip(clamped[0], 0, ch.quantizer_semantic_codebook_size - 1)
    clamped[1:] = np.clip(clamped[1:], 0, ch.quantizer_residual_codebook_size - 1)
    assert np.array_equal(co.decode(wild), co.decode(clamped))


def test_window_attention_limits_context(small):
    """With the window mask (8 frames here) and 2 layers, a code change at
    frame 0 reaches the transformer output of frames < 15 only; the causal
    decoder carries it a receptive field (< 13 frames here) further, and no
    further: the tail of a 40-frame clip is untouched."""
    ch, co = small
    codes = synthetic.codec_codes(ch, 40, seed=4)
    a = co.decode(codes)
    changed = codes.copy()
    changed[0, 0] = (changed[0, 0] + 1) % ch.quantizer_semantic_codebook_size
    b = co.decode(changed)
    diff = np.nonzero(a != b)[0]
    assert diff.size > 0 and diff[0] < ch.samples_per_frame
    assert diff[-1] < 28 * ch.samples_per_frame


@pytest.mark.parametrize("total,stride,context", [(100, 16, -1), (37, 16, -1), (16, 16, -1), (5, 16, -1),
                                                   (90, 7, 12), (64, 16, 0)])
def test_offline_windows_tile_the_utterance(small, total, stride, context):
    ch, co = small
    ws = co.windows_offline(total, stride, context)
    covered = []
    for start, wf, eb, ee in ws:
        assert 0 <= start and start + wf <= total and 0 <= eb <= ee <= wf
        covered += list(range(start + eb, start + ee))
    assert covered == list(range(total))  # every frame emitted once, in order
    hist = context if context >= 0 else co.history_frames()
    for start, wf, eb, ee in ws[:-1]:
        assert eb <= hist  # at most `history` frames of context before what a window emits


@pytest.mark.parametrize("total,stride,context,holdback", [(30, 4, -1, -1), (50, 4, 8, 2), (9, 4, 0, 0),
                                                            (3, 4, -1, -1), (41, 1, 6, 3)])
def test_stream_windows_tile_the_utterance(small, total, stride, context, holdback):
    ch, co = small
    ws = co.windows_stream(total, stride, context, holdback)
    covered = []
    for seen, start, wf, eb, ee in ws:
        assert start + wf == seen <= total
        covered += list(range(start + eb, start + ee))
    assert covered == list(range(total))


def test_windowed_decode_matches_window_decodes(small):
    ch, co = small
    codes = synthetic.codec_codes(ch, 70, seed=6)
    got = co.decode_windowed(codes, 16)
    spf = ch.samples_per_frame
    parts = [co.decode(codes[:, s:s + wf])[eb * spf: ee * spf] for s, wf, eb, ee in co.windows_offline(70, 16)]
    assert np.array_equal(got, np.concatenate(parts))
    assert got.shape == (70 * spf,)


def test_history_frames_formula(small):
    """streaming_history_frames = ceil8(window - 1 + 16) (src/s2_codec.cpp:870-874)"""
    ch, co = small
    assert co.history_frames() == 24
    s2 = synthetic.codec_preset("s2pro")
    assert ((s2.rvq_window_size - 1 + 16 + 7) // 8) * 8 == 144


def test_accumulation_order_drift_is_small(small):
    """Two valid accumulation orders of the same fp16-rounded graph (double,
    or float in sequence) agree to ~1e-4 of the audio -- the floor the GPU
    parity bar is measured against -- and not bit for bit: fp16 roundings
    that land on the other side compound through the decoder stack."""
    ch, co = small
    codes = synthetic.codec_codes(ch, 40, seed=8)
    a, b = co.decode(codes), co.decode(codes, f32_accum=True)
    d = np.abs(a.astype(np.float64) - b)
    assert 0 < np.sqrt(np.mean(d * d)) < 1e-3 and d.max() < 5e-3
    assert np.array_equal(co.decode(codes), a)  # the switch resets
