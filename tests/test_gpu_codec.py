"""GPU parity of the codec decode (s2k_codec_*, AudioCodec::decode,
src/s2_codec.cpp:1297-1447) against the CPU oracle, through the C ABI.

Bars.  Against the oracle: the reference graph rounds operands to fp16 at
every matrix product and convolution, as the tensor-core GEMMs do, but a
different accumulation order lands some roundings on the other side, and
those flips compound through the decoder stack.  The oracle itself drifts by
that much between two valid accumulation orders (double vs. float in
sequence: rms ~2e-4 on the small codec, ~1e-3 at S2 Pro widths, audio std
0.25-0.45).  So the bar is relative to that drift, measured on the same
input: max and rms |GPU - oracle| <= 3x the oracle's own max / rms drift
(+1e-5 / 1e-6).  Between GPU paths (a window decoded whole vs. the
truncated decode of the emitted range, the windowed / streaming drivers vs.
their windows decoded one by one): bit-exact."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
import s2k
import synthetic

pytestmark = pytest.mark.gpu

def _dev(a: np.ndarray, b: np.ndarray):
    d = np.abs(a.astype(np.float64) - b.astype(np.float64))
    return float(d.max(initial=0.0)), float(np.sqrt(np.mean(d * d))) if d.size else 0.0


def assert_audio_close(got: np.ndarray, want: np.ndarray, want_f32acc: np.ndarray, what: str) -> None:
    """got vs the oracle (want), bounded by the oracle's own drift between
    its two accumulation orders (want vs want_f32acc)"""
    assert got.shape == want.shape == want_f32acc.shape, (what, got.shape, want.shape)
    assert np.isfinite(got).all(), what
    fmax, frms = _dev(want, want_f32acc)
    gmax, grms = _dev(got, want)
    assert gmax <= 3 * fmax + 1e-5 and grms <= 3 * frms + 1e-6, (
        f"{what}: |gpu - oracle| max {gmax:.3g} rms {grms:.3g}; oracle drift max {fmax:.3g} rms {frms:.3g}")


@pytest.fixture(scope="module")
def small():
    ch = synthetic.codec_preset("small")
    tensors = list(synthetic.make_codec(ch, seed=5))
    c = s2k.AudioCodec(ch)
    c.load_tensors(tensors)
    co = oracle.CodecOracle(ch)
    co.load_tensors(tensors)
    yield ch, c, co
    c.close()
    co.close()


def test_small_decode_matches_oracle(small):
    ch, c, co = small
    assert c.samples_per_code_frame() == ch.samples_per_frame
    assert c.num_codebooks() == ch.num_codebooks
    assert c.streaming_history_frames() == co.history_frames()
    for n, seed in ((1, 1), (7, 2), (40, 3), (130, 4)):
        codes = synthetic.codec_codes(ch, n, seed=seed)
        assert_audio_close(c.decode(codes), co.decode(codes), co.decode(codes, True), f"small decode n={n}")


def test_small_codes_clamped(small):
    ch, c, co = small
    codes = synthetic.codec_codes(ch, 12, seed=9)
    wild = codes.copy()
    wild[0, 1] = -7
    wild[0, 4] = 10 ** 6
    wild[3, 9] = ch.quantizer_residual_codebook_size + 3
    got = c.decode(wild)
    clamped = wild.copy()
    clamped[0] = np.clip(clamped[0], 0, ch.quantizer_semantic_codebook_size - 1)
    clamped[1:] = np.clip(clamped[1:], 0, ch.quantizer_residual_codebook_size - 1)
    assert np.array_equal(got, c.decode(clamped))
    assert_audio_close(got, co.decode(wild), co.decode(wild, True), "clamped codes")


def test_small_range_is_exact_slice(small):
    """decode_range computes only what frames [b, e) depend on (the
    transformer over [0, e), the decoder from b - receptive_frames): the
    samples equal the whole-window decode's, bit for bit."""
    ch, c, co = small
    spf = ch.samples_per_frame
    codes = synthetic.codec_codes(ch, 90, seed=12)
    full = c.decode(codes)
    rf = c.receptive_frames()
    assert 1 <= rf < 40
    for b, e in ((0, 90), (0, 5), (30, 46), (rf, rf + 1), (rf + 1, 90), (89, 90), (60, 60)):
        got = c.decode_range(codes, b, e)
        assert np.array_equal(got, full[b * spf: e * spf]), (b, e)


def test_small_windowed_matches_windows(small):
    """decode_codes_windowed: each window's emitted samples equal that window
    decoded whole (bit-exact), and the oracle's windowed decode (tolerance)."""
    ch, c, co = small
    spf = ch.samples_per_frame
    for total, stride, ctx in ((100, 16, -1), (37, 16, -1), (70, 7, 12), (9, 16, -1)):
        codes = synthetic.codec_codes(ch, total, seed=total)
        got, ms, nb = c.decode_windowed(codes, stride, ctx)
        wins = co.windows_offline(total, stride, ctx)
        assert nb == len(wins) and ms > 0
        parts = [c.decode(codes[:, s:s + wf])[eb * spf: ee * spf] for s, wf, eb, ee in wins]
        assert np.array_equal(got, np.concatenate(parts)), (total, stride, ctx)
        assert_audio_close(got, co.decode_windowed(codes, stride, ctx), co.decode_windowed(codes, stride, ctx, True),
                           f"windowed {total}/{stride}/{ctx}")


@pytest.mark.parametrize("stride,ctx,hold", [(4, -1, -1), (4, 8, 2), (1, 6, 0), (5, 0, 3)])
def test_small_stream_matches_windows(small, stride, ctx, hold):
    ch, c, co = small
    spf = ch.samples_per_frame
    total = 45
    codes = synthetic.codec_codes(ch, total, seed=70 + stride)
    st = c.stream(stride, ctx, hold)
    parts = [st.push(codes[:, f]) for f in range(total)]
    parts.append(st.finish())
    st.close()
    got = np.concatenate(parts)
    want = [c.decode(codes[:, s:s + wf])[eb * spf: ee * spf] for _, s, wf, eb, ee in co.windows_stream(total, stride, ctx, hold)]
    assert np.array_equal(got, np.concatenate(want))
    assert got.shape == (total * spf,)


def test_small_errors(small):
    ch, c, co = small
    codes = synthetic.codec_codes(ch, 4, seed=1)
    with pytest.raises(s2k.S2KError):
        c.decode(codes[:, :0])
    with pytest.raises(s2k.S2KError):
        c.decode_range(codes, 3, 5)  # past the window
    with pytest.raises(s2k.S2KError):
        c.decode_windowed(codes[:2], 16)  # wrong codebook count


def test_codec_gguf_combined_and_codec_only(tmp_path):
    pytest.importorskip("gguf")
    from gguf_fixture import write_codec_gguf
    ch = synthetic.codec_preset("small")
    tensors = list(synthetic.make_codec(ch, seed=8))
    ref = s2k.AudioCodec(ch)
    ref.load_tensors(tensors)
    codes = synthetic.codec_codes(ch, 30, seed=31)
    want = ref.decode(codes)
    for combined in (True, False):
        path = os.path.join(tmp_path, f"codec_{combined}.gguf")
        write_codec_gguf(path, ch, tensors, combined=combined)
        c = s2k.AudioCodec.from_gguf(path)
        try:
            assert c.samples_per_code_frame() == ch.samples_per_frame
            assert np.array_equal(c.decode(codes), want)
        finally:
            c.close()
    ref.close()


@pytest.fixture(scope="module")
def s2pro():
    ch = synthetic.codec_preset("s2pro")
    tensors = list(synthetic.make_codec(ch, seed=6))
    c = s2k.AudioCodec(ch)
    c.load_tensors(tensors)
    yield ch, c, tensors
    c.close()


def test_s2pro_decode_matches_oracle(s2pro):
    """The S2 Pro codec widths (1024-wide 8-layer post-module transformer,
    1536 -> 96 channel decoder, 2048 samples per frame) on 6 frames."""
    ch, c, tensors = s2pro
    co = oracle.CodecOracle(ch)
    try:
        co.load_tensors(tensors)
        codes = synthetic.codec_codes(ch, 6, seed=21)
        assert_audio_close(c.decode(codes), co.decode(codes), co.decode(codes, True), "s2pro decode")
    finally:
        co.close()


def test_s2pro_range_and_windowed_exact(s2pro):
    ch, c, _ = s2pro
    spf = ch.samples_per_frame
    codes = synthetic.codec_codes(ch, 40, seed=22)
    full = c.decode(codes)
    rf = c.receptive_frames()
    assert 8 <= rf <= 16
    for b, e in ((20, 24), (rf + 2, 40), (0, 3)):
        assert np.array_equal(c.decode_range(codes, b, e), full[b * spf: e * spf]), (b, e)
    got, _, _ = c.decode_windowed(codes, 16, 12)
    wins = oracle.codec_windows_offline(40, 16, 12)
    parts = [c.decode(codes[:, s:s + wf])[eb * spf: ee * spf] for s, wf, eb, ee in wins]
    assert np.array_equal(got, np.concatenate(parts))
