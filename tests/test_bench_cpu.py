"""CPU: the bench workloads are the configurations they claim to be."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402
import synthetic  # noqa: E402


def test_ragged_requests_match_config():
    """64 utterances, prompts ~U[64, 1024] tokens, frames ~U[100, 1500], seeded."""
    hp = synthetic.preset("s2pro")
    a = bench.ragged_requests(hp, 64)
    b = bench.ragged_requests(hp, 64)
    assert len(a) == 64
    cols = np.array([p.shape[1] for _, p, _ in a])
    frames = np.array([f for _, _, f in a])
    assert cols.min() >= 64 and cols.max() <= 1024
    assert frames.min() >= 100 and frames.max() <= 1500
    assert all(np.array_equal(p, q) and f == g for (_, p, f), (_, q, g) in zip(a, b))
    # round-robin dealing covers every utterance once
    world = 8
    dealt = sorted(i for r in range(world) for i, _, _ in a if i % world == r)
    assert dealt == list(range(64))


def test_frame_bytes_match_survey():
    """Per-frame algorithmic bytes of the S2 Pro Q8_0 frame loop: Slow
    4,283,760,640 B + 9 x Fast 440,074,240 B + 147,456 B per cached position."""
    hp = synthetic.preset("s2pro")
    slow, fast = bench.weight_stream_bytes(hp, "q8_0")
    assert slow == 4283760640
    assert fast == 440074240
    one = bench.frame_bytes(hp, 64, 1)
    assert one == slow + 9 * fast + 147456 * 65


def test_frame_metric_names_the_weight_scheme():
    """The default (Q8_0) run reports the headline metric unchanged; other
    weight schemes name themselves instead of claiming Q8_0."""
    assert bench.frame_metric("q8_0") == bench.METRIC
    assert "Q4_K_M" in bench.frame_metric("q4_k_m") and "Q8_0" not in bench.frame_metric("q4_k_m")
    assert "F16" in bench.frame_metric("f16")


def test_codec_flops_counts_the_graph():
    """bench.codec_flops: linear in frames, and on the small codec equal to a
    hand count of its products (transformer, upsample, decoder)."""
    import synthetic
    ch = synthetic.codec_preset("small")
    f1, f2 = bench.codec_flops(ch, 10, 10), bench.codec_flops(ch, 20, 20)
    assert abs(f2 - 2 * f1) < 1e-6 * f2
    d, hd, ff = 128, 32, 256
    H, Hk = 4, 2
    keys = 8
    n = 10
    want = 2 * 2.0 * n * (d * (H + 2 * Hk) * hd + H * hd * d + 3 * d * ff + 2 * H * hd * keys)
    L, C = n, d
    for fac in (2, 3):
        want += 2.0 * L * fac * C * C
        L *= fac
        want += 2.0 * L * C * (7 + 2 * 512)
    want += 2.0 * L * 256 * C * 7
    C = 256
    for r in (4, 2):
        co = C // 2
        want += 2.0 * L * (r * co) * (2 * C)
        L *= r
        want += 3 * 2.0 * L * co * co * 8
        C = co
    want += 2.0 * L * C * 7
    assert abs(f1 - want) < 1e-9 * want
