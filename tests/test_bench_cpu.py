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
