"""s2k_sample_noalloc: the allocation-free sampler entry (fixed static device
scratch) against s2k_sample on the same logits and uniform draws.

It exists for callers that may not allocate device memory, for instance a
host that runs under a fixed device-memory budget set up front.  Collected
last (file name) so it runs both alone and after every other GPU test on a
device whose allocator has already been exercised.  Tokens are integers: the
two entries must agree exactly, on two calls in a row.  The calls must leave
the model's device bytes and the device's free memory unchanged.
"""
from __future__ import annotations

import numpy as np
import pytest

import s2k

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(small_model_data):
    hp, tensors = small_model_data
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    yield m
    m.close()


@pytest.mark.parametrize("n", [1, 1000, 4097, s2k.SAMPLE_NOALLOC_MAX_N])
def test_noalloc_matches_sample(model, n):
    rng = np.random.default_rng(1000 + n)
    cases = [(0.0, 0.8, 30), (1.0, 0.9, 30), (0.7, 0.9, 0), (1.3, 1.0, 5), (0.8, 0.8, 4096)]
    for trial in range(4):
        x = (rng.standard_normal(n) * rng.uniform(0.5, 4)).astype(np.float32)
        for temp, top_p, top_k in cases:
            u = float(rng.uniform())
            want = model.sample(x, temp, top_p, top_k, u)
            first = model.sample_noalloc(x, temp, top_p, top_k, u)
            second = model.sample_noalloc(x, temp, top_p, top_k, u)
            assert first == second == want, (n, trial, temp, top_p, top_k, u, first, second, want)


def test_noalloc_consecutive_different_rows(model):
    """Back-to-back calls with different rows: the second call sees only its
    own logits (no stale scratch from the first, which was longer)."""
    rng = np.random.default_rng(3)
    a = rng.standard_normal(6000).astype(np.float32)
    b = rng.standard_normal(700).astype(np.float32)
    b[123] = 50.0
    assert model.sample_noalloc(a, 0.0, 1.0, 0) == model.sample(a, 0.0, 1.0, 0)
    assert model.sample_noalloc(b, 0.0, 1.0, 0) == 123
    assert model.sample_noalloc(b, 0.0, 1.0, 0) == model.sample(b, 0.0, 1.0, 0) == 123


def test_noalloc_rejects_oversize(model):
    x = np.zeros(s2k.SAMPLE_NOALLOC_MAX_N + 1, np.float32)
    with pytest.raises(s2k.S2KError) as e:
        model.sample_noalloc(x, 0.0, 1.0, 0)
    assert e.value.status == -1
    assert "fixed scratch" in str(e.value)
    # a rejected call leaves the entry usable
    y = np.zeros(16, np.float32)
    y[5] = 1.0
    assert model.sample_noalloc(y, 0.0, 1.0, 0) == 5


def test_noalloc_allocates_nothing(model):
    """After a first call (which looks up the scratch array's address), calls
    of every size leave the model's device bytes and the device's free memory
    unchanged."""
    rng = np.random.default_rng(9)
    x = rng.standard_normal(s2k.SAMPLE_NOALLOC_MAX_N).astype(np.float32)
    model.sample_noalloc(x, 0.8, 0.9, 30, 0.5)
    held = model.device_bytes()
    free0, _ = s2k.device_mem_info(model.device)
    for n in (1, 777, 4096, s2k.SAMPLE_NOALLOC_MAX_N):
        for _ in range(2):
            model.sample_noalloc(x[:n], 0.8, 0.9, 30, float(rng.uniform()))
    free1, _ = s2k.device_mem_info(model.device)
    assert model.device_bytes() == held
    assert free1 == free0
