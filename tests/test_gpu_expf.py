"""The device exp (det_expf: every softmax, SiLU and sampler kernel) against
the CPU oracle's so_det_expf, bit for bit, over every regime of its input:
the shared exp is what lets the GPU and the oracle agree on attention,
SwiGLU and sampling."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import s2k
from test_oracle_golden import _expf_inputs

pytestmark = pytest.mark.gpu


def test_device_det_expf_bit_exact():
    x = _expf_inputs(seed=11)
    got = s2k.det_expf(x)
    want = oracle.det_expf(x)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    # the subnormal results (k < -126) are where the scaling rounds
    sub = (want > 0) & (want < np.finfo(np.float32).tiny)
    assert sub.sum() > 1000


def test_device_det_expf_empty_and_errors():
    assert s2k.det_expf(np.zeros(0, np.float32)).size == 0
    with pytest.raises(s2k.S2KError):  # NULL arrays with n > 0
        s2k._check(s2k.lib().s2k_debug_det_expf(0, None, None, 5))
