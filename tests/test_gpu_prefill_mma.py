"""GPU: the tensor-core prefill GEMM (tcgen05 int8 MMAs with the double-
precision block-scale epilogue) on prompts of one to three token tiles,
ragged last tile and split-K partials included, against the CPU oracle.
Each int8 MMA over a 32-column block is one exact Q8_0 block sum, so the
prefill is bit-exact with the oracle."""
from __future__ import annotations

import numpy as np
import pytest

import s2k
import synthetic
from parity_util import assert_exact

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [8, 64, 150])
def test_prefill_mma_matches_oracle(small_model_data, small_oracle, n):
    hp, tensors = small_model_data
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    p = synthetic.semantic_prompt(hp, n, seed=n)
    m.init_kv_cache(n + 4)
    small_oracle.init_kv_cache(n + 4)
    hg, lg = m.prefill_fast(p.T.reshape(-1), n)
    ho, lo = small_oracle.eval(p.T.reshape(-1), n)
    m.close()
    assert_exact(hg, ho, f"{n}-token tensor-core prefill hidden")
    assert_exact(lg, lo, f"{n}-token tensor-core prefill logits")
