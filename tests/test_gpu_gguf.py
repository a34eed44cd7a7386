"""GPU: a model read from a GGUF file by s2k_model_load_gguf (the reader
without ggml) is the model uploaded tensor by tensor: same device weight
bytes and the same greedy frames as the oracle, for the Q8_0, Q4_K_M and F16
schemes."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
import s2k
import synthetic
from gguf_fixture import write_model_gguf

pytestmark = pytest.mark.gpu
pytest.importorskip("gguf")


@pytest.mark.parametrize("quant", ["q8_0", "q4_k_m", "f16"])
def test_load_gguf_matches_upload(tmp_path, quant):
    hp = synthetic.preset("small")
    tensors = list(synthetic.make_model(hp, seed=8, quant=quant, norm_std=0.1))
    path = os.path.join(tmp_path, f"m_{quant}.gguf")
    write_model_gguf(path, hp, tensors)
    m = s2k.SlowARModel.from_gguf(path)
    ref = s2k.SlowARModel(hp)
    om = oracle.OracleModel(hp)
    try:
        ref.load_tensors(tensors)
        om.load_tensors(tensors)
        assert m.weight_bytes() == ref.weight_bytes()
        p = synthetic.text_prompt(hp, 12, seed=12)
        got = m.generate(p, 16, temperature=0.0, seed=3, im_end_id=-1)
        assert np.array_equal(got, ref.generate(p, 16, temperature=0.0, seed=3, im_end_id=-1))
        assert np.array_equal(got, om.generate(p, 16, temperature=0.0, seed=3, im_end_id=-1))
    finally:
        m.close()
        ref.close()
        om.close()
