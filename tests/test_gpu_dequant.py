"""GPU dequantization bit-exact against gguf-py's published vectors.

The golden blocks of tests/golden/quants.npz (random valid Q8_0 / Q4_K / Q6_K
blocks and their values from gguf-py 0.19.0's dequantize_blocks, documented
there as matching ggml's dequantize_row_*) are tiled into a token-embedding
table, uploaded through s2k_model_upload_tensor (so they pass the device
re-layout) and read back row by row with s2k_get_rows, which uses the
element dequantization every embedding gather of the decode path uses.  F16
rows must come back as numpy's float16 -> float32.  Bar: array_equal.
"""
from __future__ import annotations

import numpy as np
import pytest

import s2k
import synthetic

pytestmark = pytest.mark.gpu

GOLDEN_BLOCKS = {synthetic.GGML_Q8_0: ("q8_0_blocks", "q8_0_deq"), synthetic.GGML_Q4_K: ("q4_k_blocks", "q4_k_deq"),
                 synthetic.GGML_Q6_K: ("q6_k_blocks", "q6_k_deq")}


def table_from_golden(golden, ggml_type: int, rows: int, dim: int):
    """A [rows][dim] table of golden blocks (tiled) and its expected values."""
    bkey, dkey = GOLDEN_BLOCKS[ggml_type]
    blocks, deq = golden[bkey], golden[dkey]
    per_block = deq.size // blocks.shape[0]
    nb = rows * dim // per_block
    idx = (np.arange(nb) * 7 + np.arange(nb) // blocks.shape[0]) % blocks.shape[0]  # varied order
    raw = blocks[idx].reshape(-1)
    vals = deq.reshape(blocks.shape[0], per_block)[idx].reshape(rows, dim)
    return raw, vals


@pytest.mark.parametrize("ggml_type", [synthetic.GGML_Q8_0, synthetic.GGML_Q4_K, synthetic.GGML_Q6_K,
                                       synthetic.GGML_F16])
def test_get_rows_bit_exact(golden, ggml_type):
    hp = synthetic.preset("small")
    tensors = list(synthetic.make_model(hp, seed=5, norm_std=0.1))
    dim = hp.embedding_length
    if ggml_type == synthetic.GGML_F16:
        rng = np.random.default_rng(16)
        h = (rng.standard_normal((hp.vocab_size, dim)) * rng.uniform(1e-3, 30, (hp.vocab_size, 1))).astype(np.float16)
        h.reshape(-1)[:6] = np.array([0.0, -0.0, 6.1e-5, -6.0e-8, 65504.0, -1.0], np.float16)  # zero, subnormal, max
        raw, want = h.view(np.uint8).reshape(-1), h.astype(np.float32)
    else:
        raw, want = table_from_golden(golden, ggml_type, hp.vocab_size, dim)
    out = []
    for spec, buf in tensors:
        if spec.name == "embeddings.weight":
            spec = synthetic.TensorSpec(spec.name, ggml_type, spec.ne0, spec.ne1, spec.std)
            buf = raw
        out.append((spec, buf))
    m = s2k.SlowARModel(hp)
    try:
        m.load_tensors(out)
        ids = np.array([0, 1, 2, 3, 5, 8, 13, 100, hp.vocab_size - 1], np.int32)
        got = m.get_rows("embeddings.weight", ids)
        assert np.array_equal(got.view(np.uint32), want[ids].view(np.uint32)), \
            f"type {ggml_type}: {int((got != want[ids]).sum())} values differ"
    finally:
        m.close()
