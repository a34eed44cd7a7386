"""Generates the committed golden fixtures in this directory.

Run in a container that has gguf-py (0.19.0 was used):
    python tests/golden/make_golden.py

quants.npz
    Random valid Q8_0 / Q4_K / Q6_K blocks and their dequantized values from
    gguf-py's gguf/quants.py (documented there as matching ggml's
    dequantize_row_*), plus random f32 rows and their Q8_0 blocks from
    gguf.quants.Q8_0.quantize_blocks (documented as bit-exact with ggml's
    reference quantizer quantize_row_q8_0_ref).  These pin the oracle's block
    codecs and the synthetic-weight quantizer.
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _f16_scale(rng, n, lo=1e-4, hi=5e-2):
    return rng.uniform(lo, hi, size=n).astype(np.float16)


def q8_0_blocks(rng, n):
    d = _f16_scale(rng, n).view(np.uint8).reshape(n, 2)
    q = rng.integers(-128, 128, size=(n, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    return np.concatenate([d, q], axis=1)


def q4_k_blocks(rng, n):
    d = _f16_scale(rng, n).view(np.uint8).reshape(n, 2)
    dmin = _f16_scale(rng, n).view(np.uint8).reshape(n, 2)
    scales = rng.integers(0, 256, size=(n, 12), dtype=np.int16).astype(np.uint8)
    qs = rng.integers(0, 256, size=(n, 128), dtype=np.int16).astype(np.uint8)
    return np.concatenate([d, dmin, scales, qs], axis=1)


def q6_k_blocks(rng, n):
    ql = rng.integers(0, 256, size=(n, 128), dtype=np.int16).astype(np.uint8)
    qh = rng.integers(0, 256, size=(n, 64), dtype=np.int16).astype(np.uint8)
    sc = rng.integers(-128, 128, size=(n, 16), dtype=np.int16).astype(np.int8).view(np.uint8)
    d = _f16_scale(rng, n).view(np.uint8).reshape(n, 2)
    return np.concatenate([ql, qh, sc, d], axis=1)


def main() -> None:
    from gguf import quants

    rng = np.random.default_rng(20261201)
    out = {}
    b = q8_0_blocks(rng, 64)
    out["q8_0_blocks"] = b
    out["q8_0_deq"] = quants.Q8_0.dequantize_blocks(b).astype(np.float32).reshape(-1)
    b = q4_k_blocks(rng, 16)
    out["q4_k_blocks"] = b
    out["q4_k_deq"] = quants.Q4_K.dequantize_blocks(b).astype(np.float32).reshape(-1)
    b = q6_k_blocks(rng, 16)
    out["q6_k_blocks"] = b
    out["q6_k_deq"] = quants.Q6_K.dequantize_blocks(b).astype(np.float32).reshape(-1)
    x = (rng.standard_normal((48, 32)) * rng.uniform(0.001, 3.0, size=(48, 1))).astype(np.float32)
    x[0] = 0.0  # all-zero block (d = 0)
    x[1, :] = 0.0
    x[1, 5] = -1.0  # single negative max
    out["q8_0_src"] = x.reshape(-1)
    out["q8_0_quant"] = quants.Q8_0.quantize_blocks(x).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "quants.npz"), **out)
    print("wrote", os.path.join(HERE, "quants.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
