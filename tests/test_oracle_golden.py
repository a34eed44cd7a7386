"""CPU: pins the oracle's block codecs and helpers against gguf-py golden
vectors (tests/golden/quants.npz, made by tests/golden/make_golden.py) and
hand-derived known answers."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
import synthetic

Q8_0, Q4_K, Q6_K, F16 = 8, 12, 14, 1


@pytest.mark.parametrize("name,ggml_type,blk", [("q8_0", Q8_0, 32), ("q4_k", Q4_K, 256), ("q6_k", Q6_K, 256)])
def test_dequant_bit_exact_vs_gguf(golden, name, ggml_type, blk):
    blocks = golden[f"{name}_blocks"]
    want = golden[f"{name}_deq"]
    got = oracle.dequant_row(ggml_type, blocks.reshape(-1), blocks.shape[0] * blk)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_synth_q8_0_quantizer_bit_exact_vs_gguf(golden):
    x = golden["q8_0_src"]
    want = golden["q8_0_quant"]
    out = np.empty_like(want)
    synthetic._lib().s2synth_quantize_q8_0.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    synthetic._lib().s2synth_quantize_q8_0(x.ctypes.data, x.size, out.ctypes.data)
    assert np.array_equal(out, want)


def test_fp16_conversion_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * 10,
        np.array([0.0, -0.0, 65504.0, 65520.0, -65536.0, 6e-8, 3e-8, 1e-8, 5.96e-8, np.inf, -np.inf], np.float32),
        (rng.standard_normal(500) * 1e-5).astype(np.float32),
    ])
    for v in vals:
        got = oracle.lib().so_fp32_to_fp16(float(v))
        want = int(np.array([v], np.float32).astype(np.float16).view(np.uint16)[0])
        assert got == want, (v, hex(got), hex(want))
        back = oracle.lib().so_fp16_to_fp32(want)
        assert np.float32(back) == np.float16(np.uint16(want).view(np.float16)).astype(np.float32) or np.isnan(back)


def test_activation_q8_0_x86_rule():
    # amax 127 -> id = 1: ties round half to even (2.5 -> 2, 3.5 -> 4, -2.5 -> -2)
    x = np.zeros(32, np.float32)
    x[:5] = [127.0, 2.5, 3.5, -2.5, 0.49]
    b = oracle.quantize_act_q8_0(x)
    d = np.frombuffer(b[:2].tobytes(), np.float16)[0]
    q = b[2:].view(np.int8)
    assert d == np.float16(1.0)
    assert list(q[:5]) == [127, 2, 4, -2, 0]
    # zero block: d = 0, q = 0
    z = oracle.quantize_act_q8_0(np.zeros(32, np.float32))
    assert not z.any()
    # numpy restatement on random data
    rng = np.random.default_rng(1)
    x = rng.standard_normal(32 * 40).astype(np.float32)
    b = oracle.quantize_act_q8_0(x).reshape(-1, 34)
    xb = x.reshape(-1, 32)
    amax = np.abs(xb).max(1)
    ident = (np.float32(127.0) / amax).astype(np.float32)
    q = np.rint(xb * ident[:, None]).astype(np.int8)
    assert np.array_equal(b[:, 2:].view(np.int8), q)
    assert np.array_equal(b[:, :2].copy().view(np.float16)[:, 0], (amax / np.float32(127)).astype(np.float16))


def test_activation_q8_K_rule():
    rng = np.random.default_rng(2)
    x = rng.standard_normal(512).astype(np.float32)
    b = oracle.quantize_act_q8_K(x).reshape(-1, 292)
    for i, xb in enumerate(x.reshape(-1, 256)):
        j = int(np.argmax(np.abs(xb)))
        iscale = np.float32(-127.0) / xb[j]
        q = np.minimum(np.rint(iscale * xb), 127).astype(np.int8)
        assert np.array_equal(b[i, 4:260].view(np.int8), q)
        assert np.frombuffer(b[i, :4].tobytes(), np.float32)[0] == np.float32(1.0) / iscale
        bs = np.frombuffer(b[i, 260:].tobytes(), np.int16)
        assert np.array_equal(bs, q.astype(np.int32).reshape(16, 16).sum(1))


def test_vec_dot_matches_dequantized_dot():
    """The integer block dots equal dequant(W) . dequant(quant(x)) up to f32 rounding."""
    rng = np.random.default_rng(3)
    n = 512
    x = rng.standard_normal(n).astype(np.float32)
    for t, blk in [(Q8_0, 32)]:
        w = synthetic.make_tensor(synthetic.TensorSpec("w", t, n, 1, 0.02), seed=4)
        a = oracle.quantize_act_q8_0(x)
        got = oracle.vec_dot(t, w, a, n)
        wd = oracle.dequant_row(t, w, n).astype(np.float64)
        xd = oracle.dequant_row(Q8_0, a, n).astype(np.float64)
        assert abs(got - float(wd @ xd)) < 1e-5 * max(1.0, abs(float(wd @ xd)))


def test_philox_uniform_properties():
    u = np.array([oracle.philox_uniform(42, f, p, 0) for f in range(200) for p in range(12)])
    assert (u >= 0).all() and (u < 1).all()
    assert abs(u.mean() - 0.5) < 0.03
    assert oracle.philox_uniform(42, 3, 2, 0) == oracle.philox_uniform(42, 3, 2, 0)
    assert oracle.philox_uniform(42, 3, 2, 0) != oracle.philox_uniform(43, 3, 2, 0)
    assert oracle.philox_uniform(42, 3, 2, 0) != oracle.philox_uniform(42, 3, 2, 1)


def _expf_inputs(seed: int = 3) -> np.ndarray:
    """Every regime of the exp: random x over its whole finite range, a dense
    sweep where results turn subnormal (k < -126) and where they overflow,
    reductions that land on k = 0, and the special values."""
    rng = np.random.default_rng(seed)
    parts = [rng.uniform(-110.0, 95.0, 200_000), np.linspace(-104.5, -86.0, 100_001),
             np.linspace(87.0, 89.0, 20_001), rng.uniform(-0.4, 0.4, 20_000),
             np.array([0.0, -0.0, 1.0, -1.0, 88.72283935546875, 88.7228394, -103.972084045410156, -103.9721,
                       np.inf, -np.inf, np.nan])]
    return np.concatenate(parts).astype(np.float32)


def test_det_expf_scaling_equals_ldexpf():
    """The oracle's exp scales by 2^k with two IEEE products (so_pow2_scale),
    as the CUDA det_expf does: it must equal the C library's ldexpf (exact,
    or correctly rounded into the subnormals) for every reachable k."""
    assert oracle.check_pow2_scale(4000) == 0
    x = _expf_inputs()
    y = oracle.det_expf(x)
    fin = np.isfinite(x) & (x > -103.972084045410156) & (x < 88.72283935546875)
    ref = np.exp(x[fin].astype(np.float64))
    rel = np.abs(y[fin].astype(np.float64) - ref) / np.maximum(ref, np.finfo(np.float32).tiny)
    normal = ref >= np.finfo(np.float32).tiny
    assert rel[normal].max() < 4e-7  # ~2 ulp
    assert np.isnan(y[np.isnan(x)]).all() and y[x == np.inf][0] == np.inf and y[x == -np.inf][0] == 0.0
