"""GPU parity for F16 (unquantized) weights against the CPU oracle, through
the C ABI.  The F16 mat-vec rounds the activation to fp16 (ggml's vec_dot_type
for F16 weights) and sums the exact fp16 x fp16 products in double, on both
sides, so decode is held to the same bars as Q8_0: bit-exact logits, identical
greedy codes, and batched frames equal to single-sequence frames.  Prompts of
8+ tokens prefill through the fp16 tensor-core GEMM (fp32 sums), which, and
the steps reading the K/V it cached, are held to 1e-2 * std(logits)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import s2k
import synthetic
from parity_util import assert_close, assert_exact

pytestmark = pytest.mark.gpu



@pytest.fixture(scope="module")
def f16_pair():
    hp = synthetic.preset("small")
    tensors = list(synthetic.make_model(hp, seed=23, quant="f16", norm_std=0.1))
    assert {spec.type for spec, _ in tensors if spec.ne1 > 1} == {synthetic.GGML_F16}
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    yield hp, m, om
    m.close()
    om.close()


def test_f16_steps_and_fast(f16_pair):
    hp, m, om = f16_pair
    p = synthetic.semantic_prompt(hp, 6)
    m.init_kv_cache(64)
    om.init_kv_cache(64)
    hg, lg = m.prefill_fast(p.T.reshape(-1), 6)
    ho, lo = om.eval(p.T.reshape(-1), 6)
    assert_exact(hg, ho, "f16 prefill hidden")
    assert_exact(lg, lo, "f16 prefill logits")
    rng = np.random.default_rng(3)
    for i in range(4):
        tok = np.zeros(hp.num_codebooks + 1, np.int32)
        tok[1:] = rng.integers(0, hp.codebook_size, hp.num_codebooks)
        tok[0] = hp.semantic_begin_id + tok[1] if i % 2 == 0 else rng.integers(0, hp.semantic_begin_id)
        hg, lg = m.step(tok)
        ho, lo = om.eval(tok, 1)
        assert_exact(lg, lo, f"f16 step {i} logits")
    for n in range(hp.num_codebooks):
        prefix = rng.integers(0, hp.codebook_size, n).astype(np.int32)
        assert_exact(m.fast_decode(ho, prefix), om.fast_decode(ho, prefix), f"f16 fast_decode {n}")


def test_f16_generate_greedy_64(f16_pair):
    hp, m, om = f16_pair
    p = synthetic.text_prompt(hp, 7)
    want = om.generate(p, 64, temperature=0.0, seed=7, im_end_id=-1)
    got = m.generate(p, 64, temperature=0.0, seed=7, im_end_id=-1)
    assert got.shape == want.shape == (hp.num_codebooks, 64)
    assert np.array_equal(got, want)


def test_f16_generate_sampled(f16_pair):
    hp, m, om = f16_pair
    p = synthetic.semantic_prompt(hp, 5)
    kw = dict(temperature=0.7, top_p=0.9, top_k=0, seed=11, im_end_id=-1)
    assert np.array_equal(m.generate(p, 24, **kw), om.generate(p, 24, **kw))


def test_f16_batched_frames(f16_pair):
    hp, m, _ = f16_pair
    reqs = [(synthetic.text_prompt(hp, 5 + i, seed=40 + i), 6 + 3 * i,
             dict(temperature=0.7 if i % 2 else 0.0, top_p=0.9, top_k=0, seed=100 + i, seq_id=i, im_end_id=-1))
            for i in range(3)]
    sc = s2k.BatchScheduler(m, 3, 48)
    ids = [sc.submit(p, f, **kw) for p, f, kw in reqs]
    sc.run()
    for i, (p, f, kw) in zip(ids, reqs):
        assert np.array_equal(sc.result(i), m.generate(p, f, **kw)), i
    sc.close()


def test_f16_weight_bytes(f16_pair):
    """Device bytes equal the GGUF bytes of every matrix (2 B per weight)."""
    hp, m, _ = f16_pair
    gguf = sum(spec.nbytes for spec in synthetic.tensor_specs(hp, "f16", 0.1) if spec.ne1 > 1)
    assert m.weight_bytes() == gguf


@pytest.mark.parametrize("T", [8, 64, 300])
def test_f16_prefill_tensor_cores(f16_pair, T):
    """Prompts of 8+ tokens prefill through the fp16 tensor-core GEMM (fp32
    accumulation; 64- and 256-token tiles, a partial last tile at 300):
    logits within the tolerance of the oracle, then decode steps too."""
    hp, m, om = f16_pair
    p = synthetic.text_prompt(hp, T, seed=T)
    m.init_kv_cache(T + 8)
    om.init_kv_cache(T + 8)
    hg, lg = m.prefill_fast(p.T.reshape(-1), T)
    ho, lo = om.eval(p.T.reshape(-1), T)
    assert_close(hg, ho, f"f16 tc prefill hidden T={T}")
    assert_close(lg, lo, f"f16 tc prefill logits T={T}")
    for i in range(2):
        tok = np.zeros(hp.num_codebooks + 1, np.int32)
        tok[0] = 3 + i
        hg, lg = m.step(tok)
        ho, lo = om.eval(tok, 1)
        assert_close(lg, lo, f"f16 step {i} after tc prefill T={T}")


def test_f16_mid_real_widths():
    """S2 Pro widths (d 2560, GQA 32/8, ff 9728, vocab 155,648), F16: a
    72-token tensor-core prefill and decode steps against the oracle."""
    hp = synthetic.preset("mid")
    tensors = list(synthetic.make_model(hp, seed=29, quant="f16", norm_std=0.1))
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    p = synthetic.semantic_prompt(hp, 72, seed=2)
    m.init_kv_cache(80)
    om.init_kv_cache(80)
    _, lg = m.prefill_fast(p.T.reshape(-1), 72)
    ho, lo = om.eval(p.T.reshape(-1), 72)
    assert_close(lg, lo, "f16 mid prefill logits")
    tok = np.zeros(hp.num_codebooks + 1, np.int32)
    tok[0] = 1000
    _, lg = m.step(tok)
    ho, lo = om.eval(tok, 1)
    assert_close(lg, lo, "f16 mid step logits")
    assert_exact(m.fast_decode(ho, np.array([5, 9], np.int32)), om.fast_decode(ho, np.array([5, 9], np.int32)),
                 "f16 mid fast_decode")
    m.close()
    om.close()
