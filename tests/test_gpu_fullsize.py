"""GPU parity on the full S2 Pro model the benchmark times: 36 Slow layers +
4 Fast layers at d 2560, GQA 32/8, ff 9728, vocab 155,648, Q8_0 weights
N(0, 0.02), norm weights N(1, 0.1), against the CPU oracle on the same
seeded weights and inputs.

  * the Slow step over a cache of 512 N(0,1) f16 positions with a seeded text
    token (the single-step workload: src/s2_model.cpp:860-1097): logits and
    hidden state bit-exact;
  * 64 greedy frames after a 64-token seeded text prompt (the frame-loop
    workload: src/s2_generate.cpp:11-216): identical semantic and codebook
    tokens, and the first Slow step of that loop bit-exact;
  * sampled frames (T 0.7, top-p 0.9, top-k 30, seeded device RNG): identical
    codes.
The persistent kernel runs every layer's split counters and activation tags at
full depth here (36 layers x 148 CTAs).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import s2k
import synthetic
from parity_util import assert_exact

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def s2pro_pair():
    hp = synthetic.preset("s2pro")
    tensors = list(synthetic.make_model(hp, seed=41, norm_std=0.1))
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    yield hp, m, om
    m.close()
    om.close()


def random_kv(hp, n_pos: int, seed: int):
    rng = np.random.default_rng(seed)
    shape = (hp.block_count, n_pos, hp.head_count_kv, hp.head_dim)
    return (rng.standard_normal(shape, dtype=np.float32).astype(np.float16),
            rng.standard_normal(shape, dtype=np.float32).astype(np.float16))


def test_slow_step_over_512_cached_positions(s2pro_pair):
    hp, m, om = s2pro_pair
    k, v = random_kv(hp, 512, seed=512)
    m.init_kv_cache(520)
    om.init_kv_cache(520)
    m.load_kv(k, v)
    om.load_kv(k, v)
    assert m.n_past == om.n_past == 512
    rng = np.random.default_rng(77)
    for i in range(2):
        tok = np.zeros(hp.num_codebooks + 1, np.int32)
        tok[0] = rng.integers(0, hp.semantic_begin_id)  # a text token: the codebook sum is masked out
        hg, lg = m.step(tok)
        ho, lo = om.eval(tok, 1)
        assert_exact(hg, ho, f"S2 Pro step {i} hidden at {512 + i} cached positions")
        assert_exact(lg, lo, f"S2 Pro step {i} logits at {512 + i} cached positions")
    assert m.n_past == om.n_past == 514


def test_greedy_64_frames_after_64_token_prompt(s2pro_pair):
    hp, m, om = s2pro_pair
    p = synthetic.text_prompt(hp, 64, seed=64)
    want = om.generate(p, 64, temperature=0.0, seed=3, im_end_id=-1)
    got = m.generate(p, 64, temperature=0.0, seed=3, im_end_id=-1)
    assert got.shape == want.shape == (hp.num_codebooks, 64)
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"first differing (codebook, frame): {bad[0].tolist()}"


def test_prefill_then_step_logits(s2pro_pair):
    """The 64-token prefill (tensor-core GEMMs) and the Slow step after it."""
    hp, m, om = s2pro_pair
    p = synthetic.text_prompt(hp, 64, seed=64)
    m.init_kv_cache(72)
    om.init_kv_cache(72)
    hg, lg = m.prefill_fast(p.T.reshape(-1), 64)
    ho, lo = om.eval(p.T.reshape(-1), 64)
    assert_exact(lg, lo, "S2 Pro 64-token prefill logits")
    tok = np.zeros(hp.num_codebooks + 1, np.int32)
    tok[1:] = np.arange(hp.num_codebooks) * 401 % hp.codebook_size
    tok[0] = hp.semantic_begin_id + tok[1]
    hg, lg = m.step(tok)
    ho, lo = om.eval(tok, 1)
    assert_exact(lg, lo, "S2 Pro semantic step logits")
    for n in (1, 9):
        prefix = (np.arange(n) * 733 % hp.codebook_size).astype(np.int32)
        assert_exact(m.fast_decode(ho, prefix), om.fast_decode(ho, prefix), f"S2 Pro fast_decode prefix {n}")


def test_sampled_frames(s2pro_pair):
    hp, m, om = s2pro_pair
    p = synthetic.semantic_prompt(hp, 24, seed=5)
    kw = dict(temperature=0.7, top_p=0.9, top_k=30, seed=11, im_end_id=-1)
    want = om.generate(p, 16, **kw)
    got = m.generate(p, 16, **kw)
    assert np.array_equal(got, want)
