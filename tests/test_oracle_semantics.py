"""CPU: the oracle follows the reference's sampler / generate / eval rules
(src/s2_sampler.cpp:42-99, src/s2_generate.cpp:11-216, src/s2_model.cpp:860-1255)."""
from __future__ import annotations

import numpy as np

import oracle
import synthetic


def test_sampler_greedy_and_ties():
    x = np.array([0.1, 2.0, 2.0, -1.0], np.float32)
    assert oracle.sample_token(x, 0.0, 0.8, 30) == 1  # tie -> lowest index
    assert oracle.sample_token(x, -1.0, 0.8, 30) == 1


def test_sampler_top_k_top_p_and_draw():
    x = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float32))
    # top_k = 1: only the best survives whatever u is
    for u in (0.0, 0.5, 0.999):
        assert oracle.sample_token(x, 1.0, 1.0, 1, u) == 0
    # top_p = 0.6: cumsum 0.5 (kept, i=0), 0.8 > 0.6 -> only item 0
    assert oracle.sample_token(x, 1.0, 0.6, 0, 0.9) == 0
    # top_p = 0.85 keeps {0, 1}: renormalised 0.625 / 0.375
    assert oracle.sample_token(x, 1.0, 0.85, 0, 0.6) == 0
    assert oracle.sample_token(x, 1.0, 0.85, 0, 0.63) == 1
    # full distribution, temperature 1: cdf 0.5 0.8 0.95 1.0
    assert oracle.sample_token(x, 1.0, 1.0, 0, 0.49) == 0
    assert oracle.sample_token(x, 1.0, 1.0, 0, 0.79) == 1
    assert oracle.sample_token(x, 1.0, 1.0, 0, 0.94) == 2
    assert oracle.sample_token(x, 1.0, 1.0, 0, 0.99) == 3


def test_eval_prefill_equals_incremental_up_to_f16_kv(small_oracle, small_model_data):
    """Prefill of T tokens vs (T-1)-prefill + step: the reference rounds only
    the *past* K/V to f16, so the two paths agree closely but not exactly."""
    hp, _ = small_model_data
    om = small_oracle
    p = synthetic.text_prompt(hp, 12)
    tm = p.T.copy()
    om.init_kv_cache(64)
    h1, l1 = om.eval(tm.reshape(-1), 12)
    om.init_kv_cache(64)
    om.eval(tm[:11].reshape(-1), 11)
    h2, l2 = om.eval(tm[11:].reshape(-1), 1)
    assert om.n_past == 12
    assert np.abs(l1 - l2).max() < 0.1 * l1.std()
    assert not np.array_equal(l1, l2)


def test_fast_decode_prefix_semantics(small_oracle, small_model_data):
    hp, _ = small_model_data
    om = small_oracle
    om.init_kv_cache(32)
    p = synthetic.semantic_prompt(hp, 4)
    h, _ = om.eval(p.T.reshape(-1), 4)
    a = om.fast_decode(h, [5])
    b = om.fast_decode(h, [5])
    assert np.array_equal(a, b)
    c = om.fast_decode(h, [6])
    assert not np.array_equal(a, c)
    assert om.fast_decode(h, []).shape == (hp.codebook_size,)


def test_generate_rules(small_oracle, small_model_data):
    hp, _ = small_model_data
    om = small_oracle
    p = synthetic.text_prompt(hp, 8)
    codes = om.generate(p, 20, temperature=0.0, seed=3, im_end_id=-1)
    assert codes.shape == (hp.num_codebooks, 20)
    assert (codes >= 0).all() and (codes < hp.codebook_size).all()
    # determinism of the seeded RNG path (RAS resampling included)
    assert np.array_equal(codes, om.generate(p, 20, temperature=0.0, seed=3, im_end_id=-1))
    # im_end = the token greedy picks first, blocked for the first 5 frames
    _, logits = (om.init_kv_cache(64), om.eval(p.T.reshape(-1), 8))[1]
    masked = np.full_like(logits, -np.inf)
    masked[hp.semantic_begin_id:hp.semantic_end_id + 1] = logits[hp.semantic_begin_id:hp.semantic_end_id + 1]
    first = int(np.argmax(masked))
    stop = om.generate(p, 20, temperature=0.0, seed=3, im_end_id=first)
    assert stop.shape[1] == 0  # the first sampled token is im_end -> no frame
    blocked = om.generate(p, 20, temperature=0.0, seed=3, im_end_id=first, min_tokens_before_end=5)
    assert blocked.shape[1] >= 5
