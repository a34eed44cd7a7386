"""GPU parity at long contexts (S2 Pro widths, 2 Slow + 1 Fast layer, Q8_0,
norm weights N(1, 0.1)), where every attention path runs many 64-key splits:

  * the prompt-prefill attention (one CTA per kv head and 64 query vectors)
    over 1,024 and 4,096 prompt tokens, then the persistent kernel's
    attention in the frame loop at 1,024+ and 4,096+ cached positions;
  * the standalone attention kernels of single steps and short calls over a
    restored cache of 4,096 N(0,1) positions (src/s2_model.cpp:1007-1039);
  * the split-parallel attention of batched frames with more splits per row
    than CTAs per row (8 sequences at ~1,300 positions: each CTA strides over
    several splits).
All bit-exact against the oracle (logits) or code-identical (frames).
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
def mid_pair():
    hp = synthetic.preset("mid")
    tensors = list(synthetic.make_model(hp, seed=31, norm_std=0.1))
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    yield hp, m, om
    m.close()
    om.close()


@pytest.mark.parametrize("T", [1024, 4096])
def test_long_prompt_prefill_and_frames(mid_pair, T):
    hp, m, om = mid_pair
    p = synthetic.text_prompt(hp, T, seed=T)
    m.init_kv_cache(T + 8)
    om.init_kv_cache(T + 8)
    hg, lg = m.prefill_fast(p.T.reshape(-1), T)
    ho, lo = om.eval(p.T.reshape(-1), T)
    assert_exact(hg, ho, f"{T}-token prefill hidden")
    assert_exact(lg, lo, f"{T}-token prefill logits")
    want = om.generate(p, 6, temperature=0.0, seed=2, im_end_id=-1)
    got = m.generate(p, 6, temperature=0.0, seed=2, im_end_id=-1)
    assert np.array_equal(got, want), f"frames after a {T}-token prompt"


def test_steps_over_restored_4096_cache(mid_pair):
    hp, m, om = mid_pair
    rng = np.random.default_rng(4096)
    shape = (hp.block_count, 4096, hp.head_count_kv, hp.head_dim)
    k = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    v = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    m.init_kv_cache(4200)
    om.init_kv_cache(4200)
    m.load_kv(k, v)
    om.load_kv(k, v)
    # a single step (split-parallel attention, one CTA per split)
    tok = np.zeros(hp.num_codebooks + 1, np.int32)
    tok[0] = 777
    hg, lg = m.step(tok)
    ho, lo = om.eval(tok, 1)
    assert_exact(lg, lo, "step at 4,096 cached positions")
    # a 4-token call (one CTA per kv head and row over all splits)
    p = synthetic.semantic_prompt(hp, 4, seed=4)
    hg, lg = m.prefill_fast(p.T.reshape(-1), 4)
    ho, lo = om.eval(p.T.reshape(-1), 4)
    assert_exact(lg, lo, "4-token call at 4,097 cached positions")
    # a 40-token call (query-block attention over 4,101+ keys)
    p = synthetic.text_prompt(hp, 40, seed=40)
    hg, lg = m.prefill_fast(p.T.reshape(-1), 40)
    ho, lo = om.eval(p.T.reshape(-1), 40)
    assert_exact(lg, lo, "40-token call at 4,101 cached positions")
    assert m.n_past == om.n_past == 4141


def test_batched_frames_many_splits(mid_pair):
    hp, m, om = mid_pair
    sc = s2k.BatchScheduler(m, max_batch=8, max_seq_len=1408)
    prompts = [synthetic.text_prompt(hp, 1280 + 16 * i, seed=100 + i) for i in range(8)]
    ids = [sc.submit(p, 3, temperature=0.0, seed=1, seq_id=i, im_end_id=-1) for i, p in enumerate(prompts)]
    sc.run()
    for i, (rid, p) in enumerate(zip(ids, prompts)):
        want = om.generate(p, 3, temperature=0.0, seed=1, seq_id=i, im_end_id=-1)
        assert np.array_equal(sc.result(rid), want), f"request {i}"
    sc.close()
