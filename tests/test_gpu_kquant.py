"""GPU parity for K-quant weights (the mixed Q4_K_M scheme: Q4_K attention /
FFN-up / embedding tables, Q6_K FFN-down and output projections) against the
CPU oracle, through the C ABI.  Same bars as the Q8_0 parity tests:
bit-exact logits, identical greedy codes."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import s2k
import synthetic
from parity_util import assert_exact

pytestmark = pytest.mark.gpu



@pytest.fixture(scope="module")
def kq_pair():
    hp = synthetic.preset("small")
    tensors = list(synthetic.make_model(hp, seed=21, quant="q4_k_m", norm_std=0.1))
    assert {spec.type for spec, _ in tensors} >= {synthetic.GGML_Q4_K, synthetic.GGML_Q6_K}
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    yield hp, m, om
    m.close()
    om.close()


def test_kquant_prefill_steps_fast(kq_pair):
    hp, m, om = kq_pair
    p = synthetic.semantic_prompt(hp, 16)
    m.init_kv_cache(64)
    om.init_kv_cache(64)
    hg, lg = m.prefill_fast(p.T.reshape(-1), 16)
    ho, lo = om.eval(p.T.reshape(-1), 16)
    assert_exact(hg, ho, "kquant prefill hidden")
    assert_exact(lg, lo, "kquant prefill logits")
    rng = np.random.default_rng(3)
    for i in range(4):
        tok = np.zeros(hp.num_codebooks + 1, np.int32)
        tok[1:] = rng.integers(0, hp.codebook_size, hp.num_codebooks)
        tok[0] = hp.semantic_begin_id + tok[1] if i % 2 == 0 else rng.integers(0, hp.semantic_begin_id)
        hg, lg = m.step(tok)
        ho, lo = om.eval(tok, 1)
        assert_exact(lg, lo, f"kquant step {i} logits")
    for n in range(hp.num_codebooks):
        prefix = rng.integers(0, hp.codebook_size, n).astype(np.int32)
        assert_exact(m.fast_decode(ho, prefix), om.fast_decode(ho, prefix), f"kquant fast_decode {n}")


def test_kquant_generate_greedy_64(kq_pair):
    hp, m, om = kq_pair
    p = synthetic.text_prompt(hp, 20)
    want = om.generate(p, 64, temperature=0.0, seed=7, im_end_id=-1)
    got = m.generate(p, 64, temperature=0.0, seed=7, im_end_id=-1)
    assert got.shape == want.shape == (hp.num_codebooks, 64)
    assert np.array_equal(got, want)


def test_kquant_weight_bytes(kq_pair):
    """Device bytes equal the GGUF bytes of every matrix (the re-layout keeps 144 / 210 B per super-block)."""
    hp, m, _ = kq_pair
    gguf = sum(spec.nbytes for spec in synthetic.tensor_specs(hp, "q4_k_m", 0.1) if spec.ne1 > 1)
    assert m.weight_bytes() == gguf


def test_kquant_prefill_long_prompt(kq_pair):
    """A 96-token prompt: the Slow stack's GEMMs run on the int8 tensor cores
    over the K-quant prefill copies (Q8_K rows, exact super-block terms in the
    epilogue; a 16-bit-activation path would leave the reference's Q8_K
    arithmetic by ~8 % of the logits' std), then decode steps."""
    hp, m, om = kq_pair
    p = synthetic.semantic_prompt(hp, 96, seed=4)
    m.init_kv_cache(128)
    om.init_kv_cache(128)
    hg, lg = m.prefill_fast(p.T.reshape(-1), 96)
    ho, lo = om.eval(p.T.reshape(-1), 96)
    assert_exact(hg, ho, "kquant long prefill hidden")
    assert_exact(lg, lo, "kquant long prefill logits")
    for i in range(3):
        tok = np.zeros(hp.num_codebooks + 1, np.int32)
        tok[0] = 17 + i
        hg, lg = m.step(tok)
        ho, lo = om.eval(tok, 1)
        assert_exact(lg, lo, f"kquant step {i} after long prefill")


@pytest.mark.parametrize("T", [64, 150])
def test_kquant_tensor_core_prefill_tiles(kq_pair, T):
    """The tensor-core K-quant prefill on one full 64-token tile and on three
    tiles with a partial last one (150 tokens), against the oracle's prefill
    of the same prompt (prefill semantics: every K/V row of the call in f32),
    then a decode step reading the cached f16 rows."""
    hp, m, om = kq_pair
    p = synthetic.text_prompt(hp, T, seed=100 + T)
    flat = p.T.reshape(-1)
    m.init_kv_cache(T + 4)
    om.init_kv_cache(T + 4)
    hg, lg = m.prefill_fast(flat, T)
    ho, lo = om.eval(flat, T)
    assert_exact(hg, ho, f"kquant tc prefill hidden T={T}")
    assert_exact(lg, lo, f"kquant tc prefill logits T={T}")
    tok = np.zeros(hp.num_codebooks + 1, np.int32)
    tok[0] = 9
    _, lg = m.step(tok)
    _, lo = om.eval(tok, 1)
    assert_exact(lg, lo, f"kquant step after tc prefill T={T}")


def test_kquant_tensor_core_prefill_real_widths():
    """S2 Pro widths (d 2560, GQA 32/8, ff 9728: Q4_K attention / FFN-up,
    Q6_K FFN-down over K = 9728), 2 Slow layers: a 72-token prefill through
    the tensor cores against the oracle, then a step."""
    hp = synthetic.preset("mid")
    tensors = list(synthetic.make_model(hp, seed=33, quant="q4_k_m", norm_std=0.1))
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    p = synthetic.semantic_prompt(hp, 72, seed=5)
    m.init_kv_cache(80)
    om.init_kv_cache(80)
    hg, lg = m.prefill_fast(p.T.reshape(-1), 72)
    ho, lo = om.eval(p.T.reshape(-1), 72)
    assert_exact(hg, ho, "kquant mid prefill hidden")
    assert_exact(lg, lo, "kquant mid prefill logits")
    tok = np.zeros(hp.num_codebooks + 1, np.int32)
    tok[0] = 1000
    _, lg = m.step(tok)
    _, lo = om.eval(tok, 1)
    assert_exact(lg, lo, "kquant mid step logits")
    m.close()
    om.close()


def test_kquant_batch_of_64_matches_single_sequence(kq_pair):
    """64 live sequences: the batched Slow GEMMs take 64 rows, so they run on
    the tensor-core K-quant path (the Fast-AR stack stays on the tile GEMV);
    every request's codes equal its single-sequence frame loop's."""
    hp, m, _ = kq_pair
    rng = np.random.default_rng(64)
    reqs = []
    for i in range(64):
        cols = int(rng.integers(4, 9))
        p = synthetic.text_prompt(hp, cols, seed=500 + i) if i % 2 else synthetic.semantic_prompt(hp, cols, seed=500 + i)
        kw = dict(temperature=0.0 if i % 3 == 0 else 0.7, top_p=0.9, top_k=30, seed=900 + i, seq_id=i, im_end_id=-1)
        reqs.append((p, 3, kw))
    sc = s2k.BatchScheduler(m, 64, 16)
    ids = [sc.submit(p, f, **kw) for p, f, kw in reqs]
    sc.run()
    st = sc.stats()
    got = [sc.result(i) for i in ids]
    sc.close()
    assert st["max_live"] == 64
    for i, (p, f, kw) in enumerate(reqs):
        assert np.array_equal(got[i], m.generate(p, f, **kw)), f"request {i}"


def test_kquant_prefill_layer_slots():
    """The tensor-core K-quant prefill reads int8 copies that are built one
    layer ahead into two alternating layer slots: a 6-layer model (every slot
    rebuilt three times per pass) against the oracle at 64 and 150 tokens,
    then a batched frame of 64 sequences; the copies take two layers of
    device memory, not one per layer."""
    import dataclasses
    hp = dataclasses.replace(synthetic.preset("small"), block_count=6)
    tensors = list(synthetic.make_model(hp, seed=61, quant="q4_k_m", norm_std=0.1))
    m = s2k.SlowARModel(hp)
    om = oracle.OracleModel(hp)
    try:
        m.load_tensors(tensors)
        om.load_tensors(tensors)
        layer_copy = sum(spec.ne0 * spec.ne1 * (2 if spec.type == synthetic.GGML_Q6_K else 1)
                         for spec, _ in tensors if spec.name.startswith("layers.0.") and spec.ne1 > 1)
        # weights + the two layer slots (plus workspaces), well under one copy per layer
        assert m.device_bytes() - m.weight_bytes() < 4 * layer_copy + (64 << 20)
        for T in (64, 150):
            p = synthetic.text_prompt(hp, T, seed=T + 1)
            m.init_kv_cache(T + 4)
            om.init_kv_cache(T + 4)
            hg, lg = m.prefill_fast(p.T.reshape(-1), T)
            ho, lo = om.eval(p.T.reshape(-1), T)
            assert_exact(lg, lo, f"6-layer kquant prefill logits T={T}")
            tok = np.zeros(hp.num_codebooks + 1, np.int32)
            tok[0] = 4
            _, lg = m.step(tok)
            _, lo = om.eval(tok, 1)
            assert_exact(lg, lo, f"6-layer kquant step after T={T}")
        sc = s2k.BatchScheduler(m, max_batch=64, max_seq_len=32)
        prompts = [synthetic.text_prompt(hp, 6 + i % 5, seed=200 + i) for i in range(64)]
        ids = [sc.submit(pp, 3, temperature=0.0, seed=1, seq_id=i, im_end_id=-1) for i, pp in enumerate(prompts)]
        sc.run()
        for i in (0, 17, 63):
            want = om.generate(prompts[i], 3, temperature=0.0, seed=1, seq_id=i, im_end_id=-1)
            assert np.array_equal(sc.result(ids[i]), want), i
        sc.close()
    finally:
        m.close()
        om.close()
