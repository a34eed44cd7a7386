"""GPU parity of continuous batching: every request decoded inside a ragged,
continuously refilled batch must give exactly the codes the single-sequence
frame loop gives for it, and those of the CPU oracle.

Batching changes no arithmetic (the batched GEMMs, attention and samplers
compute each row as the single-sequence kernels do, and the sampling draws
are keyed by (seed, frame, seq_id)), so the bar is equality of every code,
greedy and sampled alike.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import s2k
import synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_gpu(small_model_data):
    hp, tensors = small_model_data
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    yield m
    m.close()


def _requests(hp, n, seed, max_prompt=40, max_frames=40):
    """Ragged requests: text / semantic prompts of seeded lengths, greedy and
    sampled parameters, distinct seeds and seq ids."""
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        cols = int(rng.integers(4, max_prompt + 1))
        p = (synthetic.text_prompt(hp, cols, seed=seed * 100 + i) if i % 2 == 0
             else synthetic.semantic_prompt(hp, cols, seed=seed * 100 + i))
        frames = int(rng.integers(1, max_frames + 1))
        kw = dict(temperature=0.0 if i % 3 == 0 else 0.7, top_p=0.9, top_k=30, seed=1000 + i, seq_id=i,
                  im_end_id=-1)
        out.append((p, frames, kw))
    return out


def _run_sched(m, reqs, max_batch, max_seq_len, pool_pages=0):
    sc = s2k.BatchScheduler(m, max_batch, max_seq_len, pool_pages)
    ids = [sc.submit(p, f, **kw) for p, f, kw in reqs]
    sc.run()
    res = [sc.result(i) for i in ids]
    st = sc.stats()
    sc.close()
    return res, st


def test_sched_matches_single_sequence(small_gpu, small_model_data):
    """12 ragged requests through 10 batch slots: batches of 10 (tensor-core
    GEMMs) shrink to 1 (tile GEMV) as requests finish and others join."""
    hp, _ = small_model_data
    reqs = _requests(hp, 12, seed=3)
    got, st = _run_sched(small_gpu, reqs, max_batch=10, max_seq_len=96)
    assert st["admitted"] == st["finished"] == 12
    assert st["max_live"] == 10
    assert st["frames"] == sum(f for _, f, _ in reqs)
    assert st["free_pages"] == st["pool_pages"]
    for i, (p, f, kw) in enumerate(reqs):
        want = small_gpu.generate(p, f, **kw)
        assert got[i].shape == want.shape == (hp.num_codebooks, f), i
        assert np.array_equal(got[i], want), f"request {i}"


def test_sched_matches_oracle(small_gpu, small_oracle, small_model_data):
    hp, _ = small_model_data
    reqs = _requests(hp, 5, seed=8, max_frames=24)
    got, _ = _run_sched(small_gpu, reqs, max_batch=3, max_seq_len=80)
    for i, (p, f, kw) in enumerate(reqs):
        want = small_oracle.generate(p, f, **kw)
        assert np.array_equal(got[i], want), f"request {i}"


def test_sched_page_pool_pressure(small_gpu, small_model_data):
    """A pool that holds two requests at a time: the others wait for pages
    that finished requests return."""
    hp, _ = small_model_data
    reqs = _requests(hp, 6, seed=11, max_prompt=30, max_frames=30)
    need = max((p.shape[1] + f + 1 + 15) // 16 for p, f, _ in reqs)
    got, st = _run_sched(small_gpu, reqs, max_batch=6, max_seq_len=80, pool_pages=2 * need)
    assert st["finished"] == 6 and st["free_pages"] == 2 * need
    assert st["max_live"] <= 2
    for i, (p, f, kw) in enumerate(reqs):
        assert np.array_equal(got[i], small_gpu.generate(p, f, **kw)), f"request {i}"


def test_sched_stops_at_im_end(small_gpu, small_model_data):
    """Requests with an end token leave the batch when they sample it."""
    hp, _ = small_model_data
    p = synthetic.text_prompt(hp, 10, seed=5)
    free = small_gpu.generate(p, 30, temperature=0.0, seed=2)
    ends = list(dict.fromkeys(int(hp.semantic_begin_id + t) for t in free[0]))
    reqs = []
    for i, c in enumerate(ends[:4]):
        reqs.append((p, 30, dict(temperature=0.0, seed=2, seq_id=0, im_end_id=c, min_tokens_before_end=2)))
    reqs.append((p, 12, dict(temperature=0.0, seed=2, seq_id=0, im_end_id=-1)))
    got, st = _run_sched(small_gpu, reqs, max_batch=5, max_seq_len=64)
    for i, (pp, f, kw) in enumerate(reqs):
        assert np.array_equal(got[i], small_gpu.generate(pp, f, **kw)), f"request {i}"
    assert any(g.shape[1] < 30 for g in got[:4])


def test_low_level_batch_frame(small_gpu, small_model_data):
    """s2k_seq_begin + s2k_batch_frame: sequences of different lengths; the
    finished ones drop out of later frames."""
    hp, _ = small_model_data
    reqs = _requests(hp, 3, seed=21, max_frames=12)
    seqs = []
    for p, f, kw in reqs:
        s = s2k.Sequence(small_gpu, p.shape[1] + f + 1)
        s.begin(p, f, **kw)
        seqs.append(s)
    for _ in range(max(f for _, f, _ in reqs) + 2):
        if s2k.batch_frame(small_gpu, seqs) == 0:
            break
    for s, (p, f, kw) in zip(seqs, reqs):
        codes, done = s.frames()
        assert done
        assert np.array_equal(codes, small_gpu.generate(p, f, **kw))
        s.close()


def test_sched_rejects_oversized_request(small_gpu, small_model_data):
    hp, _ = small_model_data
    sc = s2k.BatchScheduler(small_gpu, 2, 32)
    with pytest.raises(s2k.S2KError) as e:
        sc.submit(synthetic.text_prompt(hp, 20), 20)
    assert e.value.status == -4
    sc.close()


@pytest.fixture(scope="module")
def mid_model():
    hp = synthetic.preset("mid")
    tensors = list(synthetic.make_model(hp, seed=21, norm_std=0.1))
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    yield hp, m
    m.close()


def test_mid_batch_real_widths(mid_model):
    """S2 Pro widths (d 2560, GQA 32/8, ff 9728, vocab 155,648): 9 requests in
    one batch (tensor-core GEMMs on every projection and both LM heads)."""
    hp, m = mid_model
    reqs = _requests(hp, 9, seed=31, max_prompt=24, max_frames=10)
    got, st = _run_sched(m, reqs, max_batch=9, max_seq_len=48)
    assert st["max_live"] == 9
    for i, (p, f, kw) in enumerate(reqs):
        assert np.array_equal(got[i], m.generate(p, f, **kw)), f"request {i}"
