"""GPU failure detection, in the forms that fault, trap or hang no GPU:

  * a bounded device wait that runs out: the model's wait limit is set to
    ~1 ms and a warp waits for an activation tag nobody writes; the call
    returns S2K_ERR_TIMEOUT and, with the default limit back, the model
    decodes exactly as before;
  * an injected device-allocation failure (host-side hook in the model's
    allocator): the call returns S2K_ERR_OOM, leaves no half-built state, and
    the model's device bytes go back to where they were;
  * a scheduler request whose admission fails: it alone is marked FAILED, the
    other requests finish with their single-sequence codes and every KV page
    returns to the pool.
"""
from __future__ import annotations

import numpy as np
import pytest

import s2k
import synthetic

pytestmark = pytest.mark.gpu

ERR_OOM, ERR_TIMEOUT = -2, -6


@pytest.fixture(scope="module")
def small_gpu(small_model_data):
    hp, tensors = small_model_data
    m = s2k.SlowARModel(hp)
    m.load_tensors(tensors)
    yield m
    m.close()


def test_wait_timeout_returns_status_and_model_recovers(small_gpu, small_oracle, small_model_data):
    hp, _ = small_model_data
    p = synthetic.text_prompt(hp, 10, seed=6)
    before = small_gpu.generate(p, 12, temperature=0.0, seed=1, im_end_id=-1)
    small_gpu.set_wait_limit(2_000_000)  # ~1 ms of SM cycles
    with pytest.raises(s2k.S2KError) as e:
        small_gpu.wait_probe()
    assert e.value.status == ERR_TIMEOUT
    small_gpu.set_wait_limit(0)  # back to the default
    after = small_gpu.generate(p, 12, temperature=0.0, seed=1, im_end_id=-1)
    assert np.array_equal(before, after)
    assert np.array_equal(after, small_oracle.generate(p, 12, temperature=0.0, seed=1, im_end_id=-1))


def test_injected_oom_then_recovery(small_model_data, small_oracle):
    hp, tensors = small_model_data
    m = s2k.SlowARModel(hp)
    try:
        m.load_tensors(tensors)
        base = m.device_bytes()
        p = synthetic.text_prompt(hp, 40, seed=7)  # 40 tokens: a larger Slow workspace than finalize made
        m.init_kv_cache(64)
        with_seq = m.device_bytes()
        assert with_seq > base
        m.fail_alloc(0)
        with pytest.raises(s2k.S2KError) as e:
            m.prefill_fast(p.T.reshape(-1), 40)
        assert e.value.status == ERR_OOM
        assert m.n_past == 0
        # the failed workspace was released, not left half-built
        assert m.device_bytes() <= with_seq
        hg, lg = m.prefill_fast(p.T.reshape(-1), 40)
        small_oracle.init_kv_cache(64)
        ho, lo = small_oracle.eval(p.T.reshape(-1), 40)
        assert np.array_equal(lg, lo)
        # an OOM while creating a sequence leaves nothing allocated
        grown = m.device_bytes()
        m.fail_alloc(1)  # the second allocation of s2k_seq_create (V pages) fails
        with pytest.raises(s2k.S2KError) as e:
            m.init_kv_cache(128)
        assert e.value.status == ERR_OOM
        assert m.device_bytes() == grown - (with_seq - base)  # the old sequence was freed, no new bytes held
    finally:
        m.close()


def test_sched_admission_failure_isolated(small_gpu, small_model_data):
    hp, _ = small_model_data
    sc = s2k.BatchScheduler(small_gpu, max_batch=4, max_seq_len=64)
    prompts = [synthetic.text_prompt(hp, 8 + i, seed=30 + i) for i in range(3)]
    ids = [sc.submit(p, 10, temperature=0.0, seed=1, seq_id=i, im_end_id=-1) for i, p in enumerate(prompts)]
    small_gpu.fail_alloc(0)  # the first admission's first device allocation fails
    sc.run()
    small_gpu.fail_alloc(-1)
    st, nf, rs = sc.poll_status(ids[0])
    assert st == s2k.REQ_FAILED and rs == ERR_OOM and nf == 0
    for i in (1, 2):
        assert sc.poll(ids[i])[0] == s2k.REQ_DONE
        want = small_gpu.generate(prompts[i], 10, temperature=0.0, seed=1, seq_id=i, im_end_id=-1)
        assert np.array_equal(sc.result(ids[i]), want)
    stats = sc.stats()
    assert stats["failed"] == 1 and stats["finished"] == 2
    assert stats["free_pages"] == stats["pool_pages"]
    with pytest.raises(s2k.S2KError):
        sc.result(ids[0])
    sc.close()
