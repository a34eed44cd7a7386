"""GPU: the streaming frame hand-off of generate (src/s2_generate.cpp:150-163,
src/s2_pipeline.cpp:1100-1115).

on_frame is called for each frame as soon as its codes reach host memory,
while later frames still decode on the device; a False return stops
generation within the look-ahead (no more than 4 frames past the aborted
one are decoded), keeps frames 0..f, and leaves n_past at cols + f, where the
reference's model stands when it breaks before the aborted frame's step().
The same hand-off per request in the continuous-batching scheduler, and its
cancel.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

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


def test_callback_aborts_at_frame_4_of_200(small_gpu, small_oracle, small_model_data):
    hp, _ = small_model_data
    p = synthetic.text_prompt(hp, 12, seed=3)
    want = small_oracle.generate(p, 200, temperature=0.0, seed=8, im_end_id=-1)
    # launches of the prefill and of one frame graph, from runs of 10 and 20 frames
    s2k.launch_count(reset=True)
    small_gpu.generate(p, 10, temperature=0.0, seed=8, im_end_id=-1)
    ten = s2k.launch_count(reset=True)
    small_gpu.generate(p, 20, temperature=0.0, seed=8, im_end_id=-1)
    twenty = s2k.launch_count(reset=True)
    per_frame = (twenty - ten) // 10
    prefill = ten - 10 * per_frame
    assert per_frame > 0 and twenty - ten == 10 * per_frame
    seen = []

    def cb(codes, idx, total):
        seen.append((idx, total, codes.copy()))
        return idx < 4

    got = small_gpu.generate(p, 200, temperature=0.0, seed=8, im_end_id=-1, on_frame=cb)
    aborted = s2k.launch_count(reset=True)
    assert got.shape == (hp.num_codebooks, 5)
    assert np.array_equal(got, want[:, :5])
    assert [s[0] for s in seen] == [0, 1, 2, 3, 4] and [s[1] for s in seen] == [1, 2, 3, 4, 5]
    for idx, _, c in seen:
        assert np.array_equal(c, want[:, idx])
    assert small_gpu.n_past == p.shape[1] + 4
    # no more frames decoded than the 5 handed over plus the look-ahead
    frames_launched = (aborted - prefill) / per_frame
    assert frames_launched <= 8, frames_launched


def test_callbacks_interleave_with_decoding(small_gpu, small_model_data):
    hp, _ = small_model_data
    p = synthetic.text_prompt(hp, 8, seed=4)
    stamps = []

    def cb(codes, idx, total):
        stamps.append(time.perf_counter())
        return True

    plain = small_gpu.generate(p, 200, temperature=0.0, seed=1, im_end_id=-1)  # also captures the frame graph
    t0 = time.perf_counter()
    out = small_gpu.generate(p, 200, temperature=0.0, seed=1, im_end_id=-1, on_frame=cb)
    t1 = time.perf_counter()
    assert out.shape[1] == 200 and len(stamps) == 200
    # frames reach the caller while decoding goes on: the first one long
    # before generate returns, and the callbacks spread over the decode
    assert stamps[0] - t0 < 0.25 * (t1 - t0)
    assert stamps[-1] - stamps[0] > 0.5 * (t1 - t0)
    # without a callback the codes are the same
    assert np.array_equal(out, plain)


def test_abort_then_continue_with_steps(small_gpu, small_oracle, small_model_data):
    """After an abort at frame f the sequence holds cols + f positions, so a
    step() continues from there as the reference's model would."""
    hp, _ = small_model_data
    p = synthetic.text_prompt(hp, 10, seed=5)
    codes = small_gpu.generate(p, 50, temperature=0.0, seed=2, im_end_id=-1, on_frame=lambda c, i, t: i < 6)
    assert codes.shape[1] == 7 and small_gpu.n_past == 10 + 6
    om = small_oracle
    assert np.array_equal(om.generate(p, 7, temperature=0.0, seed=2, im_end_id=-1), codes)
    # the oracle's model where the reference stops: prefill, then step() of frames 0..5
    om.init_kv_cache(40)
    om.eval(p.T.reshape(-1), p.shape[1])
    for f in range(6):
        sem = min(max(int(codes[0, f]), 0), hp.codebook_size - 1)
        tok = np.concatenate([[hp.semantic_begin_id + sem], codes[:, f]]).astype(np.int32)
        om.eval(tok, 1)
    tok = np.zeros(hp.num_codebooks + 1, np.int32)
    tok[0] = 11
    hg, lg = small_gpu.step(tok)
    ho, lo = om.eval(tok, 1)
    assert np.array_equal(lg, lo)
    assert small_gpu.n_past == om.n_past == 17


def test_sched_frame_callback_and_cancel(small_gpu, small_oracle, small_model_data):
    hp, _ = small_model_data
    sc = s2k.BatchScheduler(small_gpu, max_batch=4, max_seq_len=64)
    prompts = [synthetic.text_prompt(hp, 6 + 2 * i, seed=20 + i) for i in range(4)]
    ids = [sc.submit(p, 12, temperature=0.0, seed=1, seq_id=i, im_end_id=-1) for i, p in enumerate(prompts)]
    got = {rid: [] for rid in ids}

    def cb(rid, codes, idx):
        got[rid].append((idx, codes.copy()))
        return not (rid == ids[1] and idx == 2)  # request 1 stops after its frame 2

    sc.set_frame_callback(cb)
    sc.step()
    sc.step()
    sc.cancel(ids[3])  # a live request cancelled between frames
    sc.run()
    st = sc.stats()
    assert st["free_pages"] == st["pool_pages"]
    assert st["cancelled"] == 2
    for i, rid in enumerate(ids):
        want = small_oracle.generate(prompts[i], 12, temperature=0.0, seed=1, seq_id=i, im_end_id=-1)
        res = sc.result(rid)
        state = sc.poll(rid)[0]
        if i == 1:
            assert state == s2k.REQ_CANCELLED and res.shape[1] == 3
        elif i == 3:
            assert state == s2k.REQ_CANCELLED and res.shape[1] == 2
        else:
            assert state == s2k.REQ_DONE and res.shape[1] == 12
        assert np.array_equal(res, want[:, : res.shape[1]])
        assert [g[0] for g in got[rid]] == list(range(len(got[rid])))
        for idx, c in got[rid]:
            assert np.array_equal(c, want[:, idx])
    sc.close()


def test_generate_metrics(small_gpu, small_model_data):
    """The [Metrics] split of generate (src/s2_generate.cpp:185-199), device-timed."""
    hp, _ = small_model_data
    p = synthetic.text_prompt(hp, 9, seed=9)
    out = small_gpu.generate(p, 40, temperature=0.0, seed=1, im_end_id=-1)
    gm = small_gpu.last_metrics()
    assert gm["n_frames"] == out.shape[1] == 40 and gm["prompt_tokens"] == 9
    assert gm["prefill_ms"] > 0 and gm["loop_ms"] > 0
    assert abs(gm["total_ms"] - gm["prefill_ms"] - gm["loop_ms"]) < 1e-6
    assert abs(gm["ms_per_frame"] * 40 - gm["loop_ms"]) < 1e-6
    small_gpu.generate(p, 30, temperature=0.0, seed=1, im_end_id=-1, on_frame=lambda c, i, t: i < 2)
    assert small_gpu.last_metrics()["n_frames"] == 3
