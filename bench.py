#!/usr/bin/env python
"""Benchmark of the per-frame dual-AR decode path (frames/s).

Workload (one "step"): one utterance through the full dual-AR frame loop on
the S2 Pro shape with Q8_0 weights at batch 1: a 64-token seeded text prompt
is prefilled, then 200 frames are decoded greedily (each frame = 9 Fast-AR
passes + samples + one Slow-AR step + sample).  Weights are seeded synthetic
N(0, 0.02) quantized to Q8_0 (no checkpoints offline).  min_tokens_before_end
is set to the frame count so every step yields exactly 200 frames.

Multi-GPU: one process per GPU (torchrun); each rank decodes its own
utterance with no collective on the data path (request-level sharding,
"weak" scaling).  Timing: CUDA events on the library's stream, barrier +
synchronize on both sides, max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python bench.py --workload ragged [--utterances 64] [--steps 1] [--warmup 1]

--workload ragged measures continuous batching instead: 64 utterances
(prompts ~U[64, 1024] tokens, ~U[100, 1500] frames, stop by length) dealt
round-robin to the GPUs, each GPU decoding its share as one continuously
refilled batch (s2k_sched_*); frames/s over the whole job, prefills included.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "s2.cpp_b200"))

import shard  # noqa: E402
import synthetic  # noqa: E402

PROMPT = 64
FRAMES = 200
SEED = 1234
METRIC = "codec frames/s (dual-AR frame loop, Q8_0, bs=1 per GPU)"


def frame_metric(quant: str) -> str:
    """The frame-loop metric for a weight scheme (the headline one for Q8_0)."""
    return METRIC if quant == "q8_0" else METRIC.replace("Q8_0", quant.upper())
WORKLOAD = ("dual-AR frame loop, S2 Pro shape (36+4 layers, d2560, GQA 32/8, ff 9728, vocab 155648), "
            "Q8_0, bs=1: 64-token text prompt prefill + 200 greedy frames")


# DRAM traffic / algorithmic bytes of the persistent kernel, measured with
# ncu (dram__bytes_read.sum + dram__bytes_write.sum) on the same kernel with
# 2 Slow + 1 Fast-AR layers at full widths (bench.py --preset mid, launches
# 18 and 19): Slow segment 645.58 MB for 638.36 MB, Fast-AR segment 121.95 MB
# for 118.37 MB.  Traffic grows with the bytes streamed, so full-size
# launches are scaled by these ratios.
TRAFFIC_RATIO_SLOW = 645.58 / 638.36
TRAFFIC_RATIO_FAST = 121.95 / 118.37


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "tflops": float(d.get("bf16_tflops", 1590.0)), "src": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "src": "fallback"}


def codec_flops(ch, n_tr: int, n_dec: int) -> float:
    """Algorithmic FLOPs (2 per multiply-add) of a codec decode over n_tr
    transformer frames and n_dec decoder frames: the matrix products and
    convolutions of the reference graph (each transposed convolution once, as
    the reference computes it)."""
    d, hd, ff = ch.rvq_dim, ch.rvq_head_dim, ch.rvq_ff
    H = d // hd
    Hk = ch.rvq_n_local_heads if ch.rvq_n_local_heads > 0 else H
    keys = min(ch.rvq_window_size, n_tr) if ch.rvq_window_size > 0 else n_tr
    f = ch.rvq_n_layer * 2.0 * n_tr * (d * (H + 2 * Hk) * hd + H * hd * d + 3 * d * ff + 2 * H * hd * keys)
    L, C = n_dec, d
    for fac in reversed(ch.quantizer_downsample_factor):
        f += 2.0 * L * fac * C * C
        L *= fac
        f += 2.0 * L * C * (ch.dw_kernel + 2 * ch.convnext_hidden)
    f += 2.0 * L * ch.decoder_dim * C * 7
    C = ch.decoder_dim
    for r in ch.decoder_rates:
        co = C // 2
        f += 2.0 * L * (r * co) * (2 * C)
        L *= r
        f += 3 * 2.0 * L * co * co * 8
        C = co
    return f + 2.0 * L * C * 7


def codec_decode(with_cpu: bool, reps: int = 10, warmup: int = 3) -> dict:
    """The codec decode after the frame loop (AudioCodec::decode,
    src/s2_codec.cpp:1297-1447) on the S2 Pro codec shapes with seeded F16
    weights: one decode of a 160-frame window (the offline windowed decode's
    transformer span at stride 16 / history 144) timed with the library's CUDA
    events, the tensor-core FLOP rate against the measured dense bf16/f16
    peak, and the windowed decode of a 215-frame (10 s) utterance.  Beside
    it the CPU oracle on a 2-frame sample."""
    import s2k  # noqa: E402
    ch = synthetic.codec_preset("s2pro")
    tensors = list(synthetic.make_codec(ch, seed=6))
    c = s2k.AudioCodec(ch)
    c.load_tensors(tensors)
    out = {"workload": "codec decode, S2 Pro codec shapes (8-layer 1024-wide windowed transformer, 1536->96 "
                       "channel decoder, 2048 samples/frame), F16 weights"}
    n = 160
    codes = synthetic.codec_codes(ch, n, seed=160)
    dev = []
    for i in range(warmup + reps):
        _, ms, _ = c.decode_windowed(codes, n, 0)  # one window: the whole 160 frames
        if i >= warmup:
            dev.append(ms)
    ms = float(np.median(dev))
    fl = codec_flops(ch, n, n)
    pk = peaks()
    out["window_160"] = {"ms": ms, "flops": fl, "achieved_tflops": fl / (ms / 1e3) / 1e12,
                         "peak_tflops": pk["tflops"], "frac": fl / (ms / 1e3) / 1e12 / pk["tflops"],
                         "peak_src": pk["src"], "audio_s": n * ch.samples_per_frame / ch.sample_rate}
    utt = synthetic.codec_codes(ch, 215, seed=215)
    c.decode_windowed(utt, 16)
    t = time.perf_counter()
    audio, wms, nb = c.decode_windowed(utt, 16)
    wall = (time.perf_counter() - t) * 1e3
    out["windowed_215"] = {"device_ms": wms, "wall_ms": wall, "windows": nb, "audio_s": audio.size / ch.sample_rate,
                           "rtf": wall / 1e3 / (audio.size / ch.sample_rate),
                           "receptive_frames": c.receptive_frames()}
    if with_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle  # noqa: E402  (cpu_baseline leg only)
        oracle.set_threads(os.cpu_count() or 1)
        co = oracle.CodecOracle(ch)
        co.load_tensors(tensors)
        sample = synthetic.codec_codes(ch, 2, seed=2)
        t = time.perf_counter()
        want = co.decode(sample)
        cpu_s = time.perf_counter() - t
        got = c.decode(sample)
        d = np.abs(got.astype(np.float64) - want)
        out["cpu_oracle"] = {"ms_per_frame": cpu_s * 1e3 / 2, "cores": os.cpu_count() or 1, "sample": "2 frames",
                             "gpu_max_abs_diff": float(d.max()), "gpu_rms_diff": float(np.sqrt(np.mean(d * d)))}
        co.close()
    c.close()
    return out


def workload(preset: str, quant: str, prompt: int, frames: int) -> str:
    if preset != "s2pro":
        return f"{preset} preset (profiling only)"
    if quant == "q8_0" and prompt == PROMPT and frames == FRAMES:
        return WORKLOAD
    return (f"dual-AR frame loop, S2 Pro shape, {quant}, bs=1: {prompt}-token text prompt prefill + "
            f"{frames} greedy frames")


def weight_stream_bytes(hp, quant: str) -> tuple[float, float]:
    """GGUF bytes of the matrices one Slow step and one Fast-AR pass stream in
    full (the embedding tables are gathered row by row and not counted)."""
    slow = fast = 0.0
    for spec in synthetic.tensor_specs(hp, quant):
        if spec.ne1 <= 1 or spec.name in ("codebook_embeddings.weight", "fast_embeddings.weight"):
            continue
        if spec.name.startswith("fast_"):
            fast += spec.nbytes
        else:
            slow += spec.nbytes
    return slow, fast


def frame_bytes(hp, ctx0: int, frames: int, quant: str = "q8_0") -> float:
    """Algorithmic bytes of one step's frames: weights streamed per frame (Slow
    step + 9 Fast-AR passes) + f16 KV read by the Slow step."""
    slow, fast = weight_stream_bytes(hp, quant)
    kv_per_pos = hp.block_count * 2 * hp.head_count_kv * hp.head_dim * 2
    total = 0.0
    for f in range(frames):
        total += slow + (hp.num_codebooks - 1) * fast + kv_per_pos * (ctx0 + f + 1)
    return total


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    def __init__(self, dev: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(dev), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 7:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def build_weights(hp, threads: int, quant: str = "q8_0"):
    synthetic._lib().s2synth_set_threads(threads)
    return list(synthetic.make_model(hp, seed=SEED, quant=quant, norm_std=0.0))


def cpu_sample(hp, tensors, frames_sample: int, prompt_len: int = PROMPT, frames: int = FRAMES) -> dict:
    """The CPU oracle (C restatement of the reference path) on a bounded sample:
    the prompt prefill + `frames_sample` frames, scaled to the step's frames."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402  (cpu_baseline leg only)
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    prompt = synthetic.text_prompt(hp, prompt_len, seed=7)
    _, pre_ms, loop_ms = om.generate_timed(prompt, frames_sample, temperature=0.0, seed=SEED,
                                           min_tokens_before_end=frames_sample)
    om.close()
    per_frame = loop_ms / frames_sample
    step_s = (pre_ms + frames * per_frame) / 1e3
    return {"value": frames / step_s, "unit": "frames/s", "cores": cores, "kind": "port",
            "sample": f"oracle generate: {prompt_len}-token prefill ({pre_ms / 1e3:.1f} s) + {frames_sample} frames "
                      f"({per_frame / 1e3:.2f} s/frame), scaled to {frames} frames",
            "prefill_s": pre_ms / 1e3, "s_per_frame": per_frame / 1e3}


def frame_config(hp, quant: str, preset: str, prompt: int, frames: int, world: int) -> dict:
    """The `config` of the frame-loop workload, the same on both arms."""
    return {"workload": workload(preset, quant, prompt, frames),
            "prompt_tokens": prompt, "frames": frames, "batch_per_gpu": 1,
            "weights": f"seeded N(0,0.02) -> {quant}",
            "l2": f"inputs larger than L2 ({weight_stream_bytes(hp, quant)[0] / 1e9:.1f} GB of Slow weights per frame)",
            "parallelism": f"request-level x{world}, no collectives"}


def run_reference(args, rank: int, world: int) -> None:
    """--impl reference: the reference's CPU path on the host cores.  ggml is an
    un-vendored submodule of s2.cpp (absent), so the reference cannot be built;
    its restatement in oracle/ is timed instead, with every host thread.

    One step runs a bounded sample of the workload (the prompt prefill + a few
    frames; a whole 200-frame step takes minutes on the CPU): steps and
    ms_per_step are what ran.  value is the workload's rate from the measured
    prefill time and time per frame (medians over the steps)."""
    if rank != 0:
        return
    hp = synthetic.preset("s2pro")
    tensors = build_weights(hp, os.cpu_count() or 1)
    walls, runs = [], []
    for i in range(args.warmup + args.steps):
        t = time.perf_counter()
        r = cpu_sample(hp, tensors, args.cpu_frames)
        if i >= args.warmup:
            walls.append(time.perf_counter() - t)
            runs.append(r)
    pre_s = float(np.median([r["prefill_s"] for r in runs]))
    frame_s = float(np.median([r["s_per_frame"] for r in runs]))
    v = FRAMES / (pre_s + FRAMES * frame_s)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * float(np.mean(walls)),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q8_0", "data": "synthetic",
        "config": frame_config(hp, "q8_0", "s2pro", PROMPT, FRAMES, world),
        "step": {"frames_run": args.cpu_frames, "prompt_tokens": PROMPT,
                 "note": (f"each step ran the {PROMPT}-token prefill + {args.cpu_frames} greedy frames; value = "
                          f"{FRAMES} / (prefill_s + {FRAMES} x s_per_frame)"),
                 "prefill_s": pre_s, "s_per_frame": frame_s},
        "cpu_baseline": {k: runs[-1][k] for k in ("unit", "cores", "kind", "sample")} | {"value": v},
        "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "ggml (s2.cpp's compute backend) is an absent submodule; the C restatement in oracle/ is timed",
    }
    print(json.dumps(line), flush=True)


def slow_step_at_512(m, hp, tensors, with_cpu: bool, reps: int = 20, warmup: int = 3) -> dict:
    """The single-step workload: one Slow-AR step (s2k_eval, 1 text token, host
    token in and host logits out) over an f16 cache of 512 N(0,1) positions.
    Every rep restores the cache to exactly 512 positions first (untimed) and
    times the step with CUDA events on the model stream; median of `reps`
    after `warmup`.  Beside it the CPU oracle's step on the same cache."""
    import torch
    rng = np.random.default_rng(512)
    shape = (hp.block_count, 512, hp.head_count_kv, hp.head_dim)
    k = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    v = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    tok = np.zeros(hp.num_codebooks + 1, np.int32)
    tok[0] = int(rng.integers(0, hp.semantic_begin_id))
    m.init_kv_cache(513)
    dev = torch.device("cuda", m.device)
    stream = torch.cuda.ExternalStream(m.stream(), device=dev)
    times = []
    for i in range(warmup + reps):
        m.load_kv(k, v)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        _, logits = m.step(tok)
        e1.record(stream)
        torch.cuda.synchronize()
        if i >= warmup:
            times.append(e0.elapsed_time(e1))
    slow_b, _ = weight_stream_bytes(hp, "q8_0")
    kv_b = 512 * hp.block_count * 2 * hp.head_count_kv * hp.head_dim * 2
    ms = float(np.median(times))
    out = {"workload": "Slow-AR step, Q8_0, bs=1, 512 cached N(0,1) f16 positions, text token; host logits out",
           "ms_per_step": ms, "reps": reps, "warmup": warmup, "bytes": slow_b + kv_b,
           "achieved_gbs": (slow_b + kv_b) / (ms / 1e3) / 1e9}
    out["frac"] = out["achieved_gbs"] / peaks()["hbm_gbs"]
    if with_cpu and tensors is not None:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle  # noqa: E402  (cpu_baseline leg only)
        oracle.set_threads(os.cpu_count() or 1)
        om = oracle.OracleModel(hp)
        om.load_tensors(tensors)
        om.init_kv_cache(513)
        cpu = []
        for _ in range(3):
            om.load_kv(k, v)
            t = time.perf_counter()
            _, lo = om.eval(tok, 1)
            cpu.append(time.perf_counter() - t)
        om.close()
        out["cpu_oracle_ms_per_step"] = 1e3 * float(np.median(cpu))
        out["cpu_cores"] = os.cpu_count() or 1
        out["logits_equal_cpu"] = bool(np.array_equal(lo, logits))
    return out


RAGGED_UTTS = 64
RAGGED_METRIC = "codec frames/s, continuous ragged batching (Q8_0), aggregate over GPUs"


def ragged_requests(hp, n_utts: int, frames_scale: float = 1.0):
    """The continuous-batching workload: n_utts independent utterances with
    seeded prompt lengths ~U[64, 1024] and target frame counts ~U[100, 1500]
    (scaled by frames_scale), stop by length (no end token)."""
    rng = np.random.default_rng(SEED)
    out = []
    for i in range(n_utts):
        cols = int(rng.integers(64, 1025))
        frames = max(1, int(round(int(rng.integers(100, 1501)) * frames_scale)))
        prompt = synthetic.text_prompt(hp, cols, seed=SEED + 17 * i)
        out.append((i, prompt, frames))
    return out


def run_ragged(args, rank: int, world: int, local: int) -> None:
    """Continuous ragged batching: the utterances are dealt round-robin to the
    ranks; each rank's scheduler admits, prefills and decodes its share as one
    continuously refilled batch over a 16-token-page KV pool."""
    import torch
    import torch.distributed as dist
    import s2k  # noqa: E402

    dist_on = world > 1
    if dist_on:
        torch.cuda.set_device(local)
        shard.init("nccl", local, timeout_s=600)
    torch.cuda.set_device(local)
    hp = synthetic.preset(args.preset)
    threads = max(1, (os.cpu_count() or 8) // max(world, 1))
    tensors = build_weights(hp, threads, args.quant)
    m = s2k.SlowARModel(hp, device=local)
    m.load_tensors(tensors)
    del tensors
    reqs = [r for r in ragged_requests(hp, args.utterances, args.frames_scale) if r[0] % world == rank]
    max_len = max(p.shape[1] + f + 1 for _, p, f in reqs)
    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))
    kw = dict(temperature=0.0, top_p=0.8, top_k=30, im_end_id=-1, seed=SEED)

    def job(rs, sched):
        for i, p, f in rs:
            sched.submit(p, f, seq_id=i, **kw)
        sched.run()

    sc = s2k.BatchScheduler(m, max_batch=len(reqs), max_seq_len=max_len)
    # warm-up: every batch size once (one more request finishes each frame),
    # so the timed run instantiates no frame graph
    warm = [(i, synthetic.text_prompt(hp, 16, seed=i), i + 1) for i in range(len(reqs))]
    for _ in range(args.warmup):
        job(warm, sc)
    torch.cuda.synchronize()
    if dist_on:
        dist.barrier()
    st0 = sc.stats()
    clocks = Clocks(local)
    s2k.launch_count(reset=True)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        job(reqs, sc)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t_wall) * 1e3
    launches = s2k.launch_count()
    clk = clocks.stop()
    st1 = sc.stats()
    ms = ev0.elapsed_time(ev1)
    frames_rank = sum(f for _, _, f in reqs) * args.steps
    assert st1["frames"] - st0["frames"] == frames_rank, (st1, st0, frames_rank)
    if dist_on:
        dist.barrier()
    ms_max = shard.max_over_ranks(ms, f"cuda:{local}")
    wall_max = shard.max_over_ranks(wall_ms, f"cuda:{local}")
    frames_all = sum(f for _, _, f in ragged_requests(hp, args.utterances, args.frames_scale)) * args.steps
    value = frames_all / (ms_max / 1e3)
    e2e = frames_all / (wall_max / 1e3)
    slow_b, fast_b = weight_stream_bytes(hp, args.quant)
    kv_per_pos = hp.block_count * 2 * hp.head_count_kv * hp.head_dim * 2
    steps_run = st1["steps"] - st0["steps"]
    dec_bytes = steps_run * (slow_b + (hp.num_codebooks - 1) * fast_b) + (st1["kv_positions"] - st0["kv_positions"]) * kv_per_pos
    pk = peaks()
    res = sc.result(len(warm) * args.warmup)  # first timed request: shape check
    assert res.shape == (hp.num_codebooks, reqs[0][2]), res.shape
    sc.close()
    m.close()
    if rank == 0:
        line = {
            "metric": RAGGED_METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.quant, "data": "synthetic",
            "config": {"workload": (f"{args.utterances} utterances, prompts ~U[64,1024] tokens, frames ~U[100,1500]"
                                    f" x{args.frames_scale:g}, stop by length, S2 Pro shape, {args.quant}; round-robin "
                                    f"over {world} GPU(s), one continuous batch per GPU, 16-token KV pages"),
                       "utterances": args.utterances, "frames_total": frames_all // args.steps,
                       "max_batch_per_gpu": st1["max_live"],
                       "l2": "inputs larger than L2 (4.3 GB of Slow weights per batched frame)",
                       "parallelism": f"request-level x{world}, no collectives"},
            "e2e": {"value": e2e, "unit": "frames/s", "h2d_bytes_per_step": int(sum(p.nbytes for _, p, _ in reqs)),
                    "d2h_bytes_per_step": int(4 * hp.num_codebooks * frames_rank // args.steps),
                    "note": "host prompts in, host codes out through s2k_sched_*; wall clock"},
            "frame_roofline": {"achieved": dec_bytes / (ms / 1e3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                               "frac": dec_bytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"],
                               "bytes": dec_bytes, "batched_frames": steps_run,
                               "note": "weights once per batched frame + f16 KV of every live sequence, over the "
                                       "whole job's time (prefill included)"},
            "prefill_tokens": st1["prefill_tokens"] - st0["prefill_tokens"],
            "clocks": clk,
            "gpu_launches": int(launches),
        }
        print(json.dumps(line), flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


LONG_UTTS = 8
LONG_PROMPT = 4096
LONG_FRAMES = 2000
LONG_METRIC = "codec frames/s, F16 weights, long context (4096-token prompt + 2000 sampled frames), aggregate"


def run_long(args, rank: int, world: int, local: int) -> None:
    """F16 long-context decode: LONG_UTTS utterances, each a LONG_PROMPT-token
    prompt then --frames-scale x LONG_FRAMES frames sampled at temperature 0.7,
    top-p 0.9 with the device RNG, dealt round-robin to the GPUs.  A GPU with
    one utterance runs the batch-1 frame loop (s2k_generate_device); a GPU
    with several decodes them as one continuous batch (s2k_sched_*)."""
    import torch
    import torch.distributed as dist
    import s2k  # noqa: E402

    dist_on = world > 1
    if dist_on:
        torch.cuda.set_device(local)
        shard.init("nccl", local, timeout_s=900)
    torch.cuda.set_device(local)
    hp = synthetic.preset(args.preset)
    threads = max(1, (os.cpu_count() or 8) // max(world, 1))
    tensors = build_weights(hp, threads, "f16")
    m = s2k.SlowARModel(hp, device=local)
    m.load_tensors(tensors)
    del tensors
    frames = max(1, int(round(LONG_FRAMES * args.frames_scale)))
    P = args.long_prompt
    mine = [i for i in range(args.utterances) if i % world == rank]
    prompts = {i: synthetic.semantic_prompt(hp, P, seed=SEED + 31 * i) for i in mine}
    kw = dict(temperature=0.7, top_p=0.9, top_k=0, im_end_id=-1, seed=SEED, min_tokens_before_end=frames)
    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))
    if len(mine) == 1:
        i = mine[0]
        m.init_kv_cache(P + frames + 1)
        d_prompt = torch.from_numpy(np.ascontiguousarray(prompts[i].T)).to(f"cuda:{local}")
        d_codes = torch.zeros((hp.num_codebooks, frames), dtype=torch.int32, device=f"cuda:{local}")

        def job(nf):
            n = m.generate_device(d_prompt.data_ptr(), P, d_codes.data_ptr(), nf, seq_id=i, **dict(kw, min_tokens_before_end=nf))
            assert n == nf, n
        warm = lambda: job(4)  # noqa: E731
        mode = "batch-1 frame loop"
    else:
        sc = s2k.BatchScheduler(m, max_batch=len(mine), max_seq_len=P + frames + 1)

        def job(nf):
            for i in mine:
                sc.submit(prompts[i], nf, seq_id=i, **dict(kw, min_tokens_before_end=nf))
            sc.run()
        warm = lambda: [job(k) for k in (len(mine),)]  # noqa: E731
        mode = f"continuous batch of {len(mine)}"
    for _ in range(args.warmup):
        warm()
    torch.cuda.synchronize()
    if dist_on:
        dist.barrier()
    clocks = Clocks(local)
    s2k.launch_count(reset=True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        job(frames)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t_wall) * 1e3
    launches = s2k.launch_count()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if dist_on:
        dist.barrier()
    ms_max = shard.max_over_ranks(ms, f"cuda:{local}")
    wall_max = shard.max_over_ranks(wall_ms, f"cuda:{local}")
    frames_all = args.utterances * frames * args.steps
    slow_b, fast_b = weight_stream_bytes(hp, "f16")
    if len(mine) > 1:
        sc.close()
    m.close()
    if rank == 0:
        line = {
            "metric": LONG_METRIC, "value": frames_all / (ms_max / 1e3), "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": (f"{args.utterances} utterances x ({P}-token prompt + {frames} frames at T=0.7, "
                                    f"top-p 0.9, device RNG), S2 Pro shape, F16 weights; round-robin over {world} "
                                    f"GPU(s), {mode} per GPU"),
                       "weights_per_frame_bytes": slow_b + (hp.num_codebooks - 1) * fast_b,
                       "l2": "inputs larger than L2 (8.1 GB of Slow weights per frame)",
                       "parallelism": f"request-level x{world}, no collectives"},
            "e2e": {"value": frames_all / (wall_max / 1e3), "unit": "frames/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0, "note": "wall clock of the same run"},
            "clocks": clk,
            "gpu_launches": int(launches),
        }
        print(json.dumps(line), flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--frames", type=int, default=FRAMES)
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens prefilled before the frames")
    ap.add_argument("--quant", choices=sorted(synthetic.QUANT_SCHEMES), default="q8_0",
                    help="weight quantization scheme (q4_k_m: the mixed Q4_K / Q6_K workload)")
    ap.add_argument("--cpu-frames", type=int, default=2, help="frames in the CPU oracle sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-slow-step", action="store_true", help="skip the Slow step at 512 cached positions")
    ap.add_argument("--no-codec", action="store_true", help="skip the codec decode measurement")
    ap.add_argument("--preset", choices=["s2pro", "mid"], default="s2pro",
                    help="model shape; 'mid' (2+1 layers, real widths) is for small profiler captures only")
    ap.add_argument("--workload", choices=["frames", "ragged", "f16long"], default="frames",
                    help="frames: one utterance per GPU at batch 1 (default); ragged: continuous batching of "
                         "--utterances utterances dealt round-robin to the GPUs; f16long: F16 weights, 8 "
                         "utterances of a 4096-token prompt + 2000 sampled frames")
    ap.add_argument("--utterances", type=int, default=None)
    ap.add_argument("--long-prompt", type=int, default=LONG_PROMPT)
    ap.add_argument("--frames-scale", type=float, default=1.0,
                    help="ragged: scale of the target frame counts (1.0 = U[100, 1500])")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    rank, world, local = shard.dist_env()

    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "ragged":
        args.utterances = args.utterances or RAGGED_UTTS
        run_ragged(args, rank, world, local)
        return
    if args.workload == "f16long":
        args.utterances = args.utterances or LONG_UTTS
        run_long(args, rank, world, local)
        return

    import torch
    import torch.distributed as dist
    import s2k  # noqa: E402

    dist_on = world > 1
    if dist_on:
        torch.cuda.set_device(local)
        shard.init("nccl", local, timeout_s=300)
    torch.cuda.set_device(local)
    hp = synthetic.preset(args.preset)
    threads = max(1, (os.cpu_count() or 8) // max(world, 1))
    t0 = time.time()
    tensors = build_weights(hp, threads, args.quant)
    t_synth = time.time() - t0
    m = s2k.SlowARModel(hp, device=local)
    m.load_tensors(tensors)
    if not (rank == 0 and world == 1 and not args.no_cpu_baseline):
        del tensors
        tensors = None
    frames = args.frames
    utt = shard.utterance_for_rank(rank)  # this rank's utterance
    P = args.prompt
    prompt = synthetic.text_prompt(hp, P, seed=utt["prompt_seed"])
    m.init_kv_cache(P + frames + 1)  # + 1: the slot the kernel profile below writes
    d_prompt = torch.from_numpy(np.ascontiguousarray(prompt.T)).to(f"cuda:{local}")
    d_codes = torch.zeros((hp.num_codebooks, frames), dtype=torch.int32, device=f"cuda:{local}")
    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))
    kw = dict(temperature=0.0, top_p=0.8, top_k=30, min_tokens_before_end=frames, im_end_id=-1, seed=SEED,
              seq_id=utt["seq_id"])

    def step():
        n = m.generate_device(d_prompt.data_ptr(), P, d_codes.data_ptr(), frames, **kw)
        assert n == frames, n

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist_on:
        dist.barrier()
    clocks = Clocks(local)
    torch.cuda.synchronize()
    s2k.launch_count(reset=True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = s2k.launch_count()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if dist_on:
        dist.barrier()
    ms = shard.max_over_ranks(ms, f"cuda:{local}")
    ms_per_step = ms / args.steps
    value = shard.aggregate_rate(world, args.steps, frames, ms)

    timed_codes = d_codes.cpu().numpy()
    # end to end through the host API: host prompt in, host codes out
    e2e_times = []
    for _ in range(args.steps):
        torch.cuda.synchronize()
        a = time.perf_counter()
        out = m.generate(prompt, frames, **kw)
        e2e_times.append(time.perf_counter() - a)
        assert out.shape == (hp.num_codebooks, frames)
    # the timed run decoded the request the host API decodes
    codes_match = bool(np.array_equal(timed_codes, out))
    assert codes_match, "timed frames differ from an untimed generate of the same request"
    e2e_s = shard.max_over_ranks(float(np.sum(e2e_times)), f"cuda:{local}")
    e2e_value = shard.aggregate_rate(world, args.steps, frames, e2e_s * 1e3)

    # dominant kernel: the persistent decode kernel (mega_kernel), one launch per
    # Fast-AR pass and one per Slow step; each launch event-timed on its stream
    ms_s, ms_f, b_s, b_f = m.profile_frame(reps=5)
    nf = hp.num_codebooks - 1
    mk_bytes = (b_s + nf * b_f) / (nf + 1)
    mk_ms = (ms_s + nf * ms_f) / (nf + 1)
    pk = peaks()
    achieved = mk_bytes / (mk_ms / 1e3) / 1e9
    # the standalone GEMV kernel of s2k_eval / s2k_fast_decode, for comparison
    gb, gms, glaunch = m.profile_gemv(reps=5)
    fb = frame_bytes(hp, P, frames, args.quant)
    step_bytes = fb  # + prefill weights, counted separately below
    frame_achieved = step_bytes / (ms_per_step / 1e3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and tensors is not None:
        try:
            cpu = cpu_sample(hp, tensors, args.cpu_frames, P, frames)
        except Exception as e:  # reported, never fatal
            cpu = {"value": None, "error": str(e)}
    step512 = None
    if args.preset == "s2pro" and args.quant == "q8_0" and not args.no_slow_step:
        step512 = slow_step_at_512(m, hp, tensors, with_cpu=cpu is not None and cpu.get("value") is not None)
    codec = None
    if rank == 0 and world == 1 and not args.no_codec:
        try:
            codec = codec_decode(with_cpu=cpu is not None and cpu.get("value") is not None)
        except Exception as e:  # reported, never fatal
            codec = {"error": str(e)}

    if rank == 0:
        line = {
            "metric": frame_metric(args.quant), "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.quant, "data": "synthetic",
            "config": frame_config(hp, args.quant, args.preset, P, frames, world),
            "e2e": {"value": e2e_value, "unit": "frames/s", "h2d_bytes_per_step": int(prompt.nbytes),
                    "d2h_bytes_per_step": int(hp.num_codebooks * frames * 4)},
            "roofline": {"bound": "hbm", "kernel": "mega_kernel (persistent decode kernel, 9 Fast-pass + 1 Slow-step "
                                                   "launches per frame)",
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "peak_src": pk["src"],
                         "traffic": (TRAFFIC_RATIO_SLOW * b_s + nf * TRAFFIC_RATIO_FAST * b_f) / (nf + 1),
                         "traffic_src": "ncu dram bytes of the same kernel at 2+1 layers, scaled by bytes streamed",
                         "bytes_per_launch": mk_bytes,
                         "launch_ms": mk_ms, "slow_launch": {"ms": ms_s, "bytes": b_s},
                         "fast_launch": {"ms": ms_f, "bytes": b_f}},
            "gemv_roofline": {"kernel": "gemv_q8_0 (standalone, s2k_eval path): Slow-step weight GEMV chain",
                              "achieved": gb / (gms / 1e3) / 1e9, "frac": gb / (gms / 1e3) / 1e9 / pk["hbm_gbs"],
                              "unit": "GB/s", "launches": glaunch, "ms_per_pass": gms},
            "frame_roofline": {"achieved": frame_achieved, "frac": frame_achieved / pk["hbm_gbs"], "unit": "GB/s",
                               "bytes_per_step": step_bytes},
            "cpu_baseline": cpu,
            "slow_step_512": step512,
            "codec_decode": codec,
            "timed_codes_match_generate": codes_match,
            "clocks": clk,
            "gpu_launches": int(launches),
            "setup_s": {"synth": t_synth},
        }
        print(json.dumps(line), flush=True)
    m.close()
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
