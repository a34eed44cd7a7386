#!/usr/bin/env python
"""Profiling entry points of the decode path (B200), for the summaries kept
with the repository.

  python s2.cpp_b200/s2k_profile.py prefill [--preset s2pro] [--quant q8_0] [--tokens 64,256,1024]
      CUDA-event time of prefill_fast (the whole Slow stack over a text
      prompt) and its dense-equivalent GEMM rate.

  python s2.cpp_b200/s2k_profile.py ops [--preset s2pro] [--quant q8_0] [--frames 200]
      Generates `frames` greedy frames after a 64-token prompt, then traces one
      Fast-AR pass and the Slow step of the persistent decode kernel
      (s2k_profile_trace) and prints, per op kind of a layer, the mean span and
      its parts: grid-barrier release, activation prologue, median / slowest
      CTA's work; and the attention op's phase stamps.

  python s2.cpp_b200/s2k_profile.py batch [--preset s2pro] [--sizes 1,8,16,32,64] [--context 512]
      CUDA-event time of one batched frame (s2k_batch_frame: every sequence's
      Fast-AR passes and Slow step as batched kernels) for each batch size,
      all sequences at `context` cached positions.  With --profile-one, one
      frame of the last size runs between cudaProfilerStart / Stop (for
      `ncu --profile-from-start off`).

  python s2.cpp_b200/s2k_profile.py codec [--frames 160] [--reps 2]
      The codec decode (s2k_codec_decode) of `frames` code frames on the S2
      Pro codec shapes, `reps` times: kernel launches per decode, host wall
      time per decode and the library's device time of one decode.  With
      --reps 2 the second decode is the one to capture (skip the first
      decode's launches).

Seeded synthetic weights (no checkpoints offline).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import s2k  # noqa: E402
import synthetic  # noqa: E402

OP_NAMES = ["qkv", "attn", "wo", "w13", "w2"]


def _model(preset: str, quant: str):
    hp = synthetic.preset(preset)
    synthetic._lib().s2synth_set_threads(os.cpu_count() or 8)
    m = s2k.SlowARModel(hp)
    m.load_tensors(synthetic.make_model(hp, seed=1234, quant=quant, norm_std=0.0))
    return hp, m


def cmd_prefill(a) -> None:
    import torch
    hp, m = _model(a.preset, a.quant)
    stream = torch.cuda.ExternalStream(m.stream())
    d, ff = hp.embedding_length, hp.feed_forward_length
    qkv = (hp.head_count + 2 * hp.head_count_kv) * hp.head_dim
    params = hp.block_count * (d * qkv + hp.head_count * hp.head_dim * d + 3 * d * ff)
    for T in [int(x) for x in a.tokens.split(",")]:
        p = synthetic.text_prompt(hp, T, seed=5).T.reshape(-1).copy()
        m.init_kv_cache(T + 8)
        m.prefill_fast(p, T)
        best = None
        for _ in range(3):
            m.init_kv_cache(T + 8)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            m.prefill_fast(p, T)
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        print(json.dumps(dict(preset=a.preset, quant=a.quant, tokens=T, ms=round(best, 3),
                              gemm_tflops_equiv=round(2 * params * T / (best / 1e3) / 1e12, 1),
                              weight_gb=round(m.weight_bytes() / 1e9, 3),
                              device_gb=round(m.device_bytes() / 1e9, 3))), flush=True)
    m.close()


def _layer_table(tr: np.ndarray, kinds: np.ndarray) -> dict:
    T = tr.astype(np.int64)
    n = T.shape[0] - 1
    st, pro, dn = T[:, :, 0], T[:, :, 1], T[:, :, 2]
    t0 = st[0].min()
    rows = []
    for i in range(n):
        prev = dn[i - 1].max() if i > 0 else t0
        nxt = st[i + 1].min()
        rows.append(dict(span=(nxt - prev) / 1e3, barrier=(np.median(st[i]) - prev) / 1e3,
                         prologue=np.median(pro[i] - st[i]) / 1e3, work_med=np.median(dn[i] - pro[i]) / 1e3,
                         work_max=(dn[i] - pro[i]).max() / 1e3))
    k = list(kinds)
    first = k.index(2) - 1
    nl = (n - first - 1) // 5
    out = {}
    for j, name in enumerate(OP_NAMES):
        sel = [rows[first + 5 * l + j] for l in range(nl)]
        out[name] = {key: round(float(np.mean([r[key] for r in sel])), 2) for key in sel[0]}
    out["layers"] = nl
    out["launch_us"] = round(float((st[n].max() - t0) / 1e3), 1)
    phases = {}
    names = {8: "qkv_rotated", 9: "cta_barrier", 4: "kv_in_smem", 5: "scores", 6: "softmax", 7: "values",
             10: "partials_fenced", 3: "arrival_counted", 2: "done"}
    for slot, nm in names.items():
        v = []
        for i in range(n):
            if kinds[i] != 2:
                continue
            for c in range(T.shape[1]):
                if T[i, c, 4] > 0 and T[i, c, slot] > 0:
                    v.append((T[i, c, slot] - T[i, c, 0]) / 1e3)
        if v:
            phases[nm] = [round(float(np.median(v)), 2), round(float(np.max(v)), 2)]
    out["attention_phases_us_median_max"] = phases
    return out


def _gemv_shapes(hp, fast: bool) -> dict:
    """(R, K) of the layer GEMVs of a segment, by op name."""
    if fast:
        d, H, Hkv, hd, ff = (hp.fast_embedding_length, hp.fast_head_count, hp.fast_head_count_kv, hp.fast_head_dim,
                             hp.fast_feed_forward_length)
    else:
        d, H, Hkv, hd, ff = hp.embedding_length, hp.head_count, hp.head_count_kv, hp.head_dim, hp.feed_forward_length
    return {"qkv": ((H + 2 * Hkv) * hd, d), "wo": (d, H * hd), "w13": (2 * ff, d), "w2": (d, ff)}


def _critical_table(tr: np.ndarray, kinds: np.ndarray, shapes: dict) -> dict:
    """Per op of a layer (mean over layers): `lat` = last CTA done of this op
    minus last CTA done of the previous op (the op's share of the launch's
    critical path).  For the GEMV ops, on the CTA that finished last (times
    after the previous op's last done): `quantized` = its activation
    quantized [7] (also the median and slowest CTA with work), for RMSNorm'd
    inputs `warp0` / `all_warps` = warp 0's squares summed [4] / every
    warp's, the norm scale known [5]; then `tile0` = first weight tile
    ready [6] after the prologue end [1], `tiles` = done [2] after [6], `n` =
    its weight tiles in the op, `issued` = the producer's last tile of the op issued [3]
    relative to [1] (negative: every tile was requested before the consumers
    needed it); `us_per_tile` = median over CTAs with work of ([2] - [6]) / n."""
    T = tr.astype(np.int64)
    n = T.shape[0] - 1
    G = T.shape[1]
    dn = T[:, :, 2]
    k = list(kinds)
    first = k.index(2) - 1
    nl = (n - first - 1) // 5
    acc = {nm: [] for nm in OP_NAMES}
    for l in range(nl):
        for j, nm in enumerate(OP_NAMES):
            i = first + 5 * l + j
            prev = dn[i - 1].max()
            c = int(dn[i].argmax())
            row = dict(lat=(dn[i].max() - prev) / 1e3)
            if nm in shapes:
                R, K = shapes[nm]
                RT, NKT = R // 32, K // 512
                ntile = np.array([(RT * (cc + 1) // G - RT * cc // G) * NKT for cc in range(G)])
                w = ntile > 0
                qz = T[i, :, 7] - prev
                row.update(quantized=(T[i, c, 7] - prev) / 1e3, quantized_med=float(np.median(qz[w])) / 1e3,
                           quantized_max=float(qz[w].max()) / 1e3, tile0=(T[i, c, 6] - T[i, c, 1]) / 1e3,
                           tiles=(T[i, c, 2] - T[i, c, 6]) / 1e3, n=int(ntile[c]),
                           issued=(T[i, c, 3] - T[i, c, 1]) / 1e3)
                if nm in ("qkv", "w13"):  # RMSNorm'd input: [4] warp 0's squares summed, [5] scale known
                    row.update(warp0=(T[i, c, 4] - prev) / 1e3, all_warps=(T[i, c, 5] - prev) / 1e3,
                               warp0_med=float(np.median(T[i, w, 4] - prev)) / 1e3,
                               all_warps_med=float(np.median(T[i, w, 5] - prev)) / 1e3)
                row["us_per_tile"] = float(np.median((T[i, w, 2] - T[i, w, 6]) / ntile[w])) / 1e3
            acc[nm].append(row)
    return {nm: {key: round(float(np.mean([r[key] for r in rows])), 2) for key in rows[0]} for nm, rows in acc.items()}


def cmd_ops(a) -> None:
    hp, m = _model(a.preset, a.quant)
    prompt = synthetic.text_prompt(hp, 64, seed=7)
    m.init_kv_cache(64 + a.frames + 1)
    m.generate(prompt, a.frames, temperature=0.0, min_tokens_before_end=a.frames, im_end_id=-1, seed=1234)
    ms_s, ms_f, b_s, b_f = m.profile_frame(reps=5)
    print(json.dumps(dict(ms_slow=round(ms_s, 4), ms_fast=round(ms_f, 4), frame_ms=round(ms_s + 9 * ms_f, 4))))
    for seg, label in ((1, "fast_ar_pass"), (-1, "slow_step")):
        tr = m.profile_trace(seg)
        _, kinds = m.profile_ops(seg, reps=1)
        print(json.dumps({label: _layer_table(tr, kinds)}), flush=True)
        crit = _critical_table(tr, kinds, _gemv_shapes(hp, seg > 0))
        print(json.dumps({label + "_critical_path": crit}), flush=True)
    m.close()


def cmd_batch(a) -> None:
    import torch
    hp, m = _model(a.preset, a.quant)
    stream = torch.cuda.ExternalStream(m.stream())
    sizes = [int(x) for x in a.sizes.split(",")]
    for n in sizes:
        seqs = []
        for i in range(n):
            s = s2k.Sequence(m, a.context + a.frames + 8)
            s.begin(synthetic.text_prompt(hp, a.context, seed=i), a.frames + 4, temperature=0.0, seed=1, seq_id=i,
                    min_tokens_before_end=a.frames + 4)
            seqs.append(s)
        for _ in range(3):
            s2k.batch_frame(m, seqs)
        torch.cuda.synchronize()
        if a.profile_one and n == sizes[-1]:
            torch.cuda.profiler.start()
            s2k.batch_frame(m, seqs)
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
        else:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(a.frames):
                s2k.batch_frame(m, seqs)
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / a.frames
            print(json.dumps(dict(preset=a.preset, quant=a.quant, sequences=n, context=a.context,
                                  ms_per_batched_frame=round(ms, 3), frames_per_s=round(n / ms * 1e3, 1))),
                  flush=True)
        for s in seqs:
            s.close()
    m.close()


def cmd_codec(a) -> None:
    import time
    ch = synthetic.codec_preset("s2pro")
    c = s2k.AudioCodec(ch)
    c.load_tensors(synthetic.make_codec(ch, seed=6))
    codes = synthetic.codec_codes(ch, a.frames, seed=a.frames)
    for i in range(a.reps):
        s2k.launch_count(True)
        t = time.perf_counter()
        c.decode(codes)
        wall = (time.perf_counter() - t) * 1e3
        print(json.dumps({"decode": i, "frames": a.frames, "launches": s2k.launch_count(True), "wall_ms": wall}))
    _, ms, _ = c.decode_windowed(codes, a.frames, 0)
    print(json.dumps({"device_ms": ms, "receptive_frames": c.receptive_frames()}))
    c.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("prefill")
    p.add_argument("--preset", default="s2pro")
    p.add_argument("--quant", default="q8_0")
    p.add_argument("--tokens", default="64,256,1024")
    o = sub.add_parser("ops")
    o.add_argument("--preset", default="s2pro")
    o.add_argument("--quant", default="q8_0")
    o.add_argument("--frames", type=int, default=200)
    b = sub.add_parser("batch")
    b.add_argument("--preset", default="s2pro")
    b.add_argument("--quant", default="q8_0")
    b.add_argument("--sizes", default="1,8,16,32,64")
    b.add_argument("--context", type=int, default=512)
    b.add_argument("--frames", type=int, default=20)
    b.add_argument("--profile-one", action="store_true")
    k = sub.add_parser("codec")
    k.add_argument("--frames", type=int, default=160)
    k.add_argument("--reps", type=int, default=2)
    a = ap.parse_args()
    {"prefill": cmd_prefill, "ops": cmd_ops, "batch": cmd_batch, "codec": cmd_codec}[a.cmd](a)


if __name__ == "__main__":
    main()
