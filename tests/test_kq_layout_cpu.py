"""CPU checks of the K-quant layouts and formulations the CUDA kernels use,
against ggml's definitions and the CPU oracle (no GPU).

* q4k_scales4 (s2k_tgemv.cuh): the eight 6-bit scales and mins of a Q4_K
  header decoded with byte masks equal ggml's get_scale_min_k4.
* q8k_swz (s2k_tgemv.cuh): the Q8_K activation swizzle is a permutation of
  every 512-byte block, and the eight lanes of each quarter-warp of the Q4_K
  and Q6_K consumers read eight different 16-byte bank groups.
* The tensor-core K-quant prefill (prefill_q8_kernel<64, KQ>, kq_build_kernel,
  quant_rows_q8k_kernel in s2k_prefill.cu) forms its super-block terms from
  per-block integer sums: Q4_K from 32-value sub-block sums with the Q8_K
  16-value block sums paired per sub-block, Q6_K from its 16-value sub-blocks
  each zero-padded to a 32-column block.  Restated here in numpy, row dots
  equal the oracle's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle

Q4_K, Q6_K = 12, 14


def get_scale_min_k4(j: int, q: np.ndarray) -> tuple[int, int]:
    """ggml get_scale_min_k4 over the 12 packed bytes q."""
    q = [int(v) for v in q]
    if j < 4:
        return q[j] & 63, q[j + 4] & 63
    return (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4), (q[j + 4] >> 4) | ((q[j] >> 6) << 4)


def scales4(q: np.ndarray) -> tuple[list[int], list[int]]:
    """q4k_scales4: byte masks over the words w0, w1, w2 of the 12 bytes."""
    w0, w1, w2 = (int(np.frombuffer(q[4 * i:4 * i + 4].tobytes(), "<u4")[0]) for i in range(3))
    sc_lo = w0 & 0x3F3F3F3F
    mn_lo = w1 & 0x3F3F3F3F
    sc_hi = (w2 & 0x0F0F0F0F) | ((w0 >> 2) & 0x30303030)
    mn_hi = ((w2 >> 4) & 0x0F0F0F0F) | ((w1 >> 2) & 0x30303030)
    sc = [(sc_lo >> (8 * j)) & 0xFF for j in range(4)] + [(sc_hi >> (8 * j)) & 0xFF for j in range(4)]
    mn = [(mn_lo >> (8 * j)) & 0xFF for j in range(4)] + [(mn_hi >> (8 * j)) & 0xFF for j in range(4)]
    return sc, mn


def test_q4k_register_scale_decode():
    rng = np.random.default_rng(0)
    for _ in range(2000):
        q = rng.integers(0, 256, 12, dtype=np.uint8)
        sc, mn = scales4(q)
        for j in range(8):
            assert (sc[j], mn[j]) == get_scale_min_k4(j, q), (q, j)


def q8k_swz(o: int, q6: bool) -> int:
    return o ^ (((o >> 6) & 6) << 4) if q6 else o ^ (((o >> 7) & 3) << 4)


@pytest.mark.parametrize("q6", [False, True])
def test_q8k_swizzle_permutation_and_banks(q6):
    for base in (0, 512, 4096):
        img = sorted(q8k_swz(base + o, q6) for o in range(512))
        assert img == list(range(base, base + 512))
    # the consumers' quarter-warps: 8 lanes of one weight row r, lane s = lane % 8
    for kt in range(3):
        for step in range(4):
            groups = []
            for s in range(8):
                sb = s >> 2
                if q6:
                    h, is_ = (s >> 1) & 1, s & 1
                    o = (kt * 2 + sb) * 256 + 128 * h + 16 * is_ + 32 * step
                else:
                    c = s & 3
                    o = (kt * 2 + sb) * 256 + 64 * c + 16 * step
                groups.append((q8k_swz(o, q6) >> 4) & 7)  # 16-byte bank group within 128 bytes
            assert len(set(groups)) == 8, (q6, kt, step, groups)


def random_q4k(rng, nsb: int) -> np.ndarray:
    blocks = rng.integers(0, 256, (nsb, 144), dtype=np.uint8)
    for b in range(nsb):
        for k, v in ((0, rng.uniform(1e-3, 4e-3)), (2, rng.uniform(1e-4, 2e-3))):
            blocks[b, k:k + 2] = np.frombuffer(np.float16(v).tobytes(), np.uint8)
    return blocks.reshape(-1)


def random_q6k(rng, nsb: int) -> np.ndarray:
    blocks = rng.integers(0, 256, (nsb, 210), dtype=np.uint8)
    for b in range(nsb):
        blocks[b, 192:208] = rng.integers(-60, 61, 16).astype(np.int8).view(np.uint8)
        blocks[b, 208:210] = np.frombuffer(np.float16(rng.uniform(1e-4, 1e-3)).tobytes(), np.uint8)
    return blocks.reshape(-1)


def q8k_parts(act: np.ndarray, nsb: int):
    """Q8_K super-blocks (oracle layout: float d, 256 int8, 16 int16 sums)."""
    a = act.reshape(nsb, 292)
    d = a[:, 0:4].copy().view(np.float32)[:, 0]
    q = a[:, 4:260].view(np.int8).astype(np.int64)
    bs = a[:, 260:292].copy().view(np.int16).astype(np.int64)
    return d, q, bs


def f16(b: np.ndarray) -> np.float32:
    return np.float32(b.copy().view(np.float16)[0])


def prefill_dot_q4k(w: np.ndarray, act: np.ndarray, nsb: int) -> np.float32:
    """The K-quant epilogue for Q4_K: per super-block isum = sum_j sc_j * s_j
    (s_j: the 32-value sub-block sum an int8 MMA block gives), msum =
    sum_j m_j * (bs[2j] + bs[2j+1]) (the slot's block sum), term =
    fma(d_w*d_x, isum, -((dmin_w*d_x) * msum)) in double."""
    dx, qx, bs = q8k_parts(act, nsb)
    blk = w.reshape(nsb, 144)
    acc = 0.0
    for b in range(nsb):
        d, dmin = f16(blk[b, 0:2]), f16(blk[b, 2:4])
        sc, mn = scales4(blk[b, 4:16])
        qs = blk[b, 16:144].astype(np.int64)
        isum = msum = 0
        for j in range(8):
            g = qs[32 * (j >> 1):32 * (j >> 1) + 32]
            qj = (g >> 4) if (j & 1) else (g & 0xF)  # the copy block's 32 quants
            isum += sc[j] * int(np.dot(qj, qx[b, 32 * j:32 * j + 32]))
            msum += mn[j] * int(bs[b, 2 * j] + bs[b, 2 * j + 1])
        dd = float(np.float32(d * dx[b]))
        dm = float(np.float32(dmin * dx[b]))
        # fma(dd, isum, -(dm * msum)): both products are exact in double
        # (24-bit float times a < 2^26 integer), so the fused form equals
        # one rounding of their difference
        acc += dd * isum - dm * msum
    return np.float32(acc)


def prefill_dot_q6k(w: np.ndarray, act: np.ndarray, nsb: int) -> np.float32:
    """The K-quant epilogue for Q6_K: each 16-value sub-block j fills its own
    32-column block (16 quants q - 32, 16 zeros), isum = sum_j sc_j * s_j,
    term = (double)(d_w*d_x) * isum."""
    dx, qx, _ = q8k_parts(act, nsb)
    blk = w.reshape(nsb, 210)
    acc = 0.0
    for b in range(nsb):
        ql = blk[b, 0:128].astype(np.int64)
        qh = blk[b, 128:192].astype(np.int64)
        sc = blk[b, 192:208].view(np.int8).astype(np.int64)
        d = f16(blk[b, 208:210])
        q = np.empty(256, np.int64)
        for v in range(256):
            h, k, l = v >> 7, (v >> 5) & 3, v & 31
            lo = ql[64 * h + l + ((k & 1) << 5)]
            q[v] = (((lo >> 4) if (k & 2) else (lo & 0xF)) | (((qh[32 * h + l] >> (2 * k)) & 3) << 4)) - 32
        isum = 0
        for j in range(16):
            padded_w = np.concatenate([q[16 * j:16 * j + 16], np.zeros(16, np.int64)])
            padded_x = np.concatenate([qx[b, 16 * j:16 * j + 16], np.zeros(16, np.int64)])
            isum += int(sc[j]) * int(np.dot(padded_w, padded_x))
        acc += float(np.float32(d * dx[b])) * float(isum)
    return np.float32(acc)


@pytest.mark.parametrize("ggml_type", [Q4_K, Q6_K])
def test_kquant_prefill_terms_match_oracle(ggml_type):
    rng = np.random.default_rng(ggml_type)
    n = 1024
    nsb = n // 256
    for trial in range(25):
        w = random_q4k(rng, nsb) if ggml_type == Q4_K else random_q6k(rng, nsb)
        x = (rng.standard_normal(n) * rng.uniform(0.2, 3.0)).astype(np.float32)
        act = oracle.quantize_act_q8_K(x)
        want = np.float32(oracle.vec_dot(ggml_type, w, act, n))
        got = prefill_dot_q4k(w, act, nsb) if ggml_type == Q4_K else prefill_dot_q6k(w, act, nsb)
        assert got.tobytes() == want.tobytes(), (ggml_type, trial, got, want)
