"""ctypes binding of the CPU oracle (libs2oracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the
"port" CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg import this module.  See s2_oracle.h for the reference
functions it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libs2oracle.so")

_lib = None


def build() -> str:
    src = [os.path.join(HERE, f) for f in ("s2_oracle.c", "s2_codec_oracle.c", "s2_oracle.h", "Makefile")]
    if not os.path.exists(LIB_PATH) or any(os.path.getmtime(s) > os.path.getmtime(LIB_PATH) for s in src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class _HP(ctypes.Structure):
    pass


def _hp_fields():
    from_fields = [
        "context_length", "vocab_size", "embedding_length", "feed_forward_length", "block_count", "head_count",
        "head_count_kv", "head_dim", "codebook_size", "num_codebooks", "semantic_begin_id", "semantic_end_id",
        "rope_freq_base", "rms_norm_eps", "tie_word_embeddings", "attention_qk_norm", "scale_codebook_embeddings",
        "fast_context_length", "fast_embedding_length", "fast_feed_forward_length", "fast_block_count",
        "fast_head_count", "fast_head_count_kv", "fast_head_dim", "fast_rope_freq_base", "fast_rms_norm_eps",
        "fast_attention_qk_norm", "fast_has_project_in", "has_fast_decoder"]
    floats = {"rope_freq_base", "rms_norm_eps", "fast_rope_freq_base", "fast_rms_norm_eps"}
    return [(f, ctypes.c_float if f in floats else ctypes.c_int32) for f in from_fields]


_HP._fields_ = _hp_fields()


class _GP(ctypes.Structure):
    _fields_ = [("max_new_tokens", ctypes.c_int32), ("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("top_k", ctypes.c_int32), ("min_tokens_before_end", ctypes.c_int32), ("im_end_id", ctypes.c_int32),
                ("seed", ctypes.c_uint64), ("seq_id", ctypes.c_uint32)]


class _CodecHP(ctypes.Structure):
    """so_codec_hparams (the same fields as s2k_codec_hparams)"""
    _fields_ = [("sample_rate", ctypes.c_int32), ("hop_length", ctypes.c_int32), ("latent_dim", ctypes.c_int32),
                ("decoder_dim", ctypes.c_int32), ("n_decoder_rates", ctypes.c_int32),
                ("decoder_rates", ctypes.c_int32 * 8), ("quantizer_input_dim", ctypes.c_int32),
                ("quantizer_codebook_dim", ctypes.c_int32), ("quantizer_residual_codebooks", ctypes.c_int32),
                ("quantizer_residual_codebook_size", ctypes.c_int32),
                ("quantizer_semantic_codebook_size", ctypes.c_int32), ("n_downsample", ctypes.c_int32),
                ("quantizer_downsample_factor", ctypes.c_int32 * 8), ("rvq_window_size", ctypes.c_int32),
                ("rvq_block_size", ctypes.c_int32), ("rvq_n_layer", ctypes.c_int32),
                ("rvq_n_local_heads", ctypes.c_int32), ("rvq_head_dim", ctypes.c_int32), ("rvq_dim", ctypes.c_int32),
                ("rvq_rope_base", ctypes.c_float), ("rvq_norm_eps", ctypes.c_float)]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        sig = {
            "so_row_bytes": ([ctypes.c_int, i64], i64),
            "so_dequant_row": ([ctypes.c_int, vp, vp, i64], ctypes.c_int),
            "so_quantize_act_q8_0": ([vp, i64, vp], None),
            "so_quantize_act_q8_K": ([vp, i64, vp], None),
            "so_vec_dot": ([ctypes.c_int, vp, vp, i64], ctypes.c_float),
            "so_matvec": ([ctypes.c_int, vp, i64, i64, vp, vp], None),
            "so_fp32_to_fp16": ([ctypes.c_float], ctypes.c_uint16),
            "so_fp16_to_fp32": ([ctypes.c_uint16], ctypes.c_float),
            "so_philox4x32_10": ([vp, vp, vp], None),
            "so_philox_uniform": ([ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32], ctypes.c_double),
            "so_model_create": ([ctypes.POINTER(_HP)], vp),
            "so_model_free": ([vp], None),
            "so_model_set_tensor": ([vp, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(i64), vp, ctypes.c_size_t], ctypes.c_int),
            "so_model_check": ([vp], ctypes.c_int),
            "so_kv_init": ([vp, i32], ctypes.c_int),
            "so_kv_clear": ([vp], None),
            "so_kv_load": ([vp, vp, vp, i32], ctypes.c_int),
            "so_n_past": ([vp], i32),
            "so_eval": ([vp, vp, i32, vp, vp], ctypes.c_int),
            "so_fast_decode": ([vp, vp, vp, i32, vp], ctypes.c_int),
            "so_sample_token": ([vp, i32, ctypes.c_float, ctypes.c_float, i32, ctypes.c_double], i32),
            "so_generate": ([vp, vp, i32, ctypes.POINTER(_GP), vp, ctypes.POINTER(i32)], ctypes.c_int),
            "so_set_threads": ([ctypes.c_int], None),
            "so_generate_timed": ([vp, vp, i32, ctypes.POINTER(_GP), vp, ctypes.POINTER(i32),
                                   ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
            "so_codec_create": ([ctypes.POINTER(_CodecHP)], vp),
            "so_codec_free": ([vp], None),
            "so_codec_set_tensor": ([vp, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(i64), vp], ctypes.c_int),
            "so_codec_samples": ([vp, i32], i64),
            "so_codec_decode": ([vp, vp, i32, vp, i64, ctypes.POINTER(i64)], ctypes.c_int),
            "so_codec_set_f32_accum": ([ctypes.c_int], None),
            "so_det_expf": ([ctypes.c_float], ctypes.c_float),
            "so_det_expf_array": ([vp, vp, i64], None),
            "so_check_pow2_scale": ([i64, ctypes.c_uint32], i64),
        }
        for name, (a, r) in sig.items():
            f = getattr(L, name)
            f.argtypes = a
            f.restype = r
        _lib = L
    return _lib


def det_expf(x: np.ndarray) -> np.ndarray:
    """so_det_expf of every element (float32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().so_det_expf_array(x.ctypes.data, y.ctypes.data, x.size)
    return y


def check_pow2_scale(n: int, seed: int = 1) -> int:
    """Mismatches of the oracle's power-of-two scaling against ldexpf."""
    return int(lib().so_check_pow2_scale(n, seed))


def set_threads(n: int) -> None:
    lib().so_set_threads(n)


def dequant_row(ggml_type: int, data: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    rc = lib().so_dequant_row(ggml_type, np.ascontiguousarray(data).ctypes.data, out.ctypes.data, n)
    assert rc == 0
    return out


def quantize_act_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib().so_quantize_act_q8_0(x.ctypes.data, x.size, out.ctypes.data)
    return out


def quantize_act_q8_K(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 256 * 292, dtype=np.uint8)
    lib().so_quantize_act_q8_K(x.ctypes.data, x.size, out.ctypes.data)
    return out


def vec_dot(ggml_type: int, wrow: np.ndarray, act: np.ndarray, n: int) -> float:
    return float(lib().so_vec_dot(ggml_type, np.ascontiguousarray(wrow).ctypes.data,
                                  np.ascontiguousarray(act).ctypes.data, n))


def matvec(ggml_type: int, w: np.ndarray, rows: int, n: int, x: np.ndarray) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib().so_matvec(ggml_type, np.ascontiguousarray(w).ctypes.data, rows, n, x.ctypes.data, y.ctypes.data)
    return y


def philox(ctr, key):
    c = (ctypes.c_uint32 * 4)(*ctr)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    lib().so_philox4x32_10(c, k, o)
    return list(o)


def philox_uniform(seed: int, frame: int, purpose: int, seq: int = 0) -> float:
    return float(lib().so_philox_uniform(seed, frame, purpose, seq))


def sample_token(logits: np.ndarray, temperature: float, top_p: float, top_k: int, u: float = 0.0) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().so_sample_token(x.ctypes.data, x.size, temperature, top_p, top_k, u))


class OracleModel:
    """CPU restatement of s2::SlowARModel's compute (eval_cached, fast_decode)."""

    def __init__(self, hp):
        h = _HP()
        for name, _ in _HP._fields_:
            setattr(h, name, getattr(hp, name))
        self.hp = hp
        self._m = lib().so_model_create(ctypes.byref(h))
        self._keep = []

    def set_tensor(self, name: str, ggml_type: int, ne, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        self._keep.append(data)
        ne4 = (ctypes.c_int64 * 4)(*[int(x) for x in (list(ne) + [1, 1, 1, 1])[:4]])
        rc = lib().so_model_set_tensor(self._m, name.encode(), ggml_type, ne4, data.ctypes.data, data.nbytes)
        if rc != 0:
            raise RuntimeError(f"oracle rejected tensor {name} ({rc})")

    def load_tensors(self, tensors) -> None:
        for spec, buf in tensors:
            self.set_tensor(spec.name, spec.type, spec.ne, buf)
        rc = lib().so_model_check(self._m)
        if rc != 0:
            raise RuntimeError(f"oracle model incomplete ({rc})")

    def init_kv_cache(self, max_seq_len: int) -> None:
        assert lib().so_kv_init(self._m, max_seq_len) == 0

    def clear_kv_cache(self) -> None:
        lib().so_kv_clear(self._m)

    def load_kv(self, k: np.ndarray, v: np.ndarray) -> None:
        """Restore the cache: k, v f16 [layer][pos][kv_head][head_dim]; n_past = pos."""
        k = np.ascontiguousarray(k, dtype=np.float16)
        v = np.ascontiguousarray(v, dtype=np.float16)
        assert lib().so_kv_load(self._m, k.ctypes.data, v.ctypes.data, int(k.shape[1])) == 0

    @property
    def n_past(self) -> int:
        return int(lib().so_n_past(self._m))

    def eval(self, flat_tokens: np.ndarray, n_tokens: int):
        flat = np.ascontiguousarray(flat_tokens, dtype=np.int32)
        hidden = np.empty(self.hp.embedding_length, dtype=np.float32)
        logits = np.empty(self.hp.vocab_size, dtype=np.float32)
        rc = lib().so_eval(self._m, flat.ctypes.data, n_tokens, hidden.ctypes.data, logits.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"oracle eval failed ({rc})")
        return hidden, logits

    def fast_decode(self, hidden: np.ndarray, prefix) -> np.ndarray:
        h = np.ascontiguousarray(hidden, dtype=np.float32)
        p = np.ascontiguousarray(np.asarray(prefix, dtype=np.int32))
        out = np.empty(self.hp.codebook_size, dtype=np.float32)
        rc = lib().so_fast_decode(self._m, h.ctypes.data, p.ctypes.data if p.size else None, int(p.size),
                                  out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"oracle fast_decode failed ({rc})")
        return out

    def generate(self, prompt: np.ndarray, max_new_tokens: int, temperature: float = 0.0, top_p: float = 0.8,
                 top_k: int = 30, min_tokens_before_end: int = 0, im_end_id: int = -1, seed: int = 0,
                 seq_id: int = 0) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        rows, cols = p.shape
        self.init_kv_cache(cols + max_new_tokens)
        ncb = max(self.hp.num_codebooks, 1)
        codes = np.zeros(ncb * max(max_new_tokens, 1), dtype=np.int32)
        nf = ctypes.c_int32(0)
        gp = _GP(max_new_tokens, temperature, top_p, top_k, min_tokens_before_end, im_end_id, seed, seq_id)
        rc = lib().so_generate(self._m, p.ctypes.data, cols, ctypes.byref(gp), codes.ctypes.data, ctypes.byref(nf))
        if rc != 0:
            raise RuntimeError(f"oracle generate failed ({rc})")
        n = nf.value
        return codes[: ncb * n].reshape(ncb, n)

    def generate_timed(self, prompt: np.ndarray, max_new_tokens: int, **kw):
        """generate() plus the reference's [Metrics] split: (codes, prefill_ms, loop_ms)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        rows, cols = p.shape
        self.init_kv_cache(cols + max_new_tokens)
        ncb = max(self.hp.num_codebooks, 1)
        codes = np.zeros(ncb * max(max_new_tokens, 1), dtype=np.int32)
        nf = ctypes.c_int32(0)
        gp = _GP(max_new_tokens, kw.get("temperature", 0.0), kw.get("top_p", 0.8), kw.get("top_k", 30),
                 kw.get("min_tokens_before_end", 0), kw.get("im_end_id", -1), kw.get("seed", 0), kw.get("seq_id", 0))
        pm, lm = ctypes.c_double(0), ctypes.c_double(0)
        rc = lib().so_generate_timed(self._m, p.ctypes.data, cols, ctypes.byref(gp), codes.ctypes.data,
                                     ctypes.byref(nf), ctypes.byref(pm), ctypes.byref(lm))
        if rc != 0:
            raise RuntimeError(f"oracle generate failed ({rc})")
        n = nf.value
        return codes[: ncb * n].reshape(ncb, n), pm.value, lm.value

    def close(self) -> None:
        if self._m:
            lib().so_model_free(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CodecOracle:
    """CPU restatement of s2::AudioCodec::decode (src/s2_codec.cpp:1297-1447)
    and of its windowed callers (src/s2_pipeline.cpp:198-289, :1034-1115)."""

    def __init__(self, ch):
        h = _CodecHP()
        for name, _ in _CodecHP._fields_:
            if name in ("decoder_rates", "quantizer_downsample_factor"):
                vals = list(getattr(ch, name))
                arr = getattr(h, name)
                for k, v in enumerate(vals):
                    arr[k] = int(v)
                setattr(h, "n_decoder_rates" if name == "decoder_rates" else "n_downsample", len(vals))
            elif name not in ("n_decoder_rates", "n_downsample"):
                setattr(h, name, getattr(ch, name))
        self.ch = ch
        self._c = lib().so_codec_create(ctypes.byref(h))

    def set_tensor(self, name: str, arr: np.ndarray, ne) -> None:
        arr = np.ascontiguousarray(arr)
        t = 1 if arr.dtype == np.float16 else 0
        ne4 = (ctypes.c_int64 * 4)(*[int(x) for x in (list(ne) + [1, 1, 1, 1])[:4]])
        if lib().so_codec_set_tensor(self._c, name.encode(), t, ne4, arr.ctypes.data) != 0:
            raise RuntimeError(f"codec oracle rejected {name}")

    def load_tensors(self, tensors) -> None:
        for spec, arr in tensors:
            self.set_tensor(spec.name, arr, spec.ne)

    def samples_per_frame(self) -> int:
        return int(lib().so_codec_samples(self._c, 1))

    def decode(self, codes: np.ndarray, f32_accum: bool = False) -> np.ndarray:
        """f32_accum: sum the dot products in float, in sequence (a second
        valid accumulation order) instead of double"""
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        n = codes.shape[1]
        cap = int(lib().so_codec_samples(self._c, n))
        out = np.empty(cap, dtype=np.float32)
        ns = ctypes.c_int64(0)
        lib().so_codec_set_f32_accum(1 if f32_accum else 0)
        try:
            rc = lib().so_codec_decode(self._c, codes.ctypes.data, n, out.ctypes.data, cap, ctypes.byref(ns))
        finally:
            lib().so_codec_set_f32_accum(0)
        if rc != 0:
            raise RuntimeError(f"codec oracle decode failed ({rc})")
        return out[: ns.value]

    def history_frames(self) -> int:
        """streaming_history_frames (src/s2_codec.cpp:870-874)"""
        h = ((max(0, self.ch.rvq_window_size - 1) + 16 + 7) // 8) * 8
        return h if h > 0 else 160

    def windows_offline(self, total: int, stride: int = 16, context: int = -1):
        return codec_windows_offline(total, stride, context if context >= 0 else self.history_frames())

    def decode_windowed(self, codes: np.ndarray, stride: int = 16, context: int = -1,
                        f32_accum: bool = False) -> np.ndarray:
        spf = self.samples_per_frame()
        parts = []
        for start, wf, eb, ee in self.windows_offline(codes.shape[1], stride, context):
            if ee > eb:
                pcm = self.decode(codes[:, start:start + wf], f32_accum)
                parts.append(pcm[eb * spf: ee * spf])
        return np.concatenate(parts) if parts else np.zeros(0, np.float32)

    def windows_stream(self, total: int, stride: int = 4, context: int = -1, holdback: int = -1):
        ctx = context if context >= 0 else self.history_frames()
        return codec_windows_stream(total, stride, ctx, holdback if holdback >= 0 else ctx)

    def close(self) -> None:
        if getattr(self, "_c", None):
            lib().so_codec_free(self._c)
            self._c = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def codec_windows_offline(total: int, stride: int, history: int):
    """(start, frames, emit_begin, emit_end) of every window
    decode_codes_windowed decodes (src/s2_pipeline.cpp:198-289)."""
    stride = max(1, stride if stride > 0 else 16)
    out, committed = [], 0

    def window(avail, fin):
        nonlocal committed
        if avail <= 0 or avail <= committed:
            return
        stable = avail if fin else max(0, avail - history)
        if stable <= committed and not fin:
            return
        start = max(0, committed - history)
        wf = avail - start
        if wf <= 0:
            return
        eb = max(0, committed - start)
        ee = wf if fin else min(wf, max(0, stable - start))
        out.append((start, wf, eb, ee))
        committed = avail if fin else stable

    avail = min(total, stride)
    while avail < total:
        window(avail, False)
        avail += stride
    window(total, True)
    return out


def codec_windows_stream(total: int, stride: int, context: int, holdback: int):
    """Windows of the streaming path: on_frame after every frame, a window
    once stride frames arrived since the last decode, then the final one
    (src/s2_pipeline.cpp:1034-1115, :1136-1141); entries are
    (frames seen, start, frames, emit_begin, emit_end)."""
    stride = stride if stride > 0 else 4
    out, committed, last = [], 0, 0

    def window(tot, fin):
        nonlocal committed, last
        if tot <= 0 or tot <= committed:
            return
        stable = tot if fin else max(0, tot - holdback)
        if stable <= committed and not fin:
            return
        start = max(0, committed - context)
        wf = tot - start
        if wf <= 0:
            return
        eb = max(0, committed - start)
        ee = wf if fin else min(wf, max(0, stable - start))
        out.append((tot, start, wf, eb, ee))
        committed = tot if fin else stable
        last = tot

    for f in range(1, total + 1):
        if f - last >= stride:
            window(f, False)
    if total > last or committed < total:
        window(total, True)
    return out
