"""Python binding of the s2k C ABI (include/s2k.h) and a mirror of the
reference's model interface for the dual-AR decode path.

`SlowARModel` keeps s2::SlowARModel's method names and argument meaning
(include/s2_model.h:92-130): init_kv_cache, clear_kv_cache, reset,
prefill_fast, prefill, step, fast_decode, hparams.  `generate` mirrors
s2::generate (include/s2_generate.h:40-45).  Results come back as numpy
arrays; failures raise S2KError with the library's message (the reference
returns false and prints to stderr).

The library is the in-tree libs2k.so built by build.py; importing this module
on a machine without it raises, there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
from typing import Callable, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libs2k.so")

S2K_OK = 0
SAMPLE_NOALLOC_MAX_N = 8192  # S2K_SAMPLE_NOALLOC_MAX_N
STATUS = {-1: "ERR_ARG", -2: "ERR_OOM", -3: "ERR_CUDA", -4: "ERR_KV_FULL", -5: "ERR_STATE",
          -6: "ERR_TIMEOUT", -7: "ERR_UNSUPPORTED", -8: "ERR_NO_DEVICE"}

# symbols declared in include/s2k.h (checked by the CPU tests)
EXPORTED = [
    "s2k_abi_version", "s2k_last_error", "s2k_device_count", "s2k_model_create", "s2k_model_upload_tensor",
    "s2k_model_finalize", "s2k_model_free", "s2k_model_get_hparams", "s2k_model_weight_bytes",
    "s2k_model_stream", "s2k_seq_create", "s2k_seq_reset", "s2k_seq_free", "s2k_seq_n_past", "s2k_eval",
    "s2k_fast_decode", "s2k_generate", "s2k_generate_device", "s2k_sample", "s2k_launch_count",
    "s2k_profile_gemv", "s2k_debug_copy", "s2k_sample_noalloc",
    "s2k_profile_frame", "s2k_profile_ops", "s2k_profile_trace",
    "s2k_seq_begin", "s2k_batch_frame", "s2k_seq_frames", "s2k_sched_create", "s2k_sched_free",
    "s2k_sched_submit", "s2k_sched_step", "s2k_sched_run", "s2k_sched_poll", "s2k_sched_result",
    "s2k_sched_get_stats", "s2k_sched_poll_status", "s2k_sched_cancel", "s2k_sched_set_frame_callback",
    "s2k_seq_load_kv", "s2k_get_rows", "s2k_model_set_wait_limit", "s2k_debug_wait_probe", "s2k_debug_fail_alloc", "s2k_debug_det_expf",
    "s2k_model_device_bytes", "s2k_device_mem_info", "s2k_gguf_read_hparams", "s2k_gguf_tensor_info",
    "s2k_model_load_gguf", "s2k_build_prompt", "s2k_seq_last_metrics",
    "s2k_codec_create", "s2k_codec_upload_tensor", "s2k_codec_finalize", "s2k_codec_load_gguf", "s2k_codec_free",
    "s2k_codec_get_hparams", "s2k_codec_samples_per_frame", "s2k_codec_history_frames", "s2k_codec_num_codebooks",
    "s2k_codec_receptive_frames", "s2k_codec_decode", "s2k_codec_decode_range", "s2k_codec_decode_windowed",
    "s2k_codec_stream_create", "s2k_codec_stream_free", "s2k_codec_stream_push", "s2k_codec_stream_finish",
    "s2k_codec_stream_max_release",
]

REQ_WAITING, REQ_LIVE, REQ_DONE, REQ_FAILED, REQ_CANCELLED = 0, 1, 2, 3, 4  # S2K_REQ_*


class S2KError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class _HParams(ctypes.Structure):
    _fields_ = [
        ("context_length", ctypes.c_int32), ("vocab_size", ctypes.c_int32), ("embedding_length", ctypes.c_int32),
        ("feed_forward_length", ctypes.c_int32), ("block_count", ctypes.c_int32), ("head_count", ctypes.c_int32),
        ("head_count_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("codebook_size", ctypes.c_int32),
        ("num_codebooks", ctypes.c_int32), ("semantic_begin_id", ctypes.c_int32),
        ("semantic_end_id", ctypes.c_int32), ("rope_freq_base", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
        ("tie_word_embeddings", ctypes.c_int32), ("attention_qk_norm", ctypes.c_int32),
        ("scale_codebook_embeddings", ctypes.c_int32), ("fast_context_length", ctypes.c_int32),
        ("fast_embedding_length", ctypes.c_int32), ("fast_feed_forward_length", ctypes.c_int32),
        ("fast_block_count", ctypes.c_int32), ("fast_head_count", ctypes.c_int32),
        ("fast_head_count_kv", ctypes.c_int32), ("fast_head_dim", ctypes.c_int32),
        ("fast_rope_freq_base", ctypes.c_float), ("fast_rms_norm_eps", ctypes.c_float),
        ("fast_attention_qk_norm", ctypes.c_int32), ("fast_has_project_in", ctypes.c_int32),
        ("has_fast_decoder", ctypes.c_int32),
    ]


class _GenParams(ctypes.Structure):
    _fields_ = [("max_new_tokens", ctypes.c_int32), ("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("top_k", ctypes.c_int32), ("min_tokens_before_end", ctypes.c_int32),
                ("im_end_id", ctypes.c_int32), ("seed", ctypes.c_uint64), ("seq_id", ctypes.c_uint32)]


class _SchedStats(ctypes.Structure):
    _fields_ = [("steps", ctypes.c_int64), ("frames", ctypes.c_int64), ("prefill_tokens", ctypes.c_int64),
                ("admitted", ctypes.c_int64), ("finished", ctypes.c_int64), ("kv_positions", ctypes.c_int64),
                ("max_live", ctypes.c_int32),
                ("free_pages", ctypes.c_int32), ("pool_pages", ctypes.c_int32), ("pad_", ctypes.c_int32),
                ("cancelled", ctypes.c_int64), ("failed", ctypes.c_int64)]


class _GenMetrics(ctypes.Structure):
    _fields_ = [("prefill_ms", ctypes.c_double), ("loop_ms", ctypes.c_double), ("total_ms", ctypes.c_double),
                ("ms_per_frame", ctypes.c_double), ("n_frames", ctypes.c_int32), ("prompt_tokens", ctypes.c_int32)]


class _CodecHParams(ctypes.Structure):
    """s2k_codec_hparams"""
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


def codec_hp_struct(ch, cls=_CodecHParams):
    """A ctypes codec hyper-parameter struct from an object with the
    CodecHParams attributes (decoder_rates / quantizer_downsample_factor as
    sequences)."""
    h = cls()
    for name, _ in cls._fields_:
        if name in ("decoder_rates", "quantizer_downsample_factor"):
            vals = list(getattr(ch, name))
            arr = getattr(h, name)
            for k, v in enumerate(vals):
                arr[k] = int(v)
            setattr(h, "n_decoder_rates" if name == "decoder_rates" else "n_downsample", len(vals))
        elif name not in ("n_decoder_rates", "n_downsample"):
            setattr(h, name, getattr(ch, name))
    return h


FRAME_CB = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, ctypes.c_int32,
                            ctypes.c_int32, ctypes.c_void_p)
ENCODE_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                             ctypes.c_void_p)
SCHED_FRAME_CB = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                                  ctypes.c_int32, ctypes.c_void_p)

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libs2k.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python s2.cpp_b200/build.py` (needs nvcc)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64p = ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_int64)
    sig = {
        "s2k_abi_version": ([], i32),
        "s2k_last_error": ([], ctypes.c_char_p),
        "s2k_device_count": ([ctypes.POINTER(i32)], i32),
        "s2k_model_create": ([i32, ctypes.POINTER(_HParams), ctypes.POINTER(vp)], i32),
        "s2k_model_upload_tensor": ([vp, ctypes.c_char_p, i32, i64p, vp, ctypes.c_size_t], i32),
        "s2k_model_finalize": ([vp], i32),
        "s2k_model_free": ([vp], None),
        "s2k_model_get_hparams": ([vp, ctypes.POINTER(_HParams)], i32),
        "s2k_model_weight_bytes": ([vp], ctypes.c_size_t),
        "s2k_model_stream": ([vp], vp),
        "s2k_seq_create": ([vp, i32, ctypes.POINTER(vp)], i32),
        "s2k_seq_reset": ([vp], i32),
        "s2k_seq_free": ([vp], None),
        "s2k_seq_n_past": ([vp], i32),
        "s2k_eval": ([vp, vp, vp, i32, vp, vp], i32),
        "s2k_fast_decode": ([vp, vp, vp, i32, vp], i32),
        "s2k_generate": ([vp, vp, vp, i32, ctypes.POINTER(_GenParams), vp, ctypes.POINTER(i32), FRAME_CB, vp], i32),
        "s2k_generate_device": ([vp, vp, vp, i32, ctypes.POINTER(_GenParams), vp, ctypes.POINTER(i32)], i32),
        "s2k_sample": ([vp, vp, i32, ctypes.c_float, ctypes.c_float, i32, ctypes.c_double, ctypes.POINTER(i32)], i32),
        "s2k_sample_noalloc": ([vp, vp, i32, ctypes.c_float, ctypes.c_float, i32, ctypes.c_double,
                                ctypes.POINTER(i32)], i32),
        "s2k_launch_count": ([i32], ctypes.c_uint64),
        "s2k_profile_gemv": ([vp, i32, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                              ctypes.POINTER(i32)], i32),
        "s2k_debug_copy": ([vp, vp, ctypes.c_char_p, vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)], i32),
        "s2k_profile_frame": ([vp, vp, i32] + [ctypes.POINTER(ctypes.c_double)] * 4, i32),
        "s2k_profile_ops": ([vp, vp, i32, i32, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i32), i32,
                             ctypes.POINTER(i32)], i32),
        "s2k_profile_trace": ([vp, vp, i32, ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t, ctypes.POINTER(i32),
                               ctypes.POINTER(i32)], i32),
        "s2k_seq_begin": ([vp, vp, vp, i32, ctypes.POINTER(_GenParams)], i32),
        "s2k_batch_frame": ([vp, ctypes.POINTER(vp), i32, ctypes.POINTER(i32)], i32),
        "s2k_seq_frames": ([vp, vp, i32, ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
        "s2k_sched_create": ([vp, i32, i32, i32, ctypes.POINTER(vp)], i32),
        "s2k_sched_free": ([vp], None),
        "s2k_sched_submit": ([vp, vp, i32, ctypes.POINTER(_GenParams), ctypes.POINTER(i32)], i32),
        "s2k_sched_step": ([vp, ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
        "s2k_sched_run": ([vp], i32),
        "s2k_sched_poll": ([vp, i32, ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
        "s2k_sched_result": ([vp, i32, vp, i32, ctypes.POINTER(i32)], i32),
        "s2k_sched_get_stats": ([vp, ctypes.POINTER(_SchedStats)], i32),
        "s2k_sched_poll_status": ([vp, i32, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
        "s2k_sched_cancel": ([vp, i32], i32),
        "s2k_sched_set_frame_callback": ([vp, SCHED_FRAME_CB, vp], i32),
        "s2k_seq_load_kv": ([vp, vp, vp, i32], i32),
        "s2k_get_rows": ([vp, ctypes.c_char_p, vp, i32, vp], i32),
        "s2k_model_set_wait_limit": ([vp, ctypes.c_int64], i32),
        "s2k_debug_wait_probe": ([vp], i32),
        "s2k_debug_fail_alloc": ([vp, ctypes.c_int64], i32),
        "s2k_debug_det_expf": ([i32, vp, vp, ctypes.c_int64], i32),
        "s2k_model_device_bytes": ([vp], ctypes.c_size_t),
        "s2k_device_mem_info": ([i32, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)], i32),
        "s2k_gguf_read_hparams": ([ctypes.c_char_p, ctypes.POINTER(_HParams)], i32),
        "s2k_gguf_tensor_info": ([ctypes.c_char_p, i32, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(i32), i64p,
                                  ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                  ctypes.POINTER(i32)], i32),
        "s2k_model_load_gguf": ([i32, ctypes.c_char_p, ctypes.POINTER(vp)], i32),
        "s2k_seq_last_metrics": ([vp, ctypes.POINTER(_GenMetrics)], i32),
        "s2k_build_prompt": ([ENCODE_FN, vp, ctypes.c_char_p, ctypes.c_char_p, vp, i32, i32, i32, i32, i32, vp,
                              ctypes.c_size_t, ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
        "s2k_codec_create": ([i32, ctypes.POINTER(_CodecHParams), ctypes.POINTER(vp)], i32),
        "s2k_codec_upload_tensor": ([vp, ctypes.c_char_p, i32, i64p, vp, ctypes.c_size_t], i32),
        "s2k_codec_finalize": ([vp], i32),
        "s2k_codec_load_gguf": ([i32, ctypes.c_char_p, ctypes.POINTER(vp)], i32),
        "s2k_codec_free": ([vp], None),
        "s2k_codec_get_hparams": ([vp, ctypes.POINTER(_CodecHParams)], i32),
        "s2k_codec_samples_per_frame": ([vp], i32),
        "s2k_codec_history_frames": ([vp], i32),
        "s2k_codec_num_codebooks": ([vp], i32),
        "s2k_codec_receptive_frames": ([vp], i32),
        "s2k_codec_decode": ([vp, vp, i32, vp, ctypes.c_size_t, i64p], i32),
        "s2k_codec_decode_range": ([vp, vp, i32, i32, i32, vp, ctypes.c_size_t, i64p], i32),
        "s2k_codec_decode_windowed": ([vp, vp, i32, i32, i32, i32, vp, ctypes.c_size_t, i64p,
                                       ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i32)], i32),
        "s2k_codec_stream_create": ([vp, i32, i32, i32, ctypes.POINTER(vp)], i32),
        "s2k_codec_stream_free": ([vp], None),
        "s2k_codec_stream_push": ([vp, vp, vp, ctypes.c_size_t, i64p], i32),
        "s2k_codec_stream_finish": ([vp, vp, ctypes.c_size_t, i64p], i32),
        "s2k_codec_stream_max_release": ([vp], ctypes.c_int64),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc != S2K_OK:
        raise S2KError(rc, lib().s2k_last_error().decode(errors="replace"))


def device_count() -> int:
    n = ctypes.c_int32(0)
    rc = lib().s2k_device_count(ctypes.byref(n))
    return n.value if rc == S2K_OK else 0


def device_mem_info(device: int = 0):
    """(free, total) bytes of a device (cudaMemGetInfo)."""
    f, t = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _check(lib().s2k_device_mem_info(device, ctypes.byref(f), ctypes.byref(t)))
    return f.value, t.value


def build_prompt(encode: Callable[[str], list], text: str, prompt_text: str = "", prompt_codes=None,
                 num_codebooks: int = 10, im_end_id: int = 151645, voice_id: int = 151673,
                 semantic_begin_id: int = 151678) -> np.ndarray:
    """s2::build_prompt through s2k_build_prompt: the PromptTensor grid
    [num_codebooks+1][cols].  encode(text) -> token ids stands in for the
    tokenizer; prompt_codes [num_codebooks][T_prompt] is the reference clip."""
    def _enc(txt, ids, cap, user):
        try:
            toks = list(encode(txt.decode()))
        except Exception:
            return -1
        for i in range(min(cap, len(toks))):
            ids[i] = toks[i]
        return len(toks)
    cb = ENCODE_FN(_enc)
    codes = None if prompt_codes is None else np.ascontiguousarray(prompt_codes, dtype=np.int32)
    T = 0 if codes is None else int(codes.shape[1])
    cptr = None if codes is None else _ptr(codes)
    rows, cols = ctypes.c_int32(0), ctypes.c_int32(0)
    args = (cb, None, text.encode(), prompt_text.encode(), cptr, num_codebooks, T, im_end_id, voice_id,
            semantic_begin_id)
    _check(lib().s2k_build_prompt(*args, None, 0, ctypes.byref(rows), ctypes.byref(cols)))
    out = np.zeros((rows.value, cols.value), dtype=np.int32)
    _check(lib().s2k_build_prompt(*args, _ptr(out), out.size, ctypes.byref(rows), ctypes.byref(cols)))
    return out


def gguf_read_hparams(path: str) -> dict:
    """Hyper-parameters of a GGUF file (s2k_gguf_read_hparams), by field name."""
    h = _HParams()
    _check(lib().s2k_gguf_read_hparams(os.fsencode(path), ctypes.byref(h)))
    return {name: getattr(h, name) for name, _ in _HParams._fields_}


def gguf_tensors(path: str) -> list:
    """[(name, ggml type, ne[4], absolute data offset, nbytes)] of a GGUF file."""
    n = ctypes.c_int32(0)
    _check(lib().s2k_gguf_tensor_info(os.fsencode(path), -1, None, 0, None, None, None, None, ctypes.byref(n)))
    out = []
    for i in range(n.value):
        name = ctypes.create_string_buffer(512)
        t = ctypes.c_int32(0)
        ne = (ctypes.c_int64 * 4)()
        off, nb = ctypes.c_uint64(0), ctypes.c_uint64(0)
        _check(lib().s2k_gguf_tensor_info(os.fsencode(path), i, name, 512, ctypes.byref(t), ne, ctypes.byref(off),
                                          ctypes.byref(nb), None))
        out.append((name.value.decode(), t.value, tuple(ne), off.value, nb.value))
    return out


def _hp_struct(hp) -> _HParams:
    s = _HParams()
    for name, _ in _HParams._fields_:
        setattr(s, name, getattr(hp, name))
    return s


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class SlowARModel:
    """The dual-AR model on one CUDA device, mirroring s2::SlowARModel."""

    def __init__(self, hparams, device: int = 0):
        self._m = ctypes.c_void_p()
        self._seq = ctypes.c_void_p()
        self._hp = hparams
        _check(lib().s2k_model_create(device, ctypes.byref(_hp_struct(hparams)), ctypes.byref(self._m)))
        self.device = device

    @classmethod
    def from_gguf(cls, path: str, device: int = 0) -> "SlowARModel":
        """A finalized model read from a GGUF file (s2k_model_load_gguf)."""
        import types
        self = cls.__new__(cls)
        self._m = ctypes.c_void_p()
        self._seq = ctypes.c_void_p()
        _check(lib().s2k_model_load_gguf(device, os.fsencode(path), ctypes.byref(self._m)))
        h = _HParams()
        _check(lib().s2k_model_get_hparams(self._m, ctypes.byref(h)))
        self._hp = types.SimpleNamespace(**{name: getattr(h, name) for name, _ in _HParams._fields_})
        self.device = device
        return self

    # --- loading (SlowARModel::load_shared + read_tensor_data) ---
    def upload_tensor(self, name: str, ggml_type: int, ne, data: np.ndarray) -> None:
        ne4 = (ctypes.c_int64 * 4)(*[int(x) for x in (list(ne) + [1, 1, 1, 1])[:4]])
        data = np.ascontiguousarray(data)
        _check(lib().s2k_model_upload_tensor(self._m, name.encode(), ggml_type, ne4, _ptr(data), data.nbytes))

    def finalize(self) -> None:
        _check(lib().s2k_model_finalize(self._m))

    def load_tensors(self, tensors) -> None:
        """tensors: iterable of (spec, bytes) as produced by synthetic.make_model."""
        for spec, buf in tensors:
            self.upload_tensor(spec.name, spec.type, spec.ne, buf)
        self.finalize()

    def hparams(self):
        return self._hp

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._m

    @property
    def seq_handle(self) -> ctypes.c_void_p:
        return self._seq

    def weight_bytes(self) -> int:
        return int(lib().s2k_model_weight_bytes(self._m))

    def device_bytes(self) -> int:
        """Device bytes the model holds (s2k_model_device_bytes)."""
        return int(lib().s2k_model_device_bytes(self._m))

    def set_wait_limit(self, cycles: int) -> None:
        """Bound of every device-side wait, in SM cycles (0 = default)."""
        _check(lib().s2k_model_set_wait_limit(self._m, int(cycles)))

    def wait_probe(self) -> None:
        """A bounded wait on a tag nobody writes (raises S2KError ERR_TIMEOUT)."""
        _check(lib().s2k_debug_wait_probe(self._m))

    def fail_alloc(self, after: int) -> None:
        """Test hook: the device allocation `after` allocations ahead fails once (-1 disarms)."""
        _check(lib().s2k_debug_fail_alloc(self._m, int(after)))

    def get_rows(self, table: str, ids) -> np.ndarray:
        """Rows of a weight table dequantized on the device (s2k_get_rows)."""
        i = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        out = np.empty((i.size, self._hp.embedding_length), dtype=np.float32)
        _check(lib().s2k_get_rows(self._m, table.encode(), _ptr(i), int(i.size), _ptr(out)))
        return out

    def load_kv(self, k: np.ndarray, v: np.ndarray) -> None:
        """Restore the KV cache: k, v f16 [layer][pos][kv_head][head_dim]; n_past = pos."""
        k = np.ascontiguousarray(k, dtype=np.float16)
        v = np.ascontiguousarray(v, dtype=np.float16)
        if k.shape != v.shape or k.ndim != 4:
            raise S2KError(-1, "k and v must both be [layer][pos][kv_head][head_dim]")
        _check(lib().s2k_seq_load_kv(self._seq, _ptr(k), _ptr(v), int(k.shape[1])))

    def stream(self) -> int:
        return int(lib().s2k_model_stream(self._m) or 0)

    # --- KV cache (init_kv_cache / reset / clear_kv_cache) ---
    def init_kv_cache(self, max_seq_len: int) -> None:
        self.clear_kv_cache()
        _check(lib().s2k_seq_create(self._m, max_seq_len, ctypes.byref(self._seq)))
        self._max_seq_len = max_seq_len

    def reset(self) -> None:
        _check(lib().s2k_seq_reset(self._seq))

    def clear_kv_cache(self) -> None:
        if self._seq:
            lib().s2k_seq_free(self._seq)
            self._seq = ctypes.c_void_p()
        self._max_seq_len = 0

    @property
    def n_past(self) -> int:
        return int(lib().s2k_seq_n_past(self._seq)) if self._seq else 0

    # --- eval_cached / prefill_fast / prefill / step ---
    def _eval(self, flat_tokens: np.ndarray, n_tokens: int):
        flat = np.ascontiguousarray(flat_tokens, dtype=np.int32)
        if flat.size != n_tokens * (self._hp.num_codebooks + 1):
            raise S2KError(-1, f"expected {n_tokens * (self._hp.num_codebooks + 1)} ints, got {flat.size}")
        hidden = np.empty(self._hp.embedding_length, dtype=np.float32)
        logits = np.empty(self._hp.vocab_size, dtype=np.float32)
        _check(lib().s2k_eval(self._m, self._seq, _ptr(flat), n_tokens, _ptr(hidden), _ptr(logits)))
        return hidden, logits

    def prefill_fast(self, flat_tokens: np.ndarray, n_tokens: int):
        return self._eval(flat_tokens, n_tokens)

    def prefill(self, flat_tokens: np.ndarray, n_tokens: int):
        return self._eval(flat_tokens, n_tokens)

    def step(self, flat_tokens: np.ndarray):
        return self._eval(flat_tokens, 1)

    def fast_decode(self, hidden: np.ndarray, prefix_codes) -> np.ndarray:
        h = np.ascontiguousarray(hidden, dtype=np.float32)
        p = np.ascontiguousarray(np.asarray(prefix_codes, dtype=np.int32))
        out = np.empty(self._hp.codebook_size, dtype=np.float32)
        _check(lib().s2k_fast_decode(self._m, _ptr(h), _ptr(p) if p.size else None, int(p.size), _ptr(out)))
        return out

    def sample(self, logits: np.ndarray, temperature: float, top_p: float, top_k: int, u: float = 0.0) -> int:
        x = np.ascontiguousarray(logits, dtype=np.float32)
        tok = ctypes.c_int32(0)
        _check(lib().s2k_sample(self._m, _ptr(x), int(x.size), temperature, top_p, top_k, u, ctypes.byref(tok)))
        return tok.value

    def sample_noalloc(self, logits: np.ndarray, temperature: float, top_p: float, top_k: int,
                       u: float = 0.0) -> int:
        """`sample` through s2k_sample_noalloc: fixed device scratch, at most
        SAMPLE_NOALLOC_MAX_N logits; concurrent calls on one device race."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        tok = ctypes.c_int32(0)
        _check(lib().s2k_sample_noalloc(self._m, _ptr(x), int(x.size), temperature, top_p, top_k, u,
                                        ctypes.byref(tok)))
        return tok.value

    # --- generate ---
    def generate(self, prompt: np.ndarray, max_new_tokens: int = 1024, temperature: float = 0.8,
                 top_p: float = 0.8, top_k: int = 30, min_tokens_before_end: int = 0, im_end_id: int = -1,
                 seed: int = 0, seq_id: int = 0,
                 on_frame: Optional[Callable[[np.ndarray, int, int], bool]] = None) -> np.ndarray:
        """prompt: PromptTensor grid [num_codebooks+1][cols].  Returns codes
        [num_codebooks][n_frames] (GenerateResult.codes)."""
        hp = self._hp
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        rows, cols = p.shape
        if rows != hp.num_codebooks + 1:
            raise S2KError(-1, f"prompt must have {hp.num_codebooks + 1} rows")
        need = cols + max_new_tokens
        if not self._seq or self._max_seq() < need:
            self.init_kv_cache(need)
        ncb = max(hp.num_codebooks, 1)
        codes = np.zeros(ncb * max(max_new_tokens, 1), dtype=np.int32)
        nf = ctypes.c_int32(0)
        gp = _GenParams(max_new_tokens, temperature, top_p, top_k, min_tokens_before_end, im_end_id, seed, seq_id)
        if on_frame is not None:
            def _cb(codes_ptr, idx, total, ncb_, user):
                arr = np.ctypeslib.as_array(codes_ptr, shape=(ncb_,)).copy()
                return 1 if on_frame(arr, idx, total) else 0
            cb = FRAME_CB(_cb)
        else:
            cb = FRAME_CB()
        _check(lib().s2k_generate(self._m, self._seq, _ptr(p), cols, ctypes.byref(gp), _ptr(codes),
                                  ctypes.byref(nf), cb, None))
        n = nf.value
        return codes[: ncb * n].reshape(ncb, n)

    def last_metrics(self) -> dict:
        """Device-timed prefill / frame-loop split of the last generate (s2k_seq_last_metrics)."""
        gm = _GenMetrics()
        _check(lib().s2k_seq_last_metrics(self._seq, ctypes.byref(gm)))
        return {name: getattr(gm, name) for name, _ in _GenMetrics._fields_}

    def _max_seq(self) -> int:
        return getattr(self, "_max_seq_len", 0)

    def debug_buffer(self, name: str, dtype=np.float32, nbytes: int = 1 << 30) -> np.ndarray:
        """Copy of a named device buffer (see s2k_debug_copy)."""
        buf = np.empty(nbytes // np.dtype(dtype).itemsize, dtype=dtype) if nbytes < (1 << 30) else None
        if buf is None:
            # size probe: copy into a small buffer first is not possible; allocate generously
            buf = np.empty((256 << 20) // np.dtype(dtype).itemsize, dtype=dtype)
        got = ctypes.c_size_t(0)
        _check(lib().s2k_debug_copy(self._m, self._seq, name.encode(), _ptr(buf), buf.nbytes, ctypes.byref(got)))
        return buf[: got.value // np.dtype(dtype).itemsize].copy()

    def profile_gemv(self, reps: int = 5):
        """(bytes per pass, ms per pass, launches per pass) of the Slow-step GEMVs."""
        b, ms, n = ctypes.c_double(0), ctypes.c_double(0), ctypes.c_int32(0)
        _check(lib().s2k_profile_gemv(self._m, reps, ctypes.byref(b), ctypes.byref(ms), ctypes.byref(n)))
        return b.value, ms.value, n.value

    def profile_frame(self, reps: int = 5):
        """Persistent decode kernel, event-timed per launch: (ms Slow segment,
        ms Fast pass, bytes Slow segment, bytes Fast pass).  Needs a prior
        generate on this model's sequence with a free KV position."""
        v = [ctypes.c_double(0) for _ in range(4)]
        _check(lib().s2k_profile_frame(self._m, self._seq, reps, *[ctypes.byref(x) for x in v]))
        return tuple(x.value for x in v)

    def profile_ops(self, segment: int, reps: int = 5):
        """Per-op device time (us) and kind of one persistent-kernel segment
        (s2k_profile_ops); segment -1 is the Slow step."""
        cap = 4096
        us = (ctypes.c_double * cap)()
        kind = (ctypes.c_int32 * cap)()
        n = ctypes.c_int32(0)
        if segment < 0:
            segment += self._hp.num_codebooks
        _check(lib().s2k_profile_ops(self._m, self._seq, segment, reps, us, kind, cap, ctypes.byref(n)))
        return np.array(us[: n.value]), np.array(kind[: n.value], dtype=np.int32)

    def profile_trace(self, segment: int) -> np.ndarray:
        """Per-op, per-CTA stamps of one persistent-kernel segment launch
        (s2k_profile_trace): uint64 ns array [n_ops + 1][n_ctas][12]."""
        if segment < 0:
            segment += self._hp.num_codebooks
        cap = 1 << 20
        buf = (ctypes.c_uint64 * cap)()
        n, g = ctypes.c_int32(0), ctypes.c_int32(0)
        _check(lib().s2k_profile_trace(self._m, self._seq, segment, buf, cap, ctypes.byref(n), ctypes.byref(g)))
        a = np.frombuffer(buf, dtype=np.uint64, count=(n.value + 1) * g.value * 12).copy()
        return a.reshape(n.value + 1, g.value, 12)

    def generate_device(self, d_prompt_tm: int, cols: int, d_codes: int, max_new_tokens: int,
                        temperature: float = 0.0, top_p: float = 0.8, top_k: int = 30,
                        min_tokens_before_end: int = 0, im_end_id: int = -1, seed: int = 0, seq_id: int = 0) -> int:
        """s2k_generate_device on device pointers; returns the frame count."""
        need = cols + max_new_tokens
        if not self._seq or self._max_seq() < need:
            self.init_kv_cache(need)
        nf = ctypes.c_int32(0)
        gp = _GenParams(max_new_tokens, temperature, top_p, top_k, min_tokens_before_end, im_end_id, seed, seq_id)
        _check(lib().s2k_generate_device(self._m, self._seq, ctypes.c_void_p(d_prompt_tm), cols, ctypes.byref(gp),
                                         ctypes.c_void_p(d_codes), ctypes.byref(nf)))
        return nf.value

    def close(self) -> None:
        if getattr(self, "_m", None):
            self.clear_kv_cache()
            lib().s2k_model_free(self._m)
            self._m = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Sequence:
    """One utterance's decode state (s2k_seq) for batched frames: begin()
    prefills the prompt, SlowARModel.batch_frame advances several together."""

    def __init__(self, model: "SlowARModel", max_seq_len: int):
        self._model = model
        self._hp = model._hp
        h = ctypes.c_void_p()
        _check(lib().s2k_seq_create(model.handle, max_seq_len, ctypes.byref(h)))
        self._s = h
        self._cap = 0

    def begin(self, prompt: np.ndarray, max_new_tokens: int, temperature: float = 0.8, top_p: float = 0.8,
              top_k: int = 30, min_tokens_before_end: int = 0, im_end_id: int = -1, seed: int = 0,
              seq_id: int = 0) -> None:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        gp = _GenParams(max_new_tokens, temperature, top_p, top_k, min_tokens_before_end, im_end_id, seed, seq_id)
        _check(lib().s2k_seq_begin(self._model.handle, self._s, _ptr(p), p.shape[1], ctypes.byref(gp)))
        self._cap = max(max_new_tokens, 1)

    def frames(self):
        """(codes [num_codebooks][n_frames], done)."""
        ncb = max(self._hp.num_codebooks, 1)
        buf = np.zeros(ncb * max(self._cap, 1), dtype=np.int32)
        nf, done = ctypes.c_int32(0), ctypes.c_int32(0)
        _check(lib().s2k_seq_frames(self._s, _ptr(buf), self._cap, ctypes.byref(nf), ctypes.byref(done)))
        return buf[: ncb * nf.value].reshape(ncb, nf.value), bool(done.value)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._s

    def close(self) -> None:
        if getattr(self, "_s", None):
            lib().s2k_seq_free(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def batch_frame(model: "SlowARModel", seqs) -> int:
    """One batched frame over the unfinished sequences in `seqs`; returns how
    many are still unfinished."""
    arr = (ctypes.c_void_p * len(seqs))(*[s.handle for s in seqs])
    live = ctypes.c_int32(0)
    _check(lib().s2k_batch_frame(model.handle, arr, len(seqs), ctypes.byref(live)))
    return live.value


class BatchScheduler:
    """Continuous batching over independent utterances (s2k_sched_*): submit
    requests, run, collect each request's codes [num_codebooks][n_frames]."""

    def __init__(self, model: "SlowARModel", max_batch: int, max_seq_len: int, pool_pages: int = 0):
        self._model = model
        self._hp = model._hp
        h = ctypes.c_void_p()
        _check(lib().s2k_sched_create(model.handle, max_batch, max_seq_len, pool_pages, ctypes.byref(h)))
        self._sc = h

    def submit(self, prompt: np.ndarray, max_new_tokens: int, temperature: float = 0.8, top_p: float = 0.8,
               top_k: int = 30, min_tokens_before_end: int = 0, im_end_id: int = -1, seed: int = 0,
               seq_id: int = 0) -> int:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        if p.shape[0] != self._hp.num_codebooks + 1:
            raise S2KError(-1, f"prompt must have {self._hp.num_codebooks + 1} rows")
        gp = _GenParams(max_new_tokens, temperature, top_p, top_k, min_tokens_before_end, im_end_id, seed, seq_id)
        rid = ctypes.c_int32(0)
        _check(lib().s2k_sched_submit(self._sc, _ptr(p), p.shape[1], ctypes.byref(gp), ctypes.byref(rid)))
        return rid.value

    def step(self):
        """(live, waiting) after admitting, one batched frame and retiring."""
        nl, nw = ctypes.c_int32(0), ctypes.c_int32(0)
        _check(lib().s2k_sched_step(self._sc, ctypes.byref(nl), ctypes.byref(nw)))
        return nl.value, nw.value

    def run(self) -> None:
        _check(lib().s2k_sched_run(self._sc))

    def poll(self, req_id: int):
        st, nf = ctypes.c_int32(0), ctypes.c_int32(0)
        _check(lib().s2k_sched_poll(self._sc, req_id, ctypes.byref(st), ctypes.byref(nf)))
        return st.value, nf.value

    def poll_status(self, req_id: int):
        """(state, n_frames, status of a failed request)."""
        st, nf, rs = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_int32(0)
        _check(lib().s2k_sched_poll_status(self._sc, req_id, ctypes.byref(st), ctypes.byref(nf), ctypes.byref(rs)))
        return st.value, nf.value, rs.value

    def cancel(self, req_id: int) -> None:
        _check(lib().s2k_sched_cancel(self._sc, req_id))

    def set_frame_callback(self, fn: Optional[Callable[[int, np.ndarray, int], bool]]) -> None:
        """fn(req_id, codes [num_codebooks], frame_index) after each frame; False cancels the request."""
        if fn is None:
            self._cb = None
            _check(lib().s2k_sched_set_frame_callback(self._sc, SCHED_FRAME_CB(), None))
            return

        def _cb(rid, codes_ptr, idx, ncb_, user):
            arr = np.ctypeslib.as_array(codes_ptr, shape=(ncb_,)).copy()
            return 1 if fn(rid, arr, idx) else 0
        self._cb = SCHED_FRAME_CB(_cb)  # kept alive while the scheduler holds it
        _check(lib().s2k_sched_set_frame_callback(self._sc, self._cb, None))

    def result(self, req_id: int) -> np.ndarray:
        nf = ctypes.c_int32(0)
        _check(lib().s2k_sched_result(self._sc, req_id, None, 0, ctypes.byref(nf)))
        ncb = max(self._hp.num_codebooks, 1)
        buf = np.zeros(ncb * max(nf.value, 1), dtype=np.int32)
        _check(lib().s2k_sched_result(self._sc, req_id, _ptr(buf), nf.value, ctypes.byref(nf)))
        return buf[: ncb * nf.value].reshape(ncb, nf.value)

    def stats(self) -> dict:
        st = _SchedStats()
        _check(lib().s2k_sched_get_stats(self._sc, ctypes.byref(st)))
        return {name: getattr(st, name) for name, _ in _SchedStats._fields_}

    def close(self) -> None:
        if getattr(self, "_sc", None):
            lib().s2k_sched_free(self._sc)
            self._sc = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass



def det_expf(x: np.ndarray, device: int = 0) -> np.ndarray:
    """The device exp every softmax / SiLU / sampler kernel uses, over x
    (float32), through s2k_debug_det_expf."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    _check(lib().s2k_debug_det_expf(device, x.ctypes.data, y.ctypes.data, x.size))
    return y

def launch_count(reset: bool = False) -> int:
    return int(lib().s2k_launch_count(1 if reset else 0))


class AudioCodec:
    """Mirror of s2::AudioCodec's decode side (include/s2_codec.h:14-60):
    decode (AudioCodec::decode), samples_per_code_frame,
    streaming_history_frames, num_codebooks, plus the windowed decode of
    offline synthesis (decode_codes_windowed) and a streaming decoder.
    Codes are [num_codebooks][n_frames] int32, audio float32."""

    def __init__(self, hparams, device: int = 0):
        self._hp = hparams
        self._c = ctypes.c_void_p()
        h = codec_hp_struct(hparams)
        _check(lib().s2k_codec_create(device, ctypes.byref(h), ctypes.byref(self._c)))

    @classmethod
    def from_gguf(cls, path: str, device: int = 0) -> "AudioCodec":
        self = cls.__new__(cls)
        self._hp = None
        self._c = ctypes.c_void_p()
        _check(lib().s2k_codec_load_gguf(device, path.encode(), ctypes.byref(self._c)))
        return self

    def upload_tensor(self, name: str, ggml_type: int, ne, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        ne4 = (ctypes.c_int64 * 4)(*[int(x) for x in (list(ne) + [1, 1, 1, 1])[:4]])
        _check(lib().s2k_codec_upload_tensor(self._c, name.encode(), ggml_type, ne4, _ptr(data), data.nbytes))

    def load_tensors(self, tensors) -> None:
        """tensors: (spec, fp16 array) pairs as synthetic.make_codec yields"""
        for spec, arr in tensors:
            self.upload_tensor(spec.name, 1 if arr.dtype == np.float16 else 0, spec.ne, arr)
        _check(lib().s2k_codec_finalize(self._c))

    def samples_per_code_frame(self) -> int:
        return int(lib().s2k_codec_samples_per_frame(self._c))

    def streaming_history_frames(self) -> int:
        return int(lib().s2k_codec_history_frames(self._c))

    def num_codebooks(self) -> int:
        return int(lib().s2k_codec_num_codebooks(self._c))

    def receptive_frames(self) -> int:
        return int(lib().s2k_codec_receptive_frames(self._c))

    def decode(self, codes: np.ndarray) -> np.ndarray:
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        n = codes.shape[1]
        out = np.empty(n * self.samples_per_code_frame(), dtype=np.float32)
        ns = ctypes.c_int64(0)
        _check(lib().s2k_codec_decode(self._c, _ptr(codes), n, _ptr(out), out.size, ctypes.byref(ns)))
        return out[: ns.value]

    def decode_range(self, codes: np.ndarray, emit_begin: int, emit_end: int) -> np.ndarray:
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        n = codes.shape[1]
        out = np.empty(max(emit_end - emit_begin, 0) * self.samples_per_code_frame(), dtype=np.float32)
        ns = ctypes.c_int64(0)
        _check(lib().s2k_codec_decode_range(self._c, _ptr(codes), n, emit_begin, emit_end, _ptr(out), out.size,
                                            ctypes.byref(ns)))
        return out[: ns.value]

    def decode_windowed(self, codes: np.ndarray, stride_frames: int = 16, context_frames: int = -1):
        """(audio, device ms, windows) of decode_codes_windowed"""
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        ncb, n = codes.shape
        out = np.empty(n * self.samples_per_code_frame(), dtype=np.float32)
        ns, ms, nb = ctypes.c_int64(0), ctypes.c_double(0), ctypes.c_int32(0)
        _check(lib().s2k_codec_decode_windowed(self._c, _ptr(codes), n, ncb, stride_frames, context_frames, _ptr(out),
                                               out.size, ctypes.byref(ns), ctypes.byref(ms), ctypes.byref(nb)))
        return out[: ns.value], ms.value, nb.value

    def stream(self, stride_frames: int = 4, context_frames: int = -1, holdback_frames: int = -1) -> "CodecStream":
        return CodecStream(self, stride_frames, context_frames, holdback_frames)

    def close(self) -> None:
        if getattr(self, "_c", None):
            lib().s2k_codec_free(self._c)
            self._c = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CodecStream:
    """Streaming decode: push one frame of codes at a time, get the PCM each
    window releases (decode_window_and_emit, src/s2_pipeline.cpp:1034-1115)."""

    def __init__(self, codec: AudioCodec, stride_frames: int, context_frames: int, holdback_frames: int):
        self._codec = codec
        self._s = ctypes.c_void_p()
        _check(lib().s2k_codec_stream_create(codec._c, stride_frames, context_frames, holdback_frames,
                                             ctypes.byref(self._s)))

    def _buf(self) -> np.ndarray:
        return np.empty(max(int(lib().s2k_codec_stream_max_release(self._s)), 1), dtype=np.float32)

    def push(self, frame_codes) -> np.ndarray:
        fc = np.ascontiguousarray(frame_codes, dtype=np.int32)
        out = self._buf()
        n = ctypes.c_int64(0)
        _check(lib().s2k_codec_stream_push(self._s, _ptr(fc), _ptr(out), out.size, ctypes.byref(n)))
        return out[: n.value]

    def finish(self) -> np.ndarray:
        out = self._buf()
        n = ctypes.c_int64(0)
        _check(lib().s2k_codec_stream_finish(self._s, _ptr(out), out.size, ctypes.byref(n)))
        return out[: n.value]

    def close(self) -> None:
        if getattr(self, "_s", None):
            lib().s2k_codec_stream_free(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
