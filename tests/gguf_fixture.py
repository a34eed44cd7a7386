"""Writes a synthetic model as a GGUF file with gguf-py (GGUFWriter), under
the keys SlowARModel::load_shared reads (src/s2_model.cpp:245-288) and the
tensor names it binds (src/s2_model.cpp:374-423), plus one tensor of another
component (a codec-like name) that the model loader must skip.

gguf-py is present in the build container; tests that need it skip where it
is missing.
"""
from __future__ import annotations

import numpy as np

import synthetic


def write_model_gguf(path: str, hp, tensors, extra_tensor: bool = True) -> None:
    import gguf

    w = gguf.GGUFWriter(path, arch="fish-speech")
    p = "fish-speech."
    w.add_uint32(p + "context_length", hp.context_length)
    w.add_uint32(p + "vocab_size", hp.vocab_size)
    w.add_uint32(p + "embedding_length", hp.embedding_length)
    w.add_uint32(p + "feed_forward_length", hp.feed_forward_length)
    w.add_uint32(p + "block_count", hp.block_count)
    w.add_uint32(p + "attention.head_count", hp.head_count)
    w.add_uint32(p + "attention.head_count_kv", hp.head_count_kv)
    w.add_float32(p + "rope.freq_base", hp.rope_freq_base)
    w.add_float32(p + "attention.layer_norm_rms_epsilon", hp.rms_norm_eps)
    f = "fish_speech."
    w.add_uint32(f + "codebook_size", hp.codebook_size)
    w.add_uint32(f + "num_codebooks", hp.num_codebooks)
    w.add_uint32(f + "semantic_begin_id", hp.semantic_begin_id)
    w.add_uint32(f + "semantic_end_id", hp.semantic_end_id)
    w.add_bool(f + "tie_word_embeddings", bool(hp.tie_word_embeddings))
    w.add_bool(f + "attention_qk_norm", bool(hp.attention_qk_norm))
    w.add_bool(f + "scale_codebook_embeddings", bool(hp.scale_codebook_embeddings))
    w.add_uint32(f + "fast_context_length", hp.fast_context_length)
    w.add_uint32(f + "fast_embedding_length", hp.fast_embedding_length)
    w.add_uint32(f + "fast_feed_forward_length", hp.fast_feed_forward_length)
    w.add_uint32(f + "fast_block_count", hp.fast_block_count)
    w.add_uint32(f + "fast_head_count", hp.fast_head_count)
    w.add_uint32(f + "fast_head_count_kv", hp.fast_head_count_kv)
    w.add_uint32(f + "fast_head_dim", hp.fast_head_dim)
    w.add_float32(f + "fast_rope_freq_base", hp.fast_rope_freq_base)
    w.add_float32(f + "fast_layer_norm_rms_eps", hp.fast_rms_norm_eps)
    w.add_bool(f + "fast_attention_qk_norm", bool(hp.fast_attention_qk_norm))
    w.add_bool(f + "fast_project_in", bool(hp.fast_has_project_in))
    w.add_array("tokenizer.ggml.tokens", ["<a>", "<b>", "<c>"])  # a string array the reader must step over
    for spec, buf in tensors:
        if spec.type == synthetic.GGML_F32:
            w.add_tensor(spec.name, np.frombuffer(buf.tobytes(), dtype=np.float32).reshape(spec.ne1, spec.ne0)
                         if spec.ne1 > 1 else np.frombuffer(buf.tobytes(), dtype=np.float32))
        elif spec.type == synthetic.GGML_F16:
            w.add_tensor(spec.name, np.frombuffer(buf.tobytes(), dtype=np.float16).reshape(spec.ne1, spec.ne0))
        else:
            raw = np.asarray(buf, dtype=np.uint8).reshape(spec.ne1, -1)
            w.add_tensor(spec.name, raw, raw_shape=raw.shape, raw_dtype=gguf.GGMLQuantizationType(spec.type))
    if extra_tensor:
        w.add_tensor("c.decoder.conv.weight", np.arange(64, dtype=np.float32).reshape(4, 16))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def write_codec_gguf(path: str, ch, tensors, combined: bool = True) -> None:
    """A codec GGUF under the keys AudioCodec::load_shared reads
    (src/s2_codec.cpp:813-858): the combined layout ("fish-speech", tensors
    named "c.*", next to a model tensor the codec loader must skip) or a
    codec-only file ("fish-speech-codec", bare names)."""
    import gguf

    w = gguf.GGUFWriter(path, arch="fish-speech" if combined else "fish-speech-codec")
    k = "fish_speech.codec."
    w.add_uint32(k + "sample_rate", ch.sample_rate)
    w.add_uint32(k + "hop_length", ch.hop_length)
    w.add_uint32(k + "frame_length", ch.hop_length)
    w.add_uint32(k + "encoder_dim", 64)
    w.add_uint32(k + "decoder_dim", ch.decoder_dim)
    w.add_uint32(k + "latent_dim", ch.latent_dim)
    w.add_array(k + "encoder_rates", list(reversed(ch.decoder_rates)))
    w.add_array(k + "decoder_rates", list(ch.decoder_rates))
    w.add_array(k + "encoder_transformer_layers", [0] * len(ch.decoder_rates))
    w.add_array(k + "decoder_transformer_layers", [0] * len(ch.decoder_rates))
    w.add_string(k + "quantizer_type", "downsample_residual_vector_quantize")
    w.add_uint32(k + "quantizer_input_dim", ch.quantizer_input_dim)
    w.add_uint32(k + "quantizer_codebook_dim", ch.quantizer_codebook_dim)
    w.add_uint32(k + "quantizer_residual_codebooks", ch.quantizer_residual_codebooks)
    w.add_uint32(k + "quantizer_residual_codebook_size", ch.quantizer_residual_codebook_size)
    w.add_uint32(k + "quantizer_semantic_codebook_size", ch.quantizer_semantic_codebook_size)
    w.add_array(k + "quantizer_downsample_factor", list(ch.quantizer_downsample_factor))
    w.add_uint32(k + "transformer.block_size", 8192)
    w.add_int32(k + "transformer.n_local_heads", -1)
    w.add_uint32(k + "transformer.head_dim", 64)
    w.add_float32(k + "transformer.rope_freq_base", 10000.0)
    w.add_float32(k + "transformer.layer_norm_rms_eps", 1e-5)
    w.add_uint32(k + "rvq_transformer.window_size", ch.rvq_window_size)
    w.add_uint32(k + "rvq_transformer.block_size", ch.rvq_block_size)
    w.add_uint32(k + "rvq_transformer.n_layer", ch.rvq_n_layer)
    w.add_uint32(k + "rvq_transformer.n_head", ch.rvq_dim // ch.rvq_head_dim)
    w.add_int32(k + "rvq_transformer.n_local_heads", ch.rvq_n_local_heads)
    w.add_uint32(k + "rvq_transformer.head_dim", ch.rvq_head_dim)
    w.add_uint32(k + "rvq_transformer.dim", ch.rvq_dim)
    w.add_uint32(k + "rvq_transformer.feed_forward_length", ch.rvq_ff)
    w.add_float32(k + "rvq_transformer.rope_freq_base", ch.rvq_rope_base)
    w.add_float32(k + "rvq_transformer.layer_norm_rms_eps", ch.rvq_norm_eps)
    pre = "c." if combined else ""
    if combined:
        w.add_tensor("norm.weight", np.ones(64, dtype=np.float32))  # a model tensor
    for spec, arr in tensors:
        w.add_tensor(pre + spec.name, np.asarray(arr).reshape(tuple(reversed(spec.ne))))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
