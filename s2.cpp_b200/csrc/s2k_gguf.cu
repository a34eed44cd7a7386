// s2k_gguf.cu -- a GGUF reader without ggml: the model's hyper-parameters
// from the file's key/value metadata and its tensors streamed straight into
// s2k_model_upload_tensor.
//
// Reference: SlowARModel::load_shared reads the hyper-parameters with
// gguf_find_key / gguf_get_val_* and the defaults of src/s2_model.cpp:245-288;
// read_all_tensor_data (src/s2_pipeline.cpp:306-389) seeks to
// data_offset + tensor offset and hands each model tensor's bytes to
// ggml_backend_tensor_set.  Here the same bytes go to the device re-layout.
//
// File format (GGUF v2 / v3, little endian): magic "GGUF", version u32,
// tensor count u64, key/value count u64; key/value pairs (string key, u32 type,
// value); tensor infos (string name, u32 n_dims, u64 ne[n_dims], u32 ggml
// type, u64 offset relative to the data section); the data section starts at
// the end of the tensor infos rounded up to general.alignment (default 32).
// Strings are a u64 length and the bytes (no terminator).
#include "../../include/s2k.h"
#include "s2k_model.h"

#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

enum GgufType : uint32_t {
    GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6, GT_BOOL = 7,
    GT_STRING = 8, GT_ARRAY = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12
};

struct GgufValue {
    uint32_t type = 0;
    uint64_t u = 0;  // integer / bool payload
    int64_t i = 0;
    double f = 0;
    std::string s;
    std::vector<int64_t> arr;  // integer arrays (the codec's rate lists)
    uint32_t arr_type = 0;
};

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;
    uint64_t nbytes = 0;
};

struct GgufFile {
    uint32_t version = 0;
    std::map<std::string, GgufValue> kv;
    std::vector<GgufTensor> tensors;
    uint64_t data_offset = 0;
    uint64_t file_size = 0;
};

struct Reader {
    std::FILE *f = nullptr;
    bool ok = true;
    bool read(void *p, size_t n) {
        if (ok && std::fread(p, 1, n, f) != n) ok = false;
        return ok;
    }
    template <class T>
    T get() {
        T v{};
        read(&v, sizeof(T));
        return v;
    }
    bool str(std::string *out) {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 24)) return ok = false;
        out->resize(n);
        return n == 0 || read(&(*out)[0], n);
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
    }
}

// Bytes of a ggml tensor of `type` with ne[0] elements per row (the block
// formats the path uploads, and the plain types a GGUF may also hold).
bool tensor_bytes(uint32_t type, const int64_t ne[4], uint64_t *out) {
    int64_t blk = 1, bb = 0;
    switch (type) {
    case 0: bb = 4; break;                 // F32
    case 1: bb = 2; break;                 // F16
    case 8: blk = 32; bb = 34; break;      // Q8_0
    case 12: blk = 256; bb = 144; break;   // Q4_K
    case 14: blk = 256; bb = 210; break;   // Q6_K
    case 30: bb = 2; break;                // BF16
    default: return false;
    }
    if (ne[0] % blk != 0) return false;
    *out = (uint64_t)(ne[0] / blk * bb) * (uint64_t)ne[1] * (uint64_t)ne[2] * (uint64_t)ne[3];
    return true;
}

s2k_status parse(const char *path, GgufFile *g, std::FILE **keep) {
    std::FILE *f = std::fopen(path, "rb");
    if (!f) return fail(S2K_ERR_ARG, "cannot open '%s'", path);
    Reader r{f};
    auto bad = [&](const char *what) {
        std::fclose(f);
        return fail(S2K_ERR_ARG, "'%s': malformed GGUF (%s)", path, what);
    };
    char magic[4];
    if (!r.read(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) return bad("magic");
    g->version = r.get<uint32_t>();
    if (g->version < 2 || g->version > 3) return bad("version");
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) return bad("counts");
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key;
        if (!r.str(&key)) return bad("key");
        GgufValue v;
        v.type = r.get<uint32_t>();
        if (!r.ok) return bad("value type");
        if (v.type == GT_STRING) {
            if (!r.str(&v.s)) return bad("string value");
        } else if (v.type == GT_ARRAY) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            if (!r.ok) return bad("array header");
            if (et == GT_STRING) {
                std::string tmp;
                for (uint64_t i = 0; i < n; ++i)
                    if (!r.str(&tmp)) return bad("string array");
            } else {
                const size_t es = scalar_size(et);
                if (es == 0 || n > (1ull << 32)) return bad("array type");
                v.arr_type = et;
                const bool keep = n <= 64 && (et == GT_U32 || et == GT_I32 || et == GT_U64 || et == GT_I64);
                if (keep) {
                    for (uint64_t i = 0; i < n; ++i) {
                        uint64_t raw = 0;
                        if (!r.read(&raw, es)) return bad("array data");
                        v.arr.push_back(et == GT_I32 ? (int64_t)(int32_t)raw : (int64_t)raw);
                    }
                } else if (std::fseek(f, (long)(es * n), SEEK_CUR) != 0) {
                    return bad("array data");
                }
            }
        } else {
            const size_t es = scalar_size(v.type);
            if (es == 0) return bad("value type");
            uint64_t raw = 0;
            if (!r.read(&raw, es)) return bad("value");
            switch (v.type) {
            case GT_I8: v.i = (int8_t)raw; break;
            case GT_I16: v.i = (int16_t)raw; break;
            case GT_I32: v.i = (int32_t)raw; break;
            case GT_I64: v.i = (int64_t)raw; break;
            case GT_F32: {
                float x;
                std::memcpy(&x, &raw, 4);
                v.f = x;
                break;
            }
            case GT_F64: std::memcpy(&v.f, &raw, 8); break;
            default: v.u = raw; v.i = (int64_t)raw; break;
            }
        }
        g->kv[key] = v;
    }
    for (uint64_t t = 0; t < n_tensors; ++t) {
        GgufTensor ti;
        if (!r.str(&ti.name)) return bad("tensor name");
        const uint32_t nd = r.get<uint32_t>();
        if (!r.ok || nd < 1 || nd > 4) return bad("tensor dims");
        for (uint32_t d = 0; d < nd; ++d) ti.ne[d] = (int64_t)r.get<uint64_t>();
        ti.type = r.get<uint32_t>();
        ti.offset = r.get<uint64_t>();
        if (!r.ok) return bad("tensor info");
        if (!tensor_bytes(ti.type, ti.ne, &ti.nbytes)) ti.nbytes = 0;  // a type this path does not read
        g->tensors.push_back(ti);
    }
    uint64_t align = 32;
    auto it = g->kv.find("general.alignment");
    if (it != g->kv.end() && (it->second.type == GT_U32 || it->second.type == GT_I32) && it->second.u > 0)
        align = it->second.u;
    const long pos = std::ftell(f);
    if (pos < 0) return bad("position");
    g->data_offset = ((uint64_t)pos + align - 1) / align * align;
    std::fseek(f, 0, SEEK_END);
    g->file_size = (uint64_t)std::ftell(f);
    for (const GgufTensor &ti : g->tensors)
        if (ti.nbytes && g->data_offset + ti.offset + ti.nbytes > g->file_size) return bad("tensor past end of file");
    if (keep) {
        *keep = f;
    } else {
        std::fclose(f);
    }
    return S2K_OK;
}

// The hyper-parameters with the keys and defaults of SlowARModel::load_shared
// (src/s2_model.cpp:245-288).  head_dim is not a key: the reference derives
// it from the q_norm / wo shapes (src/s2_model.cpp:879-884).
void read_hparams(const GgufFile &g, s2k_hparams *hp) {
    auto find = [&](const std::string &k) -> const GgufValue * {
        auto it = g.kv.find(k);
        return it == g.kv.end() ? nullptr : &it->second;
    };
    auto u32 = [&](const std::string &k, uint32_t def) -> int32_t {
        const GgufValue *v = find(k);
        if (!v || !(v->type == GT_U32 || v->type == GT_I32 || v->type == GT_U64 || v->type == GT_I64)) return (int32_t)def;
        return (int32_t)v->i;
    };
    auto f32 = [&](const std::string &k, float def) -> float {
        const GgufValue *v = find(k);
        if (!v || !(v->type == GT_F32 || v->type == GT_F64)) return def;
        return (float)v->f;
    };
    auto flag = [&](const std::string &k, bool def) -> int32_t {
        const GgufValue *v = find(k);
        if (!v || v->type != GT_BOOL) return def ? 1 : 0;
        return v->u ? 1 : 0;
    };
    std::memset(hp, 0, sizeof(*hp));
    std::string arch = "fish-speech";
    const GgufValue *a = find("general.architecture");
    if (a && a->type == GT_STRING) arch = a->s;
    const std::string p = arch + ".";
    hp->has_fast_decoder = a && a->type == GT_STRING ? (arch == "fish-speech") : 0;
    hp->context_length = u32(p + "context_length", 32768);
    hp->vocab_size = u32(p + "vocab_size", 155776);
    hp->embedding_length = u32(p + "embedding_length", 2560);
    hp->feed_forward_length = u32(p + "feed_forward_length", 9728);
    hp->block_count = u32(p + "block_count", 36);
    hp->head_count = u32(p + "attention.head_count", 32);
    hp->head_count_kv = u32(p + "attention.head_count_kv", 8);
    hp->rope_freq_base = f32(p + "rope.freq_base", 1e6f);
    hp->rms_norm_eps = f32(p + "attention.layer_norm_rms_epsilon", 1e-6f);
    hp->codebook_size = u32("fish_speech.codebook_size", 4096);
    hp->num_codebooks = u32("fish_speech.num_codebooks", 10);
    hp->semantic_begin_id = u32("fish_speech.semantic_begin_id", 151678);
    hp->semantic_end_id = u32("fish_speech.semantic_end_id", 155773);
    hp->tie_word_embeddings = flag("fish_speech.tie_word_embeddings", true);
    hp->attention_qk_norm = flag("fish_speech.attention_qk_norm", false);
    hp->scale_codebook_embeddings = flag("fish_speech.scale_codebook_embeddings", false);
    if (hp->has_fast_decoder) {
        hp->fast_context_length = u32("fish_speech.fast_context_length", 11);
        hp->fast_embedding_length = u32("fish_speech.fast_embedding_length", 2560);
        hp->fast_feed_forward_length = u32("fish_speech.fast_feed_forward_length", 9728);
        hp->fast_block_count = u32("fish_speech.fast_block_count", 4);
        hp->fast_head_count = u32("fish_speech.fast_head_count", 32);
        hp->fast_head_count_kv = u32("fish_speech.fast_head_count_kv", 8);
        hp->fast_head_dim = u32("fish_speech.fast_head_dim", 128);
        hp->fast_rope_freq_base = f32("fish_speech.fast_rope_freq_base", 1e6f);
        hp->fast_rms_norm_eps = f32("fish_speech.fast_layer_norm_rms_eps", 1e-6f);
        hp->fast_attention_qk_norm = flag("fish_speech.fast_attention_qk_norm", false);
        hp->fast_has_project_in = flag("fish_speech.fast_project_in", false);
    }
    // head_dim from layer 0's q_norm ([head_dim]) or wo ([H * head_dim, dim])
    hp->head_dim = 128;
    for (const GgufTensor &t : g.tensors) {
        if (t.name == "layers.0.attention.q_norm.weight") {
            hp->head_dim = (int32_t)t.ne[0];
            break;
        }
        if (t.name == "layers.0.attention.wo.weight" && hp->head_count > 0) hp->head_dim = (int32_t)(t.ne[0] / hp->head_count);
    }
}

}  // namespace

S2K_API s2k_status s2k_gguf_read_hparams(const char *path, s2k_hparams *out) {
    if (!path || !out) return fail(S2K_ERR_ARG, "NULL argument");
    GgufFile g;
    s2k_status rc = parse(path, &g, nullptr);
    if (rc) return rc;
    read_hparams(g, out);
    return S2K_OK;
}

S2K_API s2k_status s2k_gguf_tensor_info(const char *path, int32_t index, char *name, size_t name_cap, int32_t *type,
                                        int64_t ne[4], uint64_t *offset, uint64_t *nbytes, int32_t *n_tensors) {
    if (!path) return fail(S2K_ERR_ARG, "NULL path");
    GgufFile g;
    s2k_status rc = parse(path, &g, nullptr);
    if (rc) return rc;
    if (n_tensors) *n_tensors = (int32_t)g.tensors.size();
    if (index < 0) return S2K_OK;  // count only
    if (index >= (int32_t)g.tensors.size()) return fail(S2K_ERR_ARG, "tensor %d of %zu", index, g.tensors.size());
    const GgufTensor &t = g.tensors[(size_t)index];
    if (name) {
        if (name_cap < t.name.size() + 1) return fail(S2K_ERR_ARG, "name buffer too small");
        std::memcpy(name, t.name.c_str(), t.name.size() + 1);
    }
    if (type) *type = (int32_t)t.type;
    if (ne)
        for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
    if (offset) *offset = g.data_offset + t.offset;
    if (nbytes) *nbytes = t.nbytes;
    return S2K_OK;
}

S2K_API s2k_status s2k_model_load_gguf(int32_t device, const char *path, s2k_model **out) {
    if (!path || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = nullptr;
    GgufFile g;
    std::FILE *f = nullptr;
    s2k_status rc = parse(path, &g, &f);
    if (rc) return rc;
    std::unique_ptr<std::FILE, int (*)(std::FILE *)> fh(f, &std::fclose);
    s2k_hparams hp;
    read_hparams(g, &hp);
    s2k_model *m = nullptr;
    rc = s2k_model_create(device, &hp, &m);
    if (rc) return rc;
    std::vector<uint8_t> buf;
    for (const GgufTensor &t : g.tensors) {
        // the model's tensors (the names SlowARModel binds); others (the
        // codec's) stay in the file, as read_all_tensor_data leaves them to
        // the codec
        if (!s2k_model_binds(m, t.name.c_str())) continue;
        if (t.nbytes == 0) {
            s2k_model_free(m);
            return fail(S2K_ERR_UNSUPPORTED, "tensor '%s' has ggml type %u, which this path does not read",
                        t.name.c_str(), t.type);
        }
        buf.resize(t.nbytes);
        if (fseeko(f, (off_t)(g.data_offset + t.offset), SEEK_SET) != 0 ||
            std::fread(buf.data(), 1, t.nbytes, f) != t.nbytes) {
            s2k_model_free(m);
            return fail(S2K_ERR_ARG, "failed to read tensor '%s'", t.name.c_str());
        }
        rc = s2k_model_upload_tensor(m, t.name.c_str(), (int32_t)t.type, t.ne, buf.data(), t.nbytes);
        if (rc) {
            std::string msg = s2k_last_error();
            s2k_model_free(m);
            return fail(rc, "%s", msg.c_str());
        }
    }
    rc = s2k_model_finalize(m);
    if (rc) {
        std::string msg = s2k_last_error();
        s2k_model_free(m);
        return fail(rc, "%s", msg.c_str());
    }
    *out = m;
    return S2K_OK;
}

// ---------------------------------------------------------------------------
// codec: AudioCodec::load_shared's keys (src/s2_codec.cpp:765-874) and the
// codec tensors ("c." names in the combined file, bare in a codec-only one)
// ---------------------------------------------------------------------------
namespace {

s2k_status read_codec_hparams(const GgufFile &g, s2k_codec_hparams *hp, std::string *prefix) {
    auto find = [&](const std::string &k) -> const GgufValue * {
        auto it = g.kv.find(k);
        return it == g.kv.end() ? nullptr : &it->second;
    };
    bool ok = true;
    std::string missing;
    auto req_int = [&](const std::string &k) -> int32_t {
        const GgufValue *v = find(k);
        if (!v || !(v->type == GT_U32 || v->type == GT_I32 || v->type == GT_U64 || v->type == GT_I64)) {
            if (ok) missing = k;
            ok = false;
            return 0;
        }
        return (int32_t)v->i;
    };
    auto req_f32 = [&](const std::string &k) -> float {
        const GgufValue *v = find(k);
        if (!v || !(v->type == GT_F32 || v->type == GT_F64)) {
            if (ok) missing = k;
            ok = false;
            return 0.f;
        }
        return (float)v->f;
    };
    auto req_arr = [&](const std::string &k, int32_t *dst, int32_t *n) {
        const GgufValue *v = find(k);
        if (!v || v->type != GT_ARRAY || v->arr.empty() || v->arr.size() > 8) {
            if (ok) missing = k;
            ok = false;
            return;
        }
        *n = (int32_t)v->arr.size();
        for (size_t i = 0; i < v->arr.size(); ++i) dst[i] = (int32_t)v->arr[i];
    };
    const GgufValue *a = find("general.architecture");
    if (!a || a->type != GT_STRING) return fail(S2K_ERR_ARG, "codec GGUF: missing general.architecture");
    if (a->s == "fish-speech") {
        *prefix = "c.";
    } else if (a->s == "fish-speech-codec") {
        *prefix = "";
    } else {
        return fail(S2K_ERR_ARG, "codec GGUF: unexpected architecture %s", a->s.c_str());
    }
    std::memset(hp, 0, sizeof(*hp));
    const std::string k = "fish_speech.codec.";
    hp->sample_rate = req_int(k + "sample_rate");
    hp->hop_length = req_int(k + "hop_length");
    hp->latent_dim = req_int(k + "latent_dim");
    hp->decoder_dim = req_int(k + "decoder_dim");
    req_arr(k + "decoder_rates", hp->decoder_rates, &hp->n_decoder_rates);
    hp->quantizer_input_dim = req_int(k + "quantizer_input_dim");
    hp->quantizer_codebook_dim = req_int(k + "quantizer_codebook_dim");
    hp->quantizer_residual_codebooks = req_int(k + "quantizer_residual_codebooks");
    hp->quantizer_residual_codebook_size = req_int(k + "quantizer_residual_codebook_size");
    hp->quantizer_semantic_codebook_size = req_int(k + "quantizer_semantic_codebook_size");
    req_arr(k + "quantizer_downsample_factor", hp->quantizer_downsample_factor, &hp->n_downsample);
    hp->rvq_window_size = req_int(k + "rvq_transformer.window_size");
    hp->rvq_block_size = req_int(k + "rvq_transformer.block_size");
    hp->rvq_n_layer = req_int(k + "rvq_transformer.n_layer");
    hp->rvq_n_local_heads = req_int(k + "rvq_transformer.n_local_heads");
    hp->rvq_head_dim = req_int(k + "rvq_transformer.head_dim");
    hp->rvq_dim = req_int(k + "rvq_transformer.dim");
    hp->rvq_rope_base = req_f32(k + "rvq_transformer.rope_freq_base");
    hp->rvq_norm_eps = req_f32(k + "rvq_transformer.layer_norm_rms_eps");
    if (!ok) return fail(S2K_ERR_ARG, "codec GGUF: missing key %s", missing.c_str());
    return S2K_OK;
}

}  // namespace

S2K_API s2k_status s2k_codec_load_gguf(int32_t device, const char *path, s2k_codec **out) {
    if (!path || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = nullptr;
    GgufFile g;
    std::FILE *f = nullptr;
    s2k_status rc = parse(path, &g, &f);
    if (rc) return rc;
    std::unique_ptr<std::FILE, int (*)(std::FILE *)> fh(f, &std::fclose);
    s2k_codec_hparams hp;
    std::string prefix;
    if ((rc = read_codec_hparams(g, &hp, &prefix))) return rc;
    s2k_codec *c = nullptr;
    if ((rc = s2k_codec_create(device, &hp, &c))) return rc;
    std::vector<uint8_t> buf;
    for (const GgufTensor &t : g.tensors) {
        if (t.name.compare(0, prefix.size(), prefix) != 0) continue;
        // codec tensors only: the quantizer and decoder trees (the encoder's
        // are left in the file, as decode does not read them)
        const std::string bare = t.name.substr(prefix.size());
        if (bare.compare(0, 10, "quantizer.") != 0 && bare.compare(0, 8, "decoder.") != 0) continue;
        if (t.type != S2K_TYPE_F32 && t.type != S2K_TYPE_F16) {
            s2k_codec_free(c);
            return fail(S2K_ERR_UNSUPPORTED, "codec tensor '%s' has ggml type %u (F32 / F16)", t.name.c_str(), t.type);
        }
        buf.resize(t.nbytes);
        if (fseeko(f, (off_t)(g.data_offset + t.offset), SEEK_SET) != 0 ||
            std::fread(buf.data(), 1, t.nbytes, f) != t.nbytes) {
            s2k_codec_free(c);
            return fail(S2K_ERR_ARG, "failed to read tensor '%s'", t.name.c_str());
        }
        rc = s2k_codec_upload_tensor(c, t.name.c_str(), (int32_t)t.type, t.ne, buf.data(), t.nbytes);
        if (rc) {
            std::string msg = s2k_last_error();
            s2k_codec_free(c);
            return fail(rc, "%s", msg.c_str());
        }
    }
    rc = s2k_codec_finalize(c);
    if (rc) {
        std::string msg = s2k_last_error();
        s2k_codec_free(c);
        return fail(rc, "%s", msg.c_str());
    }
    *out = c;
    return S2K_OK;
}
