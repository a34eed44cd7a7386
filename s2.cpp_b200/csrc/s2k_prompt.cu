// s2k_prompt.cu -- the PromptTensor grid generate() and the scheduler take:
// the chat-formatted token row of a synthesis request, with the reference
// audio's codes (voice cloning) placed under the semantic tokens.
//
// Reference: s2::build_prompt (src/s2_prompt.cpp:5-103, include/s2_prompt.h).
// The tokenizer stays with the caller (the reference's Tokenizer::encode,
// src/s2_tokenizer.cpp), passed in as a callback; the ids build_prompt takes
// from TokenizerConfig (im_end_id, voice_id, semantic_begin_id) are arguments.
// Host code only.
#include "../../include/s2k.h"
#include "s2k_model.h"

#include <cstring>
#include <string>
#include <vector>

namespace {

constexpr int32_t kNewline = 198;  // the "\n" token build_prompt appends as NEWLINE

struct Encoder {
    s2k_encode_fn fn;
    void *user;
    bool ok = true;
    std::string err;
    void append(std::vector<int32_t> &dst, const std::string &text) {
        if (!ok) return;
        // ask for the length first, then fill
        const int32_t n = fn(text.c_str(), nullptr, 0, user);
        if (n < 0) {
            ok = false;
            err = "encode callback failed on \"" + text + "\"";
            return;
        }
        const size_t at = dst.size();
        dst.resize(at + (size_t)n);
        if (n > 0 && fn(text.c_str(), dst.data() + at, n, user) != n) {
            ok = false;
            err = "encode callback returned a different length on its second call";
        }
    }
};

}  // namespace

S2K_API s2k_status s2k_build_prompt(s2k_encode_fn encode, void *user, const char *text, const char *prompt_text,
                                    const int32_t *prompt_codes, int32_t num_codebooks, int32_t T_prompt,
                                    int32_t im_end_id, int32_t voice_id, int32_t semantic_begin_id, int32_t *out,
                                    size_t cap, int32_t *rows, int32_t *cols) {
    if (!encode || !text || !rows || !cols || num_codebooks < 0 || T_prompt < 0)
        return fail(S2K_ERR_ARG, "bad argument");
    if (T_prompt > 0 && !prompt_codes) return fail(S2K_ERR_ARG, "T_prompt > 0 without prompt codes");
    const std::string ptext = prompt_text ? prompt_text : "";
    Encoder enc{encode, user};
    // a reference clip counts only with its transcript (src/s2_prompt.cpp:24)
    const bool has_reference = prompt_codes != nullptr && T_prompt > 0 && !ptext.empty();
    const bool has_speaker_tag = ptext.find("<|speaker:") != std::string::npos;
    std::vector<int32_t> pre, post;
    if (has_reference) {
        enc.append(pre, "<|im_start|>system");
        pre.push_back(kNewline);
        enc.append(pre, "convert the provided text to speech reference to the following:\n\nText:\n");
        if (!has_speaker_tag) enc.append(pre, "<|speaker:0|>");
        enc.append(pre, ptext);
        enc.append(pre, "\n\nSpeech:\n");
        post.push_back(im_end_id);
        post.push_back(kNewline);
    } else {
        enc.append(post, "<|im_start|>system");
        post.push_back(kNewline);
        enc.append(post, "convert the provided text to speech");
        post.push_back(im_end_id);
        post.push_back(kNewline);
    }
    enc.append(post, "<|im_start|>user");
    post.push_back(kNewline);
    enc.append(post, text);
    post.push_back(im_end_id);
    post.push_back(kNewline);
    enc.append(post, "<|im_start|>assistant");
    post.push_back(kNewline);
    post.push_back(voice_id);
    if (!enc.ok) return fail(S2K_ERR_ARG, "%s", enc.err.c_str());

    const int32_t R = num_codebooks + 1;
    const int32_t C = (int32_t)pre.size() + (has_reference ? T_prompt : 0) + (int32_t)post.size();
    *rows = R;
    *cols = C;
    if (!out) return S2K_OK;  // size query
    if (cap < (size_t)R * C) return fail(S2K_ERR_ARG, "prompt grid needs %d x %d ints, capacity %zu", R, C, cap);
    std::memset(out, 0, (size_t)R * C * sizeof(int32_t));
    int32_t pos = 0;
    for (int32_t v : pre) out[pos++] = v;
    if (has_reference) {
        // row 0: the semantic tokens of codebook 0; rows 1..: every codebook's codes
        for (int32_t t = 0; t < T_prompt; ++t) out[pos + t] = prompt_codes[t] + semantic_begin_id;
        for (int32_t cb = 0; cb < num_codebooks; ++cb)
            for (int32_t t = 0; t < T_prompt; ++t)
                out[(size_t)(cb + 1) * C + pos + t] = prompt_codes[(size_t)cb * T_prompt + t];
        pos += T_prompt;
    }
    for (int32_t v : post) out[pos++] = v;
    return S2K_OK;
}
