// s2k_device.h -- per-sequence device state shared by the frame-loop kernels.
#pragma once

#include "s2k_kernels.h"

namespace s2k {

// Frames of codes a sequence's host ring holds: the host reads frame f from
// slot f % kFrameRing while later frames run (at most kFrameRing - 1 frames
// may be in flight ahead of the oldest one the host has not read).
constexpr int kFrameRing = 8;

// Mapped pinned memory the host polls while frames run.  frame_commit writes
// frame f's codes into ring[f % kFrameRing], then (after a system-scope
// fence) n_frames = f + 1.
struct HostStatus {
    volatile int n_frames;
    volatile int done;
    int pad[2];
    volatile int ring[kFrameRing][16];
};

// Generation parameters as the kernels read them (device copy, so a captured
// frame graph does not depend on them).
struct SampleCfg {
    float temperature, top_p;
    int top_k;
    int min_tokens_before_end;
    int im_end;
    int max_new_tokens;
    unsigned long long seed;
    unsigned int seq_id;
    int sem_begin, sem_end, cb_size, ncb, vocab;
    int *codes_out;  // [ncb][codes_ld] cb-major
    int codes_ld;
};

struct SeqState {
    int n_past;      // positions in the KV cache
    int n_frames;    // frames completed
    int done;        // generation finished
    int main_token;  // main token of the frame being built
    int codes[16];   // codes of the frame being built
    int step_in[17]; // [main, cb0..] input of the next Slow step
    int ras[10];     // repetition-aware-sampling window
    int n_ras;
    int pad[2];
};

struct SeqDev {
    SeqState state;
    SampleCfg cfg;
    HostStatus *host;  // device alias of mapped pinned memory (may be null)
    // read by the batched-frame kernels, set when the sequence is created
    KvPaged kv;        // the sequence's paged f16 KV cache
    float *hidden;     // [embedding_length] Slow hidden state for the next Fast-AR pass
};

}  // namespace s2k
