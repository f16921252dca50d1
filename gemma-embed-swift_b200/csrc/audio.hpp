// audio.hpp -- the gemma4a audio encoder: its configuration, its weights and workspace on each
// device, and the host side of the log-mel front end (chunking, counts, tables).
//
// Reference: Sources/GemmaEmbed/Model/AudioConfig.swift (configuration), AudioWeights.swift
// (tensors), Metal/AudioTower.swift (the forward), Audio/AudioPreprocessor.swift (front end),
// AudioEmbedding.swift (batching and the text tower over each clip's rows).
#pragma once

#include <float.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "kernels.hpp"

namespace ge {

// AudioConfig (AudioConfig.swift:22-48): sizes from the file, the rest fixed by llama.cpp.
struct AudioConfig {
    int hidden = 0, layers = 0, heads = 0, head_dim = 0, ff = 0, mel_bins = 0, projection_dim = 0, output_width = 0;
    float eps = 1e-6f;  // the file's epsilon is ignored (AudioConfig.swift:26-27)
    int window = 12, relative_positions = 13, dw_kernel = 5;
    float softcap = 50.0f, ff_residual = 0.5f;
    int sub_channels[2] = {128, 32};
    // (1 / sqrt(head_dim)) / ln 2 on the queries, softplus(1) / ln 2 on the keys.
    float query_scale() const;
    float key_scale() const;
    int subsample_width() const { return (mel_bins / 4) * sub_channels[1]; }
};

// A Gemma4ClippableLinear on the device (ClippedLinear, AudioWeights.swift:7-18): the fp16
// weight, an optional bias, and its input and output bounds (the float range when absent).
struct ClippedDev {
    DevWeight w;
    float* bias = nullptr;
    float in_lo = -FLT_MAX, in_hi = FLT_MAX, out_lo = -FLT_MAX, out_hi = FLT_MAX;
};

struct AudioLayerDev {
    ClippedDev up, down, q, k, v, o, pw1, pw2, up1, down1;
    // Norm weights; the two post-FFN norms carry the half-step residual weight (0.5 w).
    float *ffn_norm = nullptr, *ffn_post_half = nullptr, *attn_pre = nullptr, *attn_post = nullptr,
          *conv_norm = nullptr, *norm_conv = nullptr, *ffn_norm1 = nullptr, *ffn_post1_half = nullptr, *ln2 = nullptr;
    float* dw_t = nullptr;    // [5][hidden] depthwise taps, tap-major
    float* rel = nullptr;     // [13][hidden]: attn_k_rel over the sinusoid of each distance
    float* qscale = nullptr;  // [head_dim]: query_scale * per_dim_scale
};

struct AudioWorkspace {
    int cap_trows = 0, cap_frames = 0, cap_t0 = 0, cap_chunks = 0;
    size_t cap_pcm = 0;
    float* pcm = nullptr;
    AudioChunk* chunks = nullptr;
    int* chunk_start = nullptr;  // per token row: its chunk's first token row
    float *mel = nullptr, *c1 = nullptr, *x = nullptr, *o32 = nullptr;
    float* vectors = nullptr;  // [token rows][projection_dim]: the rows the text tower reads
    __half *c0 = nullptr, *a1 = nullptr, *a2 = nullptr, *h = nullptr, *hk = nullptr, *hv = nullptr, *q = nullptr,
           *k = nullptr, *v = nullptr, *attn = nullptr, *act = nullptr, *t = nullptr, *glu = nullptr, *h2 = nullptr;
    DevActivation a_a1, a_a2, a_h, a_hk, a_hv, a_attn, a_act, a_h2;
    AudioChunk* h_chunks = nullptr;
    int* h_cs = nullptr;
    float* h_pcm = nullptr;  // pinned staging of the clips' samples
    std::vector<void*> allocations;
};

// The audio encoder on one device.
struct AudioDev {
    bool loaded = false;
    float *conv0_w = nullptr, *conv0_n = nullptr, *conv1_n = nullptr;  // [128][9], [128], [32]
    DevWeight conv1;  // [128 (32 used)][1152], K = (kh * 3 + kw) * 128 + c
    ClippedDev in_proj, out_proj, proj;
    std::vector<AudioLayerDev> layers;
    // Front-end tables (MelTables points into these).
    float *hann = nullptr, *cos_t = nullptr, *sin_t = nullptr, *mel_w = nullptr;
    int *bitrev = nullptr, *band = nullptr;
    int mel_nw = 0;
    AudioWorkspace ws;
    std::vector<void*> allocations;
};

// A clip ready for the tower: 16 kHz mono samples (host, or an offset into a device buffer)
// cut into 30-second chunks (PreparedAudio, AudioPreprocessor.swift:17-23).
struct PreparedAudio {
    const float* samples = nullptr;
    int64_t count = 0;
    std::vector<float> converted;  // the 16 kHz mono samples when the input needed converting
    int64_t device_offset = 0;  // with a device PCM buffer: where this clip's samples start
    int frames() const;
    int tokens() const;
};

// AudioFrontEnd's counts (AudioPreprocessor.swift:33-95).
constexpr int64_t kAudioChunkSamples = 30 * 16000;
constexpr int64_t kAudioMinimumSamples = 2;
int audio_frame_count(int64_t samples);
int audio_tokens_for_frames(int frames);
int64_t audio_token_count(int64_t samples);
// AudioFrontEnd.init's tables (AudioPreprocessor.swift:52-65, 100-123, 208-217): Hann, sin and
// cos [512], the bit reversal [512], and per filter its band [lo, hi) and weight offset into
// `w` (the filter's weights over its band, back to back).
void audio_front_tables(int mel, float* hann, float* sin_t, float* cos_t, int* bitrev, std::vector<int>& band,
                        std::vector<float>& w);

}  // namespace ge
