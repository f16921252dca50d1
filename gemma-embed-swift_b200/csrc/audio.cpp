// audio.cpp -- the gemma4a audio encoder on the GPU: configuration and weight checks, the repack
// of its weights into the device layout, the front end's tables and counts, its workspace, and
// its forward pass.
//
// Reference: AudioConfig.init (Model/AudioConfig.swift:50-85), AudioWeights.init
// (Model/AudioWeights.swift:67-135), AudioFrontEnd (Audio/AudioPreprocessor.swift:24-251) and
// AudioTower (Metal/AudioTower.swift), whose node order CPUAudioReference.forward states
// (Model/CPUAudioReference.swift:186-283).
#include <math.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <thread>

#include "model.hpp"
#include "weights.hpp"

namespace ge {

float AudioConfig::query_scale() const { return (1.0f / sqrtf(float(head_dim))) / logf(2.0f); }
float AudioConfig::key_scale() const { return logf(1.0f + expf(1.0f)) / logf(2.0f); }

// ---------------------------------------------------------------------------- front end (host)
// AudioFrontEnd.frameCount: PyTorch's unfold(321, 160) over the left-padded chunk; the integer
// division truncates toward zero, so one sample has no frame.
int audio_frame_count(int64_t samples) { return int((samples + 160 - 321) / 160 + 1); }

// AudioFrontEnd.tokenCount(frames:): two convolutions of kernel 3, stride 2, padding 1.
int audio_tokens_for_frames(int frames) {
    int n = frames;
    for (int i = 0; i < 2; i++) n = (n - 1) / 2 + 1;
    return n;
}

int64_t audio_token_count(int64_t samples) {
    int64_t total = 0;
    for (int64_t off = 0; off < samples;) {
        const int64_t n = std::min(kAudioChunkSamples, samples - off);
        total += audio_tokens_for_frames(audio_frame_count(n));
        off += n;
    }
    return total;
}

int PreparedAudio::frames() const {
    int f = 0;
    for (int64_t off = 0; off < count; off += kAudioChunkSamples)
        f += audio_frame_count(std::min(kAudioChunkSamples, count - off));
    return f;
}
int PreparedAudio::tokens() const { return int(audio_token_count(count)); }

// The tables are computed in the reference's order with separately rounded operations (this
// file is compiled without floating-point contraction), so the device front end reproduces it.
void audio_front_tables(int mel, float* hann, float* sin_t, float* cos_t, int* bitrev, std::vector<int>& band,
                        std::vector<float>& w) {
    constexpr int n = 512, win = 320, bins = n / 2 + 1;
    const float pi = 3.14159265358979323846f;
    for (int i = 0; i < n; i++) hann[i] = 0.0f;
    for (int i = 0; i < win; i++) hann[i] = 0.5f - 0.5f * cosf((2.0f * pi * float(i)) / float(win));
    for (int i = 0; i < n; i++) {
        const double a = (2.0 * 3.14159265358979323846 * double(i)) / double(n);
        sin_t[i] = sinf(float(a));
        cos_t[i] = cosf(float(a));
    }
    for (int i = 0; i < n; i++) {
        int r = 0;
        for (int b = 0; b < 9; b++)
            if (i & (1 << b)) r |= 1 << (8 - b);
        bitrev[i] = r;
    }
    // melFilterbank: HTK triangles between mel + 2 points evenly spaced in mel over 0..8 kHz,
    // sampled at the bin centres; filterBands widens each filter's nonzero bins to groups of four.
    const double bin_hz = 16000.0 / double(n);
    const double m_lo = 2595.0 * std::log10(1.0 + 0.0 / 700.0), m_hi = 2595.0 * std::log10(1.0 + 8000.0 / 700.0);
    std::vector<double> hz(size_t(mel) + 2);
    for (int i = 0; i < mel + 2; i++)
        hz[size_t(i)] = 700.0 * (std::pow(10.0, (m_lo + (m_hi - m_lo) * (double(i) / double(mel + 1))) / 2595.0) - 1.0);
    band.assign(3 * size_t(mel), 0);
    w.clear();
    std::vector<float> row(bins);
    for (int m = 0; m < mel; m++) {
        const double left = hz[size_t(m)], centre = hz[size_t(m) + 1], right = hz[size_t(m) + 2];
        const double dl = std::max(1e-30, centre - left), dr = std::max(1e-30, right - centre);
        int first = -1, last = -1;
        for (int k = 0; k < bins; k++) {
            const double f = double(k) * bin_hz;
            double v = 0.0;
            if (f >= left && f <= centre) v = (f - left) / dl;
            else if (f > centre && f <= right) v = (right - f) / dr;
            row[size_t(k)] = float(v);
            if (row[size_t(k)] != 0.0f) {
                if (first < 0) first = k;
                last = k;
            }
        }
        const int lo = first < 0 ? 0 : first / 4 * 4;
        const int hi = first < 0 ? 0 : std::min(bins, last / 4 * 4 + 4);
        band[size_t(m)] = lo;
        band[size_t(mel + m)] = hi;
        band[size_t(2 * mel + m)] = int(w.size());
        for (int k = lo; k < hi; k++) w.push_back(row[size_t(k)]);
    }
}

namespace {

// AudioConfig.init (AudioConfig.swift:50-85).
bool read_audio_config(const GgufFile& f, AudioConfig& c, LoadError& e) {
    std::string arch, proj;
    f.get_string("general.architecture", arch);
    if (arch != "clip") {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: audio encoder architecture is '" + arch + "', expected clip"};
        return false;
    }
    bool has = false;
    if (!f.get_bool("clip.has_audio_encoder", has) || !has) {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: the mmproj file has no audio encoder (clip.has_audio_encoder)"};
        return false;
    }
    f.get_string("clip.audio.projector_type", proj);
    if (proj != "gemma4a") {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: audio projector is '" + proj + "', expected gemma4a"};
        return false;
    }
    auto get = [&](const char* key, int& out) {
        int64_t v;
        if (!f.get_int(std::string("clip.audio.") + key, v)) {
            e = {GE_ERR_MISSING_METADATA, std::string("weight file lacks metadata key clip.audio.") + key};
            return false;
        }
        out = int(v);
        return true;
    };
    if (!get("embedding_length", c.hidden) || !get("attention.head_count", c.heads)) return false;
    if (c.heads <= 0 || c.hidden % c.heads) {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: audio width " + std::to_string(c.hidden) + " does not split into " +
                                      std::to_string(c.heads) + " heads"};
        return false;
    }
    if (!get("num_mel_bins", c.mel_bins)) return false;
    if (c.mel_bins % 4) {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: " + std::to_string(c.mel_bins) +
                                      " mel bins do not survive two stride-2 convolutions evenly"};
        return false;
    }
    const GgufTensor* o = f.tensor("a.pre_encode.out.weight");
    if (!o || o->shape.size() != 2 || o->shape[0] != c.hidden) {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: a.pre_encode.out.weight is missing or not [" +
                                      std::to_string(c.hidden) + ", n]"};
        return false;
    }
    c.output_width = int(o->shape[1]);
    if (!get("block_count", c.layers) || !get("feed_forward_length", c.ff) || !get("projection_dim", c.projection_dim))
        return false;
    c.head_dim = c.hidden / c.heads;
    return true;
}

// A clipped linear's tensors: `base.weight` [inputs, outputs], optional `base.bias` [outputs]
// (F32) and the four bound scalars (F32 [1]) (AudioWeights.init's linear, AudioWeights.swift:94-102).
struct ClippedHost {
    const GgufTensor* w = nullptr;
    const GgufTensor* bias = nullptr;
    float in_lo = -FLT_MAX, in_hi = FLT_MAX, out_lo = -FLT_MAX, out_hi = FLT_MAX;
};

bool clipped_host(const GgufFile& f, const std::string& base, int inputs, int outputs, ClippedHost& c, LoadError& e) {
    if (!(c.w = need_tensor(f, base + ".weight", {inputs, outputs}, false, e))) return false;
    if (f.tensor(base + ".bias") && !(c.bias = need_tensor(f, base + ".bias", {outputs}, true, e))) return false;
    const char* names[4] = {"input_min", "input_max", "output_min", "output_max"};
    float* dst[4] = {&c.in_lo, &c.in_hi, &c.out_lo, &c.out_hi};
    for (int i = 0; i < 4; i++) {
        const std::string n = base + "." + names[i];
        if (!f.tensor(n)) continue;
        const GgufTensor* t = need_tensor(f, n, {1}, true, e);
        if (!t) return false;
        memcpy(dst[i], t->data, 4);
    }
    return true;
}

std::vector<float> vec_of(const GgufTensor* t) {
    std::vector<float> v(size_t(t->elements()));
    for (int64_t r = 0; r < t->rows(); r++) dequant_row(*t, r, v.data() + r * t->cols());
    return v;
}

void free_audio_workspace(AudioWorkspace& ws) {
    for (void* p : ws.allocations) cudaFree(p);
    for (void* p : {(void*)ws.h_chunks, (void*)ws.h_cs, (void*)ws.h_pcm})
        if (p) cudaFreeHost(p);
    ws = AudioWorkspace();
}

// Grows the workspace to at least `trows` token rows (a multiple of kRowTile), `frames` log-mel
// frames, `t0` first-convolution rows, `chunks` chunks and `pcm` samples.
cudaError_t ensure_audio_workspace(const AudioConfig& c, Device& d, int trows, int frames, int t0, int chunks, size_t pcm) {
    AudioWorkspace& ws = d.aud.ws;
    if (ws.cap_trows >= trows && ws.cap_frames >= frames && ws.cap_t0 >= t0 && ws.cap_chunks >= chunks && ws.cap_pcm >= pcm)
        return cudaSuccess;
    cudaError_t e = cudaStreamSynchronize(d.stream);
    if (e != cudaSuccess) return e;
    const int R = std::max(trows, ws.cap_trows), F = std::max(frames, ws.cap_frames), T0 = std::max(t0, ws.cap_t0);
    const int C = std::max({chunks, ws.cap_chunks, 8});
    const size_t P = std::max(pcm, ws.cap_pcm);
    free_audio_workspace(ws);
    cudaError_t err = cudaSuccess;
    auto A = [&](auto** p, size_t n) {
        if (err == cudaSuccess) err = dev_alloc(ws.allocations, p, std::max<size_t>(n, 1));
    };
    const size_t r = size_t(R), dm = size_t(c.hidden);
    A(&ws.pcm, P);
    A(&ws.chunks, size_t(C));
    A(&ws.chunk_start, r);
    A(&ws.mel, size_t(F) * c.mel_bins);
    A(&ws.c0, size_t(T0) * (c.mel_bins / 2) * c.sub_channels[0]);
    A(&ws.a1, r * 32 * 9 * c.sub_channels[0]);
    A(&ws.c1, r * 32 * 128);
    A(&ws.a2, r * c.subsample_width());
    A(&ws.x, r * dm);
    A(&ws.h, r * dm);
    A(&ws.hk, r * dm);
    A(&ws.hv, r * dm);
    A(&ws.q, r * dm);
    A(&ws.k, r * dm);
    A(&ws.v, r * dm);
    A(&ws.attn, r * dm);
    A(&ws.act, r * size_t(c.ff));
    A(&ws.t, r * dm);
    A(&ws.glu, r * dm);
    A(&ws.o32, r * size_t(c.output_width));
    A(&ws.h2, r * size_t(c.output_width));
    A(&ws.vectors, r * size_t(c.projection_dim));
    if (err == cudaSuccess) err = cudaMallocHost(reinterpret_cast<void**>(&ws.h_chunks), size_t(C) * sizeof(AudioChunk));
    if (err == cudaSuccess) err = cudaMallocHost(reinterpret_cast<void**>(&ws.h_cs), r * sizeof(int));
    if (err == cudaSuccess && P > 1) err = cudaMallocHost(reinterpret_cast<void**>(&ws.h_pcm), P * sizeof(float));
    if (err != cudaSuccess) {
        free_audio_workspace(ws);
        return err;
    }
    ws.cap_trows = R;
    ws.cap_frames = F;
    ws.cap_t0 = T0;
    ws.cap_chunks = C;
    ws.cap_pcm = P;
    auto act = [&](DevActivation& a, __half* p, int nrows, int cols) {
        a.ptr = p;
        a.rows = nrows;
        a.cols = cols;
        return encode_activation_map(a);
    };
    const bool ok = act(ws.a_a1, ws.a1, R * 32, 9 * c.sub_channels[0]) && act(ws.a_a2, ws.a2, R, c.subsample_width()) &&
                    act(ws.a_h, ws.h, R, c.hidden) && act(ws.a_hk, ws.hk, R, c.hidden) && act(ws.a_hv, ws.hv, R, c.hidden) &&
                    act(ws.a_attn, ws.attn, R, c.hidden) && act(ws.a_act, ws.act, R, c.ff) &&
                    act(ws.a_h2, ws.h2, R, c.output_width);
    return ok ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

void free_audio(Device& d) {
    free_audio_workspace(d.aud.ws);
    for (void* p : d.aud.allocations) cudaFree(p);
    d.aud = AudioDev();
}

int load_audio(ge_model* m, const char* path) {
    GgufError gerr;
    if (!path) return set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: audio encoder path is NULL");
    GgufFile& f = m->audio_file;
    if (f.open(path, gerr)) return set_error(m, gerr.code, gerr.message);
    AudioConfig& c = m->acfg;
    LoadError le{0, ""};
    if (!read_audio_config(f, c, le)) return set_error(m, le.code, le.msg);
    // MetalForward.init (Metal/MetalForward.swift:90-92): the encoder projects to the text width.
    if (c.projection_dim != m->cfg.hidden)
        return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: audio encoder projects to " +
                                                     std::to_string(c.projection_dim) + " dimensions, the text model is " +
                                                     std::to_string(m->cfg.hidden) + " wide");
    // The shapes the kernels are built for (the real encoder's and BASELINE config 5's).
    auto row_width = [](int w) { return w == 512 || w == 768 || w == 1024 || w == 1536 || w == 2048; };
    if (c.mel_bins != 128 || c.head_dim != 128 || c.layers <= 0 || !row_width(c.hidden) || c.hidden % 256 ||
        c.ff % 256 || !row_width(c.output_width) || c.output_width % 256 || c.projection_dim % 256)
        return set_error(m, GE_ERR_UNSUPPORTED_ARCHITECTURE,
                         "unsupported architecture: audio encoder shape (hidden " + std::to_string(c.hidden) + ", heads " +
                             std::to_string(c.heads) + ", mel bins " + std::to_string(c.mel_bins) + ", output " +
                             std::to_string(c.output_width) + ")");
    const int d = c.hidden, ff = c.ff;
    // ---- AudioWeights.init (AudioWeights.swift:67-135)
    const GgufTensor *cw[2], *cn[2];
    for (int i = 0, in_c = 1; i < 2; i++) {
        const std::string b = "a.conv1d." + std::to_string(i);
        if (!(cw[i] = need_tensor(f, b + ".weight", {3, 3, in_c, c.sub_channels[i]}, true, le)) ||
            !(cn[i] = need_tensor(f, b + ".norm.weight", {c.sub_channels[i]}, true, le)))
            return set_error(m, le.code, le.msg);
        in_c = c.sub_channels[i];
    }
    ClippedHost in_proj, out_proj, proj;
    if (!clipped_host(f, "a.input_projection", c.subsample_width(), d, in_proj, le) ||
        !clipped_host(f, "a.pre_encode.out", d, c.output_width, out_proj, le) ||
        !clipped_host(f, "mm.a.input_projection", c.output_width, c.projection_dim, proj, le))
        return set_error(m, le.code, le.msg);
    struct LT {
        ClippedHost up, down, q, k, v, o, krel, pw1, pw2, up1, down1;
        const GgufTensor *ffn_norm, *ffn_post, *attn_pre, *attn_post, *pds, *conv_norm, *dw, *norm_conv, *ffn_norm1,
            *ffn_post1, *ln2;
    };
    std::vector<LT> lt(static_cast<size_t>(c.layers));
    for (int i = 0; i < c.layers; i++) {
        const std::string b = "a.blk." + std::to_string(i) + ".";
        LT& t = lt[size_t(i)];
        if (!(t.ffn_norm = need_tensor(f, b + "ffn_norm.weight", {d}, true, le)) ||
            !clipped_host(f, b + "ffn_up", d, ff, t.up, le) || !clipped_host(f, b + "ffn_down", ff, d, t.down, le) ||
            !(t.ffn_post = need_tensor(f, b + "ffn_post_norm.weight", {d}, true, le)) ||
            !(t.attn_pre = need_tensor(f, b + "attn_pre_norm.weight", {d}, true, le)) ||
            !clipped_host(f, b + "attn_q", d, d, t.q, le) || !clipped_host(f, b + "attn_k", d, d, t.k, le) ||
            !clipped_host(f, b + "attn_v", d, d, t.v, le) || !clipped_host(f, b + "attn_out", d, d, t.o, le) ||
            !clipped_host(f, b + "attn_k_rel", d, d, t.krel, le) ||
            !(t.pds = need_tensor(f, b + "per_dim_scale.weight", {c.head_dim}, true, le)) ||
            !(t.attn_post = need_tensor(f, b + "attn_post_norm.weight", {d}, true, le)) ||
            !(t.conv_norm = need_tensor(f, b + "conv_norm.weight", {d}, true, le)) ||
            !clipped_host(f, b + "conv_pw1", d, 2 * d, t.pw1, le) ||
            !(t.dw = need_tensor(f, b + "conv_dw.weight", {c.dw_kernel, d}, true, le)) ||
            !(t.norm_conv = need_tensor(f, b + "norm_conv.weight", {d}, true, le)) ||
            !clipped_host(f, b + "conv_pw2", d, d, t.pw2, le) ||
            !(t.ffn_norm1 = need_tensor(f, b + "ffn_norm_1.weight", {d}, true, le)) ||
            !clipped_host(f, b + "ffn_up_1", d, ff, t.up1, le) || !clipped_host(f, b + "ffn_down_1", ff, d, t.down1, le) ||
            !(t.ffn_post1 = need_tensor(f, b + "ffn_post_norm_1.weight", {d}, true, le)) ||
            !(t.ln2 = need_tensor(f, b + "ln2.weight", {d}, true, le)))
            return set_error(m, le.code, le.msg);
        // The GLU epilogue has no bias path for the interleaved halves.
        if (t.pw1.bias)
            return set_error(m, GE_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture: " + b + "conv_pw1.bias");
    }
    // SpanMarkers.audio (Model/InputRow.swift): "<|audio>" and "<audio|>" are single tokens.
    if (!m->tokenizer)
        return set_error(m, GE_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture: tokenizer model missing");
    for (int k = 0; k < 2; k++) {
        const std::string text = k == 0 ? "<|audio>" : "<audio|>";
        std::vector<int32_t> ids;
        m->tokenizer->t.encode(reinterpret_cast<const uint8_t*>(text.data()), text.size(), false, true, ids);
        if (ids.size() != 1) return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: vocabulary has no single token for " + text);
        (k == 0 ? m->audio_begin : m->audio_end) = ids[0];
    }
    // ---- host repack
    auto lin = [&](const ClippedHost& h, int N, int K) {
        return build_weight(N, K, true, [&](int r) -> std::pair<const GgufTensor*, int> { return {h.w, r}; });
    };
    // conv1: rows = output channels padded to one 128-row tile, K in tap-major order.
    HostWeight conv1;
    {
        const int taps = 9 * c.sub_channels[0], outc = c.sub_channels[1];
        conv1.N = 128;
        conv1.K = taps;
        conv1.q8 = false;
        conv1.f16.assign(size_t(conv1.N) * taps, 0);
        const float* src = reinterpret_cast<const float*>(cw[1]->data);  // [out][in][3][3]
        for (int o = 0; o < outc; o++)
            for (int ch = 0; ch < c.sub_channels[0]; ch++)
                for (int tap = 0; tap < 9; tap++)
                    conv1.f16[size_t(o) * taps + size_t(tap) * c.sub_channels[0] + ch] =
                        float_to_half_bits(src[size_t(o) * taps + size_t(ch) * 9 + tap]);
    }
    std::vector<HostWeight> hw;
    hw.push_back(lin(in_proj, d, c.subsample_width()));
    hw.push_back(lin(out_proj, c.output_width, d));
    hw.push_back(lin(proj, c.projection_dim, c.output_width));
    // The sinusoid of each relative distance (CPUAudioReference.sinusoid, CPUAudioReference.swift:105-115).
    std::vector<float> table(size_t(c.relative_positions) * d);
    {
        const int ts = d / 2;
        const float inc = logf(10000.0f) / float(std::max(ts - 1, 1));
        for (int p = 0; p < c.relative_positions; p++)
            for (int i = 0; i < ts; i++) {
                const float scaled = float(p) * expf(-float(i) * inc);
                table[size_t(p) * d + i] = sinf(scaled);
                table[size_t(p) * d + i + ts] = cosf(scaled);
            }
    }
    std::vector<std::vector<float>> rels, norms;
    for (const LT& t : lt) {
        hw.push_back(lin(t.up, ff, d));
        hw.push_back(lin(t.down, d, ff));
        hw.push_back(lin(t.q, d, d));
        hw.push_back(lin(t.k, d, d));
        hw.push_back(lin(t.v, d, d));
        hw.push_back(lin(t.o, d, d));
        // conv_pw1 for the GLU epilogue: sigmoid rows (d..2d) and value rows (0..d) interleaved in
        // blocks of kBN / 2, the sigmoid half first.
        hw.push_back(build_weight(2 * d, d, true, [&](int r) -> std::pair<const GgufTensor*, int> {
            const int blk = r / (kBN / 2), off = r % (kBN / 2);
            return {t.pw1.w, (blk & 1) ? (blk >> 1) * (kBN / 2) + off : d + (blk >> 1) * (kBN / 2) + off};
        }));
        hw.push_back(lin(t.pw2, d, d));
        hw.push_back(lin(t.up1, ff, d));
        hw.push_back(lin(t.down1, d, ff));
        // Relative keys: the clipped k_rel linear over the sinusoid table, in fp32 on the host.
        std::vector<float> wk = dequant_matrix(*t.krel.w);  // [d][d]
        std::vector<float> in(table);
        for (float& v : in) v = std::min(std::max(v, t.krel.in_lo), t.krel.in_hi);
        std::vector<float> rel(size_t(c.relative_positions) * d);
        const float* kb = t.krel.bias ? reinterpret_cast<const float*>(t.krel.bias->data) : nullptr;
        parallel_rows(d, [&](int64_t n) {
            for (int p = 0; p < c.relative_positions; p++) {
                float s = 0.f;
                for (int k = 0; k < d; k++) s += in[size_t(p) * d + k] * wk[size_t(n) * d + k];
                s = std::min(std::max(s, t.krel.out_lo), t.krel.out_hi);
                rel[size_t(p) * d + n] = s + (kb ? kb[n] : 0.f);
            }
        });
        rels.push_back(std::move(rel));
        std::vector<float> pds = vec_of(t.pds), qs(size_t(c.head_dim));
        for (int i = 0; i < c.head_dim; i++) qs[size_t(i)] = c.query_scale() * pds[size_t(i)];
        std::vector<float> fpost = vec_of(t.ffn_post), fpost1 = vec_of(t.ffn_post1);
        for (float& v : fpost) v *= c.ff_residual;
        for (float& v : fpost1) v *= c.ff_residual;
        std::vector<float> dw = vec_of(t.dw), dwt(dw.size());  // [d][5] -> [5][d]
        for (int ch = 0; ch < d; ch++)
            for (int k = 0; k < c.dw_kernel; k++) dwt[size_t(k) * d + ch] = dw[size_t(ch) * c.dw_kernel + k];
        for (auto* v : {&fpost, &fpost1, &dwt, &qs}) norms.push_back(*v);
        for (const GgufTensor* n : {t.ffn_norm, t.attn_pre, t.attn_post, t.conv_norm, t.norm_conv, t.ffn_norm1, t.ln2})
            norms.push_back(vec_of(n));
    }
    float hann[512], sin_t[512], cos_t[512];
    int bitrev[512];
    std::vector<int> band;
    std::vector<float> melw;
    audio_front_tables(c.mel_bins, hann, sin_t, cos_t, bitrev, band, melw);
    std::vector<float> c0w = vec_of(cw[0]), c0n = vec_of(cn[0]), c1n = vec_of(cn[1]);
    // ---- upload to every device
    for (Device& dv : m->devs) {
        cudaError_t e = cudaSetDevice(dv.ordinal);
        AudioDev& a = dv.aud;
        std::vector<void*>& own = a.allocations;
        auto up_lin = [&](ClippedDev& cd, const ClippedHost& h, const HostWeight& w) {
            cudaError_t x = upload_weight(own, cd.w, w);
            if (x == cudaSuccess && h.bias)
                x = dev_upload(own, &cd.bias, reinterpret_cast<const float*>(h.bias->data), size_t(h.bias->elements()));
            cd.in_lo = h.in_lo;
            cd.in_hi = h.in_hi;
            cd.out_lo = h.out_lo;
            cd.out_hi = h.out_hi;
            return x;
        };
        size_t wi = 0;
        if (e == cudaSuccess) e = dev_upload(own, &a.conv0_w, c0w.data(), c0w.size());
        if (e == cudaSuccess) e = dev_upload(own, &a.conv0_n, c0n.data(), c0n.size());
        if (e == cudaSuccess) e = dev_upload(own, &a.conv1_n, c1n.data(), c1n.size());
        if (e == cudaSuccess) e = upload_weight(own, a.conv1, conv1);
        if (e == cudaSuccess) e = up_lin(a.in_proj, in_proj, hw[wi++]);
        if (e == cudaSuccess) e = up_lin(a.out_proj, out_proj, hw[wi++]);
        if (e == cudaSuccess) e = up_lin(a.proj, proj, hw[wi++]);
        a.layers.resize(size_t(c.layers));
        for (int l = 0; l < c.layers && e == cudaSuccess; l++) {
            AudioLayerDev& L = a.layers[size_t(l)];
            const LT& t = lt[size_t(l)];
            const ClippedHost* hs[10] = {&t.up, &t.down, &t.q, &t.k, &t.v, &t.o, &t.pw1, &t.pw2, &t.up1, &t.down1};
            ClippedDev* ds[10] = {&L.up, &L.down, &L.q, &L.k, &L.v, &L.o, &L.pw1, &L.pw2, &L.up1, &L.down1};
            for (int k = 0; k < 10 && e == cudaSuccess; k++) e = up_lin(*ds[k], *hs[k], hw[wi++]);
            const std::vector<float>& rel = rels[size_t(l)];
            if (e == cudaSuccess) e = dev_upload(own, &L.rel, rel.data(), rel.size());
            float** dst[11] = {&L.ffn_post_half, &L.ffn_post1_half, &L.dw_t, &L.qscale, &L.ffn_norm, &L.attn_pre,
                               &L.attn_post, &L.conv_norm, &L.norm_conv, &L.ffn_norm1, &L.ln2};
            for (int k = 0; k < 11 && e == cudaSuccess; k++) {
                const std::vector<float>& src = norms[size_t(l) * 11 + k];
                e = dev_upload(own, dst[k], src.data(), src.size());
            }
        }
        if (e == cudaSuccess) e = dev_upload(own, &a.hann, hann, 512);
        if (e == cudaSuccess) e = dev_upload(own, &a.cos_t, cos_t, 512);
        if (e == cudaSuccess) e = dev_upload(own, &a.sin_t, sin_t, 512);
        if (e == cudaSuccess) e = dev_upload(own, &a.bitrev, bitrev, 512);
        if (e == cudaSuccess) e = dev_upload(own, &a.band, band.data(), band.size());
        if (e == cudaSuccess) e = dev_upload(own, &a.mel_w, melw.data(), melw.size());
        a.mel_nw = int(melw.size());
        if (e != cudaSuccess)
            return set_error(m, e == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                             std::string("GPU execution failed: audio encoder upload: ") + cudaGetErrorString(e));
        a.loaded = true;
    }
    m->has_audio = true;
    return GE_OK;
}

int run_audio(ge_model* m, Device& d, const AudioArgs& a) {
    const AudioConfig& c = m->acfg;
    auto report = [&](int code, const std::string& msg) {
        if (a.error) *a.error = msg;
        else m->last_error = msg;
        return code;
    };
    auto gpu_fail = [&](cudaError_t x, const char* what) {
        return report(x == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                      std::string("GPU execution failed: ") + what + ": " + cudaGetErrorString(x));
    };
    cudaError_t e = cudaSetDevice(d.ordinal);
    if (e != cudaSuccess) return gpu_fail(e, "cudaSetDevice");
    if (!d.aud.loaded)
        return report(GE_ERR_AUDIO_ENCODER_NOT_LOADED, "no audio encoder is loaded; pass the mmproj GGUF when loading the model");
    struct LaunchPolicy {
        explicit LaunchPolicy(bool on) { set_programmatic_launch(on); }
        ~LaunchPolicy() { set_programmatic_launch(false); }
    } policy(!(m->flags & GE_LOAD_NO_PDL));
    // ---- batch layout (AudioBatch, Metal/AudioTower.swift): chunks in clip order, each chunk's
    // frames, first-convolution rows and token rows back to back.
    std::vector<AudioChunk> chunks;
    int64_t pcm = 0;
    int frames = 0, t0 = 0, tokens = 0;
    for (int i = 0; i < a.n; i++) {
        const PreparedAudio& p = *a.clips[i];
        if (p.count < kAudioMinimumSamples)
            return report(GE_ERR_AUDIO_DECODING, "cannot decode audio: clip " + std::to_string(i) + " has " +
                                                     std::to_string(p.count) + " samples at 16 kHz; at least 2 are needed for one frame");
        if (p.count % kAudioChunkSamples == 1)
            return report(GE_ERR_AUDIO_DECODING, "cannot decode audio: clip " + std::to_string(i) +
                                                     ": its last 30-second chunk has 1 sample");
        const int64_t base = a.d_pcm ? p.device_offset : pcm;
        for (int64_t off = 0; off < p.count; off += kAudioChunkSamples) {
            AudioChunk ch{};
            ch.pcm_offset = base + off;
            ch.samples = int(std::min(kAudioChunkSamples, p.count - off));
            ch.frames = audio_frame_count(ch.samples);
            ch.mel_row = frames;
            ch.t0 = (ch.frames - 1) / 2 + 1;
            ch.t0_row = t0;
            ch.tokens = audio_tokens_for_frames(ch.frames);
            ch.token_row = tokens;
            frames += ch.frames;
            t0 += ch.t0;
            tokens += ch.tokens;
            chunks.push_back(ch);
        }
        pcm += p.count;
    }
    const int nch = int(chunks.size());
    const int trows = std::max(kRowTile, round_up(tokens, kRowTile));
    if ((e = staging_wait(d, kStageAudio)) != cudaSuccess) return gpu_fail(e, "staging");
    if ((e = ensure_audio_workspace(c, d, trows, frames, t0, nch, a.d_pcm ? 0 : size_t(pcm))) != cudaSuccess)
        return gpu_fail(e, "workspace");
    AudioWorkspace& ws = d.aud.ws;
    memcpy(ws.h_chunks, chunks.data(), size_t(nch) * sizeof(AudioChunk));
    for (const AudioChunk& ch : chunks)
        for (int r = 0; r < ch.tokens; r++) ws.h_cs[ch.token_row + r] = ch.token_row;
    for (int r = tokens; r < trows; r++) ws.h_cs[r] = r;
    cudaStream_t st = a.stream ? a.stream : d.stream;
    if (!a.d_pcm) {
        // The clips are gathered into pinned memory on several host threads, then copied to the
        // device in one transfer.
        std::vector<int64_t> start(size_t(a.n) + 1, 0);
        for (int i = 0; i < a.n; i++) start[size_t(i) + 1] = start[size_t(i)] + a.clips[i]->count;
        const int64_t per = std::max<int64_t>(int64_t(1) << 18, (pcm + 7) / 8);
        const int nt = int(std::min<int64_t>(8, (pcm + per - 1) / per));
        auto gather = [&](int ti) {
            const int64_t b = int64_t(ti) * per, end = std::min(pcm, b + per);
            for (int i = 0; i < a.n; i++) {
                const int64_t lo = std::max(b, start[size_t(i)]), hi = std::min(end, start[size_t(i) + 1]);
                if (lo < hi)
                    memcpy(ws.h_pcm + lo, a.clips[i]->samples + (lo - start[size_t(i)]), size_t(hi - lo) * sizeof(float));
            }
        };
        std::vector<std::thread> th;
        for (int ti = 1; ti < nt; ti++) th.emplace_back(gather, ti);
        gather(0);
        for (auto& x : th) x.join();
        e = cudaMemcpyAsync(ws.pcm, ws.h_pcm, size_t(pcm) * 4, cudaMemcpyHostToDevice, st);
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(ws.chunks, ws.h_chunks, size_t(nch) * sizeof(AudioChunk), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ws.chunk_start, ws.h_cs, size_t(trows) * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = staging_done(d, kStageAudio, st);
    if (e != cudaSuccess) return gpu_fail(e, "audio upload");
    m->h2d_bytes += int64_t((a.d_pcm ? 0 : pcm * 4) + int64_t(nch) * int64_t(sizeof(AudioChunk)) + int64_t(trows) * 4);
    const float* src = a.d_pcm ? a.d_pcm : ws.pcm;
    // ---- AudioTower.encode
    const AudioDev& A = d.aud;
    const int D = c.hidden;
    int64_t launches = 0;
    auto K = [&](const char* name, double flops, double bytes, auto&& fn) -> cudaError_t {
        if (a.profile) {
            ProfileEntry* pe = a.profile->find(name);
            if (pe) {
                pe->occurrences++;
            } else {
                cudaEvent_t e0, e1;
                cudaEventCreate(&e0);
                cudaEventCreate(&e1);
                cudaEventRecord(e0, st);
                for (int r = 0; r < a.profile->reps; r++) {
                    const cudaError_t x = fn();
                    if (x != cudaSuccess) return x;
                    launches++;
                }
                cudaEventRecord(e1, st);
                const cudaError_t x = cudaEventSynchronize(e1);
                float ms = 0.f;
                cudaEventElapsedTime(&ms, e0, e1);
                cudaEventDestroy(e0);
                cudaEventDestroy(e1);
                if (x != cudaSuccess) return x;
                a.profile->add(name, double(ms) / a.profile->reps, flops, bytes);
                return cudaSuccess;
            }
        }
        launches++;
        return fn();
    };
    auto gemm = [&](const DevActivation& X, const DevWeight& W, void* out, int ldo, int epi, float lo, float hi,
                    const float* bias = nullptr, float alo = -FLT_MAX, float ahi = FLT_MAX, int mode = GEMM_AUTO,
                    int m_rows = 0) {
        GemmLaunch g;
        g.a = &X;
        g.w = &W;
        g.m_rows = m_rows ? m_rows : trows;
        g.out = out;
        g.ldo = ldo;
        g.epilogue = epi;
        g.err = d.err;
        g.num_sms = d.num_sms;
        g.mode = mode;
        g.clamp_lo = lo;
        g.clamp_hi = hi;
        g.act_lo = alo;
        g.act_hi = ahi;
        g.bias = bias;
        return launch_gemm(g, st);
    };
    const double T = tokens;
    auto gf = [&](const DevWeight& W, double nrows) { return 2.0 * nrows * W.N * double(W.K); };
    auto gbytes = [&](const DevWeight& W, double nrows, double out_cols, double out_bytes) {
        return nrows * W.K * 2 + double(W.N) * W.K * 2 + nrows * out_cols * out_bytes;
    };
#define AK(name, flops, bytes, expr, what)                                             \
    do {                                                                               \
        cudaError_t e_ = K(name, flops, bytes, [&] { return (expr); });                \
        if (e_ != cudaSuccess) return gpu_fail(e_, what);                              \
    } while (0)
    MelTables mt;
    mt.hann = A.hann;
    mt.cos_t = A.cos_t;
    mt.sin_t = A.sin_t;
    mt.w = A.mel_w;
    mt.bitrev = A.bitrev;
    mt.band = A.band;
    mt.nw = A.mel_nw;
    mt.mel = c.mel_bins;
    AK("log_mel", 0, double(pcm) * 4 + double(frames) * c.mel_bins * 4,
       launch_log_mel(src, ws.chunks, nch, frames, mt, ws.mel, d.num_sms, st), "log-mel");
    AK("conv0", 2.0 * t0 * 64 * 128 * 9, double(frames) * c.mel_bins * 4 + double(t0) * 64 * 128 * 2,
       launch_audio_conv0(ws.mel, ws.chunks, nch, t0, A.conv0_w, A.conv0_n, c.eps, ws.c0, st), "first convolution");
    AK("im2col", 0, double(t0) * 64 * 128 * 2 + double(trows) * 32 * 1152 * 2,
       launch_audio_im2col(ws.c0, ws.chunks, nch, tokens, trows, ws.a1, st), "second convolution patches");
    AK("gemm_conv1", 2.0 * T * 32 * 32 * 1152, gbytes(A.conv1, T * 32, 128, 4),
       gemm(ws.a_a1, A.conv1, ws.c1, 128, EPI_F32, 0, 0, nullptr, -FLT_MAX, FLT_MAX, GEMM_NARROW, trows * 32),
       "second convolution");
    AK("subsample_norm", 0, T * 32 * 128 * 4 + T * c.subsample_width() * 2,
       launch_audio_subsample_norm(ws.c1, trows, A.conv1_n, c.eps, A.in_proj.in_lo, A.in_proj.in_hi, ws.a2, st),
       "subsampling norm");
    AK("gemm_in", gf(A.in_proj.w, T), gbytes(A.in_proj.w, T, D, 4),
       gemm(ws.a_a2, A.in_proj.w, ws.x, D, EPI_CLAMP_F32, A.in_proj.out_lo, A.in_proj.out_hi, A.in_proj.bias),
       "input projection");
    const double rb = T * D * 4 * 2 + T * D * 2;  // a row step: x read and written, one fp16 output
    {
        AudioRowStep s;
        s.x = ws.x;
        s.rows = trows;
        s.eps = c.eps;
        s.next_norm = 1;
        s.next_w = A.layers[0].ffn_norm;
        s.nout = 1;
        s.out[0] = ws.h;
        s.lo[0] = A.layers[0].up.in_lo;
        s.hi[0] = A.layers[0].up.in_hi;
        AK("rows", 0, rb, launch_audio_rows(s, D, st), "first norm");
    }
    double att_flops = 0;
    for (const AudioChunk& ch : chunks) {
        const double n = ch.tokens, w = c.window;
        att_flops += 2.0 * 3.0 * D * (n * w - w * (w - 1) / 2);  // content + relative scores and PV
    }
    for (int l = 0; l < c.layers; l++) {
        const AudioLayerDev& L = A.layers[size_t(l)];
        // feed-forward 1 (half step)
        AK("gemm_ffn_up", gf(L.up.w, T), gbytes(L.up.w, T, c.ff, 2),
           gemm(ws.a_h, L.up.w, ws.act, c.ff, EPI_CLAMP_SILU, L.up.out_lo, L.up.out_hi, L.up.bias, L.down.in_lo, L.down.in_hi),
           "ffn up");
        AK("gemm_ffn_down", gf(L.down.w, T), gbytes(L.down.w, T, D, 2),
           gemm(ws.a_act, L.down.w, ws.t, D, EPI_CLAMP_F16, L.down.out_lo, L.down.out_hi, L.down.bias), "ffn down");
        {
            AudioRowStep s;
            s.x = ws.x;
            s.rows = trows;
            s.eps = c.eps;
            s.branch = ws.t;
            s.branch_w = L.ffn_post_half;
            s.store_x = 1;
            s.next_norm = 1;
            s.next_w = L.attn_pre;
            s.nout = 3;
            __half* outs[3] = {ws.h, ws.hk, ws.hv};
            const ClippedDev* lins[3] = {&L.q, &L.k, &L.v};
            for (int i = 0; i < 3; i++) {
                s.out[i] = outs[i];
                s.lo[i] = lins[i]->in_lo;
                s.hi[i] = lins[i]->in_hi;
            }
            AK("rows", 0, rb + T * D * 2 * 3, launch_audio_rows(s, D, st), "ffn residual");
        }
        // attention
        AK("gemm_q", gf(L.q.w, T), gbytes(L.q.w, T, D, 2),
           gemm(ws.a_h, L.q.w, ws.q, D, EPI_CLAMP_F16, L.q.out_lo, L.q.out_hi, L.q.bias), "q projection");
        AK("gemm_k", gf(L.k.w, T), gbytes(L.k.w, T, D, 2),
           gemm(ws.a_hk, L.k.w, ws.k, D, EPI_CLAMP_F16, L.k.out_lo, L.k.out_hi, L.k.bias), "k projection");
        AK("gemm_v", gf(L.v.w, T), gbytes(L.v.w, T, D, 2),
           gemm(ws.a_hv, L.v.w, ws.v, D, EPI_CLAMP_F16, L.v.out_lo, L.v.out_hi, L.v.bias), "v projection");
        {
            AudioAttnLaunch at;
            at.q = ws.q;
            at.k = ws.k;
            at.v = ws.v;
            at.rel = L.rel;
            at.qscale = L.qscale;
            at.kscale = c.key_scale();
            at.softcap = c.softcap;
            at.lo = L.o.in_lo;
            at.hi = L.o.in_hi;
            at.chunk_start = ws.chunk_start;
            at.rows = trows;
            at.heads = c.heads;
            at.head_dim = c.head_dim;
            at.out = ws.attn;
            AK("attention", att_flops, T * D * 2 * 4, launch_audio_attention(at, st), "attention");
        }
        AK("gemm_o", gf(L.o.w, T), gbytes(L.o.w, T, D, 2),
           gemm(ws.a_attn, L.o.w, ws.t, D, EPI_CLAMP_F16, L.o.out_lo, L.o.out_hi, L.o.bias), "attention output");
        {
            AudioRowStep s;
            s.x = ws.x;
            s.rows = trows;
            s.eps = c.eps;
            s.branch = ws.t;
            s.branch_w = L.attn_post;
            s.store_x = 1;
            s.next_norm = 1;
            s.next_w = L.conv_norm;
            s.nout = 1;
            s.out[0] = ws.h;
            s.lo[0] = L.pw1.in_lo;
            s.hi[0] = L.pw1.in_hi;
            AK("rows", 0, rb + T * D * 2, launch_audio_rows(s, D, st), "attention residual");
        }
        // convolution module
        AK("gemm_pw1_glu", gf(L.pw1.w, T), gbytes(L.pw1.w, T, D, 2),
           gemm(ws.a_h, L.pw1.w, ws.glu, D, EPI_GLU, L.pw1.out_lo, L.pw1.out_hi), "pointwise 1 and GLU");
        AK("dwconv", 2.0 * T * D * c.dw_kernel, T * D * 2 * 2,
           launch_audio_dwconv(ws.glu, ws.chunk_start, trows, D, L.dw_t, L.norm_conv, c.eps, L.pw2.in_lo, L.pw2.in_hi,
                               ws.attn, st),
           "depthwise convolution");
        AK("gemm_pw2", gf(L.pw2.w, T), gbytes(L.pw2.w, T, D, 2),
           gemm(ws.a_attn, L.pw2.w, ws.t, D, EPI_CLAMP_F16, L.pw2.out_lo, L.pw2.out_hi, L.pw2.bias), "pointwise 2");
        {
            AudioRowStep s;
            s.x = ws.x;
            s.rows = trows;
            s.eps = c.eps;
            s.branch = ws.t;
            s.store_x = 1;
            s.next_norm = 1;
            s.next_w = L.ffn_norm1;
            s.nout = 1;
            s.out[0] = ws.h;
            s.lo[0] = L.up1.in_lo;
            s.hi[0] = L.up1.in_hi;
            AK("rows", 0, rb + T * D * 2, launch_audio_rows(s, D, st), "convolution residual");
        }
        // feed-forward 2 (half step), then the layer's output norm
        AK("gemm_ffn_up", gf(L.up1.w, T), gbytes(L.up1.w, T, c.ff, 2),
           gemm(ws.a_h, L.up1.w, ws.act, c.ff, EPI_CLAMP_SILU, L.up1.out_lo, L.up1.out_hi, L.up1.bias, L.down1.in_lo,
                L.down1.in_hi),
           "ffn up 1");
        AK("gemm_ffn_down", gf(L.down1.w, T), gbytes(L.down1.w, T, D, 2),
           gemm(ws.a_act, L.down1.w, ws.t, D, EPI_CLAMP_F16, L.down1.out_lo, L.down1.out_hi, L.down1.bias), "ffn down 1");
        {
            const bool last = l + 1 == c.layers;
            AudioRowStep s;
            s.x = ws.x;
            s.rows = trows;
            s.eps = c.eps;
            s.branch = ws.t;
            s.branch_w = L.ffn_post1_half;
            s.final_w = L.ln2;
            s.store_x = 1;
            s.next_norm = last ? 0 : 1;
            s.next_w = last ? nullptr : A.layers[size_t(l) + 1].ffn_norm;
            s.nout = 1;
            s.out[0] = ws.h;
            s.lo[0] = last ? A.out_proj.in_lo : A.layers[size_t(l) + 1].up.in_lo;
            s.hi[0] = last ? A.out_proj.in_hi : A.layers[size_t(l) + 1].up.in_hi;
            AK("rows", 0, rb + T * D * 2, launch_audio_rows(s, D, st), "layer output");
        }
    }
    // Output projection, its weightless RMS norm, and the multimodal projection.
    const int OW = c.output_width;
    AK("gemm_out", gf(A.out_proj.w, T), gbytes(A.out_proj.w, T, OW, 4),
       gemm(ws.a_h, A.out_proj.w, ws.o32, OW, EPI_CLAMP_F32, A.out_proj.out_lo, A.out_proj.out_hi, A.out_proj.bias),
       "output projection");
    {
        AudioRowStep s;
        s.x = ws.o32;
        s.rows = trows;
        s.eps = c.eps;
        s.next_norm = 1;
        s.nout = 1;
        s.out[0] = ws.h2;
        s.lo[0] = A.proj.in_lo;
        s.hi[0] = A.proj.in_hi;
        AK("rows", 0, T * OW * 4 + T * OW * 2, launch_audio_rows(s, OW, st), "output norm");
    }
    AK("gemm_projection", gf(A.proj.w, T), gbytes(A.proj.w, T, c.projection_dim, 4),
       gemm(ws.a_h2, A.proj.w, ws.vectors, c.projection_dim, EPI_CLAMP_F32, A.proj.out_lo, A.proj.out_hi, A.proj.bias),
       "multimodal projection");
#undef AK
    m->launches += launches;
    return GE_OK;
}

}  // namespace ge
