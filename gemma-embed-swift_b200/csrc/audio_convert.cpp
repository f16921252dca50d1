// audio_convert.cpp -- the conversion of decoded PCM to the 16 kHz mono samples the audio
// encoder reads: miniaudio 0.11.25's `ma_data_converter` path for f32 input as llama.cpp's
// decoder runs it (Sources/GemmaEmbed/Audio/MiniaudioConverter.swift): channels averaged in
// order, then `ma_linear_resampler` (fixed-point time over the gcd-reduced rates, linear
// interpolation, a 4th-order Butterworth low-pass as two transposed direct-form-2 biquads with
// coefficients in double and samples in float), and the output length of
// `ma_calculate_frame_count_after_resampling`, zero-filled where the resampler runs dry.
//
// This file is compiled without floating-point contraction; the biquad's fused multiply-adds
// are written out with fmaf where the reference's build fuses them.
#include "audio_convert.hpp"

#include <math.h>

#include <algorithm>

namespace ge {

namespace {

uint32_t gcd_u32(uint32_t a, uint32_t b) {
    while (b != 0) {
        const uint32_t t = a;
        a = b;
        b = t % a;
    }
    return a;
}

// miniaudio's cosine: sin(pi / 2 - x), which differs from cos in the last bit.
double cosd(double x) { return sin((M_PI * 0.5) - x); }

struct Biquad {
    float b0, b1, b2, a1, a2;
    float r1 = 0.f, r2 = 0.f;
    // The low-pass biquad configuration, normalised by a0 (coefficients in double, stored as float).
    Biquad(uint32_t rate, double cutoff, double q) {
        const double w = 2 * M_PI * cutoff / double(rate);
        const double s = sin(w), c = cosd(w);
        const double a = s / (2 * q);
        const double a0 = 1 + a;
        b0 = float(((1 - c) / 2) / a0);
        b1 = float((1 - c) / a0);
        b2 = float(((1 - c) / 2) / a0);
        a1 = float((-2 * c) / a0);
        a2 = float((1 - a) / a0);
    }
    // Transposed direct form 2: y = b0 x + r1 (one fma); r1 = (b1 x - a1 y) + r2 with the first
    // product fused into the subtraction of the separately rounded second; r2 likewise.
    float process(float x) {
        const float y = fmaf(b0, x, r1);
        r1 = fmaf(b1, x, -(a1 * y)) + r2;
        r2 = fmaf(b2, x, -(a2 * y));
        return y;
    }
};

struct LowPass {
    Biquad s0, s1;  // order 4: two second-order sections, q = 1 / (2 cos((2k + 1) pi / 8))
    LowPass(uint32_t rate, double cutoff)
        : s0(rate, cutoff, 1 / (2 * cosd(1 * (M_PI / 8)))), s1(rate, cutoff, 1 / (2 * cosd(3 * (M_PI / 8)))) {}
    float process(float x) { return s1.process(s0.process(x)); }
};

}  // namespace

uint64_t audio_frames_after_resampling(uint32_t rate_out, uint32_t rate_in, uint64_t frames_in) {
    if (rate_in == 0 || rate_out == 0 || frames_in == 0) return 0;
    if (rate_out == rate_in) return frames_in;
    const uint64_t ri = rate_in, ro = rate_out;
    uint64_t out = (frames_in * ro) / ri;
    const uint64_t from_frac = (out * (ri / ro)) / ro;
    const uint64_t preliminary = out * (ri % ro) + from_frac;
    if (preliminary <= frames_in) out += 1;
    return out;
}

void audio_downmix(const float* samples, int64_t frames, int channels, float* out) {
    const float div = float(channels);
    for (int64_t f = 0; f < frames; f++) {
        float t = 0.f;
        for (int c = 0; c < channels; c++) t += samples[f * channels + c];
        out[f] = t / div;
    }
}

void audio_to_mono_16k(const float* samples, int64_t frames, int channels, int rate, std::vector<float>& out) {
    std::vector<float> mono;
    const float* m = samples;
    if (channels != 1) {
        mono.resize(size_t(frames));
        audio_downmix(samples, frames, channels, mono.data());
        m = mono.data();
    }
    const uint32_t rin = uint32_t(rate), rout = 16000;
    if (rin == rout) {
        out.assign(m, m + frames);
        return;
    }
    const uint32_t g = gcd_u32(rin, rout);
    const uint32_t in_rate = rin / g, out_rate = rout / g;
    const uint32_t adv_int = in_rate / out_rate, adv_frac = in_rate % out_rate;
    LowPass lpf(std::max(in_rate, out_rate), double(std::min(in_rate, out_rate)) * 0.5 * 1.0);
    const bool down = in_rate > out_rate;
    const uint64_t length = audio_frames_after_resampling(rout, rin, uint64_t(frames));
    out.clear();
    out.reserve(size_t(length));
    uint32_t t_int = 1, t_frac = 0;
    float x0 = 0.f, x1 = 0.f;
    int64_t next = 0;
    while (out.size() < length) {
        while (t_int > 0 && next < frames) {
            x0 = x1;
            x1 = m[next];
            if (down) x1 = lpf.process(x1);
            next++;
            t_int--;
        }
        if (t_int > 0) break;
        // ma_linear_resampler_interpolate_frame_f32: three separately rounded operations.
        const float a = float(t_frac) / float(out_rate);
        float y = x0 + (x1 - x0) * a;
        if (!down) y = lpf.process(y);
        out.push_back(y);
        t_int += adv_int;
        t_frac += adv_frac;
        if (t_frac >= out_rate) {
            t_frac -= out_rate;
            t_int++;
        }
    }
    out.resize(size_t(length), 0.f);
}

}  // namespace ge
