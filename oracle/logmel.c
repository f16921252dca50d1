/*
 * logmel.c -- CPU restatement of the reference's audio front end (AudioFrontEnd,
 * Sources/GemmaEmbed/Audio/AudioPreprocessor.swift:24-251).
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker for the CUDA front end.  It also restates
 * the conversion of decoded PCM to 16 kHz mono (MiniaudioConverter, Audio/MiniaudioConverter.swift:
 * miniaudio 0.11.25's channel average, linear resampler and 4th-order Butterworth low-pass).
 * This file is compiled with -ffp-contract=off: the reference's butterflies and
 * four-bin mel sums are separate fp32 multiplies and adds in a fixed order, and a
 * fused multiply-add would change their rounding.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

enum { FFT = 512, WIN = 320, HOP = 160, BINS = FFT / 2 + 1, CHUNK = 30 * 16000 };

/* AudioFrontEnd.frameCount (AudioPreprocessor.swift:74-76); C division truncates toward zero like Swift's. */
int32_t or_audio_frame_count(int64_t samples) { return (int32_t)((samples + HOP - (WIN + 1)) / HOP + 1); }

/* AudioFrontEnd.tokenCount(frames:) (AudioPreprocessor.swift:79-83). */
int32_t or_audio_tokens_for_frames(int32_t frames) {
    int32_t n = frames;
    for (int i = 0; i < 2; i++) n = (n - 1) / 2 + 1;
    return n;
}

/* AudioFrontEnd.tokenCount(samples:) (AudioPreprocessor.swift:86-95). */
int64_t or_audio_token_count(int64_t samples) {
    int64_t total = 0;
    for (int64_t off = 0; off < samples;) {
        const int64_t n = samples - off < CHUNK ? samples - off : CHUNK;
        total += or_audio_tokens_for_frames(or_audio_frame_count(n));
        off += n;
    }
    return total;
}

/* AudioFrontEnd.init's tables (AudioPreprocessor.swift:52-65) and melFilterbank (100-123). */
void or_audio_tables(int32_t mel_bins, float* hann, float* sin_t, float* cos_t, float* filters, int32_t* band_lo,
                     int32_t* band_hi, int32_t* bitrev) {
    const float pi = 3.14159265358979323846f;
    for (int i = 0; i < FFT; i++) hann[i] = 0.0f;
    for (int i = 0; i < WIN; i++) hann[i] = 0.5f - 0.5f * cosf((2.0f * pi * (float)i) / (float)WIN);
    for (int i = 0; i < FFT; i++) {
        const double a = (2.0 * 3.14159265358979323846 * (double)i) / (double)FFT;
        sin_t[i] = sinf((float)a);
        cos_t[i] = cosf((float)a);
    }
    const double bin_hz = 16000.0 / (double)FFT;
    const double m_lo = 2595.0 * log10(1.0 + 0.0 / 700.0), m_hi = 2595.0 * log10(1.0 + 8000.0 / 700.0);
    double* hz = (double*)malloc(sizeof(double) * (size_t)(mel_bins + 2));
    for (int i = 0; i < mel_bins + 2; i++)
        hz[i] = 700.0 * (pow(10.0, (m_lo + (m_hi - m_lo) * ((double)i / (double)(mel_bins + 1))) / 2595.0) - 1.0);
    for (int m = 0; m < mel_bins; m++) {
        const double left = hz[m], centre = hz[m + 1], right = hz[m + 2];
        const double dl = centre - left > 1e-30 ? centre - left : 1e-30;
        const double dr = right - centre > 1e-30 ? right - centre : 1e-30;
        int first = -1, last = -1;
        for (int k = 0; k < BINS; k++) {
            const double f = (double)k * bin_hz;
            double w = 0.0;
            if (f >= left && f <= centre) w = (f - left) / dl;
            else if (f > centre && f <= right) w = (right - f) / dr;
            filters[(int64_t)m * BINS + k] = (float)w;
            if ((float)w != 0.0f) {
                if (first < 0) first = k;
                last = k;
            }
        }
        /* filterBands (AudioPreprocessor.swift:208-217): whole groups of four. */
        if (first < 0) {
            band_lo[m] = band_hi[m] = 0;
        } else {
            band_lo[m] = first / 4 * 4;
            band_hi[m] = last / 4 * 4 + 4 < BINS ? last / 4 * 4 + 4 : BINS;
        }
    }
    free(hz);
    for (int i = 0; i < FFT; i++) {
        int r = 0;
        for (int b = 0; b < 9; b++)
            if (i & (1 << b)) r |= 1 << (8 - b);
        bitrev[i] = r;
    }
}

/* AudioFrontEnd.fft (AudioPreprocessor.swift:223-249): bit-reversed copy, then one in-place
 * radix-2 pass per level with llama.cpp's twiddles, in its order. */
static void fft(const float* x, float* out, const float* sin_t, const float* cos_t, const int32_t* bitrev) {
    for (int i = 0; i < FFT; i++) {
        out[2 * bitrev[i]] = x[i];
        out[2 * bitrev[i] + 1] = 0.0f;
    }
    for (int count = 2; count <= FFT; count *= 2) {
        const int half = count / 2, step = FFT / count;
        for (int base = 0; base < FFT; base += count)
            for (int k = 0; k < half; k++) {
                const float re = cos_t[k * step], im = -sin_t[k * step];
                const int even = 2 * (base + k), odd = 2 * (base + k + half);
                const float ro = out[odd], io = out[odd + 1], re_e = out[even], im_e = out[even + 1];
                out[even] = re_e + re * ro - im * io;
                out[even + 1] = im_e + re * io + im * ro;
                out[odd] = re_e - re * ro + im * io;
                out[odd + 1] = im_e - re * io - im * ro;
            }
    }
}

/* AudioFrontEnd.logMel (AudioPreprocessor.swift:144-173) and melRow (178-202) over one chunk of
 * `n` samples (n <= 480000); writes frame_count(n) rows of mel_bins values and returns the count. */
int32_t or_audio_log_mel(const float* samples, int64_t n, int32_t mel_bins, float* out) {
    const int32_t frames = or_audio_frame_count(n);
    if (frames < 1) return 0;
    float hann[FFT], sin_t[FFT], cos_t[FFT];
    int32_t bitrev[FFT];
    float* filters = (float*)malloc(sizeof(float) * (size_t)mel_bins * BINS);
    int32_t* lo = (int32_t*)malloc(sizeof(int32_t) * (size_t)mel_bins);
    int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)mel_bins);
    or_audio_tables(mel_bins, hann, sin_t, cos_t, filters, lo, hi, bitrev);
    const int64_t plen = (int64_t)(frames - 1) * HOP + FFT;
    float* padded = (float*)calloc((size_t)plen, sizeof(float));
    memcpy(padded + WIN / 2, samples, sizeof(float) * (size_t)n);
#pragma omp parallel for schedule(dynamic, 16)
    for (int32_t f = 0; f < frames; f++) {
        float input[FFT], spec[2 * FFT], mag[BINS];
        for (int j = 0; j < FFT; j++) input[j] = hann[j] * padded[(int64_t)f * HOP + j];
        fft(input, spec, sin_t, cos_t, bitrev);
        for (int j = 0; j < BINS; j++) mag[j] = sqrtf(spec[2 * j] * spec[2 * j] + spec[2 * j + 1] * spec[2 * j + 1]);
        for (int m = 0; m < mel_bins; m++) {
            const float* w = filters + (int64_t)m * BINS;
            double sum = 0.0;
            int k = lo[m];
            for (; k < (hi[m] < BINS - 3 ? hi[m] : BINS - 3); k += 4) {
                const float partial = mag[k] * w[k] + mag[k + 1] * w[k + 1] + mag[k + 2] * w[k + 2] + mag[k + 3] * w[k + 3];
                sum += (double)partial;
            }
            for (; k < hi[m]; k++) sum += (double)(mag[k] * w[k]);
            const double floor_ = (double)0.001f;
            out[(int64_t)f * mel_bins + m] = (float)log(sum > floor_ ? sum : floor_);
        }
    }
    free(padded);
    free(filters);
    free(lo);
    free(hi);
    return frames;
}

/* ---- MiniaudioConverter (Audio/MiniaudioConverter.swift:18-213) */

/* ma_calculate_frame_count_after_resampling (MiniaudioConverter.swift:55-66). */
uint64_t or_audio_frames_after_resampling(uint32_t rate_out, uint32_t rate_in, uint64_t n) {
    if (rate_in == 0 || rate_out == 0 || n == 0) return 0;
    if (rate_in == rate_out) return n;
    uint64_t out = n * rate_out / rate_in;
    const uint64_t frac = out * (rate_in / rate_out) / rate_out;
    if (out * (rate_in % rate_out) + frac <= n) out++;
    return out;
}

typedef struct { float b0, b1, b2, a1, a2, r1, r2; } biquad_t;

static double mini_cos(double x) { return sin(3.14159265358979323846 * 0.5 - x); }

/* Biquad.init (MiniaudioConverter.swift:175-192). */
static void biquad_init(biquad_t* q, uint32_t rate, double cutoff, double qv) {
    const double w = 2 * 3.14159265358979323846 * cutoff / (double)rate;
    const double s = sin(w), c = mini_cos(w), a = s / (2 * qv), a0 = 1 + a;
    q->b0 = (float)(((1 - c) / 2) / a0);
    q->b1 = (float)((1 - c) / a0);
    q->b2 = (float)(((1 - c) / 2) / a0);
    q->a1 = (float)((-2 * c) / a0);
    q->a2 = (float)((1 - a) / a0);
    q->r1 = q->r2 = 0.0f;
}

/* Biquad.process (MiniaudioConverter.swift:198-203): the fused multiply-adds of llama.cpp's build. */
static float biquad_run(biquad_t* q, float x) {
    const float y = fmaf(q->b0, x, q->r1);
    q->r1 = fmaf(q->b1, x, -(q->a1 * y)) + q->r2;
    q->r2 = fmaf(q->b2, x, -(q->a2 * y));
    return y;
}

/* MiniaudioConverter.toMono16k (MiniaudioConverter.swift:23-37): writes
 * or_audio_frames_after_resampling(16000, rate, frames) samples (frames when rate is 16000). */
int64_t or_audio_to_mono16k(const float* samples, int64_t frames, int32_t channels, int32_t rate, float* out) {
    if (channels <= 0 || rate <= 0 || frames <= 0) return 0;
    float* mono = (float*)malloc(sizeof(float) * (size_t)frames);
    for (int64_t f = 0; f < frames; f++) {
        float t = 0.0f;
        for (int32_t c = 0; c < channels; c++) t += samples[f * channels + c];
        mono[f] = channels == 1 ? samples[f] : t / (float)channels;
    }
    if (rate == 16000) {
        memcpy(out, mono, sizeof(float) * (size_t)frames);
        free(mono);
        return frames;
    }
    uint32_t a = (uint32_t)rate, b = 16000;
    while (b) {
        const uint32_t t = a % b;
        a = b;
        b = t;
    }
    const uint32_t rin = (uint32_t)rate / a, rout = 16000 / a;
    const uint32_t adv_i = rin / rout, adv_f = rin % rout;
    const int down = rin > rout;
    const uint32_t lpf_rate = rin > rout ? rin : rout;
    const double cutoff = (double)(rin < rout ? rin : rout) * 0.5 * 1.0;
    biquad_t st[2];
    for (int k = 0; k < 2; k++) biquad_init(&st[k], lpf_rate, cutoff, 1 / (2 * mini_cos((double)(1 + 2 * k) * (3.14159265358979323846 / 8))));
    const int64_t len = (int64_t)or_audio_frames_after_resampling(16000, (uint32_t)rate, (uint64_t)frames);
    uint32_t ti = 1, tf = 0;
    float x0 = 0.0f, x1 = 0.0f;
    int64_t next = 0, n = 0;
    while (n < len) {
        while (ti > 0 && next < frames) {
            x0 = x1;
            x1 = mono[next++];
            if (down) x1 = biquad_run(&st[1], biquad_run(&st[0], x1));
            ti--;
        }
        if (ti > 0) break;
        const float fa = (float)tf / (float)rout;
        const float r0 = x1 - x0;
        const float r1 = r0 * fa;
        float y = x0 + r1;
        if (!down) y = biquad_run(&st[1], biquad_run(&st[0], y));
        out[n++] = y;
        ti += adv_i;
        tf += adv_f;
        if (tf >= rout) {
            tf -= rout;
            ti++;
        }
    }
    for (; n < len; n++) out[n] = 0.0f;
    free(mono);
    return len;
}
