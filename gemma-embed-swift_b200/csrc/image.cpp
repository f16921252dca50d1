// image.cpp -- host-side image sizing and resampling for the vision tower.
//
// The geometry is llama.cpp's `img_tool` as the reference ports it (Image/ImageResizer.swift):
// the target size rounds each side to a multiple of patch * merge and pulls the pixel count into
// [70, maxImageTokens] tokens; the resample is Pillow's separable bicubic (a = -0.5, 22-bit
// fixed-point taps, a horizontal pass then a vertical pass, each rounded to 8 bits), so the
// resized bytes are identical to Pillow's.  Patchification (normalisation and the fp16
// rounding) runs on the GPU (k_patchify).
#include <math.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "vision.hpp"

namespace ge {

void image_target_size(int width, int height, int alignment, int min_pixels, int max_pixels, int& out_w, int& out_h) {
    const float f = float(alignment);
    auto round_by = [&](float x) { return int(roundf(x / f)) * alignment; };
    auto ceil_by = [&](float x) { return int(ceilf(x / f)) * alignment; };
    auto floor_by = [&](float x) { return int(floorf(x / f)) * alignment; };
    int w = std::max(alignment, round_by(float(width)));
    int h = std::max(alignment, round_by(float(height)));
    if (max_pixels > 0 && int64_t(w) * h > max_pixels) {
        const float beta = sqrtf(float(height) * float(width) / float(max_pixels));
        h = std::max(alignment, floor_by(float(height) / beta));
        w = std::max(alignment, floor_by(float(width) / beta));
    } else if (min_pixels > 0 && int64_t(w) * h < min_pixels) {
        const float beta = sqrtf(float(min_pixels) / (float(height) * float(width)));
        h = ceil_by(float(height) * beta);
        w = ceil_by(float(width) * beta);
    }
    out_w = w;
    out_h = h;
}

namespace {

constexpr int kPrecision = 22;  // Pillow's PRECISION_BITS for 8-bit images: 32 - 8 - 2

double bicubic(double x) {
    constexpr double a = -0.5;
    x = fabs(x);
    if (x < 1.0) return ((a + 2.0) * x - (a + 3.0)) * x * x + 1.0;
    if (x < 2.0) return (((x - 5.0) * x + 8.0) * x - 4.0) * a;
    return 0.0;
}

// Taps of one output dimension: for output pixel i, `count[i]` inputs from `first[i]` with
// weights taps[i * stride ...] (precompute_coeffs and normalize_coeffs_8bpc in Pillow).
struct Taps {
    int stride = 0;
    std::vector<int> first, count;
    std::vector<int32_t> w;

    Taps(int in_size, int out_size) {
        const double scale = double(in_size) / double(out_size);
        const double fscale = std::max(scale, 1.0);
        const double support = 2.0 * fscale;
        stride = int(ceil(support)) * 2 + 1;
        first.assign(size_t(out_size), 0);
        count.assign(size_t(out_size), 0);
        w.assign(size_t(out_size) * size_t(stride), 0);
        std::vector<double> k(static_cast<size_t>(stride));
        const double ss = 1.0 / fscale;
        for (int i = 0; i < out_size; i++) {
            const double center = (double(i) + 0.5) * scale;
            const int lo = std::max(0, int(center - support + 0.5));  // truncation toward zero
            const int n = std::min(in_size, int(center + support + 0.5)) - lo;
            double total = 0.0;
            for (int x = 0; x < n; x++) {
                k[size_t(x)] = bicubic((double(x + lo) - center + 0.5) * ss);
                total += k[size_t(x)];
            }
            for (int x = 0; x < n; x++) {
                const double v = total != 0.0 ? k[size_t(x)] / total : k[size_t(x)];
                w[size_t(i) * stride + x] = int32_t(v * double(1 << kPrecision) + (v < 0 ? -0.5 : 0.5));
            }
            first[size_t(i)] = lo;
            count[size_t(i)] = n;
        }
    }
};

inline uint8_t to_byte(int32_t acc) {
    const int32_t v = acc >> kPrecision;
    return uint8_t(v < 0 ? 0 : (v > 255 ? 255 : v));
}

// Sums wrap in 32 bits, as Pillow's (and the reference's) integer arithmetic does.
inline int32_t mad(int32_t acc, int32_t a, int32_t b) { return int32_t(uint32_t(acc) + uint32_t(a) * uint32_t(b)); }

std::vector<uint8_t> resample(const uint8_t* in, int w, int h, int tw, int th) {
    std::vector<uint8_t> horiz;
    const uint8_t* cur = in;
    int cw = w;
    if (tw != w) {
        const Taps t(w, tw);
        horiz.resize(size_t(tw) * h * 3);
        for (int y = 0; y < h; y++) {
            const uint8_t* row = in + size_t(y) * w * 3;
            uint8_t* dst = horiz.data() + size_t(y) * tw * 3;
            for (int x = 0; x < tw; x++) {
                int32_t a0 = 1 << (kPrecision - 1), a1 = a0, a2 = a0;
                const uint8_t* p = row + size_t(t.first[size_t(x)]) * 3;
                const int32_t* k = t.w.data() + size_t(x) * t.stride;
                for (int i = 0; i < t.count[size_t(x)]; i++, p += 3) {
                    a0 = mad(a0, p[0], k[i]);
                    a1 = mad(a1, p[1], k[i]);
                    a2 = mad(a2, p[2], k[i]);
                }
                dst[3 * x] = to_byte(a0);
                dst[3 * x + 1] = to_byte(a1);
                dst[3 * x + 2] = to_byte(a2);
            }
        }
        cur = horiz.data();
        cw = tw;
    }
    const size_t rowb = size_t(cw) * 3;
    std::vector<uint8_t> out(rowb * size_t(th));
    if (th == h) {
        memcpy(out.data(), cur, out.size());
        return out;
    }
    const Taps t(h, th);
    std::vector<int32_t> acc(rowb);
    for (int y = 0; y < th; y++) {
        std::fill(acc.begin(), acc.end(), int32_t(1) << (kPrecision - 1));
        const int32_t* k = t.w.data() + size_t(y) * t.stride;
        for (int i = 0; i < t.count[size_t(y)]; i++) {
            const uint8_t* src = cur + size_t(t.first[size_t(y)] + i) * rowb;
            for (size_t e = 0; e < rowb; e++) acc[e] = mad(acc[e], src[e], k[i]);
        }
        uint8_t* dst = out.data() + size_t(y) * rowb;
        for (size_t e = 0; e < rowb; e++) dst[e] = to_byte(acc[e]);
    }
    return out;
}

}  // namespace

void image_fit(const uint8_t* rgb, int w, int h, int tw, int th, uint8_t* out) {
    if (w == tw && h == th) {
        memcpy(out, rgb, size_t(w) * h * 3);
        return;
    }
    const float scale = std::min(float(tw) / float(w), float(th) / float(h));
    const int fw = std::min(int(ceilf(float(w) * scale)), tw);
    const int fh = std::min(int(ceilf(float(h) * scale)), th);
    const std::vector<uint8_t> fitted = resample(rgb, w, h, fw, fh);
    memset(out, 0, size_t(tw) * th * 3);
    const int ox = (tw - fw) / 2, oy = (th - fh) / 2;
    for (int y = 0; y < fh; y++)
        memcpy(out + (size_t(y + oy) * tw + ox) * 3, fitted.data() + size_t(y) * fw * 3, size_t(fw) * 3);
}

void prepare_image(const VisionConfig& c, const uint8_t* rgb, int w, int h, int max_image_tokens, PreparedImage& out) {
    const int a = c.alignment();
    int tw = 0, th = 0;
    image_target_size(w, h, a, c.min_image_tokens * a * a, max_image_tokens * a * a, tw, th);
    out.width = tw;
    out.height = th;
    out.gx = tw / c.patch;
    out.gy = th / c.patch;
    out.merge = c.merge;
    out.rgb.resize(size_t(tw) * th * 3);
    image_fit(rgb, w, h, tw, th, out.rgb.data());
}

}  // namespace ge
