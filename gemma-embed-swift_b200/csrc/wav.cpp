// wav.cpp -- RIFF/WAVE bytes to interleaved float samples as miniaudio's dr_wav reads them for
// an f32 request (Sources/GemmaEmbed/Audio/WAVDecoder.swift): the chunk walk stops at `data`, so
// `fmt ` must come before it; unknown chunks are skipped with their odd-size padding; a `data`
// size that overruns the file is clamped to the bytes present and a trailing partial frame
// dropped; integer samples are scaled with dr_wav's constants, 32-bit floats copied bit for bit
// and 64-bit floats rounded to float.  Compiled without floating-point contraction.
#include "wav.hpp"

#include <string.h>

#include <algorithm>
#include <cstdio>

namespace ge {

namespace {

constexpr uint16_t kPCM = 0x0001, kIEEEFloat = 0x0003, kExtensible = 0xFFFE;

struct Reader {
    const uint8_t* b;
    int64_t n, off = 0;
    int64_t remaining() const { return n - off; }
    uint16_t u16() {
        const uint16_t v = uint16_t(b[off] | (b[off + 1] << 8));
        off += 2;
        return v;
    }
    uint32_t u32() {
        const uint32_t v = uint32_t(b[off]) | uint32_t(b[off + 1]) << 8 | uint32_t(b[off + 2]) << 16 | uint32_t(b[off + 3]) << 24;
        off += 4;
        return v;
    }
    bool four_cc(char out[4]) {
        if (remaining() < 4) return false;
        memcpy(out, b + off, 4);
        off += 4;
        return true;
    }
    // Moves the cursor (backwards too); false when that leaves the file, as dr_wav's seek fails.
    bool skip(int64_t d) {
        const int64_t t = off + d;
        if (t < 0 || t > n) return false;
        off = t;
        return true;
    }
};

struct Format {
    uint16_t tag = 0, channels = 0, block_align = 0, bits = 0, sub = 0;
    uint32_t rate = 0;
    uint16_t translated() const { return tag == kExtensible ? sub : tag; }
};

bool read_format(Reader& r, int64_t size, Format& f, std::string& why) {
    if (r.remaining() < 16) return why = "fmt chunk is truncated", false;
    f.tag = r.u16();
    f.channels = r.u16();
    f.rate = r.u32();
    r.u32();
    f.block_align = r.u16();
    f.bits = r.u16();
    if (size > 16) {
        if (r.remaining() < 2) return why = "fmt chunk is truncated", false;
        const int64_t ext = r.u16();
        int64_t consumed = 18;
        if (ext > 0) {
            if (f.tag == kExtensible) {
                if (ext != 22) return why = "extensible fmt chunk has a " + std::to_string(ext) + "-byte extension, expected 22", false;
                if (r.remaining() < 22) return why = "fmt chunk is truncated", false;
                r.u16();
                r.u32();
                f.sub = r.u16();
                r.skip(14);
            } else if (!r.skip(ext)) {
                return why = "fmt chunk is truncated", false;
            }
            consumed += ext;
        }
        if (!r.skip(size - consumed)) return why = "fmt chunk is truncated", false;
    }
    return true;
}

bool is(const char id[4], const char* want) { return memcmp(id, want, 4) == 0; }

}  // namespace

bool is_wav(const uint8_t* bytes, int64_t len) {
    return len >= 12 && memcmp(bytes, "RIFF", 4) == 0 && memcmp(bytes + 8, "WAVE", 4) == 0;
}

bool decode_wav(const uint8_t* bytes, int64_t len, DecodedWav& out, std::string& why) {
    Reader r{bytes, len};
    char id[4];
    auto fail = [&](const std::string& s) {
        why = "WAV: " + s;
        return false;
    };
    if (!r.four_cc(id) || !is(id, "RIFF")) return fail("not a RIFF file");
    if (r.remaining() < 4) return fail("not a WAVE file");
    r.u32();
    if (!r.four_cc(id) || !is(id, "WAVE")) return fail("not a WAVE file");
    Format f;
    bool have_fmt = false, have_data = false;
    int64_t data_begin = 0, data_size = 0;
    std::string w;
    while (r.remaining() >= 8) {
        r.four_cc(id);
        const uint32_t size32 = r.u32();
        const int64_t size = int64_t(size32), pad = int64_t(size32 & 1u);
        if (is(id, "fmt ")) {
            if (!read_format(r, size, f, w)) return fail(w);
            have_fmt = true;
            if (!r.skip(pad)) break;
        } else if (is(id, "data")) {
            data_begin = r.off;
            data_size = size;
            have_data = true;
            break;
        } else if (is(id, "fact")) {
            if (!r.skip(4)) return fail("fact chunk is truncated");
            if (!r.skip(size - 4 + pad)) break;
        } else if (!r.skip(size + pad)) {
            break;
        }
    }
    if (!have_fmt) return fail("no fmt chunk before the data chunk");
    if (!have_data) return fail("no data chunk");
    if (f.rate == 0 || f.rate > 384000) return fail("sample rate " + std::to_string(f.rate) + " is out of range");
    if (f.channels == 0 || f.channels > 256) return fail("channel count " + std::to_string(f.channels) + " is out of range");
    if (f.bits == 0 || f.bits > 64) return fail(std::to_string(f.bits) + " bits per sample is out of range");
    if (f.block_align == 0) return fail("block align is zero");
    const int channels = f.channels;
    const int64_t frame_bytes = f.bits % 8 == 0 ? int64_t(f.bits) * channels / 8 : int64_t(f.block_align);
    if (frame_bytes <= 0) return fail("frame size is zero");
    int64_t size = std::min(data_size, len - data_begin);
    size -= size % frame_bytes;
    const int64_t frames = size / frame_bytes, count = frames * channels;
    const uint8_t* p = bytes + data_begin;
    out.channels = channels;
    out.sample_rate = int(f.rate);
    out.samples.assign(size_t(count), 0.f);
    float* o = out.samples.data();
    const uint16_t tag = f.translated();
    if (tag == kPCM) {
        const int64_t bps = frame_bytes / channels;
        if (bps <= 0 || frame_bytes % channels != 0) {
            char buf[128];
            snprintf(buf, sizeof buf, "%d-bit PCM frames do not split evenly over %d channels", int(f.bits), channels);
            return fail(buf);
        }
        switch (bps) {
        case 1:
            for (int64_t i = 0; i < count; i++) {
                float x = float(p[i]);
                x = x * 0.00784313725490196078f;
                x = x - 1.0f;
                o[i] = x;
            }
            break;
        case 2:
            for (int64_t i = 0; i < count; i++) {
                const int16_t v = int16_t(uint16_t(p[2 * i] | (p[2 * i + 1] << 8)));
                o[i] = float(v) * 0.000030517578125f;
            }
            break;
        case 3:
            for (int64_t i = 0; i < count; i++) {
                const uint32_t u = uint32_t(p[3 * i]) << 8 | uint32_t(p[3 * i + 1]) << 16 | uint32_t(p[3 * i + 2]) << 24;
                const double x = double(int32_t(u) >> 8);
                o[i] = float(x * 0.00000011920928955078125);
            }
            break;
        case 4:
            for (int64_t i = 0; i < count; i++) {
                uint32_t u = 0;
                for (int k = 0; k < 4; k++) u |= uint32_t(p[4 * i + k]) << (8 * k);
                o[i] = float(double(int32_t(u)) / 2147483648.0);
            }
            break;
        case 5: case 6: case 7: case 8:
            for (int64_t i = 0; i < count; i++) {
                uint64_t v = 0;
                uint64_t shift = uint64_t(8 - bps) * 8;
                for (int64_t k = 0; k < bps; k++) {
                    v |= uint64_t(p[bps * i + k]) << shift;
                    shift += 8;
                }
                o[i] = float(double(int64_t(v)) / 9223372036854775807.0);
            }
            break;
        default:
            break;  // zeros, as the reference leaves them
        }
    } else if (tag == kIEEEFloat) {
        const int64_t bps = frame_bytes / channels;
        if (f.bits == 32) {
            for (int64_t i = 0; i < count; i++) memcpy(&o[i], p + 4 * i, 4);
        } else if (bps == 8) {
            for (int64_t i = 0; i < count; i++) {
                double d;
                memcpy(&d, p + 8 * i, 8);
                o[i] = float(d);
            }
        }
    } else {
        char buf[96];
        snprintf(buf, sizeof buf, "format tag 0x%x is not PCM or IEEE float", unsigned(tag));
        return fail(buf);
    }
    return true;
}

}  // namespace ge
