// wav.hpp -- RIFF/WAVE bytes to the interleaved float samples miniaudio's dr_wav reads for an f32
// request (Sources/GemmaEmbed/Audio/WAVDecoder.swift).
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

namespace ge {

struct DecodedWav {
    std::vector<float> samples;  // frames * channels, interleaved
    int channels = 0;
    int sample_rate = 0;
};

// AudioDecoder.isWAV (Audio/AudioDecoder.swift:44-46): at least 12 bytes, "RIFF" then "WAVE" at 8.
bool is_wav(const uint8_t* bytes, int64_t len);
// WAVDecoder.decode (Audio/WAVDecoder.swift:29-84); false with the reason ("WAV: ...") in `why`.
bool decode_wav(const uint8_t* bytes, int64_t len, DecodedWav& out, std::string& why);

}  // namespace ge
