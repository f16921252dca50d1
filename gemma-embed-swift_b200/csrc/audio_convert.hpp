// audio_convert.hpp -- decoded PCM (any rate, any channel count) to the 16 kHz mono samples the
// audio encoder reads, as llama.cpp's miniaudio decoder converts them
// (Sources/GemmaEmbed/Audio/MiniaudioConverter.swift).
#pragma once

#include <stdint.h>

#include <vector>

namespace ge {

// ma_calculate_frame_count_after_resampling (MiniaudioConverter.swift:55-66).
uint64_t audio_frames_after_resampling(uint32_t rate_out, uint32_t rate_in, uint64_t frames_in);
// The channels of each frame summed in order and divided by their count (MiniaudioConverter.swift:40-52).
void audio_downmix(const float* samples, int64_t frames, int channels, float* out);
// MiniaudioConverter.toMono16k (MiniaudioConverter.swift:23-37): `frames` frames of `channels`
// interleaved samples at `rate` Hz to 16 kHz mono.
void audio_to_mono_16k(const float* samples, int64_t frames, int channels, int rate, std::vector<float>& out);

}  // namespace ge
