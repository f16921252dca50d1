// vision.hpp -- the gemma4v image encoder: its configuration, its weights and workspace on each
// device, and the host-side image preparation.
//
// Reference: Sources/GemmaEmbed/Model/VisionConfig.swift (configuration), VisionWeights.swift
// (tensors), Metal/VisionTower.swift (the forward), Image/ImagePreprocessor.swift and
// Image/ImageResizer.swift (sizing, resampling, patches), EmbeddingModel+ImageEmbedding
// (ImageEmbedding.swift: batching and the text tower over each image's rows).
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

#include "kernels.hpp"

namespace ge {

class GgufFile;

// VisionConfig (VisionConfig.swift:19-81).
struct VisionConfig {
    int hidden = 0, layers = 0, heads = 0, head_dim = 0, ff = 0, patch = 0, projection_dim = 0;
    int positions = 0;  // rows in each of the two position tables
    float eps = 1e-6f;
    float mean[3] = {0, 0, 0}, std[3] = {1, 1, 1};
    // Fixed by llama.cpp for gemma4v (VisionConfig.swift:28-33).
    int merge = 3;
    float rope_theta = 100.0f;
    int min_image_tokens = 70, native_max_image_tokens = 1120;
    int area() const { return patch * patch * 3; }
    int kpad() const { return (area() + 63) / 64 * 64; }  // the patch GEMM's K
    int alignment() const { return patch * merge; }
};

struct VisionLayerDev {
    DevWeight qkv, o, gu, down;
    float *ln1 = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn = nullptr, *ln2 = nullptr,
          *post_ffn = nullptr;
};

struct VisionWorkspace {
    int cap_rows = 0, cap_tokens = 0, cap_images = 0, cap_work = 0;
    size_t cap_rgb = 0;
    uint8_t* rgb = nullptr;
    __half* patches = nullptr;
    float* x = nullptr;
    __half *h = nullptr, *qkv = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *o16 = nullptr,
           *act = nullptr, *pooled = nullptr;
    float* vectors = nullptr;  // [token rows][projection_dim]: the rows the text tower reads
    uint32_t* xy = nullptr;    // per patch row: px | py << 16
    VisionImage* imgs = nullptr;
    uint32_t* work = nullptr;  // attention schedule
    DevActivation a_patches, a_h, a_attn, a_act, a_pooled;
    // Pinned host staging.
    uint8_t* h_rgb = nullptr;
    uint32_t *h_xy = nullptr, *h_work = nullptr;
    VisionImage* h_imgs = nullptr;
    std::vector<void*> allocations;
};

// The image encoder on one device.
struct VisionDev {
    bool loaded = false;
    DevWeight patch, proj;
    float* pos = nullptr;   // [2 * positions][hidden]: the column table, then the row table
    float* rope = nullptr;  // [positions][head_dim / 4][cos, sin]
    std::vector<VisionLayerDev> layers;
    VisionWorkspace ws;
    std::vector<void*> allocations;
};

// PreparedImage (ImagePreprocessor.swift:5-29) before patchification, which runs on the GPU:
// the image resized to the tower's size, as RGB8 rows.
struct PreparedImage {
    int width = 0, height = 0, gx = 0, gy = 0, merge = 3;
    std::vector<uint8_t> rgb;
    int patches() const { return gx * gy; }
    int tokens() const { return (gx / merge) * (gy / merge); }
};

// ImageResizer.targetSize (ImageResizer.swift:11-29).
void image_target_size(int width, int height, int alignment, int min_pixels, int max_pixels, int& out_w, int& out_h);
// ImageResizer.fit (ImageResizer.swift:33-49): Pillow's bicubic resample to fit inside
// (tw, th) keeping the aspect ratio, centred on black.
void image_fit(const uint8_t* rgb, int w, int h, int tw, int th, uint8_t* out);
// ImagePreprocessor.prepare on decoded pixels (ImagePreprocessor.swift:87-97).
void prepare_image(const VisionConfig& c, const uint8_t* rgb, int w, int h, int max_image_tokens, PreparedImage& out);

}  // namespace ge
