/*
 * oracle.h -- CPU restatement of the reference's fp32 forward pass.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load it.  The product library never links or calls it.
 *
 * It restates, in plain C with fp32 arithmetic:
 *   - GGUF parsing        Sources/GemmaEmbed/GGUF/GGUFFile.swift:21-67, GGUFValue.swift:83-131
 *   - model config        Sources/GemmaEmbed/Model/ModelConfig.swift:54-112
 *   - weight views        Sources/GemmaEmbed/Model/Weights.swift:19-43, 92-132
 *   - RoPE table          Sources/GemmaEmbed/Model/RopeTable.swift:16-31
 *   - forward             Sources/GemmaEmbed/Model/CPUReference.swift:63-283
 *   - batch planning      Sources/GemmaEmbed/EmbeddingModel.swift:200-215
 *   - finish              Sources/GemmaEmbed/EmbeddingModel.swift:260-267
 *
 * Parity pins: the batch planner is pinned by the reference's known answers
 * (Tests/GemmaEmbedTests/EmbeddingModelTests.swift:101-109, committed as
 * tests/golden/batches.json); the Q8_0 block layout by the tensor offsets in
 * Tests/GemmaEmbedTests/Fixtures/model.json.  The forward's numerics are
 * "parity unpinned": the reference's golden embeddings need the real
 * embeddinggemma GGUF, which is not available, and the reference itself
 * (Swift + Accelerate) cannot be built on Linux.  The forward is a
 * line-by-line restatement checked by internal consistency tests.
 */
#ifndef GE_ORACLE_H
#define GE_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: the same numbering as include/gemma_embed.h. */
enum {
    OR_OK = 0,
    OR_ERR_FILE_NOT_READABLE = 1,
    OR_ERR_INVALID_GGUF = 2,
    OR_ERR_UNSUPPORTED_TENSOR_TYPE = 3,
    OR_ERR_UNSUPPORTED_ARCHITECTURE = 4,
    OR_ERR_MISSING_TENSOR = 5,
    OR_ERR_MISSING_METADATA = 6,
    OR_ERR_SHAPE_MISMATCH = 7,
    OR_ERR_INVALID_OPTIONS = 9,
};

typedef struct or_model or_model;

typedef struct {
    int32_t hidden, layers, heads, ff, per_layer, out_dim, dense_head, vocab, sliding_window, max_tokens;
    float eps;
    int32_t kv_heads[64], head_dim[64], sliding[64];
    float rope_base[64];
} or_info;

typedef void (*or_trace_fn)(const char* name, const float* data, int64_t count, void* user);

int or_open(const char* path, or_model** out, char* err, int errlen);
void or_close(or_model* m);
int or_get_info(const or_model* m, or_info* info);
/* Threads used by the OpenMP regions (0 = all available). */
void or_set_threads(int n);
int or_threads(void);

/* CPUReference.forward(tokens:trace:): the pooled, unnormalised vector of one sequence. */
int or_forward(or_model* m, const int32_t* tokens, int32_t T, float* pooled, or_trace_fn trace, void* user);

/* CPUReference.forward(rows:trace:) with vector rows: an id -(r + 1) is row r of `vectors`
 * ([vector_rows][hidden]), entered unscaled. */
int or_forward_rows(or_model* m, const int32_t* tokens, int32_t T, const float* vectors, int64_t vector_rows,
                    float* pooled, or_trace_fn trace, void* user);

/* ne shape (contiguous dimension first, unused dimensions 1) and dimension count of a tensor. */
int or_tensor_shape(or_model* m, const char* tensor, int64_t* shape, int32_t* ndim);

/* WeightTensor.dequantizeRow for any tensor by name. */
int or_dequantize_row(or_model* m, const char* tensor, int64_t row, float* out, int64_t n);

/* ---- gemma4v vision tower (Sources/GemmaEmbed/Model/VisionConfig.swift, VisionWeights.swift,
 * CPUVisionReference.swift) and image preprocessing (Image/ImageResizer.swift,
 * Image/ImagePreprocessor.swift). */
typedef struct {
    int32_t hidden, layers, heads, head_dim, ff, patch, projection_dim, position_count, merge;
    float eps, rope_theta;
    float mean[3], std[3];
} or_vinfo;

/* VisionConfig(gguf:) and VisionWeights(gguf:config:) over an mmproj file. */
int or_vision_open(const char* path, or_model** out, char* err, int errlen);
int or_vision_get_info(const or_model* v, or_vinfo* info);
/* CPUVisionReference.forward: `patches` is [grid_y * grid_x][3 * patch^2] (PreparedImage.patches);
 * writes (grid_x / merge) * (grid_y / merge) rows of projection_dim floats. */
int or_vision_forward(or_model* v, const float* patches, int32_t grid_x, int32_t grid_y, float* out, or_trace_fn trace,
                      void* user);
/* ImageResizer.targetSize (ImageResizer.swift:11-29). */
void or_target_size(int32_t width, int32_t height, int32_t alignment, int32_t min_pixels, int32_t max_pixels,
                    int32_t* out_width, int32_t* out_height);
/* ImageResizer.fit (ImageResizer.swift:33-49): RGB8 `in` (w x h) to `out` (tw x th). */
void or_fit_image(const uint8_t* in, int32_t w, int32_t h, int32_t tw, int32_t th, uint8_t* out);
/* PreparedImage(resized:patchSize:mergeSize:mean:std:) (ImagePreprocessor.swift:31-60): patch rows
 * [gy * gx][3 * p^2], element c * p^2 + ky * p + kx, each rounded to fp16. */
void or_patchify(const uint8_t* rgb, int32_t w, int32_t h, int32_t p, const float* mean, const float* std, float* patches);
/* Float(Float16(x)): round to the nearest fp16 value, ties to even. */
float or_round_f16(float x);

/* ---- gemma4a audio tower (Sources/GemmaEmbed/Model/AudioConfig.swift, AudioWeights.swift,
 * CPUAudioReference.swift) and the log-mel front end (Audio/AudioPreprocessor.swift, in logmel.c). */
typedef struct {
    int32_t hidden, layers, heads, head_dim, ff, mel_bins, projection_dim, output_width;
    int32_t window, relative_positions, dw_kernel, sub_channels[2];
    float eps, softcap, ff_residual;
} or_ainfo;

/* AudioConfig(gguf:) and AudioWeights(gguf:config:) over an mmproj file. */
int or_audio_open(const char* path, or_model** out, char* err, int errlen);
int or_audio_get_info(const or_model* a, or_ainfo* info);
/* CPUAudioReference.forward on one chunk: `mel` is [frames][mel_bins]; writes
 * or_audio_tokens_for_frames(frames) rows of projection_dim floats. */
int or_audio_forward(or_model* a, const float* mel, int32_t frames, float* out, or_trace_fn trace, void* user);
void or_audio_sinusoid(int32_t position, int32_t width, float* out);
void or_audio_attention(const float* q, const float* k, const float* v, const float* rel, int32_t tokens, int32_t heads,
                        int32_t hd, int32_t window, float softcap, float* out);
void or_audio_depthwise(const float* x, int32_t tokens, int32_t width, const float* w, int32_t kernel, float* out);
/* AudioFrontEnd (AudioPreprocessor.swift:74-95): frames of one chunk, tokens from frames, tokens of a clip. */
int32_t or_audio_frame_count(int64_t samples);
int32_t or_audio_tokens_for_frames(int32_t frames);
int64_t or_audio_token_count(int64_t samples);
/* AudioFrontEnd.init's tables: hann/sin/cos [512], filters [mel_bins][257], bands [mel_bins], bitrev [512]. */
void or_audio_tables(int32_t mel_bins, float* hann, float* sin_t, float* cos_t, float* filters, int32_t* band_lo,
                     int32_t* band_hi, int32_t* bitrev);
/* AudioFrontEnd.logMel on one chunk of n <= 480000 samples: writes frame_count(n) rows of mel_bins. */
int32_t or_audio_log_mel(const float* samples, int64_t n, int32_t mel_bins, float* out);
/* MiniaudioConverter (Audio/MiniaudioConverter.swift): the resampled length, and `frames` frames of
 * `channels` interleaved samples at `rate` Hz to 16 kHz mono (returns the samples written). */
uint64_t or_audio_frames_after_resampling(uint32_t rate_out, uint32_t rate_in, uint64_t frames_in);
int64_t or_audio_to_mono16k(const float* samples, int64_t frames, int32_t channels, int32_t rate, float* out);

/* Static pieces, exposed for unit tests. */
void or_matmul(const float* x, int64_t m, int64_t k, const float* w, int64_t n, float* y);
void or_rmsnorm(const float* x, int64_t rows, int64_t width, const float* weight, float eps, float* out);
float or_gelu_tanh(float x);
void or_rope_table(int32_t head_dim, float base, int32_t positions, float* values);
void or_attention(const float* q, const float* k, const float* v, int32_t tokens, int32_t heads, int32_t kv_heads,
                  int32_t hd, float scale, int32_t window, float* out);
int32_t or_batches(const int64_t* costs, int32_t n, int32_t ncost, int32_t batch_size, const int64_t* budgets,
                   int32_t* ranges);
void or_finish(const float* v, int32_t n, int32_t dims, int32_t normalise, float* out);
uint64_t or_seeded_next(uint64_t* state);

#ifdef __cplusplus
}
#endif
#endif
