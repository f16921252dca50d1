/*
 * gemma_embed.h -- C ABI of the B200 EmbeddingGemma text-encoder forward.
 *
 * This library replaces the reference's Metal forward (`MetalForward.run`,
 * Sources/GemmaEmbed/Metal/MetalForward.swift:199-204) behind its
 * `EmbeddingModel.load / embed / EmbedOptions` API
 * (Sources/GemmaEmbed/EmbeddingModel.swift:40-289, EmbedOptions.swift:34-56,
 * 171-203).  Every entry point takes plain pointers and sizes; the caller
 * owns every host array and nothing is retained after a call returns.  Calls
 * on one model handle are serialised internally (the reference's single GPU
 * queue, EmbeddingModel.swift:37, 269-281).  Every call returns a status code
 * (0 = success) and never aborts; `ge_last_error` gives the message.
 */
#ifndef GEMMA_EMBED_H
#define GEMMA_EMBED_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GE_API __attribute__((visibility("default")))

/* Status codes, one per GemmaEmbedError case that a text forward can raise
 * (Sources/GemmaEmbed/Errors.swift:6-23). */
typedef enum ge_status {
    GE_OK = 0,
    GE_ERR_FILE_NOT_READABLE = 1,      /* .fileNotReadable */
    GE_ERR_INVALID_GGUF = 2,           /* .invalidGGUF */
    GE_ERR_UNSUPPORTED_TENSOR_TYPE = 3,/* .unsupportedTensorType */
    GE_ERR_UNSUPPORTED_ARCHITECTURE = 4,/* .unsupportedArchitecture */
    GE_ERR_MISSING_TENSOR = 5,         /* .missingTensor */
    GE_ERR_MISSING_METADATA = 6,       /* .missingMetadata */
    GE_ERR_SHAPE_MISMATCH = 7,         /* .tensorShapeMismatch */
    GE_ERR_NO_DEVICE = 8,              /* .noMetalDevice: no usable sm_100 device */
    GE_ERR_INVALID_OPTIONS = 9,        /* .invalidOptions (also bad ids, sizes, positions) */
    GE_ERR_GPU_FAILURE = 10,           /* .gpuFailure */
    GE_ERR_OUT_OF_MEMORY = 11,         /* workspace growth failed (a .gpuFailure in the reference) */
    GE_ERR_TIMEOUT = 12,               /* a bounded device-side wait gave up (a .gpuFailure in the reference) */
    GE_ERR_CANCELLED = 13,             /* .cancelled */
    GE_ERR_IMAGE_DECODING = 14,        /* .imageDecoding: an image's pixels or size are unusable */
    GE_ERR_IMAGE_ENCODER_NOT_LOADED = 15, /* .imageEncoderNotLoaded */
    GE_ERR_AUDIO_DECODING = 16,        /* .audioDecoding */
    GE_ERR_AUDIO_ENCODER_NOT_LOADED = 17 /* .audioEncoderNotLoaded */
} ge_status;

typedef struct ge_model ge_model;

/* SequenceRange (MetalForward.swift:8-21): rows [start, start + length) of a packed batch. */
typedef struct ge_seq {
    uint32_t start;
    uint32_t length;
} ge_seq;

/* LoadOptions (EmbedOptions.swift:171-203), the fields a text forward uses. */
typedef struct ge_load_opts {
    uint32_t device_mask;       /* bit i selects CUDA device i; 0 selects device 0 */
    int32_t batch_token_budget; /* LoadOptions.batchTokenBudget; default 8192, at least 64 */
    uint32_t flags;             /* GE_LOAD_* bits */
    /* LoadOptions.imageEncoder: the mmproj GGUF whose gemma4v tower ge_embed_images needs;
     * NULL loads none (EmbedOptions.swift:183-187). */
    const char* image_encoder_path;
    /* Image patches per GPU batch when ge_image_opts.batch_size is 0; default 4096
     * (ImageEmbedOptions.patchBudget, EmbedOptions.swift:84-87), at least one image per batch. */
    int32_t image_patch_budget;
    /* LoadOptions.audioEncoder: the mmproj GGUF whose gemma4a tower ge_embed_audios needs; NULL
     * loads none (EmbedOptions.swift:188-191). */
    const char* audio_encoder_path;
    /* Log-mel frames per GPU batch when ge_audio_opts.batch_size is 0; default 96000 (16 minutes
     * of audio; the reference's AudioEmbedOptions.frameBudget is 12000, sized for an Apple GPU),
     * at least one clip per batch. */
    int32_t audio_frame_budget;
} ge_load_opts;

#define GE_LOAD_NO_GRAPHS 1u      /* launch kernels directly instead of replaying captured CUDA graphs */
#define GE_LOAD_Q8_ONLY 2u        /* keep only the Q8_0 planes resident; every GEMM dequantises in shared memory */
#define GE_LOAD_NO_PDL 4u         /* launch each kernel only after its predecessor completed (no programmatic
                                     dependent launch); results are bit-identical either way */
#define GE_LOAD_FUSED_RESIDUAL 8u /* fuse each residual step into the projection before it (row clusters of
                                     hidden/256 CTAs exchanging row sums through distributed shared memory) */
#define GE_LOAD_FUSED_QKV 16u     /* run the per-head q/k/v norms and RoPE of head-dim-256 layers in the q/k/v
                                     projection's epilogue; attention reads q, k and v from its rows in place */
#define GE_LOAD_SINGLE_CTA_GEMM 32u /* run every projection on single CTAs (128 x 256 tiles), never on CTA
                                       pairs; results are bit-identical either way */

/* EmbedOptions (EmbedOptions.swift:34-56) minus the task prefix, which ge_embed_texts takes
 * as a string (ge_task_prefix). */
typedef struct ge_embed_opts {
    int32_t max_tokens; /* default 2048; 2 .. ge_info.max_tokens */
    int32_t dimensions; /* 768, 512, 256 or 128 (Matryoshka prefix) */
    int32_t normalise;  /* L2-normalise the prefix */
    int32_t batch_size; /* texts per batch; 0 packs by the token budget */
} ge_embed_opts;

/* ModelInfo (ModelConfig.swift:5-27) plus the devices in use. */
typedef struct ge_info {
    char architecture[64];
    char name[128];
    int32_t layer_count;
    int32_t hidden_size;
    int32_t output_dimensions;
    int32_t feed_forward_size;
    int32_t per_layer_input_size;
    int32_t head_count;
    int32_t vocabulary_size;
    int32_t sliding_window;
    int32_t max_tokens;
    float norm_epsilon;
    char quantization[16];
    int64_t file_size;
    int32_t device_count;
    int32_t eos_id;
    int32_t bos_id;
    char device_name[128];
    int64_t kernel_launches; /* CUDA kernels this model has launched so far, on all devices */
    int64_t host_to_device_bytes; /* bytes the forwards so far copied from host to device */
    int64_t device_to_host_bytes; /* and from device to host */
    /* ImageEncoderInfo (VisionConfig.swift:5-17); all zero without an image encoder. */
    int32_t image_layer_count;
    int32_t image_hidden_size;
    int32_t image_patch_size;
    int32_t image_projection_dim;
    /* AudioEncoderInfo (AudioConfig.swift:5-19); all zero without an audio encoder. */
    int32_t audio_layer_count;
    int32_t audio_hidden_size;
    int32_t audio_head_count;
    int32_t audio_feed_forward_size;
    int32_t audio_mel_bins;
    int32_t audio_projection_dim;
    int64_t graph_captures; /* CUDA graphs captured so far: a batch shape is captured the second time it runs */
} ge_info;

/* One kernel class of a profiling forward (ge_profile). */
typedef struct ge_kernel_time {
    char name[32];
    double ms_per_launch;     /* mean over `reps` back-to-back launches, CUDA events on the launch stream */
    double flops_per_launch;  /* algorithmic FLOPs of one launch (token rows only) */
    double bytes_per_launch;  /* algorithmic HBM bytes of one launch */
    int32_t launches_per_forward;
} ge_kernel_time;

/* Progress after every batch (EmbeddingProgress, EmbedOptions.swift:155-160). Returning
 * nonzero cancels the call between batches, which then returns GE_ERR_CANCELLED
 * (the reference's Task.checkCancellation, EmbeddingModel.swift:162). */
typedef int (*ge_progress_fn)(int32_t completed_texts, int32_t total_texts, int64_t completed_tokens, void* user);

GE_API void ge_load_opts_default(ge_load_opts* opts);
GE_API void ge_embed_opts_default(ge_embed_opts* opts);

/* EmbeddingModel.load(from:options:) (EmbeddingModel.swift:40-122): parse and validate the
 * GGUF, repack its Q8_0 weights into the device layout and upload them to every selected
 * GPU, then run one warm-up forward.  On failure *out is NULL and ge_last_error(NULL) holds
 * the message. */
GE_API int ge_load(const char* gguf_path, const ge_load_opts* opts, ge_model** out);

/* Releases every device and host resource of the model. NULL is ignored. */
GE_API void ge_free(ge_model* model);

/* Message of the last failed call on `model`, or of the calling thread's last failed
 * ge_load when `model` is NULL.  Valid until the next call on the same handle. */
GE_API const char* ge_last_error(const ge_model* model);

GE_API int ge_info_get(const ge_model* model, ge_info* info);

/* MetalForward.run(_:) (MetalForward.swift:199-204) over one PackedBatch: `ntok` token ids
 * packed back to back, their positions, and `nseq` sequence ranges that tile [0, ntok) in
 * order.  Writes the pooled, unnormalised vectors, `nseq` rows of output_dimensions floats,
 * row i for sequence i.  With several devices the sequences are sharded across them and
 * gathered into `pooled_out` at their original rows. */
GE_API int ge_forward_packed(ge_model* model, const int32_t* tokens, const int32_t* positions, int32_t ntok,
                             const ge_seq* seqs, int32_t nseq, float* pooled_out);

/* The same forward over device-resident token ids on one device of the model: `d_tokens`
 * (ntok int32) and `d_pooled` (nseq * output_dimensions float) are device pointers on
 * device `device_ordinal`; `seqs` is a host array; positions are 0..length-1 per sequence.
 * Work is enqueued on `stream` (a cudaStream_t, NULL for the default stream) and the call
 * returns without synchronising. */
GE_API int ge_forward_device(ge_model* model, int32_t device_ordinal, const int32_t* d_tokens, int32_t ntok,
                             const ge_seq* seqs, int32_t nseq, float* d_pooled, void* stream);

/* Per-layer hidden state for parity checks (the `trace` names of CPUReference.forward,
 * CPUReference.swift:204-276): runs one sequence of `ntok` tokens and copies the fp32
 * residual stream after layer `layer` ("l_out-<layer>") into `hidden_out` (ntok * hidden
 * floats).  layer == -1 copies rmsnorm(x, output_norm) ("result_norm"). */
GE_API int ge_forward_trace(ge_model* model, const int32_t* tokens, int32_t ntok, int32_t layer, float* hidden_out);

/* Profiler.profile(model:texts:reps:) (Sources/GemmaEmbed/Metal/Profiler.swift:16-88): runs one forward over
 * the packed batch on the first device, timing the first launch of every kernel class over
 * `reps` back-to-back repetitions.  Fills up to `cap` entries and sets *count.  The forward's
 * output is discarded (repeated in-place kernels change it). */
GE_API int ge_profile(ge_model* model, const int32_t* tokens, int32_t ntok, const ge_seq* seqs, int32_t nseq,
                      int32_t reps, ge_kernel_time* out, int32_t cap, int32_t* count);

/* EmbeddingModel.embed over pre-tokenised texts (EmbeddingModel.swift:145-175 without the
 * tokenizer): truncation to max_tokens keeping EOS (189-196), batching by count or token
 * budget (200-215), one forward per batch, then the Matryoshka prefix and L2 (260-267) on the
 * device, with the arithmetic of ge_finish (the same bits).  `out` receives count * dimensions floats; `token_counts` and `truncated` (count entries
 * each, may be NULL) receive Embedding.tokenCount and Embedding.truncated. */
GE_API int ge_embed_tokens(ge_model* model, const int32_t* const* texts, const int32_t* lengths, int32_t count,
                           const ge_embed_opts* opts, float* out, int32_t* token_counts, int32_t* truncated,
                           ge_progress_fn progress, void* user);

/* ---- Tokenizer (Sources/GemmaEmbed/Tokenizer/Tokenizer.swift) ------------------------------ */

typedef struct ge_tokenizer ge_tokenizer;

/* Tokenizer's public properties (Tokenizer.swift:11-15) and its add-BOS/EOS flags. */
typedef struct ge_tokenizer_info {
    int32_t bos_id;
    int32_t eos_id;
    int32_t pad_id;
    int32_t unknown_id;      /* -1 when the file names none (unknownId == nil) */
    int32_t vocabulary_size;
    int32_t add_bos;         /* tokenizer.ggml.add_bos_token, default 1 */
    int32_t add_eos;         /* tokenizer.ggml.add_eos_token, default 0 */
} ge_tokenizer_info;

#define GE_ENCODE_ADD_SPECIAL 1u   /* encode(addSpecialTokens: true): BOS and EOS as the metadata asks */
#define GE_ENCODE_PARSE_SPECIAL 2u /* encode(parseSpecialTokens: true): control-token text becomes its id */

/* Tokenizer(gguf:) (Tokenizer.swift:40-56) over a GGUF file's tokenizer metadata alone: no
 * weights are read and no GPU is touched.  Fails with GE_ERR_UNSUPPORTED_ARCHITECTURE unless
 * tokenizer.ggml.model is "gemma4", GE_ERR_MISSING_METADATA without tokens, token types,
 * merges or BOS/EOS ids.  On failure *out is NULL and ge_last_error(NULL) holds the message. */
GE_API int ge_tokenizer_load(const char* gguf_path, ge_tokenizer** out);
GE_API void ge_tokenizer_free(ge_tokenizer* tokenizer);

/* EmbeddingModel.tokenizer (EmbeddingModel.swift:26): the loaded model's tokenizer, owned by
 * the model; NULL when its file carries no tokenizer.ggml.model. */
GE_API const ge_tokenizer* ge_model_tokenizer(const ge_model* model);

GE_API int ge_tokenizer_get_info(const ge_tokenizer* tokenizer, ge_tokenizer_info* info);

/* encode(_:addSpecialTokens:parseSpecialTokens:) (Tokenizer.swift:105-117) of `len` bytes of
 * UTF-8.  Sets *count to the full id count and writes the first min(count, cap) ids; a caller
 * whose buffer was too small calls again with cap >= *count.  `ids` may be NULL when cap is 0.
 * Safe to call from several threads at once. */
GE_API int ge_tokenize(const ge_tokenizer* tokenizer, const char* text, int64_t len, uint32_t flags, int32_t* ids,
                       int64_t cap, int64_t* count);

/* decode(_:) (Tokenizer.swift:120-147): UTF-8 bytes (not NUL-terminated; byte tokens may leave
 * an incomplete sequence, which the reference's String(decoding:) shows as U+FFFD).  Sets *len
 * to the full byte count and writes the first min(len, cap) bytes.  Ids outside the vocabulary
 * are skipped. */
GE_API int ge_detokenize(const ge_tokenizer* tokenizer, const int32_t* ids, int64_t n, char* text, int64_t cap,
                         int64_t* len);

/* piece(_:) (Tokenizer.swift:150-153): the vocabulary text of `id`, in the same buffer
 * convention as ge_detokenize; GE_ERR_INVALID_OPTIONS for an id outside the vocabulary (nil). */
GE_API int ge_token_piece(const ge_tokenizer* tokenizer, int32_t id, char* text, int64_t cap, int64_t* len);

/* isControl(_:) (Tokenizer.swift:155-158): 1 for a control token, else 0. */
GE_API int ge_token_is_control(const ge_tokenizer* tokenizer, int32_t id);

/* TaskPrefix (EmbedOptions.swift:5-32). */
typedef enum ge_task {
    GE_TASK_DOCUMENT = 0,       /* "title: <arg or none> | text: " */
    GE_TASK_QUERY = 1,          /* "task: <arg or search result> | query: " */
    GE_TASK_CLUSTERING = 2,     /* "task: clustering | query: " */
    GE_TASK_CLASSIFICATION = 3, /* "task: classification | query: " */
    GE_TASK_SIMILARITY = 4,     /* "task: sentence similarity | query: " */
    GE_TASK_NONE = 5            /* "" */
} ge_task;

/* TaskPrefix.prefix (EmbedOptions.swift:22-31): the prefix string of `task`; `arg` (UTF-8,
 * NUL-terminated, may be NULL) is the document title or the query's task description.  Same
 * buffer convention as ge_detokenize. */
GE_API int ge_task_prefix(int32_t task, const char* arg, char* text, int64_t cap, int64_t* len);

/* EmbeddingModel.embed(_:options:progress:) (EmbeddingModel.swift:145-175) on texts: each text
 * is `prefix` + text (prepare, 189-196: encoded with BOS/EOS as the metadata asks, truncated to
 * max_tokens keeping EOS), then batched, run and finished as ge_embed_tokens does.  `texts[i]`
 * holds lengths[i] bytes of UTF-8 (an empty text is allowed); `prefix` is NUL-terminated UTF-8
 * (ge_task_prefix), NULL for none.  The texts are encoded on several host threads. */
GE_API int ge_embed_texts(ge_model* model, const char* const* texts, const int64_t* lengths, int32_t count,
                          const char* prefix, const ge_embed_opts* opts, float* out, int32_t* token_counts,
                          int32_t* truncated, ge_progress_fn progress, void* user);

/* ---- Images (ImageEmbedding.swift, Metal/VisionTower.swift) -------------------------------- */

/* A decoded image: `height` rows of `width` RGB8 pixels, interleaved (RGBImage,
 * Image/ImageInput.swift:17-26).  Decoding files (JPEG, PNG) is the caller's. */
typedef struct ge_image {
    const uint8_t* rgb;
    int32_t width;
    int32_t height;
} ge_image;

/* ImageEmbedOptions (EmbedOptions.swift:59-88). */
typedef struct ge_image_opts {
    int32_t dimensions;       /* 768, 512, 256 or 128 */
    int32_t normalise;
    int32_t max_image_tokens; /* 1 .. 1120; default 256 */
    int32_t batch_size;       /* images per batch; 0 packs by the load options' patch budget */
} ge_image_opts;

GE_API void ge_image_opts_default(ge_image_opts* opts);

/* EmbeddingModel.embed(images:options:progress:) (ImageEmbedding.swift:17-33): each image is
 * resized to its patch grid (ImagePreprocessor.prepare), run through the vision tower, and its
 * rows, framed as [bos, <|image>, rows..., <image|>, eos], through the text tower, then finished
 * like a text.  `out` receives count * dimensions floats; `token_counts` (may be NULL) the rows
 * the text tower saw (image tokens + 4).  GE_ERR_IMAGE_ENCODER_NOT_LOADED without an encoder. */
GE_API int ge_embed_images(ge_model* model, const ge_image* images, int32_t count, const ge_image_opts* opts, float* out,
                           int32_t* token_counts, ge_progress_fn progress, void* user);

/* The image forward (vision and text towers, MetalForward.run(images:)) over device-resident
 * pixels on the caller's stream, without synchronising: `d_rgb` holds the images back to back,
 * each already at its tower size (images[i].width x height, sides multiples of patch * merge;
 * images[i].rgb is ignored); d_pooled receives [count][output_dimensions] pooled, unnormalised
 * fp32 rows.  The device counterpart of ge_embed_images' forward, for callers (and the
 * benchmark) whose pixels are already on the GPU.  NULL stream: the legacy default stream. */
GE_API int ge_image_forward_device(ge_model* model, int32_t device_ordinal, const uint8_t* d_rgb, const ge_image* images,
                                   int32_t count, float* d_pooled, void* stream);

/* Profiler.profileImages (Metal/Profiler.swift:114-200): on the first device, the whole image
 * forward ("image_forward") and the vision tower alone ("vision_tower"), mean over `reps`, then
 * each vision kernel class's first launch timed over `reps` back-to-back repetitions. */
GE_API int ge_profile_images(ge_model* model, const ge_image* images, int32_t count, int32_t max_image_tokens,
                             int32_t reps, ge_kernel_time* out, int32_t cap, int32_t* count_out);

/* PreparedImage.tokenCount (Image/ImagePreprocessor.swift:25-27) of a width x height image at
 * `max_image_tokens`: the rows ge_image_vectors returns for it; -1 without an image encoder. */
GE_API int32_t ge_image_tokens(const ge_model* model, int32_t width, int32_t height, int32_t max_image_tokens);

/* MetalForward.imageVectors (Metal/MetalForward.swift:227-238): the vision tower's projected rows
 * of each image, concatenated in order ([sum of rows][projection_dim] floats, at most cap_rows
 * rows); rows_per_image (count entries) receives each image's token count. */
GE_API int ge_image_vectors(ge_model* model, const ge_image* images, int32_t count, int32_t max_image_tokens,
                            float* out, int64_t cap_rows, int32_t* rows_per_image);

/* ---- Audio (AudioEmbedding.swift, Metal/AudioTower.swift) -------------------------------- */

/* A sound to embed (AudioInput, Audio/AudioInput.swift:6-14), in one of two forms.
 *
 * AudioInput.samples: `count` frames of `channels` interleaved PCM samples (count * channels
 * floats) in -1 .. 1 at `sample_rate` Hz, with `wav` NULL.
 *
 * AudioInput.data with WAV bytes: `wav` points at `wav_bytes` bytes of a RIFF/WAVE file, decoded
 * as miniaudio's dr_wav decodes it (PCM 8, 16, 24, 32 and 33-64 bit, IEEE float 32 and 64,
 * WAVE_FORMAT_EXTENSIBLE; WAVDecoder, Audio/WAVDecoder.swift); `samples`, `count`, `sample_rate`
 * and `channels` are ignored.  Other containers (MP3, M4A, AIFF, CAF, FLAC, which the reference
 * hands to AVFoundation) are the caller's to decode to samples.
 *
 * Clips that are not 16 kHz mono are converted as llama.cpp's miniaudio decoder converts them
 * (channels averaged in order, linear resampler with a 4th-order low-pass; MiniaudioConverter,
 * Audio/MiniaudioConverter.swift).  A non-positive rate or channel count, no samples, bytes that
 * are not a WAV file or a WAV file dr_wav refuses is GE_ERR_AUDIO_DECODING. */
typedef struct ge_audio {
    const float* samples;
    int64_t count;
    int32_t sample_rate;
    int32_t channels;
    const uint8_t* wav;
    int64_t wav_bytes;
} ge_audio;

/* WAVDecoder.decode (Audio/WAVDecoder.swift:29-84): the interleaved float samples of a RIFF/WAVE
 * file, before any downmix or resampling.  Writes min(cap, frames * channels) floats to `out` and
 * the frame count, rate and channel count to the (non-NULL) outputs.  A malformed file is
 * GE_ERR_AUDIO_DECODING with the reason ("WAV: no data chunk", ...) in ge_last_error(NULL).  Host
 * code only: needs no model and no GPU. */
GE_API int ge_audio_decode_wav(const uint8_t* bytes, int64_t length, float* out, int64_t cap, int64_t* frames,
                               int32_t* sample_rate, int32_t* channels);

/* AudioEmbedOptions (EmbedOptions.swift:91-114). */
typedef struct ge_audio_opts {
    int32_t dimensions; /* 768, 512, 256 or 128 */
    int32_t normalise;
    int32_t max_tokens; /* rows per clip including the 4 frame rows; 0: ge_info.max_tokens */
    int32_t batch_size; /* clips per batch; 0 packs by the load options' frame budget */
} ge_audio_opts;

GE_API void ge_audio_opts_default(ge_audio_opts* opts);

/* AudioDecoder.decode (Audio/AudioDecoder.swift:17-41): the 16 kHz mono samples the audio encoder
 * reads for `clip` (WAV bytes decoded first, then MiniaudioConverter.toMono16k,
 * Audio/MiniaudioConverter.swift:23-37); writes min(cap, n) of them to `out` and n to `*count`.
 * Host code only: needs no model and no GPU. */
GE_API int ge_audio_convert(const ge_audio* clip, float* out, int64_t cap, int64_t* count);

/* AudioFrontEnd.tokenCount(samples:) (Audio/AudioPreprocessor.swift:86-95): the rows a clip of
 * `samples` 16 kHz samples gives the text tower, before the 4 frame rows; 0 below 2 samples. */
GE_API int64_t ge_audio_tokens(int64_t samples);

/* EmbeddingModel.embed(audios:options:progress:) (AudioEmbedding.swift:17-33): each clip is cut
 * into 30-second chunks, turned into log-mel frames and run through the audio tower on the GPU;
 * its rows, framed as [bos, <|audio>, rows..., <audio|>, eos], go through the text tower and are
 * finished like a text.  `out` receives count * dimensions floats; `token_counts` (may be NULL)
 * the rows the text tower saw (clip tokens + 4).  A clip needing more than max_tokens rows is
 * refused (GE_ERR_INVALID_OPTIONS; audio is never cut); GE_ERR_AUDIO_ENCODER_NOT_LOADED without
 * an encoder.  Clips of a batch spread over the model's devices. */
GE_API int ge_embed_audios(ge_model* model, const ge_audio* clips, int32_t count, const ge_audio_opts* opts, float* out,
                           int32_t* token_counts, ge_progress_fn progress, void* user);

/* The audio tower's projected rows of each clip, concatenated in order ([sum of rows]
 * [projection_dim] floats, at most cap_rows rows); rows_per_clip (count entries) receives each
 * clip's token count.  Runs on the first device. */
GE_API int ge_audio_vectors(ge_model* model, const ge_audio* clips, int32_t count, float* out, int64_t cap_rows,
                            int32_t* rows_per_clip);

/* The audio forward (audio and text towers) over device-resident samples on the caller's
 * stream, without synchronising: `d_pcm` holds the clips' 16 kHz mono samples back to back
 * (clips[i].count each; clips[i].samples is ignored, clips[i].wav must be NULL); d_pooled receives [count]
 * [output_dimensions] pooled, unnormalised fp32 rows.  NULL stream: the legacy default stream. */
GE_API int ge_audio_forward_device(ge_model* model, int32_t device_ordinal, const float* d_pcm, const ge_audio* clips,
                                   int32_t count, float* d_pooled, void* stream);

/* Profiler.profileAudio (Metal/Profiler.swift:202-295): on the first device, the whole audio
 * forward ("audio_forward") and the audio tower alone ("audio_tower"), mean over `reps`, then
 * each audio kernel class's first launch timed over `reps` back-to-back repetitions. */
GE_API int ge_profile_audios(ge_model* model, const ge_audio* clips, int32_t count, int32_t reps, ge_kernel_time* out,
                             int32_t cap, int32_t* count_out);

/* ---- Mixed inputs (MultimodalEmbedding.swift) ---------------------------------------------- */

/* MultimodalInput.Part (MultimodalEmbedding.swift:7-12). */
typedef enum ge_part_kind { GE_PART_TEXT = 0, GE_PART_IMAGE = 1, GE_PART_AUDIO = 2 } ge_part_kind;

typedef struct ge_part {
    int32_t kind;      /* ge_part_kind */
    const char* text;  /* GE_PART_TEXT: text_len bytes of UTF-8 */
    int64_t text_len;
    ge_image image;    /* GE_PART_IMAGE: decoded pixels */
    ge_audio audio;    /* GE_PART_AUDIO: samples at any rate or WAV bytes */
} ge_part;

/* MultimodalInput (MultimodalEmbedding.swift:5-24): text, images and clips in reading order. */
typedef struct ge_multimodal_input {
    const ge_part* parts;
    int32_t count;
} ge_multimodal_input;

/* MultimodalEmbedOptions (EmbedOptions.swift:117-147) minus the task prefix (a string argument). */
typedef struct ge_multimodal_opts {
    int32_t max_tokens;       /* default 2048 */
    int32_t dimensions;
    int32_t normalise;
    int32_t max_image_tokens; /* default 256 */
    int32_t batch_size;       /* inputs per batch; 0 packs by the token, patch and frame budgets */
} ge_multimodal_opts;

GE_API void ge_multimodal_opts_default(ge_multimodal_opts* opts);

/* EmbeddingModel.embed(_ inputs: [MultimodalInput], options:progress:)
 * (MultimodalEmbedding.swift:100-206): each input becomes one text-tower sequence,
 * [bos] tok(prefix + text) [<|image>] rows... [<image|>] tok(text) ... [eos] with its images'
 * rows from the vision tower and its clips' [<|audio>] rows... [<audio|>] from the audio tower,
 * text cut from the end when it does not fit max_tokens; then finish.  `prefix` (NUL-terminated, NULL for none) is the task prefix.  `token_counts` and
 * `truncated` (may be NULL) receive each input's rows and whether text was cut.  An input whose
 * images and clips alone exceed max_tokens is refused (GE_ERR_INVALID_OPTIONS); image parts need
 * an image encoder and audio parts an audio encoder (GE_ERR_*_ENCODER_NOT_LOADED).  Runs on the
 * first device. */
GE_API int ge_embed_multimodal(ge_model* model, const ge_multimodal_input* inputs, int32_t count, const char* prefix,
                               const ge_multimodal_opts* opts, float* out, int32_t* token_counts, int32_t* truncated,
                               ge_progress_fn progress, void* user);

/* No counterpart in the reference.  The last stage of the forward -- mean-pool over each
 * sequence, then the dense head (or the output projection) -- for callers that cannot allocate
 * device memory: a plugin inside a host runtime that owns all device memory through its own
 * allocator, or a serving loop where an allocation could implicitly synchronise the device.
 * It calls no cudaMalloc, cudaFree or allocating library routine: its intermediates live in one
 * file-scope __device__ array of GE_NOALLOC_MAX_SEQS rows (2.5 MiB, held by every GPU that
 * loads the library until the process exits).
 *   d_hidden: device [ntok][hidden_size] fp32, the final-normed hidden states (the values
 *             ge_forward_trace returns for layer -1); d_seqs: device (start, length) uint32 pairs
 *             that tile [0, ntok); d_out: device [nseq][output_dimensions] fp32.
 * Only rows [0, ntok) of d_hidden are read: a range that runs past ntok is cut there, and a
 * range with no row inside (length 0, or a start at or past ntok) gives the head's value for a
 * zero pooled row.  The pool adds each sequence's rows in a different order than the forward's
 * chunked pool, so the output matches the forward's vectors within 1e-4 relative, not bit for
 * bit.  Work is enqueued on `stream` (a cudaStream_t; NULL is the legacy default stream) without
 * synchronising; the calling thread's current device is left as it was.  nseq above
 * GE_NOALLOC_MAX_SEQS, and hidden or dense-head widths that are not multiples of 128, return
 * GE_ERR_INVALID_OPTIONS.  ge_load looks up the array's device address (cudaGetSymbolAddress)
 * once on each of its devices; if that lookup has not succeeded, the first call on the device
 * repeats it, so make the first call before any stream capture.  All calls share the one array
 * and each overwrites what it reads: calls whose work overlaps on the GPU (other streams, other
 * host threads) race on it. */
#define GE_NOALLOC_MAX_SEQS 128
GE_API int ge_pool_head_noalloc(ge_model* model, int32_t device_ordinal, const float* d_hidden, int32_t ntok,
                                const uint32_t* d_seqs, int32_t nseq, float* d_out, void* stream);

/* EmbeddingModel.batches (EmbeddingModel.swift:200-215): splits `n` items with `ncost` costs
 * each (row-major costs[n][ncost]) into consecutive ranges, by count when batch_size > 0,
 * otherwise before the item that would take any summed cost past its budget.  Writes
 * (start, end) pairs to ranges_out (room for 2 * n) and the range count to *count_out. */
GE_API int ge_batches(const int64_t* costs, int32_t n, int32_t ncost, int32_t batch_size, const int64_t* budgets,
                      int32_t* ranges_out, int32_t* count_out);

/* EmbeddingModel.finish (EmbeddingModel.swift:260-267): the first `dims` values of `v`,
 * L2-normalised when `normalise` is nonzero and the norm is positive. */
GE_API int ge_finish(const float* v, int32_t n, int32_t dims, int32_t normalise, float* out);

#ifdef __cplusplus
}
#endif
#endif
