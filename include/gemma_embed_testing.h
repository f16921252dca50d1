/*
 * gemma_embed_testing.h -- kernel-level entry points of libgemma_embed_cuda.so for parity
 * tests, mirroring how the reference's KernelTests drive single kernels through its
 * `Kernels` encoders (Tests/GemmaEmbedTests/KernelTests.swift:89-104).  Each call allocates
 * its own device buffers, runs one kernel on the current CUDA device and copies the result
 * back; they are not for production use.
 */
#ifndef GEMMA_EMBED_TESTING_H
#define GEMMA_EMBED_TESTING_H

#include <stdint.h>

#include "gemma_embed.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Kernels.gemm (Metal/MetalForward.swift:513-557): out = a * W^T for a fp16 `a` [m][k]
 * (bit patterns) and a Q8_0 weight given as GGUF rows `w_q8_0` [n][k/32 * 34 bytes].
 * epilogue: 0 fp32 store, 1 fp16 store, 2 GeGLU over rows interleaved as the loader does
 * (out has n/2 columns), 3 gelu(acc) * aux (aux fp32 [m][n]), 5 the vision tower's GeGLU
 * with the quick GELU (interleaved like 2).  path: 0 fp16-resident
 * weights on single CTAs, 1 the in-shared-memory Q8 dequantisation, 2 fp16 weights on CTA
 * pairs (tcgen05.mma.cta_group::2), 3 fp16 weights on single CTAs with 128-wide tiles (not
 * for the GeGLU epilogue), 4 as 0 with tiles split into narrower pieces where that would
 * shorten the schedule (the last partial round, or every tile of a batch that leaves SMs idle).
 * Results are returned as fp32 [m][n] (or [m][n/2]). */
GE_API int ge_test_gemm(const uint16_t* a, int32_t m, int32_t k, const uint8_t* w_q8_0, int32_t n, int32_t epilogue,
                        int32_t path, const float* aux, float* out);

/* Mean device time of one GEMM launch (CUDA events around a CUDA graph of `reps` back-to-back
 * launches on a stream of its own, after three untimed launches and one untimed graph run) for m x k seeded fp16 activations (m a multiple
 * of 128) and an n x k seeded Q8_0 weight: epilogue 0 fp32 store, 1 fp16 store, 2 GeGLU over
 * interleaved rows; path as ge_test_gemm.  Writes microseconds per launch to *us. */
GE_API int ge_test_gemm_time(int32_t m, int32_t k, int32_t n, int32_t epilogue, int32_t path, int32_t reps, double* us);

/* The attention-output / down projection fused with the residual step (CPUReference.swift:
 * 239-243 and 252-256, Elementwise.metal:260-354): t = fp16(a * W^T); x = (x + rmsnorm(t) *
 * w_post) * scale in place on x [m][n] fp32; then, when w_next is given, y = rmsnorm(x) *
 * w_next returned as fp16 values in h_out and/or fp32 in y_out (either may be NULL).  n is
 * the hidden size, a multiple of 256 up to 1024.  path: 0 fp16-resident weights, 1 Q8. */
GE_API int ge_test_gemm_residual(const uint16_t* a, int32_t m, int32_t k, const uint8_t* w_q8_0, int32_t n,
                                 int32_t path, float* x, const float* w_post, float scale, const float* w_next,
                                 float eps, float* h_out, float* y_out);

/* Kernels.attention (Metal/MetalForward.swift:669-694): q [ntok][heads][hd], k and v
 * [ntok][kv_heads][hd] as fp16 bit patterns, sequences tiling [0, ntok); out receives fp16
 * bit patterns [ntok][heads][hd].  half_window 0 is global attention.  Head dim 256 and 512
 * run the text model's tensor-core kernel (512: one item per half of the output dims); head dim
 * 64 (heads == kv_heads, no window) the vision tower's. */
GE_API int ge_test_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t ntok, const ge_seq* seqs,
                             int32_t nseq, int32_t heads, int32_t kv_heads, int32_t hd, int32_t half_window,
                             uint16_t* out);

/* Host logic, no GPU needed. */

/* The multi-GPU dispatcher's split of a packed batch (ge_forward_packed on a model loaded on
 * several devices): device_of_seq[i] receives the device index (0..ndev-1) of sequence i. */
GE_API int ge_test_shard(const ge_seq* seqs, int32_t nseq, int32_t ndev, int32_t* device_of_seq);

/* The tensor-core attention kernel's schedule (head dim 256): items of 128 / group tokens and
 * one KV head, spread over at most max_ctas CTAs by key blocks under half_window (0: global).
 * Writes the schedule's words to out (capacity out_cap words): the items as (seq_start,
 * seq_len, first token, KV head) grouped by CTA, then ctas + 1 offsets.  *ctas and *words
 * receive the CTA count and the words written. */
GE_API int ge_test_attention_schedule(const ge_seq* seqs, int32_t nseq, int32_t kv_heads, int32_t group,
                                      int32_t half_window, int32_t max_ctas, uint32_t* out, int32_t out_cap,
                                      int32_t* ctas, int32_t* words);

/* Message of the calling thread's last failed ge_test_* call. */
/* ImagePreprocessor.prepare's sizing and resampling (Image/ImagePreprocessor.swift:87-97,
 * Image/ImageResizer.swift) on the host, without a model: the resized RGB8 image (tw x th) for
 * patch size `patch`, merge window `merge`, at least `min_tokens` and at most `max_tokens` tokens. */
GE_API int ge_test_image_prepare(int32_t patch, int32_t merge, int32_t min_tokens, const uint8_t* rgb, int32_t w,
                                 int32_t h, int32_t max_tokens, uint8_t* out, int64_t cap, int32_t* tw, int32_t* th);

/* k_patchify on one image whose sides are multiples of `patch`: fp16 patch rows
 * [(h / patch) * (w / patch)][kpad] (PreparedImage.patches, columns past 3 patch^2 zero). */
GE_API int ge_test_patchify(const uint8_t* rgb, int32_t w, int32_t h, int32_t patch, const float* mean, const float* std,
                            uint16_t* out, int32_t kpad);

/* MultimodalSequence.init (MultimodalEmbedding.swift:43-83) with one id per Unicode scalar
 * standing in for the tokenizer, as the reference's MultimodalSequenceTests do: parts given by
 * kind (0 text, 1 image, 2 audio) and, for text, NUL-terminated UTF-8; `span_rows` holds the
 * rows of each image or clip in order; images are framed by (image_begin, image_end), clips by
 * (audio_begin, audio_end).  Writes the ids (capacity `cap`), their count and whether text was
 * cut; returns GE_ERR_INVALID_OPTIONS when the spans alone do not fit (the reference's nil). */
GE_API int ge_test_multimodal_sequence(const char* prefix, const int32_t* kinds, const char* const* texts,
                                       int32_t nparts, const int32_t* span_rows, int32_t max_tokens, int32_t bos,
                                       int32_t eos, int32_t image_begin, int32_t image_end, int32_t audio_begin,
                                       int32_t audio_end, int32_t* ids, int32_t cap, int32_t* count,
                                       int32_t* truncated);

/* AudioFrontEnd.logMel (Audio/AudioPreprocessor.swift:144-202) of one chunk of `n` 16 kHz
 * samples (2 .. 480000) on the GPU: writes frame_count(n) rows of `mel_bins` (128) floats to
 * `out` and the frame count to `frames`. */
GE_API int ge_test_log_mel(const float* samples, int64_t n, int32_t mel_bins, float* out, int32_t* frames);

GE_API const char* ge_test_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
