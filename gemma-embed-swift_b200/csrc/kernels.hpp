// kernels.hpp -- host-side launchers of the sm_100a kernels used by the forward pass.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace ge {

// Rows of every activation buffer are padded to this multiple: one tcgen05 M tile.
constexpr int kRowTile = 128;

// Launch policy of the calling thread: when set, kernels are launched with programmatic
// stream serialisation, so a kernel's CTAs are scheduled while its predecessor drains and
// wait for it in pdl_wait().  Every kernel of the library calls pdl_wait() before its first
// access to activations, which keeps the launch order's data dependencies.
void set_programmatic_launch(bool on);
bool programmatic_launch();

// cudaLaunchKernelEx with the calling thread's launch policy (and an optional cluster width).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          int cluster_x, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (programmatic_launch()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = unsigned(cluster_x);
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        n++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ GEMM
enum GemmEpilogue : int {
    EPI_F32 = 0,    // out[m][n] = acc (fp32)
    EPI_F16 = 1,    // out[m][n] = acc (fp16)
    EPI_GEGLU = 2,  // weight rows interleave gate and up in blocks of BN/2: out = gelu(gate) * up (fp16)
    EPI_GELU_MUL = 3,  // out = gelu(acc) * aux[m][n] (fp16), aux fp32 with row stride ldaux
    // The residual step of k_residual_norm on whole rows: t = fp16(acc); x = (x + rmsnorm(t) *
    // w_post) * scale; then optionally y = rmsnorm(x) * w_next stored as fp16 (h16) and/or fp32
    // (y32).  N = the hidden size; the N / 256 CTAs of a cluster hold one row block's columns
    // and exchange the per-row sums of squares through distributed shared memory.
    EPI_RESIDUAL = 4,
    // As EPI_GEGLU with the quick GELU of the vision tower: out = gate / (1 + exp(-1.702 gate)) * up.
    EPI_GEGLU_QUICK = 5,
    // The audio tower's clipped linears (Gemma4ClippableLinear): v = clamp(acc, lo, hi) + bias[n]
    // (bias optional), stored as fp32 (EPI_CLAMP_F32) or fp16 (EPI_CLAMP_F16).
    EPI_CLAMP_F32 = 6,
    EPI_CLAMP_F16 = 7,
    // out = clamp(silu(clamp(acc, lo, hi) + bias[n]), act_lo, act_hi) (fp16): a clipped linear, the
    // SiLU after it, and the next clipped linear's input clamp.
    EPI_CLAMP_SILU = 8,
    // Gate/up interleaved as EPI_GEGLU: out = clamp(up) * sigmoid(clamp(gate)) (fp16), the
    // convolution module's GLU over a clipped pointwise linear.
    EPI_GLU = 9,
    // The fused q/k/v projection of a head-dim-256 layer with the per-head norms and RoPE of
    // k_qkv_norm_rope in its epilogue: each 256-column tile is one head slot (queries, then keys,
    // then values); t = fp16(acc), then t * rsqrt(mean(t^2) + eps) * (q_norm or k_norm; values
    // unweighted), then NeoX RoPE on query and key slots, stored as fp16 in place of the
    // projection.  Rows at or past ntok are stored as zeros.
    EPI_QKV = 10,
};
__host__ __device__ constexpr bool epi_is_geglu(int epi) {
    return epi == EPI_GEGLU || epi == EPI_GEGLU_QUICK || epi == EPI_GLU;
}
__host__ __device__ constexpr bool epi_is_clamp(int epi) {
    return epi == EPI_CLAMP_F32 || epi == EPI_CLAMP_F16 || epi == EPI_CLAMP_SILU || epi == EPI_GLU;
}


// One GEMM weight as the device keeps it: the Q8_0 planes (int8 values [N][K] and the fp16
// block scales transposed to [K/32][N]) and, unless disabled, the exact fp16 dequantisation
// [N][K] (each element round-to-nearest of scale * q, the value the Q8 path produces in
// shared memory).
struct DevWeight {
    int N = 0, K = 0;
    int8_t* q8 = nullptr;
    __half* scales_t = nullptr;
    __half* f16 = nullptr;
    // map_f16_half, _quarter, _eighth: boxes of BN/2, BN/4, BN/8 rows (CTA pairs and 128-wide
    // tiles take BN/2; the pieces of split tiles take BN/S, the gate and up halves of a GeGLU
    // piece BN/2S).
    CUtensorMap map_q8, map_scales, map_f16, map_f16_half, map_f16_quarter, map_f16_eighth;
};

// A row-major fp16 activation matrix that feeds GEMMs as the A operand.
struct DevActivation {
    __half* ptr = nullptr;
    int rows = 0, cols = 0;
    CUtensorMap map;
};

bool encode_weight_maps(DevWeight& w, int bn);
bool encode_activation_map(DevActivation& a);

// Which fp16-path kernel a GEMM uses: single CTAs with 128 x 256 tiles, single CTAs with
// 128 x 128 tiles, or CTA pairs (tcgen05.mma.cta_group::2, 256 x 256 tiles, 128-deep K stages).
// AUTO takes CTA pairs when their tiles fill at least two rounds of the SMs' pairs (and K is a
// multiple of 128), else single CTAs with 128 x 256 tiles: the fastest on each forward shape.
// The Q8 path always runs single CTAs with 128 x 256 tiles.
// GEMM_SPLIT runs single-CTA 128 x 256 tiles as narrower pieces where that would shorten the
// persistent schedule on paper (the last partial round, or every tile of a batch that leaves SMs
// idle; see k_gemm).  Bit-identical to whole tiles, measured no faster on any forward shape
// (bench.py's gemm_schedules), so only on request.
enum GemmMode : int { GEMM_AUTO = 0, GEMM_SINGLE = 1, GEMM_PAIR = 2, GEMM_NARROW = 3, GEMM_SPLIT = 4 };

struct GemmLaunch {
    const DevActivation* a;
    const DevWeight* w;
    int m_rows;       // rows to compute, a multiple of kRowTile
    void* out;
    int ldo;          // output row stride in elements
    int epilogue;
    const float* aux = nullptr;
    int ldaux = 0;
    bool use_q8 = false;  // dequantise Q8 tiles in shared memory instead of reading fp16 weights
    int mode = GEMM_AUTO;
    int* err;
    int num_sms;
    // EPI_RESIDUAL only: the residual stream x [m_rows][N] (read and rewritten), its norm
    // weights and the outputs of the next norm (either may be null; w_next null skips both).
    float* x = nullptr;
    const float* w_post = nullptr;
    float scale = 1.0f;
    const float* w_next = nullptr;
    float eps = 1e-6f;
    __half* h16 = nullptr;
    float* y32 = nullptr;
    // Clamp epilogues: the output bounds, the post-activation bounds (EPI_CLAMP_SILU) and an
    // optional fp32 bias per output column.
    float clamp_lo = -3.402823466e38f, clamp_hi = 3.402823466e38f;
    float act_lo = -3.402823466e38f, act_hi = 3.402823466e38f;
    const float* bias = nullptr;
    // EPI_QKV: token positions, the RoPE table ([position][128 pairs][cos, sin]), the query and
    // key norm weights (256 each), the live rows and the head counts (eps above).
    const int32_t* positions = nullptr;
    const float* rope = nullptr;
    const float* q_norm = nullptr;
    const float* k_norm = nullptr;
    int ntok = 0, heads = 0, kv_heads = 0;
};
cudaError_t launch_gemm(const GemmLaunch& g, cudaStream_t stream);
// Kernel attributes (dynamic shared-memory limits) for the current device; call once per
// device before the first launch or stream capture.
cudaError_t configure_gemm_kernels();
cudaError_t configure_attention_kernels();

// ------------------------------------------------------------------ elementwise
// x[t] = q8row(table[id]) * scale for t < ntok, 0 for padded rows; h = rmsnorm(x) * w (fp16).
// Optionally also x16 = fp16(x) (the per-layer-input GEMM's operand).  An id -(r + 1) takes
// row r of `vectors` ([*][width] fp32, device) unscaled; ids below zero need `vectors`.
cudaError_t launch_embed(const int32_t* tokens, int ntok, int rows, const int8_t* table_q, const __half* table_s,
                         int width, float scale, float* x, __half* x16, const float* norm_w, float eps, __half* h,
                         cudaStream_t stream, const float* vectors = nullptr);

// Per (token, head): q, k = rope(rmsnorm(head) * w); v = rmsnorm(head). Reads the fused
// projection output qkv (fp16, [rows][(H + 2 KV) * hd]) and writes fp16 q, k, v; rows at or
// past ntok are written as zeros.
cudaError_t launch_qkv_norm_rope(const __half* qkv, int ntok, int rows, int heads, int kv_heads, int hd,
                                 const float* q_w, const float* k_w, const int32_t* positions, const float* rope,
                                 float eps, __half* q, __half* k, __half* v, cudaStream_t stream);

// x = (x + rmsnorm(t) * w_post) * scale; then, when w_next is set,
// h16 = fp16(rmsnorm(x) * w_next) or y32 = rmsnorm(x) * w_next, and x16 = fp16(x) if set.
// t is the fp16 output of the projection; width 512 or 768.
cudaError_t launch_residual_norm(float* x, const __half* t, int rows, int width, const float* w_post, float scale,
                                 const float* w_next, float eps, __half* h16, float* y32, __half* x16,
                                 cudaStream_t stream);
// The general residual step: x' = (x + rmsnorm(t) * w_post) * scale, then, when t2 is set,
// x' += rmsnorm(t2) * w_post2; x' is stored when store_x, and the next norm of x' goes to h16
// / y32 when w_next is set (x16 = fp16(x') if set).
struct ResidualStep {
    float* x = nullptr;
    const __half* t = nullptr;
    const float* w_post = nullptr;
    float scale = 1.0f;
    const __half* t2 = nullptr;
    const float* w_post2 = nullptr;
    bool store_x = true;
    const float* w_next = nullptr;
    float eps = 1e-6f;
    __half* h16 = nullptr;
    float* y32 = nullptr;
    __half* x16 = nullptr;
};
cudaError_t launch_residual(const ResidualStep& r, int rows, int width, cudaStream_t stream);

// Per-row RMSNorm of `width`-wide chunks with a pre-scale: out = fp16(rmsnorm(x * pre) * w).
cudaError_t launch_rmsnorm_rows(const float* x, int rows, int width, float pre, const float* w, float eps, float* out,
                                cudaStream_t stream);

// pooled[s] = mean over the sequence's rows of y (fp32), in two launches: partial sums of
// chunks of rows (partial[chunk_base[s] + k], max_chunks = most chunks of any sequence),
// then the per-sequence total.  pool_chunks(len) is a sequence's chunk count.
int pool_chunks(uint32_t len);
constexpr int kPoolChunkRows = 64;  // rows per partial sum of the mean pool
cudaError_t launch_mean_pool(const float* y, int width, const uint32_t* seqs, int nseq, int max_chunks,
                             const uint32_t* chunk_base, float* partial, float* pooled, cudaStream_t stream);
// The same mean in one launch, one block per sequence (sequence ranges on the device only);
// rows at or past ntok are never read (a range is cut there, an empty one pools to zeros).
cudaError_t launch_mean_pool_seq(const float* y, int width, int ntok, const uint32_t* seqs, int nseq, float* pooled,
                                 cudaStream_t stream);

// out[s][n] = sum_k in[s][k] * w[n][k], fp32 weights [N][K].
// The forward's dense head / output projection: 64 x 64 tiles over fixed 256-wide K chunks,
// then the chunk partials added in order (`part` holds K / 256 x nrows x N floats); N a
// multiple of 64 and K of 256.  launch_dense_f32 below needs no scratch.
cudaError_t launch_dense_head(const float* in, int nrows, const float* w, int N, int K, float* part, float* out,
                              cudaStream_t stream);
int dense_head_chunks(int K);
cudaError_t launch_dense_f32(const float* in, int nrows, const float* w, int N, int K, float* out,
                             cudaStream_t stream);

// positions[start + i] = i over the sequences (start, length) pairs.
// The first `dims` of each of nseq rows of `width` values, L2-normalised when `normalise`
// (EmbeddingModel.finish), into out [nseq][dims]; bit-identical to the host's ge_finish.
cudaError_t launch_finish_rows(const float* in, int nseq, int width, int dims, int normalise, float* out,
                               cudaStream_t stream);
cudaError_t launch_positions(const uint32_t* seqs, int nseq, int32_t* positions, cudaStream_t stream);

// ------------------------------------------------------------------ vision tower
// One image of a vision batch: its bytes in the batch's RGB buffer (rows of gx * patch pixels,
// 3 bytes each), its patch grid, and where its patch rows and its pooled token rows start.
struct VisionImage {
    uint64_t rgb_offset;
    int32_t gx, gy;
    uint32_t patch_start, token_start;
};
struct NormParams {
    float mean[3], std[3];
};
// patches[patch_start + py * gx + px][c * p^2 + ky * p + kx] = fp16(2 (byte / 255 - mean[c]) /
// std[c] - 1), columns [3 p^2, kpad) zero (PreparedImage.init, ImagePreprocessor.swift:31-60).
cudaError_t launch_patchify(const uint8_t* rgb, const VisionImage* imgs, int nimg, int max_patches, int p, int kpad,
                            const NormParams& np, __half* patches, cudaStream_t stream);
// x[r] = (x[r] + pos[px]) + pos[npos + py] with (px, py) = (xy & 0xffff, xy >> 16); h = fp16(
// rmsnorm(x) * w); rows at or past ntok get h = 0.
cudaError_t launch_patch_position_norm(float* x, const uint32_t* xy, int ntok, int rows, int d, const float* pos,
                                       int npos, const float* w, float eps, __half* h, cudaStream_t stream);
// Per token and head of 64: q, k = rope2d(rmsnorm(head) * w), v = rmsnorm(head); reads the fused
// [rows][3 heads * 64] projection, writes [rows][heads * 64] each (zeros past ntok).  `rope` is
// [position][16][cos, sin] (RopeTable with head dim 32).
cudaError_t launch_vision_qkv_norm_rope(const __half* qkv, int ntok, int rows, int heads, const float* qw,
                                        const float* kw, const uint32_t* xy, const float* rope, float eps, __half* q,
                                        __half* k, __half* v, cudaStream_t stream);
// out[token_start + t] = fp16(rmsnorm(scale * sum of the token's merge x merge patch rows)).
cudaError_t launch_pool_patches_norm(const float* x, const VisionImage* imgs, int nimg, int max_tokens, int d, int merge,
                                     float scale, float eps, __half* out, cudaStream_t stream);

// ------------------------------------------------------------------ audio tower
// One 30-second (or shorter, final) chunk of a clip in a packed audio batch: where its samples,
// log-mel frames, first-convolution rows and token rows start, and how many there are.
struct AudioChunk {
    int64_t pcm_offset;
    int32_t samples, frames, mel_row, t0, t0_row, tokens, token_row, pad;
};
// The front end's tables on the device (AudioFrontEnd.init): periodic Hann, twiddles and the
// bit-reversal of the 512-point FFT, and per mel filter its band [lo, hi) of bins (whole groups
// of four) with the offset of its weights in `w`.
struct MelTables {
    const float *hann, *cos_t, *sin_t, *w;
    const int *bitrev, *band;  // band: lo[mel], hi[mel], off[mel]
    int nw, mel;
};
cudaError_t launch_log_mel(const float* pcm, const AudioChunk* chunks, int nchunks, int frames_total,
                           const MelTables& t, float* out, int num_sms, cudaStream_t stream);
cudaError_t configure_audio_kernels();
// First convolution (1 -> 128 channels, 3x3, stride 2) with LayerNorm and ReLU: out is
// [conv0 rows][64][128] fp16.  w is [128][9] (kh * 3 + kw), nw [128].
cudaError_t launch_audio_conv0(const float* mel, const AudioChunk* chunks, int nchunks, int t0_total, const float* w,
                               const float* nw, float eps, __half* out, cudaStream_t stream);
// The second convolution's patches: a [trows * 32][1152] fp16, K = (kh * 3 + kw) * 128 + c.
cudaError_t launch_audio_im2col(const __half* c0, const AudioChunk* chunks, int nchunks, int tokens, int trows, __half* a,
                                cudaStream_t stream);
// LayerNorm over the 32 channels in columns [0, 32) of c1 ([trows * 32][128] fp32), weight,
// ReLU, clamp; a2 is [trows][1024] fp16 (frequency * 32 + channel).
cudaError_t launch_audio_subsample_norm(const float* c1, int trows, const float* nw, float eps, float lo, float hi,
                                        __half* a2, cudaStream_t stream);
// A row step of the Conformer on [rows][width]: optionally x += rmsnorm(branch) * branch_w (or
// x += branch when branch_w is null), then x = rmsnorm(x) * final_w, x stored when store_x; then
// h = rmsnorm(x) * next_w (next_norm 1; next_w null: no weight) or h = x (next_norm 0), written
// to nout fp16 outputs each with its own clamp.
struct AudioRowStep {
    float* x = nullptr;
    const __half* branch = nullptr;
    const float* branch_w = nullptr;
    const float* final_w = nullptr;
    const float* next_w = nullptr;
    int next_norm = 0, nout = 0, store_x = 0, rows = 0;
    __half* out[3] = {nullptr, nullptr, nullptr};
    float lo[3] = {0, 0, 0}, hi[3] = {0, 0, 0};
    float eps = 1e-6f;
};
cudaError_t launch_audio_rows(const AudioRowStep& s, int width, cudaStream_t stream);
// Local causal attention of the audio tower: q, k, v [rows][heads * 128] fp16 (clamped linear
// outputs); scores (q * qscale) . (k * kscale + rel[t - j]) over j = max(chunk start, t - 11)
// .. t, capped at softcap tanh(s / softcap); out clamped to [lo, hi] as fp16.
struct AudioAttnLaunch {
    const __half *q, *k, *v;
    const float* rel;     // [13][heads * 128]
    const float* qscale;  // [128]
    float kscale, softcap, lo, hi;
    const int* chunk_start;  // [rows]
    int rows, heads, head_dim;
    __half* out;
};
cudaError_t launch_audio_attention(const AudioAttnLaunch& a, cudaStream_t stream);
// Causal depthwise conv (kernel 5, within each chunk), RMS norm with nw, SiLU, clamp: glu and
// out are [rows][width] fp16, dw_t [5][width].
cudaError_t launch_audio_dwconv(const __half* glu, const int* chunk_start, int rows, int width, const float* dw_t,
                                const float* nw, float eps, float lo, float hi, __half* out, cudaStream_t stream);

// Tensor-core attention for head dim 64 without a mask inside each sequence (the vision
// tower's, Shaders/Attention.metal:190-312): q, k, v [rows][heads * 64] fp16, out the same.
// `work` is build_attention_work's schedule with kv_heads = heads and group 1.
struct Attn64Launch {
    const __half* q;
    const __half* k;
    const __half* v;
    __half* out;
    int rows, heads;
    const uint32_t* work;  // items, then the CTAs' item offsets
    int sched_items, ctas;
    int* err;
};
cudaError_t launch_attention64(const Attn64Launch& a, cudaStream_t stream);
cudaError_t configure_attention64();  // part of configure_attention_kernels

// ------------------------------------------------------------------ attention
// TMA descriptors of the q, k and v buffers for the tensor-core attention kernel.
struct AttnMaps {
    CUtensorMap q, k, v;
};
// row_stride: elements between consecutive tokens' rows (0: q, k and v are dense buffers of
// heads * hd and kvh * hd columns; else they are column ranges of one fused projection row).
bool encode_attention_maps(AttnMaps& m, const __half* q, const __half* k, const __half* v, int rows, int heads, int kvh,
                           int hd, int row_stride = 0);
// A 2-D fp16 tensor map with 128-byte swizzle over a row-major [outer][inner] matrix whose rows
// are row_stride elements apart (0: inner).
bool encode_fp16_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint32_t box_inner,
                     uint32_t box_outer, uint64_t row_stride = 0);
// The same over a [d2][d1][d0] array with boxes b0 x b1 x b2; d2 steps are stride2 elements
// apart (0: d0 * d1).
bool encode_fp16_map_3d(CUtensorMap* map, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0,
                        uint32_t b1, uint32_t b2, uint64_t stride2 = 0);

struct AttnLaunch {
    const __half* q;  // [rows][heads * hd]
    const __half* k;  // [rows][kv_heads * hd]
    const __half* v;
    __half* out;      // [rows][heads * hd]
    // the schedule build_attention_work writes (items grouped by CTA, then the CTAs' item offsets)
    const uint32_t* work;
    int work_items;       // the schedule's CTA count
    int sched_items = 0;  // items in the schedule
    int heads, kv_heads, hd;  // hd 256 or 512
    int half_window;  // 0: global attention
    int* err;
    int num_sms = 148;
    const AttnMaps* maps = nullptr;  // encode_attention_maps over q, k and v
};
cudaError_t launch_attention(const AttnLaunch& a, cudaStream_t stream);
// Tokens of one tensor-core work item: its Q tile holds `group` heads per token in 128 rows
// (head dim 256) or 64 rows (head dim 512, whose 8 chunks of 64 dims fill the same 64 KB).
inline int attention_tokens_per_item(int group, int hd = 256) { return (hd == 512 ? 64 : 128) / group; }
// The tensor-core kernel's schedule for packed sequences (start, length pairs): one item per
// block of attention_tokens_per_item(group, hd) tokens and KV head (group = heads / kv_heads;
// head dim 512: two items, one per half of the output dims), spread over min(items, max_ctas)
// CTAs by longest-processing-time-first on the item's key blocks under `half_window` (0:
// global).  Layout: the items as (seq_start, seq_len, first token, KV head | half << 16),
// grouped by CTA, then CTA c's item range [off[c], off[c + 1]) as ctas + 1 offsets.  Returns
// the words written (or needed, when `out` is null); `ctas` receives the CTA count.
int build_attention_work(const uint32_t* seq_start_len, int nseq, int kv_heads, int group, int half_window,
                         int max_ctas, uint32_t* out, int* ctas, int hd = 256);

}  // namespace ge
