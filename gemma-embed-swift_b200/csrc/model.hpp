// model.hpp -- the loaded model: configuration, per-device weights and workspaces, and the
// forward pass that replaces MetalForward (Sources/GemmaEmbed/Metal/MetalForward.swift).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "gemma_embed.h"
#include "gguf.hpp"
#include "kernels.hpp"
#include "audio.hpp"
#include "tokenizer.hpp"
#include "vision.hpp"

namespace ge {

// LayerConfig (Sources/GemmaEmbed/Model/ModelConfig.swift:31-37).
struct LayerCfg {
    bool sliding = false;
    int kv = 0, hd = 0;
    float rope_base = 0.f;
    int rope_index = 0;  // which RoPE table (one per distinct head dim and base)
};

// ModelConfig (ModelConfig.swift:40-112) for the two supported architectures.
struct Config {
    std::string arch, name, quant;
    int hidden = 0, layers = 0, heads = 0, ff = 0, per_layer = 0, out_dim = 0, dense_head = 0, vocab = 0;
    int sliding_window = 0, max_tokens = 8192;
    float eps = 1e-6f, emb_scale = 1.f, pl_scale = 1.f;
    int bos_id = 2, eos_id = 1;
    bool has_ple = false, has_output = false, has_dense = false;
    std::vector<LayerCfg> layer;
    std::vector<std::pair<int, float>> ropes;  // (head dim, base) per RoPE table
    int max_q() const;
    int max_kv() const;
};

struct LayerDev {
    DevWeight qkv, o, gu, down, inp_gate, proj;
    float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn = nullptr, *ffn_norm = nullptr,
          *post_ffw = nullptr, *post_norm = nullptr;
    float out_scale = 1.f;
};

struct Workspace {
    int cap_rows = 0, cap_seqs = 0, cap_work = 0;
    int32_t *tokens = nullptr, *positions = nullptr;
    uint32_t *seqs = nullptr, *work = nullptr, *chunk_base = nullptr;
    float* pool_partial = nullptr;  // [rows / kPoolChunkRows + seqs][hidden] partial sums of the mean pool
    float *x = nullptr, *y = nullptr, *ple = nullptr;
    __half* o16 = nullptr;  // fp16 output of the o (and, with per-layer inputs, down and per-layer) projections
    __half* d16 = nullptr;  // fp16 output of the down projection, beside o16 until the FFN residual
    float *pooled = nullptr, *mid = nullptr, *out = nullptr;
    float* fin = nullptr;  // finished rows [seqs][dims] (ForwardArgs::finish_dims)
    float* head_part = nullptr;  // the dense head's per-K-chunk partial sums [chunks][seqs][N]
    __half *qkv16 = nullptr;  // fused q|k|v projection output
    __half *h = nullptr, *x16 = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *act = nullptr,
           *g = nullptr;
    // GEMM A-operand views (buffer, column count) with their TMA descriptors.
    DevActivation a_h, a_x16, a_act, a_g;
    std::vector<DevActivation> a_attn;  // one per distinct query width
    std::vector<std::pair<int, AttnMaps>> attn_maps;  // per attn_map_key(KV heads, head dim)
    // The same over the fused projection rows of qkv16 (EPI_QKV layers read q, k and v in place).
    std::vector<std::pair<int, AttnMaps>> attn_maps_fused;
    // Pinned host staging.
    int32_t *h_tokens = nullptr, *h_positions = nullptr;
    uint32_t *h_seqs = nullptr, *h_work = nullptr, *h_chunk_base = nullptr;
    float* h_out = nullptr;
    int* h_err = nullptr;
};

// A captured forward for one batch shape on one workspace.
struct GraphKey {
    int rows = 0, ntok = 0, nseq = 0, pool_chunks = 0;
    // attention schedules: (items, CTAs) for sliding and global layers of head dim 256, then 512
    int sched[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uintptr_t tokens = 0;         // the token buffer the embedding kernel reads
    uintptr_t vectors = 0;        // and the vector rows it copies (image or audio rows), if any
    int finish = 0;               // 2 * finish_dims + normalise, 0 without the device finish
    bool operator==(const GraphKey& o) const {
        if (rows != o.rows || ntok != o.ntok || nseq != o.nseq || pool_chunks != o.pool_chunks || tokens != o.tokens ||
            vectors != o.vectors || finish != o.finish)
            return false;
        for (int k = 0; k < 8; k++)
            if (sched[k] != o.sched[k]) return false;
        return true;
    }
};
// The attention tensor maps of a workspace are kept per (KV heads, head dim).
inline int attn_map_key(int kv_heads, int hd) { return kv_heads * 1024 + hd; }
struct GraphEntry {
    GraphKey key;
    cudaGraphExec_t exec = nullptr;
    int64_t launches = 0;
    uint64_t last_use = 0;
};

struct Device {
    int ordinal = 0, num_sms = 148;
    std::string name;
    cudaStream_t stream = nullptr;
    int8_t* emb_q = nullptr;
    __half* emb_s = nullptr;
    std::vector<LayerDev> layers;
    DevWeight plp;  // per_layer_model_proj (fp16 only)
    float *pl_norm = nullptr, *out_norm = nullptr;
    float *dense2 = nullptr, *dense3 = nullptr, *output = nullptr;  // fp32 [N][K]
    std::vector<float*> rope;  // per table: [position][pair][cos, sin]
    int* err = nullptr;
    Workspace ws;
    std::vector<GraphEntry> graphs;  // at most kMaxGraphs, least recently used evicted
    uint64_t graph_clock = 0;
    // Batch shapes seen once and not captured (at most kMaxSeenKeys, oldest dropped): a shape
    // is captured the second time it runs, so a stream of distinct batches never pays for a
    // capture it does not replay.
    std::vector<GraphKey> seen_keys;
    std::vector<void*> allocations;
    VisionDev vis;  // the image encoder's weights and workspace, when one is loaded
    AudioDev aud;   // the audio encoder's weights and workspace, when one is loaded
    // Mixed inputs with both images and clips: their rows gathered in sequence order.
    float* mm_vectors = nullptr;
    size_t mm_vectors_cap = 0;  // floats
    // Per path (text, image, audio): recorded after the copies out of that path's pinned staging
    // buffers (see staging_wait).
    cudaEvent_t staging[3] = {nullptr, nullptr, nullptr};
};

// Each call rewrites its path's pinned staging buffers, while the copies the previous call
// enqueued from them may still be pending: the device-resident entry points return without
// waiting for their stream.  A call therefore waits for the event recorded after the previous
// call's copies (staging_done) before it writes or regrows those buffers (staging_wait).
enum StagingKind : int { kStageText = 0, kStageImage = 1, kStageAudio = 2 };
cudaError_t staging_wait(Device& d, int kind);
cudaError_t staging_done(Device& d, int kind, cudaStream_t stream);

}  // namespace ge

struct ge_tokenizer {
    ge::Tokenizer t;
};

namespace ge {
// One host thread per device of a multi-device model, started at load and kept until the model
// is freed, so a sharded call hands each device its share without creating threads.
class DeviceWorkers {
public:
    ~DeviceWorkers() { stop(); }
    void start(int n);
    void stop();
    // Runs fn(i) for i in [0, n) (n at most the workers started), worker i on device share i,
    // and returns once every one has finished.  Not reentrant (the model's lock serialises calls).
    void run(int n, const std::function<void(int)>& fn);

private:
    void loop(int i);
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(int)>* task_ = nullptr;
    uint64_t generation_ = 0;
    int active_ = 0, pending_ = 0;
    bool stop_ = false;
};
}  // namespace ge

struct ge_model {
    ge::Config cfg;
    ge::GgufFile file;
    std::vector<ge::Device> devs;
    std::mutex mu;
    std::string last_error;
    int budget = 8192;
    uint32_t flags = 0;
    int64_t file_size = 0;
    std::atomic<int64_t> launches{0};  // kernel launches issued by this model so far
    std::atomic<int64_t> h2d_bytes{0}, d2h_bytes{0};  // host <-> device copies of the forwards so far
    std::atomic<int64_t> graph_captures{0};           // CUDA graphs captured and instantiated so far
    std::unique_ptr<ge_tokenizer> tokenizer;  // null when the file carries no tokenizer
    std::unique_ptr<ge::DeviceWorkers> workers;  // with two or more devices: one host thread each
    // The image encoder (LoadOptions.imageEncoder): its file, configuration and the tokens that
    // frame an image's rows in the text sequence (SpanMarkers.image, Model/InputRow.swift:43-45).
    bool has_vision = false;
    ge::GgufFile vision_file;
    ge::VisionConfig vcfg;
    int32_t image_begin = -1, image_end = -1;
    int patch_budget = 4096;  // ImageEmbedOptions.patchBudget unless the load options raise it
    // The audio encoder (LoadOptions.audioEncoder) and the tokens that frame a clip's rows.
    bool has_audio = false;
    ge::GgufFile audio_file;
    ge::AudioConfig acfg;
    int32_t audio_begin = -1, audio_end = -1;
    int64_t frame_budget = 96000;  // log-mel frames per audio batch
};

namespace ge {
struct ProfileEntry {
    std::string name;
    double ms = 0, flops = 0, bytes = 0;
    int occurrences = 1;
};
// Per-kernel-class timings collected by a profiling forward (ge_profile).
struct ProfileSink {
    int reps = 10;
    std::vector<ProfileEntry> entries;
    ProfileEntry* find(const std::string& n) {
        for (auto& e : entries)
            if (e.name == n) return &e;
        return nullptr;
    }
    void add(const std::string& n, double ms, double flops, double bytes) {
        ProfileEntry e;
        e.name = n;
        e.ms = ms;
        e.flops = flops;
        e.bytes = bytes;
        entries.push_back(e);
    }
};
// One forward over a packed batch on one device (the body of MetalForward.execute/encode).
// tokens/positions/out are host pointers unless the *_dev flags say otherwise.
struct ForwardArgs {
    const int32_t* tokens = nullptr;
    bool tokens_on_device = false;
    const int32_t* positions = nullptr;  // host; nullptr derives 0..len-1 per sequence
    int ntok = 0;
    const ge_seq* seqs = nullptr;  // host
    int nseq = 0;
    float* out = nullptr;
    bool out_on_device = false;
    cudaStream_t stream = nullptr;  // stream for device-resident calls; nullptr uses the device's own
    // > 0: EmbeddingModel.finish on the device (the first finish_dims of each pooled row,
    // L2-normalised when finish_normalise); out then receives [nseq][finish_dims]
    int finish_dims = 0;
    bool finish_normalise = false;
    int trace_layer = -2;           // >= -1: copy that layer's hidden state into trace_out instead
    float* trace_out = nullptr;
    std::string* error = nullptr;   // where failures are reported; nullptr: the model's last_error
    ProfileSink* profile = nullptr;  // time each kernel class instead of only running it
    // Device rows ([vector_rows][hidden] fp32) that ids below zero stand for: id -(r + 1) is
    // row r (an image's projected rows).  Checked by the caller.
    const float* vectors = nullptr;
    int vector_rows = 0;
};
int run_forward(ge_model* m, Device& d, const ForwardArgs& a);
// The image encoder: load (after the text model) and one forward over prepared images, whose
// projected rows land in d.vis.ws.vectors (image i's rows from sum of earlier token counts).
int load_vision(ge_model* m, const char* path);
void free_vision(Device& d);
struct VisionArgs {
    const PreparedImage* const* imgs = nullptr;  // grids, and the host pixels unless d_rgb is set
    int n = 0;
    const uint8_t* d_rgb = nullptr;  // device: every image's pixels back to back (skips the upload)
    cudaStream_t stream = nullptr;   // nullptr: the device's own stream
    std::string* error = nullptr;    // nullptr: the model's last_error
    ProfileSink* profile = nullptr;  // time each kernel class instead of only running it
};
int run_vision(ge_model* m, Device& d, const VisionArgs& a);
// The audio encoder: load (after the text model) and one forward over prepared clips, whose
// projected rows land in d.aud.ws.vectors (clip i's rows after the earlier clips' rows).
int load_audio(ge_model* m, const char* path);
void free_audio(Device& d);
struct AudioArgs {
    const PreparedAudio* const* clips = nullptr;  // sample counts, and the host samples unless d_pcm is set
    int n = 0;
    const float* d_pcm = nullptr;   // device: samples at each clip's device_offset (skips the upload)
    cudaStream_t stream = nullptr;  // nullptr: the device's own stream
    std::string* error = nullptr;   // nullptr: the model's last_error
    ProfileSink* profile = nullptr;  // time each kernel class instead of only running it
};
int run_audio(ge_model* m, Device& d, const AudioArgs& a);
GraphEntry* find_graph(Device& d, const GraphKey& k);
// The multi-GPU dispatcher's split of a packed batch: the sequence indices of each device,
// longest first onto the least-loaded device (cost n + n^2 / 2048), each in original order.
std::vector<std::vector<int>> shard_sequences(const ge_seq* seqs, int nseq, int ndev);
void store_graph(Device& d, const GraphKey& k, cudaGraphExec_t exec, int64_t launches);
// True when `k` ran before without a capture; otherwise remembers it and returns false.
bool seen_before(Device& d, const GraphKey& k);
void clear_graphs(Device& d);
int set_error(ge_model* m, int code, const std::string& msg);
}  // namespace ge
