// model.cpp -- loading (GGUF -> validated config -> repacked device weights) and the forward
// pass on one device.  Mirrors the reference's EmbeddingModel.init (EmbeddingModel.swift:46-122),
// ModelConfig / ModelWeights (Model/ModelConfig.swift:54-112, Model/Weights.swift:92-132) and
// MetalForward.execute / encode (Metal/MetalForward.swift:310-423).
#include "model.hpp"
#include "weights.hpp"

#include <math.h>
#include <string.h>

#include <algorithm>
#include <thread>

namespace ge {


int Config::max_q() const {
    int m = 0;
    for (auto& l : layer) m = std::max(m, heads * l.hd);
    return m;
}
int Config::max_kv() const {
    int m = 0;
    for (auto& l : layer) m = std::max(m, l.kv * l.hd);
    return m;
}

cudaError_t noalloc_setup(int device);

int set_error(ge_model* m, int code, const std::string& msg) {
    if (m) m->last_error = msg;
    return code;
}

namespace {

constexpr int kPresizeMaxRows = 262144;  // rows of the workspace reserved at load, at most


bool read_config(const GgufFile& f, Config& c, LoadError& e) {
    if (!f.get_string("general.architecture", c.arch)) c.arch.clear();
    if (c.arch != "gemma-embedding2" && c.arch != "gemma-embedding") {
        e = {GE_ERR_UNSUPPORTED_ARCHITECTURE,
             "unsupported architecture '" + c.arch + "'; supported: gemma-embedding2, gemma-embedding"};
        return false;
    }
    const std::string a = c.arch + ".";
    auto need_int = [&](const std::string& k, int& out) {
        int64_t v;
        if (!f.get_int(a + k, v)) {
            e = {GE_ERR_MISSING_METADATA, "weight file lacks metadata key " + a + k};
            return false;
        }
        out = int(v);
        return true;
    };
    auto need_float = [&](const std::string& k, float& out) {
        if (!f.get_float(a + k, out)) {
            e = {GE_ERR_MISSING_METADATA, "weight file lacks metadata key " + a + k};
            return false;
        }
        return true;
    };
    if (!need_int("block_count", c.layers) || !need_int("embedding_length", c.hidden) ||
        !need_int("attention.head_count", c.heads))
        return false;
    std::vector<int32_t> kvs;
    std::vector<bool> pattern;
    if (!f.get_int_array(a + "attention.head_count_kv", kvs) || int(kvs.size()) != c.layers) {
        e = {GE_ERR_MISSING_METADATA, "weight file lacks metadata key " + a + "attention.head_count_kv"};
        return false;
    }
    if (!f.get_bool_array(a + "attention.sliding_window_pattern", pattern) || int(pattern.size()) != c.layers) {
        e = {GE_ERR_MISSING_METADATA, "weight file lacks metadata key " + a + "attention.sliding_window_pattern"};
        return false;
    }
    int hdg, hds, vg, vs;
    if (!need_int("attention.key_length", hdg) || !need_int("attention.key_length_swa", hds) ||
        !need_int("attention.value_length", vg) || !need_int("attention.value_length_swa", vs))
        return false;
    if (vg != hdg || vs != hds) {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: key and value head sizes differ"};
        return false;
    }
    float rope_g, rope_s;
    if (!need_float("rope.freq_base", rope_g)) return false;
    if (!f.get_float(a + "rope.freq_base_swa", rope_s)) rope_s = rope_g;
    int64_t vocab;
    if (!f.get_string_array_count("tokenizer.ggml.tokens", vocab)) {
        e = {GE_ERR_MISSING_METADATA, "weight file lacks metadata key tokenizer.ggml.tokens"};
        return false;
    }
    c.vocab = int(vocab);
    if (!need_int("embedding_length_out", c.out_dim) || !need_int("feed_forward_length", c.ff) ||
        !need_int("embedding_length_per_layer_input", c.per_layer) ||
        !need_int("attention.sliding_window", c.sliding_window) ||
        !need_float("attention.layer_norm_rms_epsilon", c.eps))
        return false;
    if (!f.get_string("general.name", c.name)) c.name = c.arch;
    int64_t v;
    if (f.get_int("tokenizer.ggml.bos_token_id", v)) c.bos_id = int(v);
    if (f.get_int("tokenizer.ggml.eos_token_id", v)) c.eos_id = int(v);
    c.layer.resize(c.layers);
    for (int i = 0; i < c.layers; i++) {
        LayerCfg& l = c.layer[i];
        l.sliding = pattern[i];
        l.kv = kvs[i];
        l.hd = l.sliding ? hds : hdg;
        l.rope_base = l.sliding ? rope_s : rope_g;
        l.rope_index = -1;
        for (size_t r = 0; r < c.ropes.size(); r++)
            if (c.ropes[r].first == l.hd && c.ropes[r].second == l.rope_base) l.rope_index = int(r);
        if (l.rope_index < 0) {
            l.rope_index = int(c.ropes.size());
            c.ropes.push_back({l.hd, l.rope_base});
        }
    }
    c.emb_scale = sqrtf(float(c.hidden));
    c.pl_scale = 1.0f / sqrtf(float(c.hidden));
    c.has_ple = c.per_layer > 0;
    c.has_output = c.arch == "gemma-embedding2";
    c.has_dense = !c.has_output;
    const GgufTensor* q = f.tensor("blk.0.attn_q.weight");
    c.quant = !q ? "unknown" : q->type == GGML_Q8_0 ? "Q8_0" : q->type == GGML_F16 ? "F16" : q->type == GGML_BF16 ? "BF16" : "F32";
    return true;
}

}  // namespace

// ------------------------------------------------------------------ device memory helpers

static void free_workspace(Workspace& ws) {
    for (void* p : {(void*)ws.tokens, (void*)ws.positions, (void*)ws.seqs, (void*)ws.work, (void*)ws.x, (void*)ws.qkv16,
                    (void*)ws.o16, (void*)ws.d16, (void*)ws.y, (void*)ws.ple, (void*)ws.pooled, (void*)ws.fin, (void*)ws.chunk_base, (void*)ws.pool_partial, (void*)ws.mid, (void*)ws.head_part, (void*)ws.out,
                    (void*)ws.h, (void*)ws.x16, (void*)ws.q, (void*)ws.k, (void*)ws.v, (void*)ws.attn, (void*)ws.act,
                    (void*)ws.g})
        if (p) cudaFree(p);
    for (void* p : {(void*)ws.h_chunk_base, (void*)ws.h_tokens, (void*)ws.h_positions, (void*)ws.h_seqs, (void*)ws.h_work, (void*)ws.h_out,
                    (void*)ws.h_err})
        if (p) cudaFreeHost(p);
    ws = Workspace();
}

// Grows the workspace to at least (rows, seqs, work items) (MetalForward.workspace(forRows:),
// MetalForward.swift:173-178).  Capacities grow geometrically so repeated calls settle.
static cudaError_t ensure_workspace(const Config& c, Device& d, int rows, int seqs, int work) {
    Workspace& ws = d.ws;
    if (ws.cap_rows >= rows && ws.cap_seqs >= seqs && ws.cap_work >= work) return cudaSuccess;
    cudaError_t e = cudaStreamSynchronize(d.stream);
    if (e != cudaSuccess) return e;
    clear_graphs(d);  // captured graphs point into the old buffers
    const int R = std::max(rows, ws.cap_rows + ws.cap_rows / 2 > rows ? round_up(ws.cap_rows + ws.cap_rows / 2, kRowTile) : rows);
    const int S = std::max({seqs, ws.cap_seqs * 2, 16});
    const int W = std::max({work, ws.cap_work * 2, 64});
    free_workspace(ws);
    const size_t d_ = size_t(c.hidden), qd = size_t(c.max_q()), kvd = size_t(c.max_kv());
    const size_t qkvd = qd + 2 * kvd;
    auto A = [&](auto** p, size_t n) -> cudaError_t {
        using T = std::remove_pointer_t<std::remove_reference_t<decltype(*p)>>;
        void* q = nullptr;
        cudaError_t r = cudaMalloc(&q, std::max<size_t>(n, 1) * sizeof(T));
        *p = static_cast<T*>(q);
        return r;
    };
    auto H = [&](auto** p, size_t n) -> cudaError_t {
        using T = std::remove_pointer_t<std::remove_reference_t<decltype(*p)>>;
        void* q = nullptr;
        cudaError_t r = cudaMallocHost(&q, std::max<size_t>(n, 1) * sizeof(T));
        *p = static_cast<T*>(q);
        return r;
    };
    const size_t r = size_t(R);
    cudaError_t err = cudaSuccess;
    auto chk = [&](cudaError_t x) {
        if (err == cudaSuccess) err = x;
    };
    chk(A(&ws.tokens, r));
    chk(A(&ws.positions, r));
    chk(A(&ws.seqs, 2 * size_t(S)));
    chk(A(&ws.work, size_t(W)));
    chk(A(&ws.x, r * d_));
    chk(A(&ws.qkv16, r * qkvd));
    chk(A(&ws.o16, r * d_));
    chk(A(&ws.d16, r * d_));
    chk(A(&ws.y, r * d_));
    chk(A(&ws.h, r * d_));
    chk(A(&ws.q, r * qd));
    chk(A(&ws.k, r * kvd));
    chk(A(&ws.v, r * kvd));
    chk(A(&ws.attn, r * qd));
    chk(A(&ws.act, r * size_t(c.ff)));
    if (c.has_ple) {
        chk(A(&ws.x16, r * d_));
        chk(A(&ws.ple, r * size_t(c.layers) * c.per_layer));
        chk(A(&ws.g, r * size_t(c.per_layer)));
    }
    chk(A(&ws.pooled, size_t(S) * d_));
    chk(A(&ws.fin, size_t(S) * size_t(c.out_dim)));
    chk(A(&ws.chunk_base, size_t(S)));
    chk(A(&ws.pool_partial, (r / kPoolChunkRows + size_t(S)) * d_));
    chk(H(&ws.h_chunk_base, size_t(S)));
    chk(A(&ws.mid, size_t(S) * std::max(c.dense_head, 1)));
    const size_t head_floats = std::max({size_t(dense_head_chunks(c.hidden)) * std::max(c.dense_head, 1),
                                         size_t(dense_head_chunks(std::max(c.dense_head, 1))) * c.out_dim,
                                         size_t(dense_head_chunks(c.hidden)) * c.out_dim, size_t(1)});
    chk(A(&ws.head_part, size_t(S) * head_floats));
    chk(A(&ws.out, size_t(S) * c.out_dim));
    chk(H(&ws.h_tokens, r));
    chk(H(&ws.h_positions, r));
    chk(H(&ws.h_seqs, 2 * size_t(S)));
    chk(H(&ws.h_work, size_t(W)));
    chk(H(&ws.h_out, size_t(S) * std::max(c.out_dim, c.hidden)));
    chk(H(&ws.h_err, 1));
    if (err != cudaSuccess) {
        free_workspace(ws);
        return err;
    }
    ws.cap_rows = R;
    ws.cap_seqs = S;
    ws.cap_work = W;
    auto act = [&](DevActivation& a, __half* p, int cols) {
        a.ptr = p;
        a.rows = R;
        a.cols = cols;
        return encode_activation_map(a);
    };
    bool ok = act(ws.a_h, ws.h, c.hidden) && act(ws.a_act, ws.act, c.ff);
    if (c.has_ple) ok = ok && act(ws.a_x16, ws.x16, c.hidden) && act(ws.a_g, ws.g, c.per_layer);
    ws.attn_maps.clear();
    ws.attn_maps_fused.clear();
    for (auto& l : c.layer) {
        const int key = attn_map_key(l.kv, l.hd);
        bool have = false;
        for (auto& x : ws.attn_maps) have = have || x.first == key;
        if (!have) {
            AttnMaps am, fm;
            ok = ok && encode_attention_maps(am, ws.q, ws.k, ws.v, R, c.heads, l.kv, l.hd);
            ws.attn_maps.push_back({key, am});
            if (l.hd == 256) {  // q, k and v in place in the projection rows (GE_LOAD_FUSED_QKV)
                const int stride = (c.heads + 2 * l.kv) * l.hd;
                const __half* q = ws.qkv16;
                ok = ok && encode_attention_maps(fm, q, q + c.heads * l.hd, q + (c.heads + l.kv) * l.hd, R, c.heads, l.kv,
                                                 l.hd, stride);
                ws.attn_maps_fused.push_back({key, fm});
            }
        }
    }
    ws.a_attn.clear();
    for (auto& l : c.layer) {
        const int cols = c.heads * l.hd;
        bool have = false;
        for (auto& a : ws.a_attn) have = have || a.cols == cols;
        if (!have) {
            DevActivation a;
            ok = ok && act(a, ws.attn, cols);
            ws.a_attn.push_back(a);
        }
    }
    return ok ? cudaSuccess : cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ load
static int load_device(ge_model* m, Device& d, const std::vector<HostWeight>& hw, const std::vector<std::vector<float>>& norms,
                       const std::vector<std::vector<float>>& ropes, const std::vector<float>& dense2,
                       const std::vector<float>& dense3, const std::vector<float>& output, const HostWeight& emb,
                       const HostWeight* plp) {
    const Config& c = m->cfg;
    cudaError_t e = cudaSetDevice(d.ordinal);
    cudaDeviceProp prop;
    if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, d.ordinal);
    if (e != cudaSuccess) return set_error(m, GE_ERR_NO_DEVICE, std::string("cannot use CUDA device: ") + cudaGetErrorString(e));
    if (prop.major != 10)
        return set_error(m, GE_ERR_NO_DEVICE, std::string("device ") + prop.name + " is not an sm_100 (B200-class) GPU");
    d.num_sms = prop.multiProcessorCount;
    d.name = prop.name;
    e = cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking);
    auto fail = [&](cudaError_t x) {
        return set_error(m, x == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                         std::string("device upload failed: ") + cudaGetErrorString(x));
    };
    if (e != cudaSuccess) return fail(e);
    if ((e = dev_alloc(d.allocations, &d.err, 1)) != cudaSuccess || (e = cudaMemset(d.err, 0, sizeof(int))) != cudaSuccess) return fail(e);
    // Token embedding table: int8 plane [V][d] and fp16 scales [V][d/32].
    if ((e = dev_upload(d.allocations, &d.emb_q, emb.q.data(), emb.q.size())) != cudaSuccess) return fail(e);
    if ((e = dev_upload(d.allocations, reinterpret_cast<uint16_t**>(&d.emb_s), emb.scales_t.data(), emb.scales_t.size())) != cudaSuccess)
        return fail(e);
    size_t ni = 0, wi = 0;
    cudaError_t norm_err = cudaSuccess;
    auto norm = [&](float** p) {
        cudaError_t x = dev_upload(d.allocations, p, norms[ni].data(), norms[ni].size());
        if (norm_err == cudaSuccess) norm_err = x;
        ni++;
    };
    d.layers.resize(c.layers);
    for (int l = 0; l < c.layers; l++) {
        LayerDev& L = d.layers[l];
        for (DevWeight* w : {&L.qkv, &L.o, &L.gu, &L.down})
            if ((e = upload_weight(d.allocations, *w, hw[wi++])) != cudaSuccess) return fail(e);
        if (c.has_ple)
            for (DevWeight* w : {&L.inp_gate, &L.proj})
                if ((e = upload_weight(d.allocations, *w, hw[wi++])) != cudaSuccess) return fail(e);
        norm(&L.attn_norm);
        norm(&L.q_norm);
        norm(&L.k_norm);
        norm(&L.post_attn);
        norm(&L.ffn_norm);
        norm(&L.post_ffw);
        if (c.has_ple) {
            norm(&L.post_norm);
            L.out_scale = norms[ni++][0];
        }
    }
    norm(&d.out_norm);
    if (c.has_ple) {
        norm(&d.pl_norm);
        if ((e = upload_weight(d.allocations, d.plp, *plp)) != cudaSuccess) return fail(e);
    }
    if (norm_err != cudaSuccess) return fail(norm_err);
    for (const std::vector<float>& r : ropes) {
        float* p = nullptr;
        if ((e = dev_upload(d.allocations, &p, r.data(), r.size())) != cudaSuccess) return fail(e);
        d.rope.push_back(p);
    }
    if (c.has_dense) {
        if ((e = dev_upload(d.allocations, &d.dense2, dense2.data(), dense2.size())) != cudaSuccess) return fail(e);
        if ((e = dev_upload(d.allocations, &d.dense3, dense3.data(), dense3.size())) != cudaSuccess) return fail(e);
    }
    if (c.has_output && (e = dev_upload(d.allocations, &d.output, output.data(), output.size())) != cudaSuccess) return fail(e);
    if ((e = noalloc_setup(d.ordinal)) != cudaSuccess) return fail(e);
    if ((e = configure_gemm_kernels()) != cudaSuccess || (e = configure_attention_kernels()) != cudaSuccess ||
        (e = configure_audio_kernels()) != cudaSuccess)
        return fail(e);
    return GE_OK;
}

cudaError_t staging_wait(Device& d, int kind) {
    if (!d.staging[kind]) return cudaEventCreateWithFlags(&d.staging[kind], cudaEventDisableTiming);
    return cudaEventSynchronize(d.staging[kind]);
}

cudaError_t staging_done(Device& d, int kind, cudaStream_t stream) { return cudaEventRecord(d.staging[kind], stream); }

static void free_device(Device& d) {
    if (d.stream) {
        cudaSetDevice(d.ordinal);
        cudaStreamSynchronize(d.stream);
    }
    clear_graphs(d);
    free_workspace(d.ws);
    free_vision(d);
    free_audio(d);
    if (d.mm_vectors) cudaFree(d.mm_vectors);
    d.mm_vectors = nullptr;
    d.mm_vectors_cap = 0;
    for (cudaEvent_t& ev : d.staging) {
        if (ev) cudaEventDestroy(ev);
        ev = nullptr;
    }
    for (void* p : d.allocations) cudaFree(p);
    d.allocations.clear();
    if (d.stream) cudaStreamDestroy(d.stream);
    d.stream = nullptr;
}

int load_model(ge_model* m, const char* path, const ge_load_opts* opts) {
    GgufError ge_err;
    if (!path) return set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: weight path is NULL");
    int rc = m->file.open(path, ge_err);
    if (rc) return set_error(m, ge_err.code, ge_err.message);
    m->file_size = int64_t(m->file.size);
    LoadError le{0, ""};
    Config& c = m->cfg;
    if (!read_config(m->file, c, le)) return set_error(m, le.code, le.msg);
    if (c.layers <= 0 || (c.hidden != 512 && c.hidden != 768) || c.ff % 128 || c.heads <= 0)
        return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: unsupported dimensions");
    int kv256 = 0;  // every head-dim-256 layer shares one attention work list
    for (auto& l : c.layer)
        if (l.hd == 256 && kv256 == 0) kv256 = l.kv;
    for (auto& l : c.layer)
        if ((l.hd != 256 && l.hd != 512) || l.kv <= 0 || c.heads % l.kv ||
            c.heads + 2 * l.kv > (l.hd == 256 ? 8 : 6) ||  // the q/k/v norm kernel's slot capacity
            (l.hd == 256 && l.kv != kv256))  // one attention work list for every head-dim-256 layer
            return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: unsupported head layout");
    const GgufFile& f = m->file;
    const int d = c.hidden, ff = c.ff, pl = c.per_layer;
    // ---- shape checks (ModelWeights.init, Weights.swift:100-131)
    const GgufTensor* emb = need_tensor(f, "token_embd.weight", {d, c.vocab}, false, le);
    if (!emb) return set_error(m, le.code, le.msg);
    if (emb->type != GGML_Q8_0)
        return set_error(m, GE_ERR_UNSUPPORTED_TENSOR_TYPE, "tensor token_embd.weight must be Q8_0");
    const GgufTensor *plp = nullptr, *pln = nullptr, *outn, *outw = nullptr, *d2 = nullptr, *d3 = nullptr;
    if (c.has_ple) {
        if (!(plp = need_tensor(f, "per_layer_model_proj.weight", {d, int64_t(pl) * c.layers}, false, le)) ||
            !(pln = need_tensor(f, "per_layer_proj_norm.weight", {pl}, true, le)))
            return set_error(m, le.code, le.msg);
    }
    if (!(outn = need_tensor(f, "output_norm.weight", {d}, true, le))) return set_error(m, le.code, le.msg);
    if (c.has_output) {
        if (!(outw = need_tensor(f, "output.weight", {d, c.out_dim}, false, le))) return set_error(m, le.code, le.msg);
    } else {
        const GgufTensor* t = f.tensor("dense_2.weight");
        if (!t || t->shape.size() != 2) return set_error(m, GE_ERR_MISSING_TENSOR, "weight file lacks tensor dense_2.weight");
        c.dense_head = int(t->shape[1]);
        if (!(d2 = need_tensor(f, "dense_2.weight", {d, c.dense_head}, false, le)) ||
            !(d3 = need_tensor(f, "dense_3.weight", {c.dense_head, c.out_dim}, false, le)))
            return set_error(m, le.code, le.msg);
    }
    struct LT {
        const GgufTensor *attn_norm, *q, *k, *v, *o, *qn, *kn, *pan, *fn, *gate, *up, *down, *pfn, *ig, *proj, *pn, *os;
    };
    std::vector<LT> lt(c.layers);
    for (int i = 0; i < c.layers; i++) {
        const int hd = c.layer[i].hd, qd = c.heads * hd, kvd = c.layer[i].kv * hd;
        const std::string p = "blk." + std::to_string(i) + ".";
        LT& t = lt[i];
        if (!(t.attn_norm = need_tensor(f, p + "attn_norm.weight", {d}, true, le)) ||
            !(t.q = need_tensor(f, p + "attn_q.weight", {d, qd}, false, le)) ||
            !(t.k = need_tensor(f, p + "attn_k.weight", {d, kvd}, false, le)) ||
            !(t.v = need_tensor(f, p + "attn_v.weight", {d, kvd}, false, le)) ||
            !(t.o = need_tensor(f, p + "attn_output.weight", {qd, d}, false, le)) ||
            !(t.qn = need_tensor(f, p + "attn_q_norm.weight", {hd}, true, le)) ||
            !(t.kn = need_tensor(f, p + "attn_k_norm.weight", {hd}, true, le)) ||
            !(t.pan = need_tensor(f, p + "post_attention_norm.weight", {d}, true, le)) ||
            !(t.fn = need_tensor(f, p + "ffn_norm.weight", {d}, true, le)) ||
            !(t.gate = need_tensor(f, p + "ffn_gate.weight", {d, ff}, false, le)) ||
            !(t.up = need_tensor(f, p + "ffn_up.weight", {d, ff}, false, le)) ||
            !(t.down = need_tensor(f, p + "ffn_down.weight", {ff, d}, false, le)) ||
            !(t.pfn = need_tensor(f, p + "post_ffw_norm.weight", {d}, true, le)))
            return set_error(m, le.code, le.msg);
        if (c.has_ple) {
            if (!(t.ig = need_tensor(f, p + "inp_gate.weight", {d, pl}, false, le)) ||
                !(t.proj = need_tensor(f, p + "proj.weight", {pl, d}, false, le)) ||
                !(t.pn = need_tensor(f, p + "post_norm.weight", {d}, true, le)) ||
                !(t.os = need_tensor(f, p + "layer_output_scale.weight", {1}, true, le)))
                return set_error(m, le.code, le.msg);
        }
    }
    // ---- tokenizer (EmbeddingModel.swift:85): a file that names a tokenizer model must carry a
    // valid gemma4 one; a file without tokenizer.ggml.model still loads for token-id input and
    // the text entry points report the missing tokenizer.
    {
        std::string tm;
        if (f.get_string("tokenizer.ggml.model", tm)) {
            std::unique_ptr<ge_tokenizer> tk(new ge_tokenizer);
            if (tk->t.build(f, ge_err)) return set_error(m, ge_err.code, ge_err.message);
            if (tk->t.vocabulary_size() != c.vocab)
                return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: the tokenizer and token_embd.weight disagree on the vocabulary size");
            m->tokenizer = std::move(tk);
        }
    }
    // ---- host-side repack
    const bool want_f16 = !(m->flags & GE_LOAD_Q8_ONLY);
    std::vector<HostWeight> hw;
    for (int i = 0; i < c.layers; i++) {
        const LT& t = lt[i];
        const int hd = c.layer[i].hd, qd = c.heads * hd, kvd = c.layer[i].kv * hd;
        if ((qd + 2 * kvd) % kBN || d % kBN || (2 * ff) % kBN || (pl && pl % kBN))
            return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: projection widths must be multiples of 256");
        // Fused q, k, v projection: rows [Wq; Wk; Wv].
        hw.push_back(build_weight(qd + 2 * kvd, d, want_f16, [&](int r) -> std::pair<const GgufTensor*, int> {
            if (r < qd) return {t.q, r};
            if (r < qd + kvd) return {t.k, r - qd};
            return {t.v, r - qd - kvd};
        }));
        hw.push_back(build_weight(d, qd, want_f16, [&](int r) -> std::pair<const GgufTensor*, int> { return {t.o, r}; }));
        // Gate and up interleaved in blocks of kBN/2 rows, so one output tile holds both halves.
        hw.push_back(build_weight(2 * ff, d, want_f16, [&](int r) -> std::pair<const GgufTensor*, int> {
            const int blk = r / (kBN / 2), off = r % (kBN / 2);
            return {(blk & 1) ? t.up : t.gate, (blk >> 1) * (kBN / 2) + off};
        }));
        hw.push_back(build_weight(d, ff, want_f16, [&](int r) -> std::pair<const GgufTensor*, int> { return {t.down, r}; }));
        if (c.has_ple) {
            hw.push_back(build_weight(pl, d, want_f16, [&](int r) -> std::pair<const GgufTensor*, int> { return {t.ig, r}; }));
            hw.push_back(build_weight(d, pl, want_f16, [&](int r) -> std::pair<const GgufTensor*, int> { return {t.proj, r}; }));
        }
    }
    std::vector<std::vector<float>> norms;
    for (int i = 0; i < c.layers; i++) {
        const LT& t = lt[i];
        for (const GgufTensor* n : {t.attn_norm, t.qn, t.kn, t.pan, t.fn, t.pfn}) norms.push_back(dequant_matrix(*n));
        if (c.has_ple) {
            norms.push_back(dequant_matrix(*t.pn));
            norms.push_back(dequant_matrix(*t.os));
        }
    }
    norms.push_back(dequant_matrix(*outn));
    if (c.has_ple) norms.push_back(dequant_matrix(*pln));
    // RoPE tables (RopeTable.swift:16-31): invFreq in double, cos/sin rounded to float.
    std::vector<std::vector<float>> ropes;
    for (auto& rp : c.ropes) {
        const int hd = rp.first, pairs = hd / 2;
        std::vector<float> tab(size_t(c.max_tokens) * pairs * 2);
        for (int i = 0; i < pairs; i++) {
            const double inv = pow(double(rp.second), -2.0 * double(i) / double(hd));
            for (int pos = 0; pos < c.max_tokens; pos++) {
                const double th = double(pos) * inv;
                tab[(size_t(pos) * pairs + i) * 2] = float(cos(th));
                tab[(size_t(pos) * pairs + i) * 2 + 1] = float(sin(th));
            }
        }
        ropes.push_back(std::move(tab));
    }
    std::vector<float> dense2, dense3, output;
    if (c.has_dense) {
        dense2 = dequant_matrix(*d2);
        dense3 = dequant_matrix(*d3);
    }
    if (c.has_output) output = dequant_matrix(*outw);
    // Embedding table planes: int8 [V][d] and scales [V][d/32] (row-major, not transposed).
    HostWeight embw;
    embw.N = c.vocab;
    embw.K = d;
    embw.q.resize(size_t(c.vocab) * d);
    embw.scales_t.resize(size_t(c.vocab) * (d / 32));
    parallel_rows(c.vocab, [&](int64_t r) {
        const uint8_t* p = emb->data + r * (d / 32) * 34;
        for (int b = 0; b < d / 32; b++) {
            memcpy(&embw.scales_t[size_t(r) * (d / 32) + b], p + b * 34, 2);
            memcpy(&embw.q[size_t(r) * d + b * 32], p + b * 34 + 2, 32);
        }
    });
    HostWeight plpw;
    if (c.has_ple)
        plpw = build_weight(pl * c.layers, d, true, [&](int r) -> std::pair<const GgufTensor*, int> { return {plp, r}; });

    // ---- devices
    uint32_t mask = opts ? opts->device_mask : 0;
    if (!mask) mask = 1;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
        return set_error(m, GE_ERR_NO_DEVICE, "no CUDA device is available");
    for (int i = 0; i < 32; i++)
        if (mask & (1u << i)) {
            if (i >= count) return set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: device " + std::to_string(i) + " does not exist");
            Device dv;
            dv.ordinal = i;
            m->devs.push_back(dv);
        }
    if (m->devs.size() > 1) {
        m->workers = std::make_unique<DeviceWorkers>();
        m->workers->start(int(m->devs.size()));
    }
    for (auto& dv : m->devs) {
        rc = load_device(m, dv, hw, norms, ropes, dense2, dense3, output, embw, c.has_ple ? &plpw : nullptr);
        if (rc) return rc;
        // The workspace is sized at load for a whole batch of the token budget (or one longest
        // sequence), so a stream of batches within the budget never stops to reallocate it,
        // which would also drop every captured graph.  Larger packed batches still grow it.
        const int rows = round_up(std::min(std::max(m->budget, c.max_tokens), kPresizeMaxRows), kRowTile);
        const int seqs = 1024;
        cudaError_t e = cudaSetDevice(dv.ordinal);
        if (e == cudaSuccess) e = ensure_workspace(c, dv, rows, seqs, 16 * rows + 8 * seqs + 1024);
        if (e != cudaSuccess)
            return set_error(m, e == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                             std::string("GPU execution failed: workspace: ") + cudaGetErrorString(e));
    }
    return GE_OK;
}

void free_model(ge_model* m) {
    if (m->workers) m->workers->stop();
    for (auto& d : m->devs) free_device(d);
    m->devs.clear();
}

// ------------------------------------------------------------------ device workers
void DeviceWorkers::start(int n) {
    stop_ = false;
    for (int i = 0; i < n; i++) threads_.emplace_back(&DeviceWorkers::loop, this, i);
}

void DeviceWorkers::stop() {
    {
        std::lock_guard<std::mutex> g(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : threads_) t.join();
    threads_.clear();
}

void DeviceWorkers::loop(int i) {
    uint64_t seen = 0;
    for (;;) {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || generation_ != seen; });
        if (stop_) return;
        seen = generation_;
        const bool mine = i < active_;
        const std::function<void(int)>* task = task_;
        lk.unlock();
        if (mine) (*task)(i);
        lk.lock();
        if (mine && --pending_ == 0) done_cv_.notify_all();
    }
}

void DeviceWorkers::run(int n, const std::function<void(int)>& fn) {
    if (n <= 0) return;
    std::unique_lock<std::mutex> lk(mu_);
    task_ = &fn;
    active_ = std::min(n, int(threads_.size()));
    pending_ = active_;
    generation_++;
    cv_.notify_all();
    done_cv_.wait(lk, [&] { return pending_ == 0; });
    task_ = nullptr;
}

// ------------------------------------------------------------------ graphs
constexpr size_t kMaxGraphs = 16;

GraphEntry* find_graph(Device& d, const GraphKey& k) {
    for (auto& g : d.graphs)
        if (g.key == k) {
            g.last_use = ++d.graph_clock;
            return &g;
        }
    return nullptr;
}

void store_graph(Device& d, const GraphKey& k, cudaGraphExec_t exec, int64_t launches) {
    if (d.graphs.size() >= kMaxGraphs) {
        auto lru = std::min_element(d.graphs.begin(), d.graphs.end(),
                                    [](const GraphEntry& a, const GraphEntry& b) { return a.last_use < b.last_use; });
        cudaGraphExecDestroy(lru->exec);
        d.graphs.erase(lru);
    }
    GraphEntry g;
    g.key = k;
    g.exec = exec;
    g.launches = launches;
    g.last_use = ++d.graph_clock;
    d.graphs.push_back(g);
}

constexpr size_t kMaxSeenKeys = 64;

bool seen_before(Device& d, const GraphKey& k) {
    for (auto it = d.seen_keys.begin(); it != d.seen_keys.end(); ++it)
        if (*it == k) {
            d.seen_keys.erase(it);
            return true;
        }
    if (d.seen_keys.size() >= kMaxSeenKeys) d.seen_keys.erase(d.seen_keys.begin());
    d.seen_keys.push_back(k);
    return false;
}

void clear_graphs(Device& d) {
    for (auto& g : d.graphs) cudaGraphExecDestroy(g.exec);
    d.graphs.clear();
    d.seen_keys.clear();
}

// ------------------------------------------------------------------ forward
int run_forward(ge_model* m, Device& d, const ForwardArgs& a) {
    const Config& c = m->cfg;
    cudaError_t e = cudaSetDevice(d.ordinal);
    cudaStream_t st = a.stream ? a.stream : d.stream;
    auto report = [&](int code, const std::string& msg) {
        if (a.error) *a.error = msg;
        else m->last_error = msg;
        return code;
    };
    auto gpu_fail = [&](cudaError_t x, const char* what) {
        return report(x == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                      std::string("GPU execution failed: ") + what + ": " + cudaGetErrorString(x));
    };
    if (e != cudaSuccess) return gpu_fail(e, "cudaSetDevice");
    // Kernels of this forward overlap their set-up with their predecessor's tail unless disabled.
    struct LaunchPolicy {
        explicit LaunchPolicy(bool on) { set_programmatic_launch(on); }
        ~LaunchPolicy() { set_programmatic_launch(false); }
    } policy(!(m->flags & GE_LOAD_NO_PDL));
    const int ntok = a.ntok, nseq = a.nseq;
    const int rows = std::max(kRowTile, round_up(ntok, kRowTile));
    // Attention work stored back to back, each part starting on 16 bytes: the tensor-core
    // kernel's schedules (items of T tokens x the query heads of one KV head, spread over CTAs
    // by key blocks) for each kind of layer the model has: schedule 2 * (hd == 512) + global,
    // i.e. sliding and global head-dim-256 layers, then sliding and global head-dim-512 layers.
    static_assert(sizeof(ge_seq) == 8, "ge_seq is a (start, length) pair of uint32");
    const uint32_t* seq_pairs = reinterpret_cast<const uint32_t*>(a.seqs);
    const int hw_slide = c.sliding_window / 2;
    int kind_kv[4] = {0, 0, 0, 0};  // KV heads of the layers of each schedule (0: no such layer)
    for (auto& l : c.layer) kind_kv[2 * (l.hd == 512) + (l.sliding ? 0 : 1)] = l.kv;
    int sched[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // (items, CTAs) of each schedule
    int words[4] = {0, 0, 0, 0}, work_at[4] = {0, 0, 0, 0};
    int work_words = 0;
    for (int k = 0; k < 4; k++) {
        work_at[k] = work_words;
        if (!kind_kv[k]) continue;
        words[k] = build_attention_work(seq_pairs, nseq, kind_kv[k], c.heads / kind_kv[k], (k & 1) ? 0 : hw_slide,
                                        d.num_sms, nullptr, &sched[2 * k + 1], k >= 2 ? 512 : 256);
        sched[2 * k] = words[k] ? (words[k] - sched[2 * k + 1] - 1) / 4 : 0;
        work_words += (words[k] + 3) & ~3;
    }
    if ((e = staging_wait(d, kStageText)) != cudaSuccess) return gpu_fail(e, "staging");
    if ((e = ensure_workspace(c, d, rows, nseq, work_words)) != cudaSuccess) return gpu_fail(e, "workspace");
    Workspace& ws = d.ws;
    int64_t launches = 0;
    // ---- inputs
    int max_chunks = 0;
    uint32_t chunk_total = 0;
    for (int s = 0; s < nseq; s++) {
        ws.h_seqs[2 * s] = a.seqs[s].start;
        ws.h_seqs[2 * s + 1] = a.seqs[s].length;
        ws.h_chunk_base[s] = chunk_total;
        const int ch = pool_chunks(a.seqs[s].length);
        chunk_total += uint32_t(ch);
        max_chunks = std::max(max_chunks, ch);
    }
    for (int k = 0; k < 4; k++)
        if (words[k])
            build_attention_work(seq_pairs, nseq, kind_kv[k], c.heads / kind_kv[k], (k & 1) ? 0 : hw_slide, d.num_sms,
                                 ws.h_work + work_at[k], nullptr, k >= 2 ? 512 : 256);
    const int32_t* tokens = ws.tokens;
    int64_t h2d = int64_t(nseq) * 8 + int64_t(work_words) * 4 + int64_t(nseq) * 4;  // seqs, work, chunk bases
    if (a.tokens_on_device) {
        tokens = a.tokens;
    } else {
        h2d += int64_t(ntok) * 4;
        memcpy(ws.h_tokens, a.tokens, size_t(ntok) * 4);
        if ((e = cudaMemcpyAsync(ws.tokens, ws.h_tokens, size_t(ntok) * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
            return gpu_fail(e, "token upload");
    }
    if (a.positions == nullptr) launches++;  // the positions kernel below
    if ((e = cudaMemcpyAsync(ws.seqs, ws.h_seqs, size_t(nseq) * 8, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = cudaMemcpyAsync(ws.work, ws.h_work, size_t(work_words) * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = cudaMemcpyAsync(ws.chunk_base, ws.h_chunk_base, size_t(nseq) * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
        return gpu_fail(e, "batch upload");
    if (a.positions) {
        h2d += int64_t(ntok) * 4;
        memcpy(ws.h_positions, a.positions, size_t(ntok) * 4);
        e = cudaMemcpyAsync(ws.positions, ws.h_positions, size_t(ntok) * 4, cudaMemcpyHostToDevice, st);
    } else {
        e = launch_positions(ws.seqs, nseq, ws.positions, st);
    }
    if (e == cudaSuccess) e = staging_done(d, kStageText, st);
    if (e != cudaSuccess) return gpu_fail(e, "positions");

    cudaStream_t ks = st;  // the stream kernels are launched on (the capture stream while capturing)
    // ---- layers (MetalForward.encode, MetalForward.swift:364-423)
    const int D = c.hidden;
    // Every GEMM reads the fp16-resident weights unless the model keeps only the Q8_0 planes: the
    // in-shared-memory dequantisation was measured slower at every batch size from 128 rows up
    // (bench.py's q8_gemm sweep), where it also streams fewer weight bytes.
    const bool q8 = (m->flags & GE_LOAD_Q8_ONLY) != 0;
    auto gemm = [&](const DevActivation& A, const DevWeight& W, void* out, int ldo, int epi, const float* aux = nullptr,
                    int ldaux = 0) {
        GemmLaunch g;
        g.a = &A;
        g.w = &W;
        g.m_rows = rows;
        g.out = out;
        g.ldo = ldo;
        g.epilogue = epi;
        g.aux = aux;
        g.ldaux = ldaux;
        g.use_q8 = q8;
        if (m->flags & GE_LOAD_SINGLE_CTA_GEMM) g.mode = GEMM_SINGLE;
        g.err = d.err;
        g.num_sms = d.num_sms;
        return launch_gemm(g, ks);
    };
    // A projection fused with the residual step that follows it (x += rmsnorm(t) * w_post,
    // then the next norm into h16 or y32): one launch instead of a GEMM and k_residual_norm,
    // on request (GE_LOAD_FUSED_RESIDUAL).  Measured on B200 at 19.5k tokens it takes about
    // as long as the pair it replaces: the A and B tiles each 128 x 256 tile reloads, plus the
    // residual stream in and out, saturate the SM's L2 port.
    const bool fused = (m->flags & GE_LOAD_FUSED_RESIDUAL) != 0;
    // The q/k/v projection of a head-dim-256 layer with its per-head norms and RoPE in the GEMM
    // epilogue (EPI_QKV), attention reading q, k and v in place from the projection rows.
    // On request (GE_LOAD_FUSED_QKV).  Measured on B200 at 19.5k tokens: 61 us per layer on single
    // CTAs against 38 + 25 us for the projection and k_qkv_norm_rope, and 71 us on CTA pairs
    // against 35 + 22 us: the epilogue (one thread per token, two passes over the 256 columns,
    // each thread reading its own position's RoPE row) outlasts the K = 768 main loop it overlaps.
    const bool fused_qkv = (m->flags & GE_LOAD_FUSED_QKV) != 0;
    auto gemm_qkv = [&](const LayerDev& L, const LayerCfg& lc) {
        GemmLaunch g;
        g.a = &ws.a_h;
        g.w = &L.qkv;
        g.m_rows = rows;
        g.out = ws.qkv16;
        g.ldo = L.qkv.N;
        g.epilogue = EPI_QKV;
        g.use_q8 = q8;
        if (m->flags & GE_LOAD_SINGLE_CTA_GEMM) g.mode = GEMM_SINGLE;
        g.err = d.err;
        g.num_sms = d.num_sms;
        g.positions = ws.positions;
        g.rope = d.rope[lc.rope_index];
        g.q_norm = L.q_norm;
        g.k_norm = L.k_norm;
        g.eps = c.eps;
        g.ntok = ntok;
        g.heads = c.heads;
        g.kv_heads = lc.kv;
        return launch_gemm(g, ks);
    };
    auto gemm_residual = [&](const DevActivation& A, const DevWeight& W, const float* w_post, float scale,
                             const float* w_next, __half* h16, float* y32) {
        GemmLaunch g;
        g.a = &A;
        g.w = &W;
        g.m_rows = rows;
        g.out = nullptr;
        g.ldo = W.N;
        g.epilogue = EPI_RESIDUAL;
        g.use_q8 = q8;
        if (m->flags & GE_LOAD_SINGLE_CTA_GEMM) g.mode = GEMM_SINGLE;
        g.err = d.err;
        g.num_sms = d.num_sms;
        g.x = ws.x;
        g.w_post = w_post;
        g.scale = scale;
        g.w_next = w_next;
        g.eps = c.eps;
        g.h16 = h16;
        g.y32 = y32;
        return launch_gemm(g, ks);
    };
#define CK(expr, what)                                  \
    do {                                                \
        cudaError_t e_ = (expr);                        \
        if (e_ != cudaSuccess) return gpu_fail(e_, what); \
    } while (0)
    // Every kernel launch goes through K: it counts launches and, when profiling, times the
    // first launch of each kernel class over `reps` back-to-back repetitions (the reference's
    // Profiler, Metal/Profiler.swift:16-88).
    auto K = [&](const char* name, double flops, double bytes, auto&& fn, int kernels = 1) -> cudaError_t {
        if (a.profile) {
            ProfileEntry* pe = a.profile->find(name);
            if (pe) {
                pe->occurrences++;
            } else {
                // The repetitions are captured into a CUDA graph and the graph is timed, so the
                // time is the kernels' own and not the host's launch rate (a short kernel
                // launched back to back from the host measures the host).
                cudaGraph_t graph = nullptr;
                cudaGraphExec_t exec = nullptr;
                cudaError_t x = cudaStreamBeginCapture(ks, cudaStreamCaptureModeThreadLocal);
                if (x != cudaSuccess) return x;
                for (int r = 0; r < a.profile->reps && x == cudaSuccess; r++) {
                    x = fn();
                    launches += kernels;
                }
                const cudaError_t xe = cudaStreamEndCapture(ks, &graph);
                if (x == cudaSuccess) x = xe;
                if (x == cudaSuccess) x = cudaGraphInstantiate(&exec, graph, 0);
                if (graph) cudaGraphDestroy(graph);
                if (x != cudaSuccess) return x;
                cudaEvent_t e0 = nullptr, e1 = nullptr;
                x = cudaEventCreate(&e0);
                if (x == cudaSuccess) x = cudaEventCreate(&e1);
                if (x == cudaSuccess) x = cudaGraphLaunch(exec, ks);  // warm-up run of the repetitions
                if (x == cudaSuccess) x = cudaEventRecord(e0, ks);
                if (x == cudaSuccess) x = cudaGraphLaunch(exec, ks);
                if (x == cudaSuccess) x = cudaEventRecord(e1, ks);
                if (x == cudaSuccess) x = cudaEventSynchronize(e1);
                float ms = 0.f;
                if (x == cudaSuccess) x = cudaEventElapsedTime(&ms, e0, e1);
                if (e0) cudaEventDestroy(e0);
                if (e1) cudaEventDestroy(e1);
                cudaGraphExecDestroy(exec);
                if (x != cudaSuccess) return x;
                launches += int64_t(kernels) * a.profile->reps;  // the timed run
                a.profile->add(name, double(ms) / a.profile->reps, flops, bytes);
                return cudaSuccess;
            }
        }
        launches += kernels;
        return fn();
    };
    // Algorithmic work of a GEMM launch: the rows that hold tokens, not the padding.
    auto gemm_flops = [&](const DevWeight& W) { return 2.0 * ntok * W.N * double(W.K); };
    auto gemm_bytes = [&](const DevWeight& W, double out_elem_bytes) {
        return double(ntok) * W.K * 2 + double(W.N) * W.K * (q8 ? 34.0 / 32.0 : 2.0) + double(ntok) * W.N * out_elem_bytes;
    };
    // Keys each query sees, summed over the batch, for the attention FLOP count.
    auto visible_keys = [&](int hw) {
        double sum = 0;
        for (int s = 0; s < nseq; s++) {
            const int64_t n = a.seqs[s].length;
            if (hw <= 0) {
                sum += double(n) * n;
                continue;
            }
            for (int64_t i = 0; i < n; i++) sum += double(std::min<int64_t>(n - 1, i + hw) - std::max<int64_t>(0, i - hw) + 1);
        }
        return sum;
    };
    const double vk_sliding = a.profile ? visible_keys(c.sliding_window / 2) : 0, vk_global = a.profile ? visible_keys(0) : 0;

    auto launch_all = [&]() -> int {
        CK(K("embed", 0, double(ntok) * D * (1 + 2.0 / 32 + 4 + 2),
             [&] {
                 return launch_embed(tokens, ntok, rows, d.emb_q, d.emb_s, D, c.emb_scale, ws.x, c.has_ple ? ws.x16 : nullptr,
                                     d.layers[0].attn_norm, c.eps, ws.h, ks, a.vectors);
             }),
           "embed");
        if (c.has_ple) {
            // ple = rmsnorm_pl(x0 * Wplp^T / sqrt(d)) for every layer at once (CPUReference.swift:206-210).
            const int plw = c.per_layer * c.layers;
            CK(K("gemm_per_layer_inputs", gemm_flops(d.plp), gemm_bytes(d.plp, 4),
                 [&] { return gemm(ws.a_x16, d.plp, ws.ple, plw, EPI_F32); }),
               "per-layer projection");
            CK(K("per_layer_norm", 0, double(ntok) * plw * 8,
                 [&] { return launch_rmsnorm_rows(ws.ple, rows * c.layers, c.per_layer, c.pl_scale, d.pl_norm, c.eps, ws.ple, ks); }),
               "per-layer norm");
        }
        for (int l = 0; l < c.layers; l++) {
            const LayerCfg& lc = c.layer[l];
            const LayerDev& L = d.layers[l];
            const int qd = c.heads * lc.hd;
            const bool in_place = lc.hd == 256 && fused_qkv;
            if (in_place) {
                CK(K("gemm_qkv_norm_rope", gemm_flops(L.qkv), gemm_bytes(L.qkv, 2), [&] { return gemm_qkv(L, lc); }),
                   "qkv projection with norms and rope");
            } else {
                // The projection stores fp16; the per-head norms and RoPE read it back warp per row.
                CK(K("gemm_qkv", gemm_flops(L.qkv), gemm_bytes(L.qkv, 2),
                     [&] { return gemm(ws.a_h, L.qkv, ws.qkv16, L.qkv.N, EPI_F16); }),
                   "qkv projection");
                CK(K("qkv_norm_rope", 0, double(ntok) * L.qkv.N * 4,
                     [&] {
                         return launch_qkv_norm_rope(ws.qkv16, ntok, rows, c.heads, lc.kv, lc.hd, L.q_norm, L.k_norm,
                                                     ws.positions, d.rope[lc.rope_index], c.eps, ws.q, ws.k, ws.v, ks);
                     }),
                   "q/k/v norm and rope");
            }
            AttnLaunch al;
            al.q = in_place ? ws.qkv16 : ws.q;
            al.k = in_place ? ws.qkv16 + c.heads * lc.hd : ws.k;
            al.v = in_place ? ws.qkv16 + (c.heads + lc.kv) * lc.hd : ws.v;
            al.out = ws.attn;
            const int k = 2 * (lc.hd == 512) + (lc.sliding ? 0 : 1);
            al.work = ws.work + work_at[k];
            al.work_items = sched[2 * k + 1];
            al.sched_items = sched[2 * k];
            al.num_sms = d.num_sms;
            al.heads = c.heads;
            al.kv_heads = lc.kv;
            al.hd = lc.hd;
            al.half_window = lc.sliding ? c.sliding_window / 2 : 0;
            al.err = d.err;
            for (auto& x : (in_place ? ws.attn_maps_fused : ws.attn_maps))
                if (x.first == attn_map_key(lc.kv, lc.hd)) al.maps = &x.second;
            CK(K(lc.sliding ? "attention_sliding" : "attention_global",
                 4.0 * c.heads * lc.hd * (lc.sliding ? vk_sliding : vk_global),
                 double(ntok) * (2.0 * qd + 2.0 * lc.kv * lc.hd) * 2, [&] { return launch_attention(al, ks); }),
               "attention");
            const DevActivation* aa = nullptr;
            for (auto& x : ws.a_attn)
                if (x.cols == qd) aa = &x;
            if (fused) {
                CK(K("gemm_o_residual", gemm_flops(L.o), gemm_bytes(L.o, 10),
                     [&] { return gemm_residual(*aa, L.o, L.post_attn, 1.0f, L.ffn_norm, ws.h, nullptr); }),
                   "attention output and residual");
            } else {
                CK(K("gemm_o", gemm_flops(L.o), gemm_bytes(L.o, 2), [&] { return gemm(*aa, L.o, ws.o16, D, EPI_F16); }),
                   "attention output");
                if (c.has_ple) {
                    CK(K("residual_norm", 0, double(ntok) * D * 12,
                         [&] {
                             return launch_residual_norm(ws.x, ws.o16, rows, D, L.post_attn, 1.0f, L.ffn_norm, c.eps,
                                                         ws.h, nullptr, nullptr, ks);
                         }),
                       "post-attention residual");
                } else {
                    // The attention residual x1 = x + rmsnorm(t_o) * w feeds only the FFN norm
                    // here; the FFN residual recomputes it from x and t_o instead of a store
                    // and a reload (8 + 14 bytes per element instead of 12 + 12).
                    CK(K("residual_attn", 0, double(ntok) * D * 8,
                         [&] {
                             ResidualStep r;
                             r.x = ws.x;
                             r.t = ws.o16;
                             r.w_post = L.post_attn;
                             r.store_x = false;
                             r.w_next = L.ffn_norm;
                             r.eps = c.eps;
                             r.h16 = ws.h;
                             return launch_residual(r, rows, D, ks);
                         }),
                       "post-attention residual");
                }
            }
            CK(K("gemm_gate_up", gemm_flops(L.gu), gemm_bytes(L.gu, 1), [&] { return gemm(ws.a_h, L.gu, ws.act, c.ff, EPI_GEGLU); }),
               "gate/up projection");
            const bool last = l + 1 == c.layers;
            const float* next = last ? d.out_norm : d.layers[l + 1].attn_norm;
            if (c.has_ple) {
                CK(K("gemm_down", gemm_flops(L.down), gemm_bytes(L.down, 2),
                     [&] { return gemm(ws.a_act, L.down, ws.o16, D, EPI_F16); }),
                   "down projection");
                CK(K("residual_norm", 0, double(ntok) * D * 12,
                     [&] {
                         return launch_residual_norm(ws.x, ws.o16, rows, D, L.post_ffw, 1.0f, nullptr, c.eps, nullptr, nullptr,
                                                     ws.x16, ks);
                     }),
                   "post-ffn residual");
                CK(K("gemm_inp_gate", gemm_flops(L.inp_gate), gemm_bytes(L.inp_gate, 2),
                     [&] {
                         return gemm(ws.a_x16, L.inp_gate, ws.g, c.per_layer, EPI_GELU_MUL, ws.ple + size_t(l) * c.per_layer,
                                     c.per_layer * c.layers);
                     }),
                   "per-layer gate");
                if (fused) {
                    CK(K("gemm_proj_residual", gemm_flops(L.proj), gemm_bytes(L.proj, last ? 12 : 10),
                         [&] {
                             return gemm_residual(ws.a_g, L.proj, L.post_norm, L.out_scale, next, last ? nullptr : ws.h,
                                                  last ? ws.y : nullptr);
                         }),
                       "per-layer projection and residual");
                } else {
                    CK(K("gemm_proj", gemm_flops(L.proj), gemm_bytes(L.proj, 2),
                         [&] { return gemm(ws.a_g, L.proj, ws.o16, D, EPI_F16); }),
                       "per-layer projection");
                    CK(K("residual_norm", 0, double(ntok) * D * 12,
                         [&] {
                             return launch_residual_norm(ws.x, ws.o16, rows, D, L.post_norm, L.out_scale, next, c.eps,
                                                         last ? nullptr : ws.h, last ? ws.y : nullptr, nullptr, ks);
                         }),
                       "per-layer residual");
                }
            } else if (fused) {
                CK(K("gemm_down_residual", gemm_flops(L.down), gemm_bytes(L.down, last ? 12 : 10),
                     [&] {
                         return gemm_residual(ws.a_act, L.down, L.post_ffw, 1.0f, next, last ? nullptr : ws.h,
                                              last ? ws.y : nullptr);
                     }),
                   "down projection and residual");
            } else {
                CK(K("gemm_down", gemm_flops(L.down), gemm_bytes(L.down, 2),
                     [&] { return gemm(ws.a_act, L.down, ws.d16, D, EPI_F16); }),
                   "down projection");
                CK(K("residual_ffn", 0, double(ntok) * D * 14,
                     [&] {
                         ResidualStep r;
                         r.x = ws.x;
                         r.t = ws.o16;
                         r.w_post = L.post_attn;
                         r.t2 = ws.d16;
                         r.w_post2 = L.post_ffw;
                         r.w_next = next;
                         r.eps = c.eps;
                         r.h16 = last ? nullptr : ws.h;
                         r.y32 = last ? ws.y : nullptr;
                         return launch_residual(r, rows, D, ks);
                     }),
                   "post-ffn residual");
            }
            if (a.trace_layer == l) break;
        }
        // ---- pooling and head
        if (a.trace_layer < -1) {
            CK(K("mean_pool", 0, double(ntok) * D * 4, [&] {
                     return launch_mean_pool(ws.y, D, ws.seqs, nseq, max_chunks, ws.chunk_base, ws.pool_partial,
                                             ws.pooled, ks);
                 }, 2),
               "mean pool");
            // 64 x 64 tiles over 256-wide K chunks, two launches each (launch_dense_head), where
            // the widths allow; otherwise the scratch-free kernels
            auto head = [&](const float* in, const float* w, int N, int Kd, float* out) {
                if (N % 64 == 0 && Kd % 256 == 0) return launch_dense_head(in, nseq, w, N, Kd, ws.head_part, out, ks);
                return launch_dense_f32(in, nseq, w, N, Kd, out, ks);
            };
            auto head_launches = [&](int N, int Kd) { return (N % 64 == 0 && Kd % 256 == 0) ? 2 : 1; };
            if (c.has_dense) {
                CK(K("dense_head", 2.0 * nseq * D * c.dense_head, double(D) * c.dense_head * 4,
                     [&] { return head(ws.pooled, d.dense2, c.dense_head, D, ws.mid); }, head_launches(c.dense_head, D)),
                   "dense head");
                CK(K("dense_head_out", 2.0 * nseq * D * c.dense_head, double(D) * c.dense_head * 4,
                     [&] { return head(ws.mid, d.dense3, c.out_dim, c.dense_head, ws.out); },
                     head_launches(c.out_dim, c.dense_head)),
                   "dense head");
            } else {
                CK(K("output_projection", 2.0 * nseq * D * c.out_dim, double(D) * c.out_dim * 4,
                     [&] { return head(ws.pooled, d.output, c.out_dim, D, ws.out); }, head_launches(c.out_dim, D)),
                   "output projection");
            }
            if (a.finish_dims > 0)
                CK(K("finish", 0, double(nseq) * (c.out_dim + a.finish_dims) * 4,
                     [&] {
                         return launch_finish_rows(ws.out, nseq, c.out_dim, a.finish_dims, a.finish_normalise ? 1 : 0,
                                                   ws.fin, ks);
                     }),
                   "finish");
        }
        return GE_OK;
    };
    // Captured CUDA graphs replay the whole launch sequence of a batch shape with one call
    // (kernel arguments, tensor maps included, are fixed per workspace and shape).  A shape is
    // captured the second time it runs: the first run launches directly, so a stream of
    // distinct batches (every new length mix is a new shape) costs no capture it never replays.
    bool use_graph = !(m->flags & GE_LOAD_NO_GRAPHS) && !a.profile && a.trace_layer < -1;
    GraphKey gk;
    gk.rows = rows;
    gk.ntok = ntok;
    gk.nseq = nseq;
    gk.pool_chunks = max_chunks;
    for (int k = 0; k < 8; k++) gk.sched[k] = sched[k];
    gk.tokens = reinterpret_cast<uintptr_t>(tokens);
    gk.vectors = reinterpret_cast<uintptr_t>(a.vectors);
    gk.finish = a.trace_layer < -1 && a.finish_dims > 0 ? 2 * a.finish_dims + (a.finish_normalise ? 1 : 0) : 0;
    GraphEntry* ge_ = use_graph ? find_graph(d, gk) : nullptr;
    if (use_graph && !ge_ && !seen_before(d, gk)) use_graph = false;
    if (ge_) {
        if ((e = cudaGraphLaunch(ge_->exec, st)) != cudaSuccess) return gpu_fail(e, "graph launch");
        launches += ge_->launches;
    } else if (use_graph) {
        ks = d.stream;
        const int64_t before = launches;
        if ((e = cudaStreamBeginCapture(ks, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
            return gpu_fail(e, "graph capture");
        const int rc = launch_all();
        cudaGraph_t graph = nullptr;
        e = cudaStreamEndCapture(ks, &graph);
        if (rc != GE_OK) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (e != cudaSuccess) return gpu_fail(e, "graph capture");
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return gpu_fail(e, "graph instantiation");
        store_graph(d, gk, exec, launches - before);
        m->graph_captures++;
        if ((e = cudaGraphLaunch(exec, st)) != cudaSuccess) return gpu_fail(e, "graph launch");
    } else {
        const int rc = launch_all();
        if (rc != GE_OK) return rc;
    }
    const bool finished = a.trace_layer < -1 && a.finish_dims > 0;
    const float* result = a.trace_layer >= 0 ? ws.x : a.trace_layer == -1 ? ws.y : finished ? ws.fin : ws.out;
    const int width = a.trace_layer >= -1 ? D : finished ? a.finish_dims : c.out_dim;
    const size_t out_elems = a.trace_layer >= -1 ? size_t(ntok) * D : size_t(nseq) * width;
    float* host_out = a.trace_layer >= -1 ? a.trace_out : a.out;
    m->launches += launches;
    m->h2d_bytes += h2d;
    if (a.out_on_device && a.trace_layer < -1) {
        CK(cudaMemcpyAsync(a.out, result, out_elems * 4, cudaMemcpyDeviceToDevice, st), "result copy");
        return GE_OK;
    }
    CK(cudaMemcpyAsync(ws.h_err, d.err, sizeof(int), cudaMemcpyDeviceToHost, st), "error readback");
    m->d2h_bytes += int64_t(sizeof(int)) + int64_t(out_elems) * 4;
    if (a.trace_layer >= -1) {
        // The trace spans ntok rows of D, which may exceed the pooled staging buffer.
        CK(cudaMemcpyAsync(host_out, result, out_elems * 4, cudaMemcpyDeviceToHost, st), "trace readback");
        CK(cudaStreamSynchronize(st), "synchronize");
    } else {
        CK(cudaMemcpyAsync(ws.h_out, result, out_elems * 4, cudaMemcpyDeviceToHost, st), "result readback");
        CK(cudaStreamSynchronize(st), "synchronize");
        memcpy(host_out, ws.h_out, out_elems * 4);
    }
#undef CK
    if (*ws.h_err) {
        const int code = *ws.h_err;
        cudaMemset(d.err, 0, sizeof(int));
        return report(code, "GPU execution failed: a device-side wait timed out");
    }
    return GE_OK;
}

}  // namespace ge
