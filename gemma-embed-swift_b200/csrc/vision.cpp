// vision.cpp -- the gemma4v image encoder on the GPU: configuration and weight checks, the
// repack of its weights into the device layout, its workspace, and its forward pass.
//
// Reference: VisionConfig.init (Model/VisionConfig.swift:42-81), VisionWeights.init
// (Model/VisionWeights.swift:37-83), VisionTower.upload / encode (Metal/VisionTower.swift:121-185).
#include <math.h>
#include <string.h>

#include <algorithm>
#include <cmath>

#include "model.hpp"
#include "weights.hpp"

namespace ge {

namespace {

// VisionConfig.init (VisionConfig.swift:42-81).
bool read_vision_config(const GgufFile& f, VisionConfig& c, LoadError& e) {
    std::string arch, proj;
    f.get_string("general.architecture", arch);
    if (arch != "clip") {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: image encoder architecture is '" + arch + "', expected clip"};
        return false;
    }
    f.get_string("clip.vision.projector_type", proj);
    if (proj != "gemma4v") {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: image projector is '" + proj + "', expected gemma4v"};
        return false;
    }
    auto missing = [&](const std::string& key) {
        e = {GE_ERR_MISSING_METADATA, "weight file lacks metadata key " + key};
        return false;
    };
    auto get = [&](const char* key, int& out) {
        int64_t v;
        if (!f.get_int(std::string("clip.vision.") + key, v)) return false;
        out = int(v);
        return true;
    };
    if (!f.get_float("clip.vision.attention.layer_norm_epsilon", c.eps))
        return missing("clip.vision.attention.layer_norm_epsilon");
    if (!get("embedding_length", c.hidden)) return missing("clip.vision.embedding_length");
    if (!get("attention.head_count", c.heads)) return missing("clip.vision.attention.head_count");
    if (c.heads <= 0 || c.hidden % c.heads) {
        e = {GE_ERR_INVALID_GGUF, "invalid GGUF file: vision width " + std::to_string(c.hidden) +
                                      " does not split into " + std::to_string(c.heads) + " heads"};
        return false;
    }
    if (!get("block_count", c.layers)) return missing("clip.vision.block_count");
    if (!get("patch_size", c.patch)) return missing("clip.vision.patch_size");
    if (!get("projection_dim", c.projection_dim)) return missing("clip.vision.projection_dim");
    if (!get("feed_forward_length", c.ff)) return missing("clip.vision.feed_forward_length");
    std::vector<float> mean, std_;
    if (!f.get_float_array("clip.vision.image_mean", mean) || mean.size() != 3) return missing("clip.vision.image_mean");
    if (!f.get_float_array("clip.vision.image_std", std_) || std_.size() != 3) return missing("clip.vision.image_std");
    for (int i = 0; i < 3; i++) {
        c.mean[i] = mean[size_t(i)];
        c.std[i] = std_[size_t(i)];
    }
    c.head_dim = c.hidden / c.heads;
    return true;
}

// The patch embedding [p, p, 3, d] (F32 or F16) as the fp16 GEMM weight [d][kpad], columns
// past 3 p^2 zero.
HostWeight patch_weight(const GgufTensor& t, const VisionConfig& c) {
    HostWeight w;
    w.N = c.hidden;
    w.K = c.kpad();
    w.q8 = false;
    w.f16.assign(size_t(w.N) * w.K, 0);
    const int area = c.area();
    for (int n = 0; n < w.N; n++)
        for (int k = 0; k < area; k++) {
            const size_t i = size_t(n) * area + k;
            float v;
            if (t.type == GGML_F32) {
                memcpy(&v, t.data + 4 * i, 4);
            } else {
                uint16_t h;
                memcpy(&h, t.data + 2 * i, 2);
                v = half_bits_to_float(h);
            }
            w.f16[size_t(n) * w.K + k] = float_to_half_bits(v);
        }
    return w;
}

void free_vision_workspace(VisionWorkspace& ws) {
    for (void* p : ws.allocations) cudaFree(p);
    for (void* p : {(void*)ws.h_rgb, (void*)ws.h_xy, (void*)ws.h_work, (void*)ws.h_imgs})
        if (p) cudaFreeHost(p);
    ws = VisionWorkspace();
}

// Grows the workspace to at least the given patch rows, token rows, images, RGB bytes and
// attention-schedule words (VisionTower.upload's workspace growth, VisionTower.swift:123-133).
cudaError_t ensure_vision_workspace(const VisionConfig& c, Device& d, int rows, int tokens, int images, size_t rgb,
                                    int work) {
    VisionWorkspace& ws = d.vis.ws;
    if (ws.cap_rows >= rows && ws.cap_tokens >= tokens && ws.cap_images >= images && ws.cap_rgb >= rgb &&
        ws.cap_work >= work)
        return cudaSuccess;
    cudaError_t e = cudaStreamSynchronize(d.stream);
    if (e != cudaSuccess) return e;
    const int R = std::max(rows, ws.cap_rows);
    const int T = std::max(tokens, ws.cap_tokens);
    const int I = std::max({images, ws.cap_images, 8});
    const size_t B = std::max(rgb, ws.cap_rgb);
    const int W = std::max({work, ws.cap_work, 64});
    free_vision_workspace(ws);
    cudaError_t err = cudaSuccess;
    auto A = [&](auto** p, size_t n) {
        using Tp = std::remove_pointer_t<std::remove_reference_t<decltype(*p)>>;
        if (err == cudaSuccess) err = dev_alloc(ws.allocations, p, std::max<size_t>(n, 1));
        (void)sizeof(Tp);
    };
    auto H = [&](auto** p, size_t n) {
        using Tp = std::remove_pointer_t<std::remove_reference_t<decltype(*p)>>;
        void* q = nullptr;
        if (err == cudaSuccess) err = cudaMallocHost(&q, std::max<size_t>(n, 1) * sizeof(Tp));
        *p = static_cast<Tp*>(q);
    };
    const size_t r = size_t(R), dm = size_t(c.hidden);
    A(&ws.rgb, B);
    A(&ws.patches, r * c.kpad());
    A(&ws.x, r * dm);
    A(&ws.h, r * dm);
    A(&ws.qkv, r * 3 * dm);
    A(&ws.q, r * dm);
    A(&ws.k, r * dm);
    A(&ws.v, r * dm);
    A(&ws.attn, r * dm);
    A(&ws.o16, r * dm);
    A(&ws.act, r * size_t(c.ff));
    A(&ws.pooled, size_t(T) * dm);
    A(&ws.vectors, size_t(T) * c.projection_dim);
    A(&ws.xy, r);
    A(&ws.imgs, size_t(I));
    A(&ws.work, size_t(W));
    H(&ws.h_rgb, B);
    H(&ws.h_xy, r);
    H(&ws.h_imgs, size_t(I));
    H(&ws.h_work, size_t(W));
    if (err != cudaSuccess) {
        free_vision_workspace(ws);
        return err;
    }
    ws.cap_rows = R;
    ws.cap_tokens = T;
    ws.cap_images = I;
    ws.cap_rgb = B;
    ws.cap_work = W;
    auto act = [&](DevActivation& a, __half* p, int nrows, int cols) {
        a.ptr = p;
        a.rows = nrows;
        a.cols = cols;
        return encode_activation_map(a);
    };
    const bool ok = act(ws.a_patches, ws.patches, R, c.kpad()) && act(ws.a_h, ws.h, R, c.hidden) &&
                    act(ws.a_attn, ws.attn, R, c.hidden) && act(ws.a_act, ws.act, R, c.ff) &&
                    act(ws.a_pooled, ws.pooled, T, c.hidden);
    return ok ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

void free_vision(Device& d) {
    free_vision_workspace(d.vis.ws);
    for (void* p : d.vis.allocations) cudaFree(p);
    d.vis = VisionDev();
}

int load_vision(ge_model* m, const char* path) {
    GgufError gerr;
    if (!path) return set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: image encoder path is NULL");
    GgufFile& f = m->vision_file;
    if (f.open(path, gerr)) return set_error(m, gerr.code, gerr.message);
    VisionConfig& c = m->vcfg;
    LoadError le{0, ""};
    if (!read_vision_config(f, c, le)) return set_error(m, le.code, le.msg);
    // MetalForward.init (Metal/MetalForward.swift:87-89): the encoder projects to the text width.
    if (c.projection_dim != m->cfg.hidden)
        return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: image encoder projects to " +
                                                     std::to_string(c.projection_dim) + " dimensions, the text model is " +
                                                     std::to_string(m->cfg.hidden) + " wide");
    // The shapes the kernels are built for (the real encoder's and BASELINE config 4's).
    if (c.head_dim != 64 || (c.heads != 8 && c.heads != 12 && c.heads != 16) || c.layers <= 0 ||
        (c.hidden != 512 && c.hidden != 768 && c.hidden != 1024) || c.ff % 128 || c.patch <= 0 || c.patch > 64)
        return set_error(m, GE_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture: image encoder shape (hidden " +
                                                                  std::to_string(c.hidden) + ", heads " +
                                                                  std::to_string(c.heads) + ")");
    const int d = c.hidden, ff = c.ff, p = c.patch, hd = c.head_dim;
    // ---- VisionWeights.init (VisionWeights.swift:37-83)
    const GgufTensor* pe = f.tensor("v.patch_embd.weight");
    if (!pe) return set_error(m, GE_ERR_MISSING_TENSOR, "weight file lacks tensor v.patch_embd.weight");
    if (!need_tensor(f, "v.patch_embd.weight", {p, p, 3, d}, false, le)) return set_error(m, le.code, le.msg);
    if (pe->type != GGML_F32 && pe->type != GGML_F16)
        return set_error(m, GE_ERR_UNSUPPORTED_TENSOR_TYPE,
                         "tensor v.patch_embd.weight uses unsupported storage type " + std::to_string(pe->type));
    const GgufTensor* pos = f.tensor("v.position_embd.weight");
    if (!pos) return set_error(m, GE_ERR_MISSING_TENSOR, "weight file lacks tensor v.position_embd.weight");
    if (pos->type != GGML_F32)
        return set_error(m, GE_ERR_UNSUPPORTED_TENSOR_TYPE,
                         "tensor v.position_embd.weight uses unsupported storage type " + std::to_string(pos->type));
    if (pos->shape.size() != 3 || pos->shape[0] != d || pos->shape[2] != 2 || pos->shape[1] <= 0)
        return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: v.position_embd.weight has an unexpected shape, expected [" +
                                                     std::to_string(d) + ", n, 2]");
    c.positions = int(pos->shape[1]);
    const GgufTensor* proj = need_tensor(f, "mm.input_projection.weight", {d, c.projection_dim}, false, le);
    if (!proj) return set_error(m, le.code, le.msg);
    struct LT {
        const GgufTensor *ln1, *q, *k, *v, *o, *qn, *kn, *pan, *ln2, *gate, *up, *down, *pfn;
    };
    std::vector<LT> lt(static_cast<size_t>(c.layers));
    for (int i = 0; i < c.layers; i++) {
        const std::string b = "v.blk." + std::to_string(i) + ".";
        LT& t = lt[size_t(i)];
        if (!(t.ln1 = need_tensor(f, b + "ln1.weight", {d}, true, le)) ||
            !(t.q = need_tensor(f, b + "attn_q.weight", {d, d}, false, le)) ||
            !(t.k = need_tensor(f, b + "attn_k.weight", {d, d}, false, le)) ||
            !(t.v = need_tensor(f, b + "attn_v.weight", {d, d}, false, le)) ||
            !(t.o = need_tensor(f, b + "attn_out.weight", {d, d}, false, le)) ||
            !(t.qn = need_tensor(f, b + "attn_q_norm.weight", {hd}, true, le)) ||
            !(t.kn = need_tensor(f, b + "attn_k_norm.weight", {hd}, true, le)) ||
            !(t.pan = need_tensor(f, b + "attn_post_norm.weight", {d}, true, le)) ||
            !(t.ln2 = need_tensor(f, b + "ln2.weight", {d}, true, le)) ||
            !(t.gate = need_tensor(f, b + "ffn_gate.weight", {d, ff}, false, le)) ||
            !(t.up = need_tensor(f, b + "ffn_up.weight", {d, ff}, false, le)) ||
            !(t.down = need_tensor(f, b + "ffn_down.weight", {ff, d}, false, le)) ||
            !(t.pfn = need_tensor(f, b + "ffn_post_norm.weight", {d}, true, le)))
            return set_error(m, le.code, le.msg);
    }
    // SpanMarkers.image (Model/InputRow.swift:28-45): "<|image>" and "<image|>" are single tokens.
    if (!m->tokenizer)
        return set_error(m, GE_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture: tokenizer model missing");
    for (int k = 0; k < 2; k++) {
        const std::string text = k == 0 ? "<|image>" : "<image|>";
        std::vector<int32_t> ids;
        m->tokenizer->t.encode(reinterpret_cast<const uint8_t*>(text.data()), text.size(), false, true, ids);
        if (ids.size() != 1) return set_error(m, GE_ERR_INVALID_GGUF, "invalid GGUF file: vocabulary has no single token for " + text);
        (k == 0 ? m->image_begin : m->image_end) = ids[0];
    }
    // ---- host repack
    std::vector<HostWeight> hw;
    hw.push_back(patch_weight(*pe, c));
    for (const LT& t : lt) {
        hw.push_back(build_weight(3 * d, d, true, [&](int r) -> std::pair<const GgufTensor*, int> {
            if (r < d) return {t.q, r};
            if (r < 2 * d) return {t.k, r - d};
            return {t.v, r - 2 * d};
        }));
        hw.push_back(build_weight(d, d, true, [&](int r) -> std::pair<const GgufTensor*, int> { return {t.o, r}; }));
        // Gate and up interleaved in blocks of kBN/2 rows, so one output tile holds both halves.
        hw.push_back(build_weight(2 * ff, d, true, [&](int r) -> std::pair<const GgufTensor*, int> {
            const int blk = r / (kBN / 2), off = r % (kBN / 2);
            return {(blk & 1) ? t.up : t.gate, (blk >> 1) * (kBN / 2) + off};
        }));
        hw.push_back(build_weight(d, ff, true, [&](int r) -> std::pair<const GgufTensor*, int> { return {t.down, r}; }));
    }
    hw.push_back(build_weight(c.projection_dim, d, true, [&](int r) -> std::pair<const GgufTensor*, int> { return {proj, r}; }));
    auto vec = [&](const GgufTensor* t) {
        std::vector<float> v(size_t(t->elements()));
        dequant_row(*t, 0, v.data());
        return v;
    };
    std::vector<std::vector<float>> norms;
    for (const LT& t : lt)
        for (const GgufTensor* n : {t.ln1, t.qn, t.kn, t.pan, t.ln2, t.pfn}) norms.push_back(vec(n));
    // RopeTable(headDim: hd / 2, base: 100, positions: n) (Model/RopeTable.swift:16-31): hd / 4
    // pairs per position, angles in double, cos and sin rounded to float.
    const int pairs = hd / 4;
    std::vector<float> rope(size_t(c.positions) * pairs * 2);
    for (int i = 0; i < pairs; i++) {
        const double inv = std::pow(double(c.rope_theta), -2.0 * double(i) / double(hd / 2));
        for (int ps = 0; ps < c.positions; ps++) {
            const double th = double(ps) * inv;
            rope[(size_t(ps) * pairs + i) * 2] = float(std::cos(th));
            rope[(size_t(ps) * pairs + i) * 2 + 1] = float(std::sin(th));
        }
    }
    // ---- upload to every device
    for (Device& dv : m->devs) {
        cudaError_t e = cudaSetDevice(dv.ordinal);
        VisionDev& v = dv.vis;
        std::vector<void*>& own = v.allocations;
        size_t wi = 0;
        if (e == cudaSuccess) e = upload_weight(own, v.patch, hw[wi++]);
        v.layers.resize(size_t(c.layers));
        for (int l = 0; l < c.layers && e == cudaSuccess; l++) {
            VisionLayerDev& L = v.layers[size_t(l)];
            for (DevWeight* w : {&L.qkv, &L.o, &L.gu, &L.down})
                if (e == cudaSuccess) e = upload_weight(own, *w, hw[wi++]);
            float** dst[6] = {&L.ln1, &L.q_norm, &L.k_norm, &L.post_attn, &L.ln2, &L.post_ffn};
            for (int k = 0; k < 6 && e == cudaSuccess; k++) {
                const std::vector<float>& src = norms[size_t(l) * 6 + k];
                e = dev_upload(own, dst[k], src.data(), src.size());
            }
        }
        if (e == cudaSuccess) e = upload_weight(own, v.proj, hw[wi++]);
        if (e == cudaSuccess)
            e = dev_upload(own, &v.pos, reinterpret_cast<const float*>(pos->data), size_t(pos->elements()));
        if (e == cudaSuccess) e = dev_upload(own, &v.rope, rope.data(), rope.size());
        if (e != cudaSuccess)
            return set_error(m, e == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                             std::string("GPU execution failed: image encoder upload: ") + cudaGetErrorString(e));
        v.loaded = true;
    }
    m->has_vision = true;
    return GE_OK;
}

int run_vision(ge_model* m, Device& d, const VisionArgs& a) {
    const VisionConfig& c = m->vcfg;
    const PreparedImage* const* imgs = a.imgs;
    const int n = a.n;
    auto report = [&](int code, const std::string& msg) {
        if (a.error) *a.error = msg;
        else m->last_error = msg;
        return code;
    };
    auto gpu_fail = [&](cudaError_t x, const char* what) {
        return report(x == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                      std::string("GPU execution failed: ") + what + ": " + cudaGetErrorString(x));
    };
    cudaError_t e = cudaSetDevice(d.ordinal);
    if (e != cudaSuccess) return gpu_fail(e, "cudaSetDevice");
    if (!d.vis.loaded) return report(GE_ERR_IMAGE_ENCODER_NOT_LOADED, "no image encoder is loaded; pass the mmproj GGUF when loading the model");
    struct LaunchPolicy {
        explicit LaunchPolicy(bool on) { set_programmatic_launch(on); }
        ~LaunchPolicy() { set_programmatic_launch(false); }
    } policy(!(m->flags & GE_LOAD_NO_PDL));
    // ---- batch layout (VisionBatch, Metal/VisionTower.swift:8-33)
    int patches = 0, tokens = 0, max_patches = 0, max_tokens = 0;
    size_t rgb = 0;
    for (int i = 0; i < n; i++) {
        const PreparedImage& im = *imgs[i];
        if (im.gx <= 0 || im.gy <= 0 || im.gx % c.merge || im.gy % c.merge || im.gx > c.positions ||
            im.gy > c.positions || im.gx > 0xffff || im.gy > 0xffff ||
            (!a.d_rgb && im.rgb.size() != size_t(im.gx) * im.gy * c.patch * c.patch * 3))
            return report(GE_ERR_INVALID_OPTIONS, "invalid options: image " + std::to_string(i) + " has an unusable patch grid");
        patches += im.patches();
        tokens += im.tokens();
        max_patches = std::max(max_patches, im.patches());
        max_tokens = std::max(max_tokens, im.tokens());
        rgb += size_t(im.gx) * im.gy * c.patch * c.patch * 3;
    }
    const int rows = std::max(kRowTile, (patches + kRowTile - 1) / kRowTile * kRowTile);
    const int trows = std::max(kRowTile, (tokens + kRowTile - 1) / kRowTile * kRowTile);
    std::vector<uint32_t> seq_pairs(2 * size_t(n));
    for (int i = 0, s = 0; i < n; i++) {
        seq_pairs[2 * size_t(i)] = uint32_t(s);
        seq_pairs[2 * size_t(i) + 1] = uint32_t(imgs[i]->patches());
        s += imgs[i]->patches();
    }
    int ctas = 0;
    const int words = build_attention_work(seq_pairs.data(), n, c.heads, 1, 0, d.num_sms, nullptr, &ctas);
    const int items = words ? (words - ctas - 1) / 4 : 0;
    if ((e = staging_wait(d, kStageImage)) != cudaSuccess) return gpu_fail(e, "staging");
    if ((e = ensure_vision_workspace(c, d, rows, trows, n, a.d_rgb ? 0 : rgb, words)) != cudaSuccess)
        return gpu_fail(e, "workspace");
    VisionWorkspace& ws = d.vis.ws;
    // ---- host staging and uploads
    size_t off = 0;
    for (int i = 0, ps = 0, ts = 0; i < n; i++) {
        const PreparedImage& im = *imgs[i];
        const size_t bytes = size_t(im.gx) * im.gy * c.patch * c.patch * 3;
        if (!a.d_rgb) memcpy(ws.h_rgb + off, im.rgb.data(), bytes);
        ws.h_imgs[i] = VisionImage{uint64_t(off), im.gx, im.gy, uint32_t(ps), uint32_t(ts)};
        for (int k = 0; k < im.patches(); k++)
            ws.h_xy[ps + k] = uint32_t(k % im.gx) | (uint32_t(k / im.gx) << 16);
        off += bytes;
        ps += im.patches();
        ts += im.tokens();
    }
    build_attention_work(seq_pairs.data(), n, c.heads, 1, 0, d.num_sms, ws.h_work, nullptr);
    cudaStream_t st = a.stream ? a.stream : d.stream;
    const uint8_t* src = a.d_rgb ? a.d_rgb : ws.rgb;
    if ((!a.d_rgb && (e = cudaMemcpyAsync(ws.rgb, ws.h_rgb, rgb, cudaMemcpyHostToDevice, st)) != cudaSuccess) ||
        (e = cudaMemcpyAsync(ws.imgs, ws.h_imgs, size_t(n) * sizeof(VisionImage), cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = cudaMemcpyAsync(ws.xy, ws.h_xy, size_t(patches) * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = cudaMemcpyAsync(ws.work, ws.h_work, size_t(words) * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = staging_done(d, kStageImage, st)) != cudaSuccess)
        return gpu_fail(e, "image upload");
    m->h2d_bytes += int64_t((a.d_rgb ? 0 : rgb) + size_t(n) * sizeof(VisionImage) + size_t(patches) * 4 + size_t(words) * 4);
    // Padding rows of the GEMM operands are zero (VisionTower.upload, VisionTower.swift:145-146).
    if (rows > patches &&
        (e = cudaMemsetAsync(ws.patches + size_t(patches) * c.kpad(), 0, size_t(rows - patches) * c.kpad() * 2, st)) != cudaSuccess)
        return gpu_fail(e, "padding");
    if (trows > tokens &&
        (e = cudaMemsetAsync(ws.pooled + size_t(tokens) * c.hidden, 0, size_t(trows - tokens) * c.hidden * 2, st)) != cudaSuccess)
        return gpu_fail(e, "padding");
    // ---- VisionTower.encode (VisionTower.swift:140-185)
    const VisionDev& v = d.vis;
    const int D = c.hidden;
    int64_t launches = 0;
    // Every launch goes through K: counted, and when profiling the first launch of each kernel
    // class is timed over `reps` back-to-back repetitions (Profiler.profileImages,
    // Metal/Profiler.swift:114-200).
    auto K = [&](const char* name, double flops, double bytes, auto&& fn) -> cudaError_t {
        if (a.profile) {
            ProfileEntry* pe = a.profile->find(name);
            if (pe) {
                pe->occurrences++;
            } else {
                cudaEvent_t e0, e1;
                cudaEventCreate(&e0);
                cudaEventCreate(&e1);
                cudaEventRecord(e0, st);
                for (int r = 0; r < a.profile->reps; r++) {
                    const cudaError_t x = fn();
                    if (x != cudaSuccess) return x;
                    launches++;
                }
                cudaEventRecord(e1, st);
                const cudaError_t x = cudaEventSynchronize(e1);
                float ms = 0.f;
                cudaEventElapsedTime(&ms, e0, e1);
                cudaEventDestroy(e0);
                cudaEventDestroy(e1);
                if (x != cudaSuccess) return x;
                a.profile->add(name, double(ms) / a.profile->reps, flops, bytes);
                return cudaSuccess;
            }
        }
        launches++;
        return fn();
    };
    auto gemm = [&](const DevActivation& A, const DevWeight& W, int m_rows, void* out, int ldo, int epi) {
        GemmLaunch g;
        g.a = &A;
        g.w = &W;
        g.m_rows = m_rows;
        g.out = out;
        g.ldo = ldo;
        g.epilogue = epi;
        g.err = d.err;
        g.num_sms = d.num_sms;
        return launch_gemm(g, st);
    };
    // Algorithmic work: token rows only.
    auto gf = [&](const DevWeight& W, int nrows) { return 2.0 * nrows * W.N * double(W.K); };
    auto gbytes = [&](const DevWeight& W, int nrows, int out_cols, double out_bytes) {
        return double(nrows) * W.K * 2 + double(W.N) * W.K * 2 + double(nrows) * out_cols * out_bytes;
    };
    double att_flops = 0;
    for (int i = 0; i < n; i++) att_flops += 4.0 * double(imgs[i]->patches()) * imgs[i]->patches() * D;
#define VK(name, flops, bytes, expr, what)                                             \
    do {                                                                               \
        cudaError_t e_ = K(name, flops, bytes, [&] { return (expr); });                \
        if (e_ != cudaSuccess) return gpu_fail(e_, what);                              \
    } while (0)
    NormParams np;
    for (int i = 0; i < 3; i++) {
        np.mean[i] = c.mean[i];
        np.std[i] = c.std[i];
    }
    const double P = patches;
    VK("patchify", 0, double(rgb) + P * c.kpad() * 2,
       launch_patchify(src, ws.imgs, n, max_patches, c.patch, c.kpad(), np, ws.patches, st), "patchify");
    VK("gemm_patch", gf(v.patch, patches), gbytes(v.patch, patches, D, 4),
       gemm(ws.a_patches, v.patch, rows, ws.x, D, EPI_F32), "patch embedding");
    VK("position_norm", 0, P * D * 14,
       launch_patch_position_norm(ws.x, ws.xy, patches, rows, D, v.pos, c.positions, v.layers[0].ln1, c.eps, ws.h, st),
       "position rows");
    for (int l = 0; l < c.layers; l++) {
        const VisionLayerDev& L = v.layers[size_t(l)];
        VK("gemm_qkv", gf(L.qkv, patches), gbytes(L.qkv, patches, 3 * D, 2),
           gemm(ws.a_h, L.qkv, rows, ws.qkv, 3 * D, EPI_F16), "qkv projection");
        VK("qkv_norm_rope", 0, P * 3 * D * 4,
           launch_vision_qkv_norm_rope(ws.qkv, patches, rows, c.heads, L.q_norm, L.k_norm, ws.xy, v.rope, c.eps, ws.q,
                                       ws.k, ws.v, st),
           "q/k/v norm and rope");
        Attn64Launch at;
        at.q = ws.q;
        at.k = ws.k;
        at.v = ws.v;
        at.out = ws.attn;
        at.rows = rows;
        at.heads = c.heads;
        at.work = ws.work;
        at.sched_items = items;
        at.ctas = ctas;
        at.err = d.err;
        VK("attention", att_flops, P * D * 2 * 4, launch_attention64(at, st), "attention");
        VK("gemm_o", gf(L.o, patches), gbytes(L.o, patches, D, 2), gemm(ws.a_attn, L.o, rows, ws.o16, D, EPI_F16),
           "attention output");
        VK("residual_attn", 0, P * D * 14,
           launch_residual_norm(ws.x, ws.o16, patches, D, L.post_attn, 1.0f, L.ln2, c.eps, ws.h, nullptr, nullptr, st),
           "attention residual");
        VK("gemm_gate_up", gf(L.gu, patches), gbytes(L.gu, patches, c.ff, 2),
           gemm(ws.a_h, L.gu, rows, ws.act, c.ff, EPI_GEGLU_QUICK), "gate/up");
        VK("gemm_down", gf(L.down, patches), gbytes(L.down, patches, D, 2),
           gemm(ws.a_act, L.down, rows, ws.o16, D, EPI_F16), "down");
        const float* next = l + 1 < c.layers ? v.layers[size_t(l) + 1].ln1 : nullptr;
        VK("residual_ffn", 0, P * D * (next ? 14 : 12),
           launch_residual_norm(ws.x, ws.o16, patches, D, L.post_ffn, 1.0f, next, c.eps, next ? ws.h : nullptr, nullptr,
                                nullptr, st),
           "ffn residual");
    }
    VK("pool", 0, P * D * 4 + double(tokens) * D * 2,
       launch_pool_patches_norm(ws.x, ws.imgs, n, max_tokens, D, c.merge, sqrtf(float(D)) / float(c.merge * c.merge),
                                c.eps, ws.pooled, st),
       "pool");
    VK("gemm_projection", gf(v.proj, tokens), gbytes(v.proj, tokens, c.projection_dim, 4),
       gemm(ws.a_pooled, v.proj, trows, ws.vectors, c.projection_dim, EPI_F32), "projection");
#undef VK
    m->launches += launches;
    return GE_OK;
}

}  // namespace ge
