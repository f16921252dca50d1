// testing.cpp -- kernel-level entry points for parity tests (include/gemma_embed_testing.h).
#include <string.h>

#include <string>
#include <cmath>
#include <vector>

#include "gemma_embed_testing.h"
#include "kernels.hpp"
#include "model.hpp"
#include "vision.hpp"
#include "multimodal.hpp"

namespace {

thread_local std::string t_err;

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    cudaError_t alloc(size_t bytes) { return cudaMalloc(&p, bytes ? bytes : 1); }
};

int fail(int code, const std::string& msg) {
    t_err = msg;
    return code;
}

#define TRY(expr)                                                                                    \
    do {                                                                                             \
        cudaError_t e_ = (expr);                                                                     \
        if (e_ != cudaSuccess) return fail(GE_ERR_GPU_FAILURE, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)

uint16_t f2h(float f) {
    __half h = __float2half_rn(f);
    return __half_raw(h).x;
}
float h2f(uint16_t b) {
    __half_raw r;
    r.x = b;
    return __half2float(__half(r));
}

}  // namespace

extern "C" {

const char* ge_test_last_error(void) { return t_err.c_str(); }

int ge_test_shard(const ge_seq* seqs, int32_t nseq, int32_t ndev, int32_t* device_of_seq) {
    if (nseq < 0 || ndev <= 0 || (nseq > 0 && (!seqs || !device_of_seq)))
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options");
    const auto parts = ge::shard_sequences(seqs, nseq, ndev);
    for (int d = 0; d < ndev; d++)
        for (int i : parts[size_t(d)]) device_of_seq[i] = d;
    return GE_OK;
}

int ge_test_attention_schedule(const ge_seq* seqs, int32_t nseq, int32_t kvh, int32_t group, int32_t half_window,
                               int32_t max_ctas, uint32_t* out, int32_t out_cap, int32_t* ctas, int32_t* words) {
    if (nseq < 0 || kvh <= 0 || group <= 0 || group > 128 || half_window < 0 || max_ctas <= 0 || !ctas || !words ||
        (nseq > 0 && !seqs))
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options");
    std::vector<uint32_t> pairs;
    for (int s = 0; s < nseq; s++) {
        pairs.push_back(seqs[s].start);
        pairs.push_back(seqs[s].length);
    }
    int c = 0;
    const int need = ge::build_attention_work(pairs.data(), nseq, kvh, group, half_window, max_ctas, nullptr, &c);
    *ctas = c;
    *words = need;
    if (need > out_cap || (need > 0 && !out)) return fail(GE_ERR_INVALID_OPTIONS, "output capacity too small");
    if (need > 0) ge::build_attention_work(pairs.data(), nseq, kvh, group, half_window, max_ctas, out, nullptr);
    return GE_OK;
}

// Host repack of Q8_0 rows [n][k/32 * 34 bytes] into the device planes the loader builds.
static int upload_weight(const uint8_t* w, int n, int k, DevBuf& dq, DevBuf& ds, DevBuf& dh, ge::DevWeight& W) {
    std::vector<int8_t> q(size_t(n) * k);
    std::vector<uint16_t> st(size_t(n) * (k / 32)), f16(size_t(n) * k);
    for (int r = 0; r < n; r++)
        for (int b = 0; b < k / 32; b++) {
            const uint8_t* blk = w + (size_t(r) * (k / 32) + b) * 34;
            uint16_t s;
            memcpy(&s, blk, 2);
            st[size_t(b) * n + r] = s;
            for (int j = 0; j < 32; j++) {
                const int8_t v = int8_t(blk[2 + j]);
                q[size_t(r) * k + b * 32 + j] = v;
                f16[size_t(r) * k + b * 32 + j] = f2h(h2f(s) * float(v));
            }
        }
    TRY(dq.alloc(q.size()));
    TRY(cudaMemcpy(dq.p, q.data(), q.size(), cudaMemcpyHostToDevice));
    TRY(ds.alloc(st.size() * 2));
    TRY(cudaMemcpy(ds.p, st.data(), st.size() * 2, cudaMemcpyHostToDevice));
    TRY(dh.alloc(f16.size() * 2));
    TRY(cudaMemcpy(dh.p, f16.data(), f16.size() * 2, cudaMemcpyHostToDevice));
    W.N = n;
    W.K = k;
    W.q8 = static_cast<int8_t*>(dq.p);
    W.scales_t = static_cast<__half*>(ds.p);
    W.f16 = static_cast<__half*>(dh.p);
    if (!ge::encode_weight_maps(W, 256)) return fail(GE_ERR_GPU_FAILURE, "tensor map encoding failed");
    return GE_OK;
}

static int upload_activation(const uint16_t* a, int m, int k, int rows, DevBuf& da, ge::DevActivation& A) {
    TRY(da.alloc(size_t(rows) * k * 2));
    TRY(cudaMemset(da.p, 0, size_t(rows) * k * 2));
    TRY(cudaMemcpy(da.p, a, size_t(m) * k * 2, cudaMemcpyHostToDevice));
    A.ptr = static_cast<__half*>(da.p);
    A.rows = rows;
    A.cols = k;
    if (!ge::encode_activation_map(A)) return fail(GE_ERR_GPU_FAILURE, "tensor map encoding failed");
    return GE_OK;
}

int ge_test_gemm(const uint16_t* a, int32_t m, int32_t k, const uint8_t* w, int32_t n, int32_t epilogue, int32_t use_q8,
                 const float* aux, float* out) {
    if (m <= 0 || k <= 0 || n <= 0 || k % 64 || n % 256 || !a || !w || !out || epilogue < 0 || epilogue > 5 ||
        epilogue == ge::EPI_RESIDUAL || (epilogue == 3 && !aux))
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options: shapes must be k % 64 == 0 and n % 256 == 0");
    const int rows = (m + ge::kRowTile - 1) / ge::kRowTile * ge::kRowTile;
    int dev = 0, sms = 0;
    TRY(cudaGetDevice(&dev));
    TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DevBuf da, dq, ds, dh, dout, daux, derr;
    ge::DevWeight W;
    ge::DevActivation A;
    int rc = upload_weight(w, n, k, dq, ds, dh, W);
    if (rc != GE_OK) return rc;
    if ((rc = upload_activation(a, m, k, rows, da, A)) != GE_OK) return rc;
    const int out_cols = ge::epi_is_geglu(epilogue) ? n / 2 : n;
    const size_t out_elem = epilogue == 0 ? 4 : 2;
    TRY(dout.alloc(size_t(rows) * out_cols * out_elem));
    TRY(derr.alloc(sizeof(int)));
    TRY(cudaMemset(derr.p, 0, sizeof(int)));
    if (epilogue == 3) {
        TRY(daux.alloc(size_t(rows) * n * 4));
        TRY(cudaMemset(daux.p, 0, size_t(rows) * n * 4));
        TRY(cudaMemcpy(daux.p, aux, size_t(m) * n * 4, cudaMemcpyHostToDevice));
    }
    TRY(ge::configure_gemm_kernels());
    ge::GemmLaunch g;
    g.a = &A;
    g.w = &W;
    g.m_rows = rows;
    g.out = dout.p;
    g.ldo = out_cols;
    g.epilogue = epilogue;
    g.aux = static_cast<const float*>(daux.p);
    g.ldaux = n;
    g.use_q8 = use_q8 == 1;
    g.mode = use_q8 == 2   ? ge::GEMM_PAIR
             : use_q8 == 3 ? ge::GEMM_NARROW
             : use_q8 == 4 ? ge::GEMM_SPLIT
                           : ge::GEMM_SINGLE;
    g.err = static_cast<int*>(derr.p);
    g.num_sms = sms;
    TRY(ge::launch_gemm(g, nullptr));
    TRY(cudaDeviceSynchronize());
    int herr = 0;
    TRY(cudaMemcpy(&herr, derr.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) return fail(herr, "GPU execution failed: a device-side wait timed out");
    if (out_elem == 4) {
        TRY(cudaMemcpy(out, dout.p, size_t(m) * out_cols * 4, cudaMemcpyDeviceToHost));
    } else {
        std::vector<uint16_t> h(size_t(m) * out_cols);
        TRY(cudaMemcpy(h.data(), dout.p, h.size() * 2, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < h.size(); i++) out[i] = h2f(h[i]);
    }
    return GE_OK;
}

int ge_test_gemm_time(int32_t m, int32_t k, int32_t n, int32_t epilogue, int32_t path, int32_t reps, double* us) {
    if (m <= 0 || m % ge::kRowTile || k <= 0 || n <= 0 || k % 64 || n % 256 || epilogue < 0 || epilogue > 2 ||
        path < 0 || path > 4 || reps <= 0 || !us)
        return fail(GE_ERR_INVALID_OPTIONS,
                    "invalid options: m % 128 == 0, k % 64 == 0, n % 256 == 0, epilogue 0..2, path 0..4");
    int dev = 0, sms = 0;
    TRY(cudaGetDevice(&dev));
    TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // Seeded operands of the model's scale: activations uniform in [-1, 1], Q8_0 weights with
    // scales near 1/sqrt(k) (values matter only through the power they draw).
    uint64_t state = 0x9E3779B97F4A7C15ull ^ (uint64_t(m) << 32) ^ uint64_t(n * 131 + k);
    auto next = [&]() {
        state += 0x9E3779B97F4A7C15ull;
        uint64_t z = state;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    std::vector<uint16_t> a(size_t(m) * k);
    for (auto& v : a) v = f2h(float(int(next() % 2001) - 1000) / 1000.0f);
    std::vector<uint8_t> w(size_t(n) * (k / 32) * 34);
    const uint16_t scale = f2h(1.0f / (127.0f * std::sqrt(float(k))));
    for (size_t b = 0; b < size_t(n) * (k / 32); b++) {
        memcpy(&w[b * 34], &scale, 2);
        for (int j = 0; j < 32; j++) w[b * 34 + 2 + j] = uint8_t(int(next() % 255) - 127);
    }
    DevBuf da, dq, ds, dh, dout, derr;
    ge::DevWeight W;
    ge::DevActivation A;
    int rc = upload_weight(w.data(), n, k, dq, ds, dh, W);
    if (rc != GE_OK) return rc;
    if ((rc = upload_activation(a.data(), m, k, m, da, A)) != GE_OK) return rc;
    const int out_cols = ge::epi_is_geglu(epilogue) ? n / 2 : n;
    TRY(dout.alloc(size_t(m) * out_cols * (epilogue == 0 ? 4 : 2)));
    TRY(derr.alloc(sizeof(int)));
    TRY(cudaMemset(derr.p, 0, sizeof(int)));
    TRY(ge::configure_gemm_kernels());
    ge::GemmLaunch g;
    g.a = &A;
    g.w = &W;
    g.m_rows = m;
    g.out = dout.p;
    g.ldo = out_cols;
    g.epilogue = epilogue;
    g.use_q8 = path == 1;
    g.mode = path == 2   ? ge::GEMM_PAIR
             : path == 3 ? ge::GEMM_NARROW
             : path == 4 ? ge::GEMM_SPLIT
                         : ge::GEMM_SINGLE;
    g.err = static_cast<int*>(derr.p);
    g.num_sms = sms;
    cudaStream_t st = nullptr;
    TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    // The launches are captured into a CUDA graph and the graph is timed: back-to-back host
    // launches of a short kernel would time the host's launch rate instead of the kernel.
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    for (int i = 0; i < 3 && e == cudaSuccess; i++) e = ge::launch_gemm(g, st);
    if (e == cudaSuccess) e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        for (int i = 0; i < reps && e == cudaSuccess; i++) e = ge::launch_gemm(g, st);
        const cudaError_t ee = cudaStreamEndCapture(st, &graph);
        if (e == cudaSuccess) e = ee;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, st);
    if (e == cudaSuccess) e = cudaEventRecord(e0, st);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, st);
    if (e == cudaSuccess) e = cudaEventRecord(e1, st);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaStreamDestroy(st);
    TRY(e);
    int herr = 0;
    TRY(cudaMemcpy(&herr, derr.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) return fail(herr, "GPU execution failed: a device-side wait timed out");
    *us = double(ms) * 1000.0 / reps;
    return GE_OK;
}

int ge_test_gemm_residual(const uint16_t* a, int32_t m, int32_t k, const uint8_t* w, int32_t n, int32_t path, float* x,
                          const float* w_post, float scale, const float* w_next, float eps, float* h_out, float* y_out) {
    if (m <= 0 || k <= 0 || n <= 0 || k % 64 || n % 256 || n > 1024 || !a || !w || !x || !w_post || path < 0 ||
        path > 1)
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options: k % 64 == 0, n a multiple of 256 up to 1024");
    const int rows = (m + ge::kRowTile - 1) / ge::kRowTile * ge::kRowTile;
    int dev = 0, sms = 0;
    TRY(cudaGetDevice(&dev));
    TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DevBuf da, dq, ds, dh, dx, dwp, dwn, dh16, dy, derr;
    ge::DevWeight W;
    ge::DevActivation A;
    int rc = upload_weight(w, n, k, dq, ds, dh, W);
    if (rc != GE_OK) return rc;
    if ((rc = upload_activation(a, m, k, rows, da, A)) != GE_OK) return rc;
    const size_t xe = size_t(rows) * n;
    TRY(dx.alloc(xe * 4));
    TRY(cudaMemset(dx.p, 0, xe * 4));
    TRY(cudaMemcpy(dx.p, x, size_t(m) * n * 4, cudaMemcpyHostToDevice));
    TRY(dwp.alloc(size_t(n) * 4));
    TRY(cudaMemcpy(dwp.p, w_post, size_t(n) * 4, cudaMemcpyHostToDevice));
    if (w_next) {
        TRY(dwn.alloc(size_t(n) * 4));
        TRY(cudaMemcpy(dwn.p, w_next, size_t(n) * 4, cudaMemcpyHostToDevice));
    }
    TRY(dh16.alloc(xe * 2));
    TRY(cudaMemset(dh16.p, 0xFF, xe * 2));
    TRY(dy.alloc(xe * 4));
    TRY(cudaMemset(dy.p, 0xFF, xe * 4));
    TRY(derr.alloc(sizeof(int)));
    TRY(cudaMemset(derr.p, 0, sizeof(int)));
    TRY(ge::configure_gemm_kernels());
    ge::GemmLaunch g;
    g.a = &A;
    g.w = &W;
    g.m_rows = rows;
    g.out = nullptr;
    g.ldo = n;
    g.epilogue = ge::EPI_RESIDUAL;
    g.use_q8 = path == 1;
    g.mode = ge::GEMM_SINGLE;
    g.err = static_cast<int*>(derr.p);
    g.num_sms = sms;
    g.x = static_cast<float*>(dx.p);
    g.w_post = static_cast<const float*>(dwp.p);
    g.scale = scale;
    g.w_next = w_next ? static_cast<const float*>(dwn.p) : nullptr;
    g.eps = eps;
    g.h16 = h_out ? static_cast<__half*>(dh16.p) : nullptr;
    g.y32 = y_out ? static_cast<float*>(dy.p) : nullptr;
    TRY(ge::launch_gemm(g, nullptr));
    TRY(cudaDeviceSynchronize());
    int herr = 0;
    TRY(cudaMemcpy(&herr, derr.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) return fail(herr, "GPU execution failed: a device-side wait timed out");
    TRY(cudaMemcpy(x, dx.p, size_t(m) * n * 4, cudaMemcpyDeviceToHost));
    if (h_out) {
        std::vector<uint16_t> h(size_t(m) * n);
        TRY(cudaMemcpy(h.data(), dh16.p, h.size() * 2, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < h.size(); i++) h_out[i] = h2f(h[i]);
    }
    if (y_out) TRY(cudaMemcpy(y_out, dy.p, size_t(m) * n * 4, cudaMemcpyDeviceToHost));
    return GE_OK;
}

int ge_test_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t ntok, const ge_seq* seqs,
                      int32_t nseq, int32_t heads, int32_t kvh, int32_t hd, int32_t half_window, uint16_t* out) {
    if (ntok <= 0 || nseq <= 0 || !q || !k || !v || !seqs || !out || heads <= 0 || kvh <= 0 || heads % kvh ||
        (hd != 64 && hd != 256 && hd != 512) || half_window < 0 || (hd == 64 && (kvh != heads || half_window != 0)))
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options");
    uint64_t next = 0;
    for (int s = 0; s < nseq; s++) {
        if (seqs[s].start != next || seqs[s].length == 0) return fail(GE_ERR_INVALID_OPTIONS, "sequences must tile the batch");
        next += seqs[s].length;
    }
    if (next != uint64_t(ntok)) return fail(GE_ERR_INVALID_OPTIONS, "lengths do not sum to ntok");
    const int rows = (ntok + ge::kRowTile - 1) / ge::kRowTile * ge::kRowTile;
    int dev = 0, sms = 0;
    TRY(cudaGetDevice(&dev));
    TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    std::vector<uint32_t> work;
    int items = 0, ctas = 0;
    {
        std::vector<uint32_t> pairs;
        for (int s = 0; s < nseq; s++) {
            pairs.push_back(seqs[s].start);
            pairs.push_back(seqs[s].length);
        }
        const int shd = hd == 512 ? 512 : 256;  // head dim 64 (vision) schedules like 256 with group 1
        const int words =
            ge::build_attention_work(pairs.data(), nseq, kvh, heads / kvh, half_window, sms, nullptr, &ctas, shd);
        work.resize(size_t(words));
        ge::build_attention_work(pairs.data(), nseq, kvh, heads / kvh, half_window, sms, work.data(), nullptr, shd);
        items = (words - ctas - 1) / 4;
    }
    DevBuf dq, dk, dv, dout, dwork, derr;
    const size_t qn = size_t(rows) * heads * hd, kn = size_t(rows) * kvh * hd;
    TRY(dq.alloc(qn * 2));
    TRY(dk.alloc(kn * 2));
    TRY(dv.alloc(kn * 2));
    TRY(dout.alloc(qn * 2));
    TRY(cudaMemset(dq.p, 0, qn * 2));
    TRY(cudaMemset(dk.p, 0, kn * 2));
    TRY(cudaMemset(dv.p, 0, kn * 2));
    TRY(cudaMemset(dout.p, 0xFF, qn * 2));  // NaN fill: every row of every sequence must be written
    TRY(cudaMemcpy(dq.p, q, size_t(ntok) * heads * hd * 2, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dk.p, k, size_t(ntok) * kvh * hd * 2, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dv.p, v, size_t(ntok) * kvh * hd * 2, cudaMemcpyHostToDevice));
    TRY(dwork.alloc(work.size() * 4));
    TRY(cudaMemcpy(dwork.p, work.data(), work.size() * 4, cudaMemcpyHostToDevice));
    TRY(derr.alloc(sizeof(int)));
    TRY(cudaMemset(derr.p, 0, sizeof(int)));
    TRY(ge::configure_attention_kernels());
    ge::AttnLaunch al;
    al.q = static_cast<const __half*>(dq.p);
    al.k = static_cast<const __half*>(dk.p);
    al.v = static_cast<const __half*>(dv.p);
    al.out = static_cast<__half*>(dout.p);
    al.work = static_cast<const uint32_t*>(dwork.p);
    al.work_items = ctas;
    al.sched_items = items;
    al.heads = heads;
    al.kv_heads = kvh;
    al.hd = hd;
    al.half_window = half_window;
    al.err = static_cast<int*>(derr.p);
    al.num_sms = sms;
    if (hd == 64) {
        ge::Attn64Launch a6;
        a6.q = al.q;
        a6.k = al.k;
        a6.v = al.v;
        a6.out = al.out;
        a6.rows = rows;
        a6.heads = heads;
        a6.work = al.work;
        a6.sched_items = items;
        a6.ctas = ctas;
        a6.err = al.err;
        TRY(ge::launch_attention64(a6, nullptr));
        TRY(cudaDeviceSynchronize());
        int herr = 0;
        TRY(cudaMemcpy(&herr, derr.p, sizeof(int), cudaMemcpyDeviceToHost));
        if (herr) return fail(herr, "GPU execution failed: a device-side wait timed out");
        TRY(cudaMemcpy(out, dout.p, size_t(ntok) * heads * hd * 2, cudaMemcpyDeviceToHost));
        return GE_OK;
    }
    ge::AttnMaps maps;
    if (!ge::encode_attention_maps(maps, al.q, al.k, al.v, rows, heads, kvh, hd))
        return fail(GE_ERR_GPU_FAILURE, "tensor map encoding failed");
    al.maps = &maps;
    TRY(ge::launch_attention(al, nullptr));
    TRY(cudaDeviceSynchronize());
    int herr = 0;
    TRY(cudaMemcpy(&herr, derr.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) return fail(herr, "GPU execution failed: a device-side wait timed out");
    TRY(cudaMemcpy(out, dout.p, size_t(ntok) * heads * hd * 2, cudaMemcpyDeviceToHost));
    return GE_OK;
}

int ge_test_image_prepare(int32_t patch, int32_t merge, int32_t min_tokens, const uint8_t* rgb, int32_t w, int32_t h,
                          int32_t max_tokens, uint8_t* out, int64_t cap, int32_t* tw, int32_t* th) {
    if (patch <= 0 || merge <= 0 || !rgb || w <= 0 || h <= 0 || max_tokens <= 0 || !tw || !th)
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options");
    ge::VisionConfig c;
    c.patch = patch;
    c.merge = merge;
    c.min_image_tokens = min_tokens;
    ge::PreparedImage im;
    ge::prepare_image(c, rgb, w, h, max_tokens, im);
    *tw = im.width;
    *th = im.height;
    if (int64_t(im.rgb.size()) > cap || (cap > 0 && !out)) return fail(GE_ERR_INVALID_OPTIONS, "output capacity too small");
    memcpy(out, im.rgb.data(), im.rgb.size());
    return GE_OK;
}

int ge_test_patchify(const uint8_t* rgb, int32_t w, int32_t h, int32_t patch, const float* mean, const float* std_,
                     uint16_t* out, int32_t kpad) {
    if (!rgb || w <= 0 || h <= 0 || patch <= 0 || w % patch || h % patch || !mean || !std_ || !out ||
        kpad < 3 * patch * patch)
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options");
    const int gx = w / patch, gy = h / patch;
    const size_t bytes = size_t(w) * h * 3, n = size_t(gx) * gy * kpad;
    DevBuf drgb, dimg, dout;
    TRY(drgb.alloc(bytes));
    TRY(dimg.alloc(sizeof(ge::VisionImage)));
    TRY(dout.alloc(n * 2));
    TRY(cudaMemcpy(drgb.p, rgb, bytes, cudaMemcpyHostToDevice));
    const ge::VisionImage im{0, gx, gy, 0, 0};
    TRY(cudaMemcpy(dimg.p, &im, sizeof im, cudaMemcpyHostToDevice));
    ge::NormParams np;
    for (int i = 0; i < 3; i++) {
        np.mean[i] = mean[i];
        np.std[i] = std_[i];
    }
    TRY(ge::launch_patchify(static_cast<const uint8_t*>(drgb.p), static_cast<const ge::VisionImage*>(dimg.p), 1, gx * gy,
                            patch, kpad, np, static_cast<__half*>(dout.p), nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, n * 2, cudaMemcpyDeviceToHost));
    return GE_OK;
}

int ge_test_log_mel(const float* samples, int64_t n, int32_t mel_bins, float* out, int32_t* frames) {
    if (!samples || n < ge::kAudioMinimumSamples || n > ge::kAudioChunkSamples || mel_bins != 128 || !out || !frames)
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options");
    float hann[512], sin_t[512], cos_t[512];
    int bitrev[512];
    std::vector<int> band;
    std::vector<float> w;
    ge::audio_front_tables(mel_bins, hann, sin_t, cos_t, bitrev, band, w);
    const int nf = ge::audio_frame_count(n);
    DevBuf dpcm, dch, dout, dh, dc, ds, dw, db, dband;
    TRY(dpcm.alloc(size_t(n) * 4));
    TRY(dch.alloc(sizeof(ge::AudioChunk)));
    TRY(dout.alloc(size_t(nf) * mel_bins * 4));
    TRY(dh.alloc(512 * 4));
    TRY(dc.alloc(512 * 4));
    TRY(ds.alloc(512 * 4));
    TRY(db.alloc(512 * 4));
    TRY(dw.alloc(w.size() * 4));
    TRY(dband.alloc(band.size() * 4));
    TRY(cudaMemcpy(dpcm.p, samples, size_t(n) * 4, cudaMemcpyHostToDevice));
    ge::AudioChunk ch{};
    ch.samples = int(n);
    ch.frames = nf;
    TRY(cudaMemcpy(dch.p, &ch, sizeof ch, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dh.p, hann, 512 * 4, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dc.p, cos_t, 512 * 4, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(ds.p, sin_t, 512 * 4, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(db.p, bitrev, 512 * 4, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dw.p, w.data(), w.size() * 4, cudaMemcpyHostToDevice));
    TRY(cudaMemcpy(dband.p, band.data(), band.size() * 4, cudaMemcpyHostToDevice));
    ge::MelTables t;
    t.hann = static_cast<const float*>(dh.p);
    t.cos_t = static_cast<const float*>(dc.p);
    t.sin_t = static_cast<const float*>(ds.p);
    t.w = static_cast<const float*>(dw.p);
    t.bitrev = static_cast<const int*>(db.p);
    t.band = static_cast<const int*>(dband.p);
    t.nw = int(w.size());
    t.mel = mel_bins;
    int dev = 0, sms = 148;
    TRY(cudaGetDevice(&dev));
    TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    TRY(ge::configure_audio_kernels());
    TRY(ge::launch_log_mel(static_cast<const float*>(dpcm.p), static_cast<const ge::AudioChunk*>(dch.p), 1, nf, t,
                           static_cast<float*>(dout.p), sms, nullptr));
    TRY(cudaDeviceSynchronize());
    TRY(cudaMemcpy(out, dout.p, size_t(nf) * mel_bins * 4, cudaMemcpyDeviceToHost));
    *frames = nf;
    return GE_OK;
}

int ge_test_multimodal_sequence(const char* prefix, const int32_t* kinds, const char* const* texts, int32_t nparts,
                                const int32_t* span_rows, int32_t max_tokens, int32_t bos, int32_t eos,
                                int32_t image_begin, int32_t image_end, int32_t audio_begin, int32_t audio_end,
                                int32_t* ids, int32_t cap, int32_t* count, int32_t* truncated) {
    if (nparts < 0 || (nparts > 0 && !kinds) || !count || !truncated || cap < 0 || (cap > 0 && !ids))
        return fail(GE_ERR_INVALID_OPTIONS, "invalid options");
    std::vector<ge::SeqPart> parts;
    std::vector<ge::EncoderSpan> spans;
    for (int32_t i = 0; i < nparts; i++) {
        ge::SeqPart p;
        p.kind = kinds[i];
        if (p.kind == ge::kPartText) {
            p.text = texts && texts[i] ? texts[i] : "";
        } else {
            ge::EncoderSpan sp;
            sp.rows = span_rows ? span_rows[spans.size()] : 0;
            sp.begin = p.kind == ge::kPartImage ? image_begin : audio_begin;
            sp.end = p.kind == ge::kPartImage ? image_end : audio_end;
            spans.push_back(sp);
        }
        parts.push_back(p);
    }
    // One id per Unicode scalar of the UTF-8 text.
    auto scalars = [](const std::string& t, std::vector<int32_t>& out) {
        out.clear();
        for (size_t i = 0; i < t.size();) {
            const uint8_t b = uint8_t(t[i]);
            int n = b < 0x80 ? 1 : (b & 0xE0) == 0xC0 ? 2 : (b & 0xF0) == 0xE0 ? 3 : 4;
            int32_t cp = n == 1 ? b : n == 2 ? (b & 0x1F) : n == 3 ? (b & 0x0F) : (b & 0x07);
            for (int k = 1; k < n && i + size_t(k) < t.size(); k++) cp = (cp << 6) | (uint8_t(t[i + size_t(k)]) & 0x3F);
            out.push_back(cp);
            i += size_t(n);
        }
    };
    std::vector<int32_t> v;
    bool cut = false;
    if (!ge::multimodal_sequence(prefix ? prefix : "", parts, spans, max_tokens, bos, eos, scalars, v, cut))
        return fail(GE_ERR_INVALID_OPTIONS, "the spans alone do not fit");
    *count = int32_t(v.size());
    *truncated = cut ? 1 : 0;
    if (int32_t(v.size()) > cap) return fail(GE_ERR_INVALID_OPTIONS, "output capacity too small");
    std::copy(v.begin(), v.end(), ids);
    return GE_OK;
}

}  // extern "C"
