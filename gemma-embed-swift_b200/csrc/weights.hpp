// weights.hpp -- host-side weight preparation shared by the text model and the image encoder:
// GGUF tensor checks, dequantisation, the repack of GEMM weights into the device layout
// (Q8_0 planes and the exact fp16 dequantisation) and their upload.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <thread>
#include <vector>

#include "gemma_embed.h"
#include "gguf.hpp"
#include "kernels.hpp"

namespace ge {

constexpr int kBN = 256;

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

inline float half_bits_to_float(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}
inline uint16_t float_to_half_bits(float f) {
    __half h = __float2half_rn(f);
    return __half_raw(h).x;
}

// ------------------------------------------------------------------ config
struct LoadError {
    int code;
    std::string msg;
};

// ModelWeights' shape and type checks (Weights.swift:93-98).
inline const GgufTensor* need_tensor(const GgufFile& f, const std::string& name, std::vector<int64_t> shape, bool f32_only,
                              LoadError& e) {
    const GgufTensor* t = f.tensor(name);
    auto fmt = [](const std::vector<int64_t>& s) {
        std::string r = "[";
        for (size_t i = 0; i < s.size(); i++) r += (i ? ", " : "") + std::to_string(s[i]);
        return r + "]";
    };
    if (!t) {
        e = {GE_ERR_MISSING_TENSOR, "weight file lacks tensor " + name};
        return nullptr;
    }
    if (t->shape != shape) {
        e = {GE_ERR_SHAPE_MISMATCH, "tensor " + name + " has shape " + fmt(t->shape) + ", expected " + fmt(shape)};
        return nullptr;
    }
    if (f32_only && t->type != GGML_F32) {
        e = {GE_ERR_UNSUPPORTED_TENSOR_TYPE, "tensor " + name + " uses unsupported storage type " + std::to_string(t->type)};
        return nullptr;
    }
    return t;
}

// Dequantised fp32 row of a tensor (WeightTensor.dequantizeRow, Weights.swift:19-43).
inline void dequant_row(const GgufTensor& t, int64_t row, float* out) {
    const int64_t n = t.cols();
    const uint8_t* p = t.data + row * (n / ggml_block_elems(t.type) * ggml_block_bytes(t.type));
    switch (t.type) {
    case GGML_F32: memcpy(out, p, size_t(n) * 4); break;
    case GGML_F16:
        for (int64_t i = 0; i < n; i++) {
            uint16_t h;
            memcpy(&h, p + 2 * i, 2);
            out[i] = half_bits_to_float(h);
        }
        break;
    case GGML_BF16:
        for (int64_t i = 0; i < n; i++) {
            uint16_t h;
            memcpy(&h, p + 2 * i, 2);
            uint32_t b = uint32_t(h) << 16;
            memcpy(&out[i], &b, 4);
        }
        break;
    case GGML_Q8_0:
        for (int64_t b = 0; b < n / 32; b++) {
            uint16_t h;
            memcpy(&h, p + b * 34, 2);
            const float s = half_bits_to_float(h);
            for (int j = 0; j < 32; j++) out[b * 32 + j] = s * float(int8_t(p[b * 34 + 2 + j]));
        }
        break;
    }
}

template <class F>
inline void parallel_rows(int64_t rows, F fn) {
    const int nt = std::max(1, std::min<int>(16, int(std::thread::hardware_concurrency())));
    std::vector<std::thread> th;
    for (int t = 0; t < nt; t++)
        th.emplace_back([=]() {
            for (int64_t r = t; r < rows; r += nt) fn(r);
        });
    for (auto& x : th) x.join();
}

// A GEMM weight assembled on the host from one or more GGUF tensors stacked along N.
// `rows_of(dst_row)` names the (tensor, source row) each destination row comes from.
struct HostWeight {
    int N = 0, K = 0;
    bool q8 = true;
    std::vector<int8_t> q;
    std::vector<uint16_t> scales_t;  // [K/32][N]
    std::vector<uint16_t> f16;       // [N][K]
};

template <class RowFn>
HostWeight build_weight(int N, int K, bool want_f16, RowFn src) {
    HostWeight w;
    w.N = N;
    w.K = K;
    const GgufTensor* t0 = src(0).first;
    w.q8 = t0->type == GGML_Q8_0;
    for (int r = 1; r < N && w.q8; r++) w.q8 = src(r).first->type == GGML_Q8_0;
    if (w.q8) {
        w.q.resize(size_t(N) * K);
        w.scales_t.resize(size_t(N) * (K / 32));
    }
    if (want_f16 || !w.q8) w.f16.resize(size_t(N) * K);
    parallel_rows(N, [&](int64_t r) {
        auto s = src(int(r));
        const GgufTensor& t = *s.first;
        if (w.q8) {
            const uint8_t* p = t.data + int64_t(s.second) * (K / 32) * 34;
            for (int b = 0; b < K / 32; b++) {
                uint16_t h;
                memcpy(&h, p + b * 34, 2);
                w.scales_t[size_t(b) * N + r] = h;
                const float sc = half_bits_to_float(h);
                for (int j = 0; j < 32; j++) {
                    const int8_t qv = int8_t(p[b * 34 + 2 + j]);
                    w.q[size_t(r) * K + b * 32 + j] = qv;
                    // scale * q is exact in fp32; one round to nearest gives the fp16 operand.
                    if (!w.f16.empty()) w.f16[size_t(r) * K + b * 32 + j] = float_to_half_bits(sc * float(qv));
                }
            }
        } else {
            std::vector<float> row(K);
            dequant_row(t, s.second, row.data());
            for (int k = 0; k < K; k++) w.f16[size_t(r) * K + k] = float_to_half_bits(row[k]);
        }
    });
    return w;
}

inline std::vector<float> dequant_matrix(const GgufTensor& t) {
    std::vector<float> out(size_t(t.elements()));
    parallel_rows(t.rows(), [&](int64_t r) { dequant_row(t, r, out.data() + r * t.cols()); });
    return out;
}

template <class T>
inline cudaError_t dev_alloc(std::vector<void*>& owned, T** p, size_t count) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) return e;
    owned.push_back(q);
    *p = static_cast<T*>(q);
    return cudaSuccess;
}

template <class T>
inline cudaError_t dev_upload(std::vector<void*>& owned, T** p, const T* src, size_t count) {
    cudaError_t e = dev_alloc(owned, p, count);
    if (e == cudaSuccess && count) e = cudaMemcpy(*p, src, count * sizeof(T), cudaMemcpyHostToDevice);
    return e;
}

inline cudaError_t upload_weight(std::vector<void*>& owned, DevWeight& w, const HostWeight& h) {
    w.N = h.N;
    w.K = h.K;
    cudaError_t e = cudaSuccess;
    if (h.q8) {
        e = dev_upload(owned, &w.q8, h.q.data(), h.q.size());
        if (e == cudaSuccess) e = dev_upload(owned, reinterpret_cast<uint16_t**>(&w.scales_t), h.scales_t.data(), h.scales_t.size());
    }
    if (e == cudaSuccess && !h.f16.empty())
        e = dev_upload(owned, reinterpret_cast<uint16_t**>(&w.f16), h.f16.data(), h.f16.size());
    if (e == cudaSuccess && !encode_weight_maps(w, kBN)) e = cudaErrorInvalidValue;
    return e;
}

}  // namespace ge
