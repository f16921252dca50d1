// audio.cu -- the gemma4a audio encoder's own kernels (the GEMMs run through gemm.cu with the
// clamp epilogues):
//
//   k_log_mel            16 kHz PCM -> log-mel frames, the reference's FFT and mel sums bit for bit
//                        (AudioFrontEnd.logMel / melRow / fft, Audio/AudioPreprocessor.swift:144-249)
//   k_audio_conv0        conv 3x3 stride 2 (1 -> 128 channels), LayerNorm over channels, ReLU
//                        (CPUAudioReference.subsample, Model/CPUAudioReference.swift:67-101)
//   k_audio_im2col       the second convolution's patches as GEMM rows (tap-major K)
//   k_audio_subsample_norm  its LayerNorm (32 channels) and ReLU, flattened to the Conformer's input
//   k_audio_rows         residual adds, RMS norms and the next linears' input clamps on whole rows
//   k_audio_attention    12-frame causal attention with relative keys and the 50 tanh soft cap
//                        (CPUAudioReference.attention, CPUAudioReference.swift:127-165)
//   k_audio_dwconv       causal depthwise conv k5, RMS norm, SiLU, the next input clamp
//                        (CPUAudioReference.swift:255-262 and depthwiseCausal, 168-181)
#include <float.h>

#include <algorithm>

#include "kernels.hpp"
#include "ptx.cuh"

namespace ge {

#define CK_LAUNCH(expr)                   \
    do {                                  \
        const cudaError_t e_ = (expr);    \
        if (e_ != cudaSuccess) return e_; \
    } while (0)

namespace {

constexpr int kFft = 512, kHop = 160, kPadLeft = 160, kBins = kFft / 2 + 1;
constexpr int kMel = 128, kF0 = 64, kC0 = 128, kF1 = 32, kC1 = 32, kTaps1 = 9 * kC0;

// The chunk holding packed row `r` of the field F (the chunks are in row order).
template <int32_t AudioChunk::*F>
__device__ __forceinline__ int chunk_of(const AudioChunk* __restrict__ c, int n, int r) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (c[mid].*F <= r) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

}  // namespace

// ---------------------------------------------------------------------------- log-mel
// One warp per frame: the windowed frame is written bit-reversed into the warp's buffer, nine
// in-place radix-2 levels follow with the reference's twiddles and operation order (separately
// rounded multiplies and adds, no fused multiply-add), then the magnitudes and, per mel filter,
// four-bin fp32 partial sums added into a double, floored at fp32(0.001) and logged.
__global__ void __launch_bounds__(256) k_log_mel(const float* __restrict__ pcm, const AudioChunk* __restrict__ chunks,
                                                 int nchunks, int frames_total, MelTables t, float* __restrict__ out) {
    extern __shared__ float sm[];
    float* hann = sm;
    float* cos_t = hann + kFft;
    float* sin_t = cos_t + kFft;
    float* fw = sin_t + kFft;
    int* bitrev = reinterpret_cast<int*>(fw + t.nw);
    int* band = bitrev + kFft;  // lo[mel], hi[mel], off[mel]
    float* bufs = reinterpret_cast<float*>(band + 3 * t.mel);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* buf = bufs + warp * (2 * kFft + 264);
    float* mag = buf + 2 * kFft;
    for (int i = threadIdx.x; i < kFft; i += blockDim.x) {
        hann[i] = t.hann[i];
        cos_t[i] = t.cos_t[i];
        sin_t[i] = t.sin_t[i];
        bitrev[i] = t.bitrev[i];
    }
    for (int i = threadIdx.x; i < t.nw; i += blockDim.x) fw[i] = t.w[i];
    for (int i = threadIdx.x; i < 3 * t.mel; i += blockDim.x) band[i] = t.band[i];
    pdl_wait();
    __syncthreads();
    for (int f = blockIdx.x * 8 + warp; f < frames_total; f += gridDim.x * 8) {
        const AudioChunk ch = chunks[chunk_of<&AudioChunk::mel_row>(chunks, nchunks, f)];
        const int fl = f - ch.mel_row;
        const float* s = pcm + ch.pcm_offset;
        // padded[p] = chunk[p - 160] (160 zeros in front, zeros past the end)
        for (int j = lane; j < kFft; j += 32) {
            const int idx = fl * kHop + j - kPadLeft;
            const float x = (idx >= 0 && idx < ch.samples) ? s[idx] : 0.0f;
            const int r = bitrev[j];
            buf[2 * r] = __fmul_rn(hann[j], x);
            buf[2 * r + 1] = 0.0f;
        }
        __syncwarp();
#pragma unroll 1
        for (int lg = 0; lg < 9; lg++) {
            const int half = 1 << lg, count = half << 1, step = kFft / count;
#pragma unroll 4
            for (int b = lane; b < kFft / 2; b += 32) {
                const int k = b & (half - 1);
                const int ev = 2 * ((b >> lg) * count + k), od = ev + 2 * half;
                const float re = cos_t[k * step], im = -sin_t[k * step];
                const float ro = buf[od], io = buf[od + 1], er = buf[ev], ei = buf[ev + 1];
                const float a = __fmul_rn(re, ro), bq = __fmul_rn(im, io), c = __fmul_rn(re, io), d = __fmul_rn(im, ro);
                buf[ev] = __fsub_rn(__fadd_rn(er, a), bq);
                buf[ev + 1] = __fadd_rn(__fadd_rn(ei, c), d);
                buf[od] = __fadd_rn(__fsub_rn(er, a), bq);
                buf[od + 1] = __fsub_rn(__fsub_rn(ei, c), d);
            }
            __syncwarp();
        }
        for (int j = lane; j < kBins; j += 32)
            mag[j] = __fsqrt_rn(__fadd_rn(__fmul_rn(buf[2 * j], buf[2 * j]), __fmul_rn(buf[2 * j + 1], buf[2 * j + 1])));
        __syncwarp();
        for (int m = lane; m < t.mel; m += 32) {
            const int lo = band[m], hi = band[t.mel + m];
            const float* w = fw + band[2 * t.mel + m] - lo;
            const int lim = hi < kBins - 3 ? hi : kBins - 3;
            double sum = 0.0;
            int k = lo;
            for (; k < lim; k += 4) {
                float p = __fadd_rn(__fmul_rn(mag[k], w[k]), __fmul_rn(mag[k + 1], w[k + 1]));
                p = __fadd_rn(p, __fmul_rn(mag[k + 2], w[k + 2]));
                p = __fadd_rn(p, __fmul_rn(mag[k + 3], w[k + 3]));
                sum = __dadd_rn(sum, double(p));
            }
            for (; k < hi; k++) sum = __dadd_rn(sum, double(__fmul_rn(mag[k], w[k])));
            const double floor_ = double(0.001f);
            out[size_t(f) * t.mel + m] = float(log(sum > floor_ ? sum : floor_));
        }
        __syncwarp();
    }
}

size_t log_mel_smem(const MelTables& t) {
    return size_t(3 * kFft + t.nw) * 4 + size_t(kFft + 3 * t.mel) * 4 + size_t(8) * (2 * kFft + 264) * 4;
}

cudaError_t launch_log_mel(const float* pcm, const AudioChunk* chunks, int nchunks, int frames_total,
                           const MelTables& t, float* out, int num_sms, cudaStream_t stream) {
    if (frames_total <= 0) return cudaSuccess;
    if (t.mel != kMel || t.nw > kMel * kBins) return cudaErrorInvalidValue;
    const size_t smem = log_mel_smem(t);
    const int blocks = std::min((frames_total + 7) / 8, num_sms * 4);
    CK_LAUNCH(launch_kernel(k_log_mel, dim3(blocks), dim3(256), smem, stream, 1, pcm, chunks, nchunks, frames_total, t, out));
    return cudaGetLastError();
}

cudaError_t configure_audio_kernels() {
    // The largest table set the launcher accepts: 128 filters of at most 257 weights each.
    const size_t most = size_t(3 * kFft + kMel * kBins) * 4 + size_t(kFft + 3 * kMel) * 4 + size_t(8) * (2 * kFft + 264) * 4;
    return cudaFuncSetAttribute(k_log_mel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(std::min<size_t>(most, 227 * 1024)));
}

// ---------------------------------------------------------------------------- subsampling
// One block per conv0 output time row; warp w computes frequencies 8w..8w+7, lane l channels
// 4l..4l+3.  The three mel rows it reads are staged fp16-rounded (ggml's im2col runs in fp16).
__global__ void __launch_bounds__(256) k_audio_conv0(const float* __restrict__ mel, const AudioChunk* __restrict__ chunks,
                                                     int nchunks, const float* __restrict__ w, const float* __restrict__ nw,
                                                     float eps, __half* __restrict__ out) {
    __shared__ float in[3][kMel];
    __shared__ float ws[kC0 * 9];
    __shared__ float ns[kC0];
    const int r0 = blockIdx.x;
    for (int i = threadIdx.x; i < kC0 * 9; i += 256) ws[i] = w[i];
    if (threadIdx.x < kC0) ns[threadIdx.x] = nw[threadIdx.x];
    pdl_wait();
    pdl_launch_if_one_wave();
    const AudioChunk ch = chunks[chunk_of<&AudioChunk::t0_row>(chunks, nchunks, r0)];
    const int ot = r0 - ch.t0_row;
    for (int i = threadIdx.x; i < 3 * kMel; i += 256) {
        const int kh = i / kMel, fq = i % kMel, tt = 2 * ot + kh - 1;
        const float v = (tt >= 0 && tt < ch.frames) ? mel[size_t(ch.mel_row + tt) * kMel + fq] : 0.0f;
        in[kh][fq] = __half2float(__float2half_rn(v));
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int of = warp * 8; of < warp * 8 + 8; of++) {
        float x[9];
#pragma unroll
        for (int kh = 0; kh < 3; kh++)
#pragma unroll
            for (int kw = 0; kw < 3; kw++) {
                const int fq = 2 * of + kw - 1;
                x[kh * 3 + kw] = (fq >= 0 && fq < kMel) ? in[kh][fq] : 0.0f;
            }
        float c[4];
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float* wr = ws + (4 * lane + j) * 9;
            float a = 0.f;
#pragma unroll
            for (int k = 0; k < 9; k++) a += wr[k] * x[k];
            c[j] = a;
            sum += a;
        }
        const float mean = warp_sum(sum) / float(kC0);
        float var = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) var += (c[j] - mean) * (c[j] - mean);
        var = warp_sum(var) / float(kC0);
        const float scale = 1.0f / sqrtf(var + eps);
        uint2 o;
        o.x = pack_half2(fmaxf(0.f, (c[0] - mean) * scale * ns[4 * lane]), fmaxf(0.f, (c[1] - mean) * scale * ns[4 * lane + 1]));
        o.y = pack_half2(fmaxf(0.f, (c[2] - mean) * scale * ns[4 * lane + 2]), fmaxf(0.f, (c[3] - mean) * scale * ns[4 * lane + 3]));
        *reinterpret_cast<uint2*>(out + (size_t(r0) * kF0 + of) * kC0 + 4 * lane) = o;
    }
}

cudaError_t launch_audio_conv0(const float* mel, const AudioChunk* chunks, int nchunks, int t0_total, const float* w,
                               const float* nw, float eps, __half* out, cudaStream_t stream) {
    if (t0_total <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_audio_conv0, dim3(t0_total), dim3(256), 0, stream, 1, mel, chunks, nchunks, w, nw, eps, out));
    return cudaGetLastError();
}

// One block per token row: the 32 output positions' 9 taps x 128 channels, K index
// (kh * 3 + kw) * 128 + c, zero outside the chunk's conv0 rows and the 64 frequencies.
// Rows at or past `tokens` are zero.
__global__ void __launch_bounds__(256) k_audio_im2col(const __half* __restrict__ c0, const AudioChunk* __restrict__ chunks,
                                                      int nchunks, int tokens, __half* __restrict__ a) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const int r = blockIdx.x;
    int ot = 0, t0 = 0, t0_row = 0;
    if (r < tokens) {
        const AudioChunk ch = chunks[chunk_of<&AudioChunk::token_row>(chunks, nchunks, r)];
        ot = r - ch.token_row;
        t0 = ch.t0;
        t0_row = ch.t0_row;
    }
    for (int i = threadIdx.x; i < kF1 * 9 * 16; i += 256) {
        const int pos = i / 144, rem = i % 144, tap = rem >> 4, part = rem & 15;
        const int tt = 2 * ot + tap / 3 - 1, fq = 2 * pos + tap % 3 - 1;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < tokens && tt >= 0 && tt < t0 && fq >= 0 && fq < kF0)
            v = *reinterpret_cast<const uint4*>(c0 + (size_t(t0_row + tt) * kF0 + fq) * kC0 + part * 8);
        *reinterpret_cast<uint4*>(a + (size_t(r) * kF1 + pos) * kTaps1 + tap * kC0 + part * 8) = v;
    }
}

cudaError_t launch_audio_im2col(const __half* c0, const AudioChunk* chunks, int nchunks, int tokens, int trows, __half* a,
                                cudaStream_t stream) {
    if (trows <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_audio_im2col, dim3(trows), dim3(256), 0, stream, 1, c0, chunks, nchunks, tokens, a));
    return cudaGetLastError();
}

// One warp per conv1 output position (lane = channel): LayerNorm over the 32 channels of the
// GEMM's first 32 columns, the norm weight, ReLU and the input projection's clamp; written to
// the token row at column frequency * 32 + channel.
__global__ void __launch_bounds__(256) k_audio_subsample_norm(const float* __restrict__ c1, int positions,
                                                              const float* __restrict__ nw, float eps, float lo, float hi,
                                                              __half* __restrict__ a2) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const int p = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (p >= positions) return;
    const float v = c1[size_t(p) * 128 + lane];
    const float mean = warp_sum(v) / float(kC1);
    const float var = warp_sum((v - mean) * (v - mean)) / float(kC1);
    const float scale = 1.0f / sqrtf(var + eps);
    const float y = fmaxf(0.f, (v - mean) * scale * nw[lane]);
    a2[size_t(p / kF1) * (kF1 * kC1) + (p % kF1) * kC1 + lane] = __float2half_rn(clampf(y, lo, hi));
}

cudaError_t launch_audio_subsample_norm(const float* c1, int trows, const float* nw, float eps, float lo, float hi,
                                        __half* a2, cudaStream_t stream) {
    const int positions = trows * kF1;
    if (positions <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_audio_subsample_norm, dim3((positions + 7) / 8), dim3(256), 0, stream, 1, c1, positions, nw,
                            eps, lo, hi, a2));
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------- row steps
// One warp per row; lane l holds columns (32 i + l) * 4 + [0, 4).
template <int W>
__global__ void __launch_bounds__(256) k_audio_rows(AudioRowStep s) {
    constexpr int G = W / 128;  // float4 groups per lane
    pdl_wait();
    pdl_launch_if_one_wave();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= s.rows) return;
    float4 v[G];
    float* xr = s.x + size_t(row) * W;
#pragma unroll
    for (int i = 0; i < G; i++) v[i] = *reinterpret_cast<const float4*>(xr + (i * 32 + lane) * 4);
    auto rms_inv = [&](const float4* a) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < G; i++) ss += a[i].x * a[i].x + a[i].y * a[i].y + a[i].z * a[i].z + a[i].w * a[i].w;
        ss = warp_sum(ss);
        return 1.0f / sqrtf(ss / float(W) + s.eps);
    };
    if (s.branch) {
        float4 b[G];
        const __half* br = s.branch + size_t(row) * W;
#pragma unroll
        for (int i = 0; i < G; i++) {
            const uint2 u = *reinterpret_cast<const uint2*>(br + (i * 32 + lane) * 4);
            const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            b[i] = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
        if (s.branch_w) {
            const float inv = rms_inv(b);
#pragma unroll
            for (int i = 0; i < G; i++) {
                const float4 w = *reinterpret_cast<const float4*>(s.branch_w + (i * 32 + lane) * 4);
                v[i].x += b[i].x * inv * w.x;
                v[i].y += b[i].y * inv * w.y;
                v[i].z += b[i].z * inv * w.z;
                v[i].w += b[i].w * inv * w.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < G; i++) {
                v[i].x += b[i].x;
                v[i].y += b[i].y;
                v[i].z += b[i].z;
                v[i].w += b[i].w;
            }
        }
    }
    if (s.final_w) {
        const float inv = rms_inv(v);
#pragma unroll
        for (int i = 0; i < G; i++) {
            const float4 w = *reinterpret_cast<const float4*>(s.final_w + (i * 32 + lane) * 4);
            v[i] = make_float4(v[i].x * inv * w.x, v[i].y * inv * w.y, v[i].z * inv * w.z, v[i].w * inv * w.w);
        }
    }
    if (s.store_x)
#pragma unroll
        for (int i = 0; i < G; i++) *reinterpret_cast<float4*>(xr + (i * 32 + lane) * 4) = v[i];
    if (s.nout == 0) return;
    float4 h[G];
    if (s.next_norm) {
        const float inv = rms_inv(v);
#pragma unroll
        for (int i = 0; i < G; i++) {
            const float4 w = s.next_w ? *reinterpret_cast<const float4*>(s.next_w + (i * 32 + lane) * 4)
                                      : make_float4(1.f, 1.f, 1.f, 1.f);
            h[i] = make_float4(v[i].x * inv * w.x, v[i].y * inv * w.y, v[i].z * inv * w.z, v[i].w * inv * w.w);
        }
    } else {
#pragma unroll
        for (int i = 0; i < G; i++) h[i] = v[i];
    }
#pragma unroll
    for (int o = 0; o < 3; o++) {
        if (o >= s.nout) break;
        __half* dst = s.out[o] + size_t(row) * W;
        const float lo = s.lo[o], hi = s.hi[o];
#pragma unroll
        for (int i = 0; i < G; i++) {
            uint2 u;
            u.x = pack_half2(clampf(h[i].x, lo, hi), clampf(h[i].y, lo, hi));
            u.y = pack_half2(clampf(h[i].z, lo, hi), clampf(h[i].w, lo, hi));
            *reinterpret_cast<uint2*>(dst + (i * 32 + lane) * 4) = u;
        }
    }
}

cudaError_t launch_audio_rows(const AudioRowStep& s, int width, cudaStream_t stream) {
    if (s.rows <= 0) return cudaSuccess;
    const dim3 grid((s.rows + 7) / 8);
    switch (width) {
    case 512: CK_LAUNCH(launch_kernel(k_audio_rows<512>, grid, dim3(256), 0, stream, 1, s)); break;
    case 768: CK_LAUNCH(launch_kernel(k_audio_rows<768>, grid, dim3(256), 0, stream, 1, s)); break;
    case 1024: CK_LAUNCH(launch_kernel(k_audio_rows<1024>, grid, dim3(256), 0, stream, 1, s)); break;
    case 1536: CK_LAUNCH(launch_kernel(k_audio_rows<1536>, grid, dim3(256), 0, stream, 1, s)); break;
    case 2048: CK_LAUNCH(launch_kernel(k_audio_rows<2048>, grid, dim3(256), 0, stream, 1, s)); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------- attention
// Block: 32 query rows of one head (8 warps x 4 rows).  Keys and values of rows r0 - 11 ..
// r0 + 31 are staged as fp16; query row t reads keys max(chunk start, t - 11) .. t.  Lane l holds
// head dims 4l .. 4l + 3.  The score is kscale (q' . k) + q' . rel[t - j] with q' the scaled query.
constexpr int kAttnRows = 32, kAttnWin = 12, kAttnHd = 128;
__global__ void __launch_bounds__(256) k_audio_attention(AudioAttnLaunch a) {
    __shared__ __align__(16) __half ks[kAttnRows + kAttnWin - 1][kAttnHd];
    __shared__ __align__(16) __half vs[kAttnRows + kAttnWin - 1][kAttnHd];
    __shared__ __align__(16) float rel[kAttnWin + 1][kAttnHd];
    __shared__ __align__(16) float qsc[kAttnHd];
    const int r0 = blockIdx.x * kAttnRows, h = blockIdx.y, W = a.heads * kAttnHd;
    const int base = r0 - (kAttnWin - 1);
    for (int i = threadIdx.x; i < (kAttnWin + 1) * kAttnHd; i += 256)
        rel[i / kAttnHd][i % kAttnHd] = a.rel[(i / kAttnHd) * W + h * kAttnHd + i % kAttnHd];
    if (threadIdx.x < kAttnHd) qsc[threadIdx.x] = a.qscale[threadIdx.x];
    pdl_wait();
    pdl_launch_if_one_wave();
    for (int i = threadIdx.x; i < (kAttnRows + kAttnWin - 1) * (kAttnHd / 8); i += 256) {
        const int rr = i / (kAttnHd / 8), c8 = (i % (kAttnHd / 8)) * 8, j = base + rr;
        uint4 ku = make_uint4(0, 0, 0, 0), vu = make_uint4(0, 0, 0, 0);
        if (j >= 0 && j < a.rows) {
            ku = *reinterpret_cast<const uint4*>(a.k + size_t(j) * W + h * kAttnHd + c8);
            vu = *reinterpret_cast<const uint4*>(a.v + size_t(j) * W + h * kAttnHd + c8);
        }
        *reinterpret_cast<uint4*>(&ks[rr][c8]) = ku;
        *reinterpret_cast<uint4*>(&vs[rr][c8]) = vu;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float4 qs = *reinterpret_cast<const float4*>(&qsc[4 * lane]);
    auto ld4 = [&](const __half* p) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    };
    for (int i = 0; i < kAttnRows / 8; i++) {
        const int t = r0 + warp * (kAttnRows / 8) + i;
        if (t >= a.rows) break;
        const float4 qv = ld4(a.q + size_t(t) * W + h * kAttnHd + 4 * lane);
        const float q0 = qv.x * qs.x, q1 = qv.y * qs.y, q2 = qv.z * qs.z, q3 = qv.w * qs.w;
        const int cs = a.chunk_start[t];
        const int first = max(cs, t - (kAttnWin - 1));
        const int n = t - first + 1;  // keys, oldest first: j = first + m
        float sc[kAttnWin];
        float mx = -FLT_MAX;
#pragma unroll
        for (int m = 0; m < kAttnWin; m++) {
            if (m < n) {
                const int j = first + m, dist = t - j;
                const float4 kk = ld4(&ks[j - base][4 * lane]);
                const float4 rr = *reinterpret_cast<const float4*>(&rel[dist][4 * lane]);
                float part = q0 * kk.x + q1 * kk.y + q2 * kk.z + q3 * kk.w;
                float pr = q0 * rr.x + q1 * rr.y + q2 * rr.z + q3 * rr.w;
                part = warp_sum(part);
                pr = warp_sum(pr);
                const float c = a.softcap * tanhf((part * a.kscale + pr) / a.softcap);
                sc[m] = c;
                mx = fmaxf(mx, c);
            }
        }
        float sum = 0.f;
#pragma unroll
        for (int m = 0; m < kAttnWin; m++)
            if (m < n) {
                sc[m] = expf(sc[m] - mx);
                sum += sc[m];
            }
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
        for (int m = 0; m < kAttnWin; m++)
            if (m < n) {
                const float p = sc[m] / sum;
                const float4 vv = ld4(&vs[first + m - base][4 * lane]);
                o0 += p * vv.x;
                o1 += p * vv.y;
                o2 += p * vv.z;
                o3 += p * vv.w;
            }
        uint2 o;
        o.x = pack_half2(clampf(o0, a.lo, a.hi), clampf(o1, a.lo, a.hi));
        o.y = pack_half2(clampf(o2, a.lo, a.hi), clampf(o3, a.lo, a.hi));
        *reinterpret_cast<uint2*>(a.out + size_t(t) * W + h * kAttnHd + 4 * lane) = o;
    }
}

cudaError_t launch_audio_attention(const AudioAttnLaunch& a, cudaStream_t stream) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.head_dim != kAttnHd) return cudaErrorInvalidValue;
    CK_LAUNCH(launch_kernel(k_audio_attention, dim3((a.rows + kAttnRows - 1) / kAttnRows, a.heads), dim3(256), 0, stream, 1, a));
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------- depthwise conv
// One warp per row; lane l holds channels (32 i + l) * 8 + [0, 8).  dw_t is [5][W] (tap-major),
// tap 4 on the current row; rows before the chunk's first row contribute nothing.
template <int W>
__global__ void __launch_bounds__(256) k_audio_dwconv(const __half* __restrict__ glu, const int* __restrict__ chunk_start,
                                                      int rows, const float* __restrict__ dw_t, const float* __restrict__ nw,
                                                      float eps, float lo, float hi, __half* __restrict__ out) {
    constexpr int G = W / 256;  // groups of 8 channels per lane
    pdl_wait();
    pdl_launch_if_one_wave();
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= rows) return;
    const int cs = chunk_start[t];
    float acc[G][8];
#pragma unroll
    for (int i = 0; i < G; i++)
#pragma unroll
        for (int e = 0; e < 8; e++) acc[i][e] = 0.f;
#pragma unroll
    for (int k = 0; k < 5; k++) {
        const int src = t + k - 4;
        if (src < cs) continue;
#pragma unroll
        for (int i = 0; i < G; i++) {
            const int c = (i * 32 + lane) * 8;
            const uint4 u = *reinterpret_cast<const uint4*>(glu + size_t(src) * W + c);
            const __half2* hv = reinterpret_cast<const __half2*>(&u);
            const float4 w0 = *reinterpret_cast<const float4*>(dw_t + k * W + c);
            const float4 w1 = *reinterpret_cast<const float4*>(dw_t + k * W + c + 4);
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(hv[e]);
                acc[i][2 * e] += f.x * wv[2 * e];
                acc[i][2 * e + 1] += f.y * wv[2 * e + 1];
            }
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < G; i++)
#pragma unroll
        for (int e = 0; e < 8; e++) ss += acc[i][e] * acc[i][e];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(W) + eps);
#pragma unroll
    for (int i = 0; i < G; i++) {
        const int c = (i * 32 + lane) * 8;
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float y0 = acc[i][2 * e] * inv * nw[c + 2 * e], y1 = acc[i][2 * e + 1] * inv * nw[c + 2 * e + 1];
            y0 = y0 / (1.0f + expf(-y0));
            y1 = y1 / (1.0f + expf(-y1));
            pk[e] = pack_half2(clampf(y0, lo, hi), clampf(y1, lo, hi));
        }
        *reinterpret_cast<uint4*>(out + size_t(t) * W + c) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
}

cudaError_t launch_audio_dwconv(const __half* glu, const int* chunk_start, int rows, int width, const float* dw_t,
                                const float* nw, float eps, float lo, float hi, __half* out, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const dim3 grid((rows + 7) / 8);
    switch (width) {
    case 512: CK_LAUNCH(launch_kernel(k_audio_dwconv<512>, grid, dim3(256), 0, stream, 1, glu, chunk_start, rows, dw_t, nw, eps, lo, hi, out)); break;
    case 768: CK_LAUNCH(launch_kernel(k_audio_dwconv<768>, grid, dim3(256), 0, stream, 1, glu, chunk_start, rows, dw_t, nw, eps, lo, hi, out)); break;
    case 1024: CK_LAUNCH(launch_kernel(k_audio_dwconv<1024>, grid, dim3(256), 0, stream, 1, glu, chunk_start, rows, dw_t, nw, eps, lo, hi, out)); break;
    case 1536: CK_LAUNCH(launch_kernel(k_audio_dwconv<1536>, grid, dim3(256), 0, stream, 1, glu, chunk_start, rows, dw_t, nw, eps, lo, hi, out)); break;
    case 2048: CK_LAUNCH(launch_kernel(k_audio_dwconv<2048>, grid, dim3(256), 0, stream, 1, glu, chunk_start, rows, dw_t, nw, eps, lo, hi, out)); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace ge
