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
// One warp per frame, the whole 512-point FFT in registers: after the bit-reversed copy, element
// i sits in lane i % 32, register i / 32.  Lane l therefore loads the 16 consecutive window
// samples from rev5(l) * 16 (register r takes sample rev5(l) * 16 + rev4(r)).  The nine radix-2
// levels use the reference's twiddles and operation order in separately rounded fp32 (no fused
// multiply-add): the five levels whose partners are fewer than 32 elements apart exchange
// values between lanes by shuffle (both partners compute the same products, each keeps its own
// output), the four others pair registers within a lane.  Then the magnitudes and, per mel
// filter, four-bin fp32 partial sums added into a double, floored at fp32(0.001) and logged.
constexpr int kLogMelWarpFloats = 264;  // magnitudes of the warp's frame

__global__ void __launch_bounds__(256) k_log_mel(const float* __restrict__ pcm, const AudioChunk* __restrict__ chunks,
                                                 int nchunks, int frames_total, MelTables t, float* __restrict__ out) {
    extern __shared__ float sm[];
    float* hann = sm;
    float* cos_t = hann + kFft;
    float* sin_t = cos_t + kFft;
    float* fw = sin_t + kFft;
    int* band = reinterpret_cast<int*>(fw + t.nw);  // lo[mel], hi[mel], off[mel]
    float* mags = reinterpret_cast<float*>(band + 3 * t.mel);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* mag = mags + warp * kLogMelWarpFloats;
    for (int i = threadIdx.x; i < kFft; i += blockDim.x) {
        hann[i] = t.hann[i];
        cos_t[i] = t.cos_t[i];
        sin_t[i] = t.sin_t[i];
    }
    for (int i = threadIdx.x; i < t.nw; i += blockDim.x) fw[i] = t.w[i];
    for (int i = threadIdx.x; i < 3 * t.mel; i += blockDim.x) band[i] = t.band[i];
    pdl_wait();
    __syncthreads();
    const int j0 = int(__brev(uint32_t(lane)) >> 27) * 16;  // rev5(lane) * 16
    for (int f = blockIdx.x * 8 + warp; f < frames_total; f += gridDim.x * 8) {
        const AudioChunk ch = chunks[chunk_of<&AudioChunk::mel_row>(chunks, nchunks, f)];
        const int fl = f - ch.mel_row;
        const float* s = pcm + ch.pcm_offset;
        // padded[p] = chunk[p - 160] (160 zeros in front, zeros past the end)
        const int idx0 = fl * kHop + j0 - kPadLeft;
        float w16[16];
        if (idx0 >= 0 && idx0 + 16 <= ch.samples && (reinterpret_cast<uintptr_t>(s + idx0) & 15) == 0) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 v = *reinterpret_cast<const float4*>(s + idx0 + 4 * q);
                w16[4 * q] = v.x, w16[4 * q + 1] = v.y, w16[4 * q + 2] = v.z, w16[4 * q + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int q = 0; q < 16; q++) {
                const int idx = idx0 + q;
                w16[q] = (idx >= 0 && idx < ch.samples) ? s[idx] : 0.0f;
            }
        }
        float re[16], im[16];
#pragma unroll
        for (int r = 0; r < 16; r++) {
            const int q = int(__brev(uint32_t(r)) >> 28);  // rev4(r)
            re[r] = __fmul_rn(hann[j0 + q], w16[q]);
            im[r] = 0.0f;
        }
#pragma unroll
        for (int lg = 0; lg < 5; lg++) {  // partners in other lanes
            const int half = 1 << lg, step = kFft / (half << 1);
            const int k = lane & (half - 1);
            const float c = cos_t[k * step], sn = -sin_t[k * step];
            const bool odd = lane & half;
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const float pre = __shfl_xor_sync(0xffffffffu, re[r], half);
                const float pim = __shfl_xor_sync(0xffffffffu, im[r], half);
                const float er = odd ? pre : re[r], ei = odd ? pim : im[r];
                const float ro = odd ? re[r] : pre, io = odd ? im[r] : pim;
                const float a = __fmul_rn(c, ro), bq = __fmul_rn(sn, io), cq = __fmul_rn(c, io), d = __fmul_rn(sn, ro);
                if (odd) {
                    re[r] = __fadd_rn(__fsub_rn(er, a), bq);
                    im[r] = __fsub_rn(__fsub_rn(ei, cq), d);
                } else {
                    re[r] = __fsub_rn(__fadd_rn(er, a), bq);
                    im[r] = __fadd_rn(__fadd_rn(ei, cq), d);
                }
            }
        }
#pragma unroll
        for (int lg = 5; lg < 9; lg++) {  // partners in the same lane, h registers apart
            const int h = 1 << (lg - 5), step = kFft / (2 << lg);
#pragma unroll
            for (int r = 0; r < 16; r++) {
                if (r & h) continue;
                const int k = 32 * (r & (h - 1)) + lane;
                const float c = cos_t[k * step], sn = -sin_t[k * step];
                const float er = re[r], ei = im[r], ro = re[r + h], io = im[r + h];
                const float a = __fmul_rn(c, ro), bq = __fmul_rn(sn, io), cq = __fmul_rn(c, io), d = __fmul_rn(sn, ro);
                re[r] = __fsub_rn(__fadd_rn(er, a), bq);
                im[r] = __fadd_rn(__fadd_rn(ei, cq), d);
                re[r + h] = __fadd_rn(__fsub_rn(er, a), bq);
                im[r + h] = __fsub_rn(__fsub_rn(ei, cq), d);
            }
        }
        // Bins 0..256: element j is in lane j % 32, register j / 32.
#pragma unroll
        for (int r = 0; r < 8; r++)
            mag[32 * r + lane] = __fsqrt_rn(__fadd_rn(__fmul_rn(re[r], re[r]), __fmul_rn(im[r], im[r])));
        if (lane == 0) mag[256] = __fsqrt_rn(__fadd_rn(__fmul_rn(re[8], re[8]), __fmul_rn(im[8], im[8])));
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
    return size_t(3 * kFft + t.nw) * 4 + size_t(3 * t.mel) * 4 + size_t(8) * kLogMelWarpFloats * 4;
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
    const size_t most = size_t(3 * kFft + kMel * kBins) * 4 + size_t(3 * kMel) * 4 + size_t(8) * kLogMelWarpFloats * 4;
    return cudaFuncSetAttribute(k_log_mel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(std::min<size_t>(most, 227 * 1024)));
}

// ---------------------------------------------------------------------------- subsampling
// One warp per conv0 output time row (8 per block); lane l computes channels 4l..4l+3 with their
// 36 taps in registers, for the 64 output frequencies in turn.  The three mel rows a warp reads
// are staged fp16-rounded (ggml's im2col runs in fp16).
__global__ void __launch_bounds__(256) k_audio_conv0(const float* __restrict__ mel, const AudioChunk* __restrict__ chunks,
                                                     int nchunks, int t0_total, const float* __restrict__ w,
                                                     const float* __restrict__ nw, float eps, __half* __restrict__ out) {
    __shared__ float in[8][3][kMel];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float wr[4][9], ns[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        ns[j] = nw[4 * lane + j];
#pragma unroll
        for (int k = 0; k < 9; k++) wr[j][k] = w[(4 * lane + j) * 9 + k];
    }
    pdl_wait();
    pdl_launch_if_one_wave();
    const int r0 = blockIdx.x * 8 + warp;
    if (r0 >= t0_total) return;
    const AudioChunk ch = chunks[chunk_of<&AudioChunk::t0_row>(chunks, nchunks, r0)];
    const int ot = r0 - ch.t0_row;
    float(*x3)[kMel] = in[warp];
    for (int i = lane; i < 3 * kMel; i += 32) {
        const int kh = i / kMel, fq = i % kMel, tt = 2 * ot + kh - 1;
        const float v = (tt >= 0 && tt < ch.frames) ? mel[size_t(ch.mel_row + tt) * kMel + fq] : 0.0f;
        x3[kh][fq] = __half2float(__float2half_rn(v));
    }
    __syncwarp();
    __half* dst = out + size_t(r0) * kF0 * kC0 + 4 * lane;
#pragma unroll 2
    for (int of = 0; of < kF0; of++) {
        float x[9];
#pragma unroll
        for (int kh = 0; kh < 3; kh++)
#pragma unroll
            for (int kw = 0; kw < 3; kw++) {
                const int fq = 2 * of + kw - 1;
                x[kh * 3 + kw] = fq >= 0 ? x3[kh][fq] : 0.0f;  // fq < 128 always
            }
        float c[4], sum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 9; k++) acc += wr[j][k] * x[k];
            c[j] = acc;
            sum += acc;
        }
        const float mean = warp_sum(sum) / float(kC0);
        float var = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) var += (c[j] - mean) * (c[j] - mean);
        var = warp_sum(var) / float(kC0);
        const float scale = 1.0f / sqrtf(var + eps);
        uint2 o;
        o.x = pack_half2(fmaxf(0.f, (c[0] - mean) * scale * ns[0]), fmaxf(0.f, (c[1] - mean) * scale * ns[1]));
        o.y = pack_half2(fmaxf(0.f, (c[2] - mean) * scale * ns[2]), fmaxf(0.f, (c[3] - mean) * scale * ns[3]));
        *reinterpret_cast<uint2*>(dst + of * kC0) = o;
    }
}

cudaError_t launch_audio_conv0(const float* mel, const AudioChunk* chunks, int nchunks, int t0_total, const float* w,
                               const float* nw, float eps, __half* out, cudaStream_t stream) {
    if (t0_total <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_audio_conv0, dim3((t0_total + 7) / 8), dim3(256), 0, stream, 1, mel, chunks, nchunks,
                            t0_total, w, nw, eps, out));
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
// head dims 4l .. 4l + 3 and sums its part of every key's score; one reduce-scatter leaves key m's
// score on lanes 2m and 2m + 1, which apply the soft cap and the exponent.  The score is
// q' . (kscale k + rel[t - j]) with q' the scaled query.
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
    const int idx = lane >> 1;  // the key whose score this lane holds after the reduce-scatter
    // The four rows of a warp are independent; unrolled, their shuffle chains overlap.
#pragma unroll
    for (int i = 0; i < kAttnRows / 8; i++) {
        const int t = r0 + warp * (kAttnRows / 8) + i;
        if (t >= a.rows) continue;
        const float4 qv = ld4(a.q + size_t(t) * W + h * kAttnHd + 4 * lane);
        const float q0 = qv.x * qs.x, q1 = qv.y * qs.y, q2 = qv.z * qs.z, q3 = qv.w * qs.w;
        const int first = max(a.chunk_start[t], t - (kAttnWin - 1));
        const int n = t - first + 1;  // keys, oldest first: j = first + m
        // Partial scores over this lane's 4 dims: q' . (k kscale + rel[t - j]).
        float v[16];
#pragma unroll
        for (int m = 0; m < 16; m++) v[m] = 0.f;
#pragma unroll
        for (int m = 0; m < kAttnWin; m++) {
            if (m < n) {
                const int j = first + m;
                const float4 kk = ld4(&ks[j - base][4 * lane]);
                const float4 rr = *reinterpret_cast<const float4*>(&rel[t - j][4 * lane]);
                v[m] = q0 * fmaf(kk.x, a.kscale, rr.x) + q1 * fmaf(kk.y, a.kscale, rr.y) +
                       q2 * fmaf(kk.z, a.kscale, rr.z) + q3 * fmaf(kk.w, a.kscale, rr.w);
            }
        }
        // Reduce-scatter of the 16 partial sums over the warp: lanes 2m and 2m + 1 end with key m's score.
#pragma unroll
        for (int o = 16, cnt = 8; o >= 2; o >>= 1, cnt >>= 1) {
            const bool upper = lane & o;
#pragma unroll
            for (int k = 0; k < cnt; k++) {
                const float send = upper ? v[k] : v[k + cnt];
                const float keep = upper ? v[k + cnt] : v[k];
                v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const float sfull = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
        const bool valid = idx < n;
        const float c = valid ? a.softcap * tanhf(sfull / a.softcap) : -FLT_MAX;
        const float mx = warp_max(c);
        const float e = valid ? expf(c - mx) : 0.f;
        const float sum = warp_sum((lane & 1) ? 0.f : e);
        const float p = e / sum;
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
        for (int m = 0; m < kAttnWin; m++) {
            const float pm = __shfl_sync(0xffffffffu, p, 2 * m);
            if (m < n) {
                const float4 vv = ld4(&vs[first + m - base][4 * lane]);
                o0 += pm * vv.x;
                o1 += pm * vv.y;
                o2 += pm * vv.z;
                o3 += pm * vv.w;
            }
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
// A block computes R consecutive rows; thread i owns channels C i .. C i + C - 1 (C = W / 256)
// with their 5 taps in registers.  The R + 4 source rows are loaded once into registers and each
// is added into every output row within reach (tap 4 on the current row; rows before the output
// row's chunk start contribute nothing).  The RMS norms of the R rows share one block reduction.  dw_t is [5][W] (tap-major).
template <int C>
__device__ __forceinline__ void load_halves(const __half* p, float* v) {
    if constexpr (C == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
    } else if constexpr (C == 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(h[e]);
            v[2 * e] = f.x, v[2 * e + 1] = f.y;
        }
    } else if constexpr (C == 2) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p));
        v[0] = f.x, v[1] = f.y;
    } else {
#pragma unroll
        for (int e = 0; e < C; e++) v[e] = __half2float(p[e]);
    }
}

template <int W>
__global__ void __launch_bounds__(256) k_audio_dwconv(const __half* __restrict__ glu, const int* __restrict__ chunk_start,
                                                      int rows, const float* __restrict__ dw_t, const float* __restrict__ nw,
                                                      float eps, float lo, float hi, __half* __restrict__ out) {
    constexpr int C = W / 256, R = C > 4 ? 4 : 8;
    __shared__ float red[R][8];
    const int c0 = threadIdx.x * C, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float w[5][C], nv[C];
#pragma unroll
    for (int e = 0; e < C; e++) {
        nv[e] = nw[c0 + e];
#pragma unroll
        for (int k = 0; k < 5; k++) w[k][e] = dw_t[k * W + c0 + e];
    }
    pdl_wait();
    pdl_launch_if_one_wave();
    const int r0 = blockIdx.x * R;
    int cs[R];
#pragma unroll
    for (int rr = 0; rr < R; rr++) cs[rr] = r0 + rr < rows ? chunk_start[r0 + rr] : r0 + rr;
    // Every source row first (clamped into the buffer, so all loads issue together), then the taps.
    float x[R + 4][C];
#pragma unroll
    for (int si = 0; si < R + 4; si++) {
        const int src = min(max(r0 - 4 + si, 0), rows - 1);
        load_halves<C>(glu + size_t(src) * W + c0, x[si]);
    }
    float acc[R][C];
#pragma unroll
    for (int rr = 0; rr < R; rr++) {
#pragma unroll
        for (int e = 0; e < C; e++) acc[rr][e] = 0.f;
#pragma unroll
        for (int k = 0; k < 5; k++) {
            const int src = r0 + rr + k - 4;  // source row si = rr + k
            if (src < cs[rr] || src < 0) continue;
#pragma unroll
            for (int e = 0; e < C; e++) acc[rr][e] += x[rr + k][e] * w[k][e];
        }
    }
#pragma unroll
    for (int rr = 0; rr < R; rr++) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < C; e++) ss += acc[rr][e] * acc[rr][e];
        ss = warp_sum(ss);
        if (lane == 0) red[rr][warp] = ss;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < R; rr++) {
        const int t = r0 + rr;
        if (t >= rows) break;
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < 8; k++) ss += red[rr][k];
        const float inv = 1.0f / sqrtf(ss / float(W) + eps);
        __half* dst = out + size_t(t) * W + c0;
#pragma unroll
        for (int e = 0; e < C; e++) dst[e] = __float2half_rn(clampf(silu_fast(acc[rr][e] * inv * nv[e]), lo, hi));
    }
}

cudaError_t launch_audio_dwconv(const __half* glu, const int* chunk_start, int rows, int width, const float* dw_t,
                                const float* nw, float eps, float lo, float hi, __half* out, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int r = width / 256 > 4 ? 4 : 8;
    const dim3 grid((rows + r - 1) / r);
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
