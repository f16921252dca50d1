// attention.cu -- bidirectional grouped-query attention over packed variable-length
// sequences, replacing Sources/GemmaEmbed/Shaders/Attention.metal:25-188 (dispatch in
// Metal/MetalForward.swift:669-694).
//
// Semantics (CPUReference.swift:117-174): per sequence and query head h, keys and values
// of KV head h / (H / KV); softmax(q . k * scale) with keys |i - j| > half_window masked on
// sliding-window layers; sequences never see each other's rows.
//
// Work items are (sequence start, sequence length, first query) triples, one per block of
// `queries_per_item` queries of a sequence (AttentionWork, MetalForward.swift:45-58); a
// block's key range is clipped to the window once for the whole block
// (Attention.metal:66-74), so its result depends only on its own sequence.
#include "kernels.hpp"
#include "ptx.cuh"

namespace ge {

// ---------------------------------------------------------------------------------------
// CUDA-core kernel: one CTA of 8 warps per (work item of 32 queries, head); each warp owns
// 4 queries, lane j scores key j of the 32-key block, and lane l accumulates output
// dimensions l, l + 32, ... with an online softmax in fp32.
constexpr int kSimtQueries = 32;
constexpr int kSimtKeys = 32;

template <int HD>
__global__ void __launch_bounds__(256) k_attention_simt(const __half* __restrict__ Q, const __half* __restrict__ K,
                                                        const __half* __restrict__ V, __half* __restrict__ O,
                                                        const uint32_t* __restrict__ work, int heads, int kvh,
                                                        int hw, float scale) {
    constexpr int PER = HD / 32;
    extern __shared__ float sm[];
    float* qs = sm;                          // [32][HD]
    float* ks = qs + kSimtQueries * HD;      // [32][HD + 1]
    float* vs = ks + kSimtKeys * (HD + 1);   // [32][HD]

    const uint32_t seq_start = work[3 * blockIdx.x], len = work[3 * blockIdx.x + 1], q0 = work[3 * blockIdx.x + 2];
    const int h = blockIdx.y;
    const int kh = h / (heads / kvh);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long qstride = long(heads) * HD, kvstride = long(kvh) * HD;

    for (int idx = threadIdx.x; idx < kSimtQueries * HD; idx += blockDim.x) {
        const int r = idx / HD, c = idx % HD;
        const uint32_t qi = q0 + r;
        qs[idx] = qi < len ? __half2float(Q[(seq_start + qi) * qstride + h * HD + c]) : 0.f;
    }

    int k_start = 0, k_end = int(len);
    if (hw > 0) {
        k_start = max(int(q0) - hw, 0);
        k_end = min(int(q0) + kSimtQueries - 1 + hw + 1, int(len));
    }
    k_start = k_start / kSimtKeys * kSimtKeys;

    float m[4], l[4], acc[4][PER];
#pragma unroll
    for (int r = 0; r < 4; r++) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int i = 0; i < PER; i++) acc[r][i] = 0.f;
    }

    for (int kb = k_start; kb < k_end; kb += kSimtKeys) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < kSimtKeys * HD; idx += blockDim.x) {
            const int r = idx / HD, c = idx % HD;
            const int kj = kb + r;
            const bool in = kj < int(len);
            ks[r * (HD + 1) + c] = in ? __half2float(K[(seq_start + kj) * kvstride + kh * HD + c]) : 0.f;
            vs[r * HD + c] = in ? __half2float(V[(seq_start + kj) * kvstride + kh * HD + c]) : 0.f;
        }
        __syncthreads();
        const int kj = kb + lane;
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int qr = warp * 4 + r;
            const int qi = int(q0) + qr;
            const float* qrow = qs + qr * HD;
            const float* krow = ks + lane * (HD + 1);
            float s = 0.f;
#pragma unroll 8
            for (int d = 0; d < HD; d++) s += qrow[d] * krow[d];
            bool valid = kj < int(len);
            if (hw > 0) valid = valid && abs(qi - kj) <= hw;
            s = valid ? s * scale : -INFINITY;
            const float mb = warp_max(s);
            const float m_new = fmaxf(m[r], mb);
            float p = 0.f, alpha = 1.f;
            if (m_new != -INFINITY) {
                p = valid ? expf(s - m_new) : 0.f;
                alpha = m[r] == -INFINITY ? 0.f : expf(m[r] - m_new);
            }
            l[r] = l[r] * alpha + warp_sum(p);
            m[r] = m_new;
#pragma unroll
            for (int i = 0; i < PER; i++) acc[r][i] *= alpha;
            for (int j = 0; j < kSimtKeys; j++) {
                const float pj = __shfl_sync(0xffffffffu, p, j);
                if (pj == 0.f) continue;
                const float* vrow = vs + j * HD;
#pragma unroll
                for (int i = 0; i < PER; i++) acc[r][i] += pj * vrow[lane + 32 * i];
            }
        }
    }

#pragma unroll
    for (int r = 0; r < 4; r++) {
        const uint32_t qi = q0 + warp * 4 + r;
        if (qi >= len) continue;
        const float inv = l[r] > 0.f ? 1.0f / l[r] : 0.f;
        __half* orow = O + (seq_start + qi) * qstride + h * HD;
#pragma unroll
        for (int i = 0; i < PER; i++) orow[lane + 32 * i] = __float2half_rn(acc[r][i] * inv);
    }
}

int attention_queries_per_item(int hd) {
    (void)hd;
    return kSimtQueries;
}

template <int HD>
static cudaError_t launch_simt(const AttnLaunch& a, cudaStream_t stream) {
    const int smem = (kSimtQueries * HD + kSimtKeys * (HD + 1) + kSimtKeys * HD) * 4;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_simt<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    dim3 grid(a.work_items, a.heads);
    k_attention_simt<HD><<<grid, 256, smem, stream>>>(a.q, a.k, a.v, a.out, a.work, a.heads, a.kv_heads, a.half_window,
                                                      1.0f);
    return cudaGetLastError();
}

cudaError_t launch_attention(const AttnLaunch& a, cudaStream_t stream) {
    if (a.work_items <= 0) return cudaSuccess;
    if (a.queries_per_item != kSimtQueries || a.heads % a.kv_heads) return cudaErrorInvalidValue;
    if (a.hd == 256) return launch_simt<256>(a, stream);
    if (a.hd == 512) return launch_simt<512>(a, stream);
    return cudaErrorInvalidValue;
}

}  // namespace ge
