// elementwise.cu -- row kernels of the forward pass: one warp per row, fp32 arithmetic in
// the reference's operation order, fp16 stores for every value that feeds a GEMM.
//
// Reference kernels replaced (Sources/GemmaEmbed/Shaders/Elementwise.metal):
//   embed_q8 (8-35) + rmsnorm_rows (38-75)          -> k_embed
//   rmsnorm_rope_{256,512} (97-136) + v norm        -> k_qkv_norm_rope
//   rmsnorm_residual(_norm) (260-354)               -> k_residual_norm
//   rmsnorm_rows with preScale (per-layer inputs)   -> k_rmsnorm_rows
//   mean_pool (243-256)                             -> k_mean_pool
// and the pooled dense head / output projection, which have no Metal kernel (the
// reference projects per token with its GEMM, MetalForward.swift:421).
#include "kernels.hpp"
#include "ptx.cuh"

namespace ge {

#define CK_LAUNCH(expr)                \
    do {                               \
        const cudaError_t e_ = (expr); \
        if (e_ != cudaSuccess) return e_; \
    } while (0)

namespace {
thread_local bool t_programmatic = false;
}  // namespace
void set_programmatic_launch(bool on) { t_programmatic = on; }
bool programmatic_launch() { return t_programmatic; }

constexpr int kRowsPerBlock = 8;  // warps per 256-thread block

// x = dequant(table row) * scale, h = rmsnorm(x) * w.  Embedding.swift semantics:
// CPUReference.swift:190-203 (token rows) and Elementwise.metal:8-35 (padding rows zeroed);
// an id -(r + 1) takes row r of `vectors` unscaled (an image or audio row, Elementwise.metal:26-30).
__global__ void k_embed(const int32_t* __restrict__ tokens, int ntok, int rows, const int8_t* __restrict__ tq,
                        const __half* __restrict__ ts, int width, float scale, float* __restrict__ x,
                        __half* __restrict__ x16, const float* __restrict__ w, float eps, __half* __restrict__ h,
                        const float* __restrict__ vectors) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float* xr = x + long(row) * width;
    __half* hr = h + long(row) * width;
    if (row >= ntok) {
        for (int i = lane; i < width; i += 32) {
            xr[i] = 0.f;
            hr[i] = __float2half_rn(0.f);
            if (x16) x16[long(row) * width + i] = __float2half_rn(0.f);
        }
        return;
    }
    const long id = tokens[row];
    float ss = 0.f;
    if (id < 0) {
        const float* vr = vectors + (-id - 1) * width;
        for (int i = lane; i < width; i += 32) {
            const float v = vr[i];
            xr[i] = v;
            ss += v * v;
            if (x16) x16[long(row) * width + i] = __float2half_rn(v);
        }
    } else {
        const int8_t* q = tq + id * width;
        const __half* s = ts + id * (width / 32);
        for (int i = lane; i < width; i += 32) {
            const float v = (__half2float(s[i >> 5]) * float(q[i])) * scale;
            xr[i] = v;
            ss += v * v;
            if (x16) x16[long(row) * width + i] = __float2half_rn(v);
        }
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(width) + eps);
    for (int i = lane; i < width; i += 32) hr[i] = __float2half_rn(xr[i] * inv * w[i]);
}

// k_embed with each lane owning G groups of 8 consecutive elements (group g = lane + 32 k): one
// 8-byte load of int8 values per group, the row kept in registers for the norm, 32-byte stores
// of x and 16-byte stores of h.  The same per-element arithmetic as k_embed.
template <int G>
__global__ void k_embed_vec(const int32_t* __restrict__ tokens, int ntok, int rows, const int8_t* __restrict__ tq,
                            const __half* __restrict__ ts, float scale, float* __restrict__ x, __half* __restrict__ x16,
                            const float* __restrict__ w, float eps, __half* __restrict__ h,
                            const float* __restrict__ vectors) {
    constexpr int width = G * 256;
    pdl_wait();
    pdl_launch_if_one_wave();
    const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float v[G][8];
    float ss = 0.f;
    const long id = row < ntok ? long(tokens[row]) : 0;
#pragma unroll
    for (int k = 0; k < G; k++) {
        const int e0 = 8 * (lane + 32 * k);
        if (row >= ntok) {
#pragma unroll
            for (int j = 0; j < 8; j++) v[k][j] = 0.f;
        } else if (id < 0) {
            const float4* vr = reinterpret_cast<const float4*>(vectors + (-id - 1) * width + e0);
            const float4 a = vr[0], b = vr[1];
            v[k][0] = a.x; v[k][1] = a.y; v[k][2] = a.z; v[k][3] = a.w;
            v[k][4] = b.x; v[k][5] = b.y; v[k][6] = b.z; v[k][7] = b.w;
        } else {
            const uint2 raw = *reinterpret_cast<const uint2*>(tq + id * width + e0);
            const float sc = __half2float(ts[id * (width / 32) + (e0 >> 5)]);
            const int8_t* q = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
            for (int j = 0; j < 8; j++) v[k][j] = (sc * float(q[j])) * scale;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) ss += v[k][j] * v[k][j];
        float4* xr = reinterpret_cast<float4*>(x + long(row) * width + e0);
        xr[0] = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
        xr[1] = make_float4(v[k][4], v[k][5], v[k][6], v[k][7]);
        if (x16) {
            uint4 o;
            o.x = pack_half2(v[k][0], v[k][1]);
            o.y = pack_half2(v[k][2], v[k][3]);
            o.z = pack_half2(v[k][4], v[k][5]);
            o.w = pack_half2(v[k][6], v[k][7]);
            *reinterpret_cast<uint4*>(x16 + long(row) * width + e0) = o;
        }
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(width) + eps);
#pragma unroll
    for (int k = 0; k < G; k++) {
        const int e0 = 8 * (lane + 32 * k);
        const float4 wa = *reinterpret_cast<const float4*>(w + e0), wb = *reinterpret_cast<const float4*>(w + e0 + 4);
        const float ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; j++) o[j] = row < ntok ? v[k][j] * inv * ww[j] : 0.f;
        uint4 u;
        u.x = pack_half2(o[0], o[1]);
        u.y = pack_half2(o[2], o[3]);
        u.z = pack_half2(o[4], o[5]);
        u.w = pack_half2(o[6], o[7]);
        *reinterpret_cast<uint4*>(h + long(row) * width + e0) = u;
    }
}

cudaError_t launch_embed(const int32_t* tokens, int ntok, int rows, const int8_t* table_q, const __half* table_s,
                         int width, float scale, float* x, __half* x16, const float* norm_w, float eps, __half* h,
                         cudaStream_t stream, const float* vectors) {
    if (rows <= 0) return cudaSuccess;
    if (width == 768) {
        CK_LAUNCH(launch_kernel(k_embed_vec<3>, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(256), 0, stream,
                                1, tokens, ntok, rows, table_q, table_s, scale, x, x16, norm_w, eps, h, vectors));
        return cudaGetLastError();
    }
    CK_LAUNCH(launch_kernel(k_embed, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(256), 0, stream, 1, tokens,
                            ntok, rows, table_q, table_s, width, scale, x, x16, norm_w, eps, h, vectors));
    return cudaGetLastError();
}

// One warp per TPW tokens, over the S head slots of each token's fused projection row: slots
// [0, H) are query heads, [H, H+KV) key heads, [H+KV, H+2KV) value heads.
// CPUReference.swift:225-235.  Lane l holds elements [Q*l, Q*l + Q) of each half of a head
// (Q = HD / 64), so every element and its rotation partner HD/2 away sit in the same lane; a
// token's cos/sin pairs are read once and reused for every query and key head.  Every slot of
// every token is loaded before the first is normalised, so each warp keeps TPW * S * 2
// independent loads in flight.
template <int HD, int S, int TPW>
__global__ void k_qkv_norm_rope(const __half* __restrict__ qkv, int ntok, int rows, int heads, int kvh,
                                const float* __restrict__ qw, const float* __restrict__ kw,
                                const int32_t* __restrict__ pos, const float* __restrict__ rope, float eps,
                                __half* __restrict__ q, __half* __restrict__ k, __half* __restrict__ v) {
    pdl_wait();
    pdl_launch_if_one_wave();
    constexpr int Q = HD / 64;  // elements per lane per half: 4 (hd 256) or 8 (hd 512)
    constexpr int WQ = Q / 2;   // 32-bit words per lane per half
    constexpr int HALF = HD / 2;
    const int row0 = (blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5)) * TPW;
    const int lane = threadIdx.x & 31;
    const int c = lane * Q;
    uint32_t raw[TPW][S][2][WQ];
    int32_t pv[TPW];
#pragma unroll
    for (int t = 0; t < TPW; t++) {
        const int row = row0 + t;
        const bool live = row < ntok;
        const __half* src_row = qkv + long(row) * S * HD;
        pv[t] = live ? pos[row] : 0;
#pragma unroll
        for (int s = 0; s < S; s++)
#pragma unroll
            for (int h = 0; h < 2; h++)
#pragma unroll
                for (int i = 0; i < WQ; i += 2) {
                    uint2 r = make_uint2(0u, 0u);
                    if (live) r = *reinterpret_cast<const uint2*>(src_row + s * HD + h * HALF + c + 2 * i);
                    raw[t][s][h][i] = r.x;
                    raw[t][s][h][i + 1] = r.y;
                }
    }
#pragma unroll
    for (int t = 0; t < TPW; t++) {
        const int row = row0 + t;
        if (row >= rows) break;
        const bool live = row < ntok;
        float cs_c[Q], cs_s[Q];
        if (live) {
            const float* cs = rope + long(pv[t]) * HD + 2 * c;  // [position][pair][cos, sin]
#pragma unroll
            for (int i = 0; i < Q; i += 2) {
                const float4 f = *reinterpret_cast<const float4*>(cs + 2 * i);
                cs_c[i] = f.x;
                cs_s[i] = f.y;
                cs_c[i + 1] = f.z;
                cs_s[i + 1] = f.w;
            }
        }
#pragma unroll
        for (int slot = 0; slot < S; slot++) {
            __half* dst;
            const float* w = nullptr;
            if (slot < heads) {
                dst = q + long(row) * heads * HD + slot * HD;
                w = qw;
            } else if (slot < heads + kvh) {
                dst = k + long(row) * kvh * HD + (slot - heads) * HD;
                w = kw;
            } else {
                dst = v + long(row) * kvh * HD + (slot - heads - kvh) * HD;
            }
            float a[Q], b[Q];
#pragma unroll
            for (int i = 0; i < WQ; i++) {
                const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&raw[t][slot][0][i]));
                const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&raw[t][slot][1][i]));
                a[2 * i] = fa.x;
                a[2 * i + 1] = fa.y;
                b[2 * i] = fb.x;
                b[2 * i + 1] = fb.y;
            }
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < Q; i++) ss += a[i] * a[i] + b[i] * b[i];
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / float(HD) + eps);
#pragma unroll
            for (int i = 0; i < Q; i++) {
                a[i] = a[i] * inv * (w ? w[c + i] : 1.0f);
                b[i] = b[i] * inv * (w ? w[HALF + c + i] : 1.0f);
            }
            if (w && live) {  // NeoX rotation of the pairs (c + i, HALF + c + i)
#pragma unroll
                for (int i = 0; i < Q; i++) {
                    const float a0 = a[i], b0 = b[i];
                    a[i] = a0 * cs_c[i] - b0 * cs_s[i];
                    b[i] = a0 * cs_s[i] + b0 * cs_c[i];
                }
            }
#pragma unroll
            for (int i = 0; i < Q; i += 4) {
                uint2 oa, ob;
                *reinterpret_cast<__half2*>(&oa.x) = __floats2half2_rn(a[i], a[i + 1]);
                *reinterpret_cast<__half2*>(&oa.y) = __floats2half2_rn(a[i + 2], a[i + 3]);
                *reinterpret_cast<__half2*>(&ob.x) = __floats2half2_rn(b[i], b[i + 1]);
                *reinterpret_cast<__half2*>(&ob.y) = __floats2half2_rn(b[i + 2], b[i + 3]);
                *reinterpret_cast<uint2*>(dst + c + i) = oa;
                *reinterpret_cast<uint2*>(dst + HALF + c + i) = ob;
            }
        }
    }
}

// Head dim 256: a half-warp per token (lane l of the half holds elements 8l .. 8l + 7 of each
// 128-element half of every head slot: 16-byte loads and stores), two tokens per warp, every
// slot of both tokens loaded before the first is normalised; the norm weights are read as
// float4.  Same steps as k_qkv_norm_rope (sum of squares, weighted norm, NeoX rotation of the
// pairs (j, j + 128), v unweighted), with the sum of squares reduced over 16 lanes.
template <int S>
__global__ void __launch_bounds__(256, 3) k_qkv_norm_rope_hw(const __half* __restrict__ qkv, int ntok, int rows, int heads, int kvh,
                                   const float* __restrict__ qw, const float* __restrict__ kw,
                                   const int32_t* __restrict__ pos, const float* __restrict__ rope, float eps,
                                   __half* __restrict__ q, __half* __restrict__ k, __half* __restrict__ v) {
    pdl_wait();
    pdl_launch_if_one_wave();
    constexpr int HD = 256, HALF = 128;
    const int lane = threadIdx.x & 31;
    const int row = (blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5)) * 2 + (lane >> 4);
    if (row >= rows) return;  // the two halves of a warp reduce apart, so each may leave alone
    const unsigned mask = lane < 16 ? 0x0000ffffu : 0xffff0000u;
    const int c = (lane & 15) * 8;
    const bool live = row < ntok;
    const __half* src = qkv + long(row) * S * HD;
    uint4 ra[S], rb[S];
#pragma unroll
    for (int s = 0; s < S; s++) {
        ra[s] = live ? *reinterpret_cast<const uint4*>(src + s * HD + c) : make_uint4(0u, 0u, 0u, 0u);
        rb[s] = live ? *reinterpret_cast<const uint4*>(src + s * HD + HALF + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    float cs_c[8], cs_s[8];
    if (live) {
        const float4* cs = reinterpret_cast<const float4*>(rope + long(pos[row]) * HD + 2 * c);  // [pair][cos, sin]
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 f = cs[i];
            cs_c[2 * i] = f.x;
            cs_s[2 * i] = f.y;
            cs_c[2 * i + 1] = f.z;
            cs_s[2 * i + 1] = f.w;
        }
    }
#pragma unroll
    for (int slot = 0; slot < S; slot++) {
        __half* dst;
        const float* w = nullptr;
        if (slot < heads) {
            dst = q + long(row) * heads * HD + slot * HD;
            w = qw;
        } else if (slot < heads + kvh) {
            dst = k + long(row) * kvh * HD + (slot - heads) * HD;
            w = kw;
        } else {
            dst = v + long(row) * kvh * HD + (slot - heads - kvh) * HD;
        }
        float a[8], b[8];
        const __half2* ha = reinterpret_cast<const __half2*>(&ra[slot]);
        const __half2* hb = reinterpret_cast<const __half2*>(&rb[slot]);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 fa = __half22float2(ha[i]), fb = __half22float2(hb[i]);
            a[2 * i] = fa.x;
            a[2 * i + 1] = fa.y;
            b[2 * i] = fb.x;
            b[2 * i + 1] = fb.y;
        }
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) ss += a[i] * a[i] + b[i] * b[i];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(mask, ss, o);
        const float inv = 1.0f / sqrtf(ss / float(HD) + eps);
        if (w) {
            const float4 wa0 = *reinterpret_cast<const float4*>(w + c), wa1 = *reinterpret_cast<const float4*>(w + c + 4);
            const float4 wb0 = *reinterpret_cast<const float4*>(w + HALF + c);
            const float4 wb1 = *reinterpret_cast<const float4*>(w + HALF + c + 4);
            const float wa[8] = {wa0.x, wa0.y, wa0.z, wa0.w, wa1.x, wa1.y, wa1.z, wa1.w};
            const float wb[8] = {wb0.x, wb0.y, wb0.z, wb0.w, wb1.x, wb1.y, wb1.z, wb1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                a[i] = a[i] * inv * wa[i];
                b[i] = b[i] * inv * wb[i];
            }
            if (live) {  // NeoX rotation of the pairs (c + i, HALF + c + i)
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float a0 = a[i], b0 = b[i];
                    a[i] = a0 * cs_c[i] - b0 * cs_s[i];
                    b[i] = a0 * cs_s[i] + b0 * cs_c[i];
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                a[i] = a[i] * inv;
                b[i] = b[i] * inv;
            }
        }
        uint4 oa, ob;
        __half2* pa = reinterpret_cast<__half2*>(&oa);
        __half2* pb = reinterpret_cast<__half2*>(&ob);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            pa[i] = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
            pb[i] = __floats2half2_rn(b[2 * i], b[2 * i + 1]);
        }
        *reinterpret_cast<uint4*>(dst + c) = oa;
        *reinterpret_cast<uint4*>(dst + HALF + c) = ob;
    }
}

template <int HD, int S>
static cudaError_t launch_qkv_t(const __half* qkv, int ntok, int rows, int heads, int kv_heads, const float* q_w,
                                const float* k_w, const int32_t* positions, const float* rope, float eps, __half* q,
                                __half* k, __half* v, cudaStream_t stream) {
    if (HD == 256) {
        const int blocks = (rows + kRowsPerBlock * 2 - 1) / (kRowsPerBlock * 2);
        return launch_kernel(k_qkv_norm_rope_hw<S>, dim3(blocks), dim3(256), 0, stream, 1, qkv, ntok, rows, heads,
                             kv_heads, q_w, k_w, positions, rope, eps, q, k, v);
    }
    // Head dim 512: two tokens per warp once the grid is many waves deep; one keeps small
    // batches spread over every SM.
    if (rows >= 8192) {
        const int blocks = (rows + kRowsPerBlock * 2 - 1) / (kRowsPerBlock * 2);
        return launch_kernel(k_qkv_norm_rope<HD, S, 2>, dim3(blocks), dim3(256), 0, stream, 1, qkv, ntok, rows, heads,
                             kv_heads, q_w, k_w, positions, rope, eps, q, k, v);
    }
    const int blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    return launch_kernel(k_qkv_norm_rope<HD, S, 1>, dim3(blocks), dim3(256), 0, stream, 1, qkv, ntok, rows, heads,
                         kv_heads, q_w, k_w, positions, rope, eps, q, k, v);
}

// Head slots per token: heads + 2 kv_heads, 3..8 for head dim 256 and 3..6 for 512 (the
// loader rejects other layouts).
cudaError_t launch_qkv_norm_rope(const __half* qkv, int ntok, int rows, int heads, int kv_heads, int hd,
                                 const float* q_w, const float* k_w, const int32_t* positions, const float* rope,
                                 float eps, __half* q, __half* k, __half* v, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
#define QKV_CASE(HD, S)                                                                                         \
    if (hd == HD && heads + 2 * kv_heads == S)                                                                  \
        return launch_qkv_t<HD, S>(qkv, ntok, rows, heads, kv_heads, q_w, k_w, positions, rope, eps, q, k, v, stream);
    QKV_CASE(256, 3)
    QKV_CASE(256, 4)
    QKV_CASE(256, 5)
    QKV_CASE(256, 6)
    QKV_CASE(256, 7)
    QKV_CASE(256, 8)
    QKV_CASE(512, 3)
    QKV_CASE(512, 4)
    QKV_CASE(512, 5)
    QKV_CASE(512, 6)
#undef QKV_CASE
    return cudaErrorInvalidValue;
}

// x = (x + rmsnorm(t) * w_post) * scale, then optionally the next norm of x.
// CPUReference.swift:239-243, 252-256, 266-269 and Elementwise.metal:260-354.  One warp per
// row; lane l holds the 8-element groups l, l + 32, ... (W / 256 groups) in registers.
// PAIR applies a second residual step (t2, w_post2) to the result before the next norm, so a
// layer's attention residual can be recomputed (identically: same code, same order) in its FFN
// residual instead of being stored and reloaded; store_x = false skips the store of x.
template <int W, bool PAIR>
__global__ void k_residual_norm(float* __restrict__ x, const __half* __restrict__ t, int rows,
                                const float* __restrict__ wp, float scale, const __half* __restrict__ t2,
                                const float* __restrict__ wp2, int store_x, const float* __restrict__ wn, float eps,
                                __half* __restrict__ h16, float* __restrict__ y32, __half* __restrict__ x16) {
    pdl_wait();
    pdl_launch_if_one_wave();
    constexpr int G = W / 256;  // groups of 8 per lane
    const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float* xr = x + long(row) * W;
    const __half* tr = t + long(row) * W;
    float tv[G][8], xv[G][8];
    uint4 t2raw[PAIR ? G : 1];
    float ss = 0.f, ss_b = 0.f;
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int c = (lane + 32 * g) * 8;
        const uint4 raw = *reinterpret_cast<const uint4*>(tr + c);
        if (PAIR) t2raw[g] = *reinterpret_cast<const uint4*>(t2 + long(row) * W + c);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 f = __half22float2(h2[i]);
            tv[g][2 * i] = f.x;
            tv[g][2 * i + 1] = f.y;
            ss += f.x * f.x + f.y * f.y;
        }
        const float4 a = *reinterpret_cast<const float4*>(xr + c);
        const float4 b = *reinterpret_cast<const float4*>(xr + c + 4);
        xv[g][0] = a.x; xv[g][1] = a.y; xv[g][2] = a.z; xv[g][3] = a.w;
        xv[g][4] = b.x; xv[g][5] = b.y; xv[g][6] = b.z; xv[g][7] = b.w;
    }
    if (PAIR) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            const __half2* h2 = reinterpret_cast<const __half2*>(&t2raw[g]);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f = __half22float2(h2[i]);
                ss_b += f.x * f.x + f.y * f.y;
            }
        }
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(W) + eps);
    float inv_b = 0.f;
    if (PAIR) {
        ss_b = warp_sum(ss_b);
        inv_b = 1.0f / sqrtf(ss_b / float(W) + eps);
    }
    float ss2 = 0.f;
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int c = (lane + 32 * g) * 8;
        const float4 w0 = *reinterpret_cast<const float4*>(wp + c);
        const float4 w1 = *reinterpret_cast<const float4*>(wp + c + 4);
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float v = xv[g][i] + tv[g][i] * inv * ww[i];
            if (scale != 1.0f) v *= scale;
            xv[g][i] = v;
        }
        if (PAIR) {
            const float4 u0 = *reinterpret_cast<const float4*>(wp2 + c);
            const float4 u1 = *reinterpret_cast<const float4*>(wp2 + c + 4);
            const float uu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            const __half2* h2 = reinterpret_cast<const __half2*>(&t2raw[g]);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f = __half22float2(h2[i]);
                xv[g][2 * i] = xv[g][2 * i] + f.x * inv_b * uu[2 * i];
                xv[g][2 * i + 1] = xv[g][2 * i + 1] + f.y * inv_b * uu[2 * i + 1];
            }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) ss2 += xv[g][i] * xv[g][i];
        if (store_x) {
            *reinterpret_cast<float4*>(xr + c) = make_float4(xv[g][0], xv[g][1], xv[g][2], xv[g][3]);
            *reinterpret_cast<float4*>(xr + c + 4) = make_float4(xv[g][4], xv[g][5], xv[g][6], xv[g][7]);
        }
        if (x16) {
            uint4 o;
            __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int i = 0; i < 4; i++) o2[i] = __floats2half2_rn(xv[g][2 * i], xv[g][2 * i + 1]);
            *reinterpret_cast<uint4*>(x16 + long(row) * W + c) = o;
        }
    }
    if (!wn) return;
    ss2 = warp_sum(ss2);
    const float inv2 = 1.0f / sqrtf(ss2 / float(W) + eps);
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int c = (lane + 32 * g) * 8;
        const float4 w0 = *reinterpret_cast<const float4*>(wn + c);
        const float4 w1 = *reinterpret_cast<const float4*>(wn + c + 4);
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] = xv[g][i] * inv2 * ww[i];
        if (h16) {
            uint4 o;
            __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int i = 0; i < 4; i++) o2[i] = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
            *reinterpret_cast<uint4*>(h16 + long(row) * W + c) = o;
        }
        if (y32) {
            *reinterpret_cast<float4*>(y32 + long(row) * W + c) = make_float4(y[0], y[1], y[2], y[3]);
            *reinterpret_cast<float4*>(y32 + long(row) * W + c + 4) = make_float4(y[4], y[5], y[6], y[7]);
        }
    }
}

cudaError_t launch_residual(const ResidualStep& r, int rows, int width, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    const int store_x = r.store_x ? 1 : 0;
#define RES_CASE(W, P)                                                                                                \
    if (width == W && (r.t2 != nullptr) == P)                                                                         \
        return launch_kernel(k_residual_norm<W, P>, dim3(blocks), dim3(256), 0, stream, 1, r.x, r.t, rows, r.w_post,    \
                             r.scale, r.t2, r.w_post2, store_x, r.w_next, r.eps, r.h16, r.y32, r.x16);
    RES_CASE(768, false)
    RES_CASE(768, true)
    RES_CASE(512, false)
    RES_CASE(512, true)
#undef RES_CASE
    return cudaErrorInvalidValue;
}

cudaError_t launch_residual_norm(float* x, const __half* t, int rows, int width, const float* w_post, float scale,
                                 const float* w_next, float eps, __half* h16, float* y32, __half* x16,
                                 cudaStream_t stream) {
    ResidualStep r;
    r.x = x;
    r.t = t;
    r.w_post = w_post;
    r.scale = scale;
    r.w_next = w_next;
    r.eps = eps;
    r.h16 = h16;
    r.y32 = y32;
    r.x16 = x16;
    return launch_residual(r, rows, width, stream);
}

// out = rmsnorm(x * pre) * w over `width`-wide rows (the per-layer-input norm,
// CPUReference.swift:206-209 and Elementwise.metal:38-75 with preScale).
__global__ void k_rmsnorm_rows(const float* __restrict__ x, long rows, int width, float pre,
                               const float* __restrict__ w, float eps, float* __restrict__ out) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const long row = long(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * width;
    float* o = out + row * width;
    float ss = 0.f;
    for (int i = lane; i < width; i += 32) {
        const float v = xr[i] * pre;
        ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(width) + eps);
    for (int i = lane; i < width; i += 32) o[i] = (xr[i] * pre) * inv * w[i];
}

cudaError_t launch_rmsnorm_rows(const float* x, int rows, int width, float pre, const float* w, float eps, float* out,
                                cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_rmsnorm_rows, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(256), 0, stream, 1,
                            x, rows, width, pre, w, eps, out));
    return cudaGetLastError();
}

// pooled[s][c] = sum over the sequence's rows / length (Elementwise.metal:243-256), in two
// levels with a fixed order, so a sequence's mean depends only on its own rows:
//   k_pool_partial: one block per (sequence, chunk of kPoolChunk rows counted from the
//   sequence start); warp w sums rows w, w + 8, ... of the chunk, then the 8 warp sums of a
//   column are added in warp order into partial[chunk][c];
//   k_pool_final: one block per sequence adds its chunks in order and divides by the length.
constexpr int kPoolChunk = kPoolChunkRows;

__global__ void k_pool_partial(const float* __restrict__ y, int width, const uint32_t* __restrict__ seqs,
                               const uint32_t* __restrict__ chunk_base, float* __restrict__ partial) {
    pdl_wait();
    pdl_launch_if_one_wave();
    extern __shared__ float part[];  // [8][width]
    const int s = blockIdx.y;
    const uint32_t start = seqs[2 * s], len = seqs[2 * s + 1];
    const uint32_t r0 = blockIdx.x * kPoolChunk;
    if (r0 >= len) return;
    const uint32_t r1 = min(len, r0 + kPoolChunk);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int c0 = lane * 4; c0 < width; c0 += 128) {
        // The chunk's kPoolChunk / 8 rows of this warp are loaded before they are added in order.
        float4 v[kPoolChunk / 8];
#pragma unroll
        for (int k = 0; k < kPoolChunk / 8; k++) {
            const uint32_t r = r0 + warp + 8 * k;
            v[k] = r < r1 ? *reinterpret_cast<const float4*>(y + long(start + r) * width + c0)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kPoolChunk / 8; k++) {
            if (r0 + warp + 8 * k >= r1) break;
            acc.x += v[k].x;
            acc.y += v[k].y;
            acc.z += v[k].z;
            acc.w += v[k].w;
        }
        *reinterpret_cast<float4*>(part + warp * width + c0) = acc;
    }
    __syncthreads();
    float* out = partial + (long(chunk_base[s]) + blockIdx.x) * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
        float acc = 0.f;
        for (int w = 0; w < 8; w++) acc += part[w * width + c];
        out[c] = acc;
    }
}

__global__ void k_pool_final(const float* __restrict__ partial, int width, const uint32_t* __restrict__ seqs,
                             const uint32_t* __restrict__ chunk_base, float* __restrict__ pooled) {
    pdl_wait();
    pdl_launch_if_one_wave();
    // Block (s, y) owns columns [256 y, 256 y + 256) of sequence s, four per thread; the chunks
    // are added in order, eight loads in flight at a time.
    const int s = blockIdx.x;
    const int c = blockIdx.y * 256 + threadIdx.x * 4;
    if (c >= width) return;
    const uint32_t len = seqs[2 * s + 1];
    const uint32_t nchunks = (len + kPoolChunk - 1) / kPoolChunk;
    const float* in = partial + long(chunk_base[s]) * width + c;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t k = 0;
    for (; k + 8 <= nchunks; k += 8) {
        float4 t[8];
#pragma unroll
        for (int j = 0; j < 8; j++) t[j] = *reinterpret_cast<const float4*>(in + long(k + j) * width);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            acc.x += t[j].x;
            acc.y += t[j].y;
            acc.z += t[j].z;
            acc.w += t[j].w;
        }
    }
    for (; k < nchunks; k++) {
        const float4 t = *reinterpret_cast<const float4*>(in + long(k) * width);
        acc.x += t.x;
        acc.y += t.y;
        acc.z += t.z;
        acc.w += t.w;
    }
    const float n = float(len);
    *reinterpret_cast<float4*>(pooled + long(s) * width + c) = make_float4(acc.x / n, acc.y / n, acc.z / n, acc.w / n);
}

int pool_chunks(uint32_t len) { return int((len + kPoolChunk - 1) / kPoolChunk); }

// Single-launch mean pool for callers that only hold the sequence ranges on the device: one
// block per sequence, warp w summing rows w, w + 8, ..., then the 8 warp sums in order.  The
// ranges come straight from the caller's device memory, so only rows inside [0, ntok) are read:
// a range is cut at ntok, and a range with no row left (length 0, or a start at or past ntok)
// gives a zero vector.
__global__ void k_mean_pool_seq(const float* __restrict__ y, int width, uint32_t ntok,
                                const uint32_t* __restrict__ seqs, float* __restrict__ pooled) {
    pdl_wait();
    pdl_launch_if_one_wave();
    extern __shared__ float part[];  // [8][width]
    const uint32_t start = seqs[2 * blockIdx.x];
    const uint32_t len = start >= ntok ? 0u : min(seqs[2 * blockIdx.x + 1], ntok - start);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int c0 = lane * 4; c0 < width; c0 += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t r = warp; r < len; r += 8) {
            const float4 v = *reinterpret_cast<const float4*>(y + long(start + r) * width + c0);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        *reinterpret_cast<float4*>(part + warp * width + c0) = acc;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
        float acc = 0.f;
        for (int w = 0; w < 8; w++) acc += part[w * width + c];
        pooled[long(blockIdx.x) * width + c] = len ? acc / float(len) : 0.f;
    }
}

cudaError_t launch_mean_pool_seq(const float* y, int width, int ntok, const uint32_t* seqs, int nseq, float* pooled,
                                 cudaStream_t stream) {
    if (nseq <= 0) return cudaSuccess;
    if (width % 128 || ntok < 0) return cudaErrorInvalidValue;
    CK_LAUNCH(launch_kernel(k_mean_pool_seq, dim3(nseq), dim3(256), 8 * width * sizeof(float), stream, 1, y, width,
                            uint32_t(ntok), seqs, pooled));
    return cudaGetLastError();
}

cudaError_t launch_mean_pool(const float* y, int width, const uint32_t* seqs, int nseq, int max_chunks,
                             const uint32_t* chunk_base, float* partial, float* pooled, cudaStream_t stream) {
    if (nseq <= 0) return cudaSuccess;
    if (width % 128) return cudaErrorInvalidValue;
    CK_LAUNCH(launch_kernel(k_pool_partial, dim3(max_chunks, nseq), dim3(256), 8 * width * sizeof(float), stream, 1, y,
                            width, seqs, chunk_base, partial));
    CK_LAUNCH(launch_kernel(k_pool_final, dim3(nseq, (width + 255) / 256), dim3(64), 0, stream, 1, partial, width, seqs,
                            chunk_base, pooled));
    return cudaGetLastError();
}

// EmbeddingModel.finish (EmbeddingModel.swift:260-267) on the device: the first `dims` values of
// each pooled row, divided by their L2 norm when `normalise` (and the norm is positive).  One
// thread per row adds the squares in order with separately rounded products and sums, the same
// operations as the host's ge_finish, so the rows match it bit for bit.
__global__ void k_finish_rows(const float* __restrict__ in, int nseq, int width, int dims, int normalise,
                              float* __restrict__ out) {
    pdl_wait();
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= nseq) return;
    const float* v = in + long(s) * width;
    float* o = out + long(s) * dims;
    const int k = min(dims, width);
    float norm = 0.f;
    if (normalise) {
        float acc = 0.f;
        for (int i = 0; i < k; i++) acc = __fadd_rn(acc, __fmul_rn(v[i], v[i]));
        norm = sqrtf(acc);
    }
    for (int i = 0; i < k; i++) o[i] = norm > 0.f ? __fdiv_rn(v[i], norm) : v[i];
}

cudaError_t launch_finish_rows(const float* in, int nseq, int width, int dims, int normalise, float* out,
                               cudaStream_t stream) {
    if (nseq <= 0) return cudaSuccess;
    if (dims <= 0 || dims > width) return cudaErrorInvalidValue;
    CK_LAUNCH(launch_kernel(k_finish_rows, dim3((nseq + 63) / 64), dim3(64), 0, stream, 1, in, nseq, width, dims,
                            normalise, out));
    return cudaGetLastError();
}

// positions[start + i] = i for every sequence (PackedBatch.append, MetalForward.swift:17-21).
__global__ void k_positions(const uint32_t* __restrict__ seqs, int32_t* __restrict__ positions) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const uint32_t start = seqs[2 * blockIdx.x], len = seqs[2 * blockIdx.x + 1];
    for (uint32_t i = threadIdx.x; i < len; i += blockDim.x) positions[start + i] = int32_t(i);
}

cudaError_t launch_positions(const uint32_t* seqs, int nseq, int32_t* positions, cudaStream_t stream) {
    if (nseq <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_positions, dim3(nseq), dim3(256), 0, stream, 1, seqs, positions));
    return cudaGetLastError();
}

// out[s][n] = sum_k in[s][k] * w[n][k] in fp32 with an fp32 weight matrix.  k_dense_rows: C
// weight rows per warp held in registers (lane l holds k = 4 l + 128 i), input rows staged in
// shared memory R at a time and shared by the block's 8 warps; grid.y splits the input rows.
// Each output is lane partial sums over increasing k, then a warp sum.  k_dense_f32 (one warp
// per n, input rows read from global memory by every warp) serves other widths: at K = 3072
// (the head's second projection, 64 rows) it measured 38 us against 55 us for k_dense_rows
// with one weight row per warp, whose shared-memory stages then hold two input rows each.
constexpr int kDenseRows = 16;
constexpr int kDenseRowsPerBlock = 16;

template <int C, int KV>
__global__ void __launch_bounds__(256) k_dense_rows(const float* __restrict__ in, int nrows, const float* __restrict__ w,
                                                    int N, float* __restrict__ out, int R) {
    extern __shared__ float4 xs[];  // [R][KV * 32]
    constexpr int K4 = KV * 32;     // float4 per row
    pdl_wait();
    pdl_launch_if_one_wave();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * 8 + warp) * C;
    float4 wr[C][KV];
#pragma unroll
    for (int c = 0; c < C; c++)
#pragma unroll
        for (int i = 0; i < KV; i++)
            wr[c][i] = n0 + c < N ? *reinterpret_cast<const float4*>(w + long(n0 + c) * (K4 * 4) + 4 * lane + 128 * i)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    const int r_begin = blockIdx.y * kDenseRowsPerBlock, r_end = min(nrows, r_begin + kDenseRowsPerBlock);
    for (int r0 = r_begin; r0 < r_end; r0 += R) {
        const int nr = min(R, r_end - r0);
        __syncthreads();
        const float4* src = reinterpret_cast<const float4*>(in + long(r0) * (K4 * 4));
        for (int idx = threadIdx.x; idx < nr * K4; idx += blockDim.x) xs[idx] = src[idx];
        __syncthreads();
        // Two rows at a time: 2 * C independent sums per lane.
        for (int r = 0; r < nr; r += 2) {
            const int r1 = r + 1 < nr ? r + 1 : r;
            float acc[2][C];
#pragma unroll
            for (int c = 0; c < C; c++) acc[0][c] = acc[1][c] = 0.f;
#pragma unroll
            for (int i = 0; i < KV; i++) {
                const float4 xa = xs[r * K4 + lane + 32 * i];
                const float4 xb = xs[r1 * K4 + lane + 32 * i];
#pragma unroll
                for (int c = 0; c < C; c++) {
                    acc[0][c] += xa.x * wr[c][i].x + xa.y * wr[c][i].y + xa.z * wr[c][i].z + xa.w * wr[c][i].w;
                    acc[1][c] += xb.x * wr[c][i].x + xb.y * wr[c][i].y + xb.z * wr[c][i].z + xb.w * wr[c][i].w;
                }
            }
#pragma unroll
            for (int c = 0; c < C; c++) {
                const float v0 = warp_sum(acc[0][c]), v1 = warp_sum(acc[1][c]);
                if (lane == 0 && n0 + c < N) {
                    out[long(r0 + r) * N + n0 + c] = v0;
                    if (r1 != r) out[long(r0 + r1) * N + n0 + c] = v1;
                }
            }
        }
    }
}

template <int C, int KV>
static cudaError_t launch_dense_rows(const float* in, int nrows, const float* w, int N, float* out, cudaStream_t stream) {
    const int K = KV * 128;
    const int R = (24 * 1024) / (K * 4);  // input rows per shared-memory stage (24 KB)
    const dim3 grid((N + 8 * C - 1) / (8 * C), (nrows + kDenseRowsPerBlock - 1) / kDenseRowsPerBlock);
    return launch_kernel(k_dense_rows<C, KV>, grid, dim3(256), R * K * 4, stream, 1, in, nrows, w, N, out, R);
}
__global__ void k_dense_f32(const float* __restrict__ in, int nrows, const float* __restrict__ w, int N, int K,
                            float* __restrict__ out) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const int n = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    const float* wr = w + long(n) * K;
    const int s_end = min(nrows, int(blockIdx.y + 1) * kDenseRows);
    for (int s0 = int(blockIdx.y) * kDenseRows; s0 < s_end; s0 += 4) {
        const int ns = min(4, s_end - s0);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 6
        for (int k = lane * 4; k < K; k += 128) {
            const float4 wv = *reinterpret_cast<const float4*>(wr + k);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (j < ns) {
                    const float4 xv = *reinterpret_cast<const float4*>(in + long(s0 + j) * K + k);
                    acc[j] += xv.x * wv.x + xv.y * wv.y + xv.z * wv.z + xv.w * wv.w;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float v = warp_sum(acc[j]);
            if (lane == 0 && j < ns) out[long(s0 + j) * N + n] = v;
        }
    }
}

// The dense head of the forward: out[s][n] = sum_k in[s][k] * w[n][k] in fp32, as 64-row x
// 64-column tiles over fixed 256-wide K chunks.  Pass 1: one block per (column tile, K chunk,
// row tile); each thread keeps a 4 x 4 block of outputs in registers and adds its chunk's
// products in increasing k, with the chunk's inputs and weights staged 32 k at a time in shared
// memory (k-major, so each thread reads its 4 rows and 4 columns as two float4).  Pass 2 adds
// the chunk partials in chunk order.  Every output's summation order depends only on K, not on
// the number of rows, so a sequence's vector does not depend on its batch.
constexpr int kHeadTile = 64, kHeadChunk = 256, kHeadStep = 32;

__global__ void __launch_bounds__(256) k_dense_head_part(const float* __restrict__ in, int nrows,
                                                         const float* __restrict__ w, int N, int K,
                                                         float* __restrict__ part) {
    pdl_wait();
    pdl_launch_if_one_wave();
    __shared__ float4 xs[kHeadStep][kHeadTile / 4 + 1];  // [k][row / 4], padded
    __shared__ float4 ws[kHeadStep][kHeadTile / 4 + 1];  // [k][column / 4]
    const int n0 = blockIdx.x * kHeadTile, k0 = blockIdx.y * kHeadChunk, r0 = blockIdx.z * kHeadTile;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};
    // Staging: thread t loads row (or column) t % 64 of the tile at k offsets (t / 64) * 8 .. + 7
    // (one whole 32-byte sector per thread), so a warp's shared-memory writes fall on 32
    // consecutive words.
    const int lr = tid & 63, lk = (tid >> 6) * 8;
    const bool row_live = r0 + lr < nrows;
    const float* xin = in + long(r0 + lr) * K + k0 + lk;
    const float* win = w + long(n0 + lr) * K + k0 + lk;
    // Loads run kPre steps ahead of the products (a ring of register sets, one per step in
    // flight), so each thread has up to 3 x 64 bytes outstanding while it computes.
    constexpr int kSteps = kHeadChunk / kHeadStep, kPre = 3;
    float4 ring[kPre][4];
    auto load = [&](float4 (&r)[4], int kk) {
        r[0] = r[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row_live) {
            r[0] = *reinterpret_cast<const float4*>(xin + kk);
            r[1] = *reinterpret_cast<const float4*>(xin + kk + 4);
        }
        r[2] = *reinterpret_cast<const float4*>(win + kk);
        r[3] = *reinterpret_cast<const float4*>(win + kk + 4);
    };
#pragma unroll
    for (int i = 0; i < kPre; i++) load(ring[i], i * kHeadStep);
#pragma unroll
    for (int st = 0; st < kSteps; st++) {
        float4(&r)[4] = ring[st % kPre];
        __syncthreads();
        const float xv[8] = {r[0].x, r[0].y, r[0].z, r[0].w, r[1].x, r[1].y, r[1].z, r[1].w};
        const float wv[8] = {r[2].x, r[2].y, r[2].z, r[2].w, r[3].x, r[3].y, r[3].z, r[3].w};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            reinterpret_cast<float*>(&xs[lk + j][lr >> 2])[lr & 3] = xv[j];
            reinterpret_cast<float*>(&ws[lk + j][lr >> 2])[lr & 3] = wv[j];
        }
        __syncthreads();
        if (st + kPre < kSteps) load(r, (st + kPre) * kHeadStep);
#pragma unroll 8
        for (int k = 0; k < kHeadStep; k++) {
            const float4 a = xs[k][ty];
            const float4 b = ws[k][tx];
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
    }
    float* dst = part + (long(blockIdx.y) * nrows) * N;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = r0 + ty * 4 + i;
        if (r < nrows)
            *reinterpret_cast<float4*>(dst + long(r) * N + n0 + tx * 4) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
}

__global__ void k_dense_head_sum(const float* __restrict__ part, int chunks, long count, float* __restrict__ out) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const long i = (long(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= count) return;
    float4 s = *reinterpret_cast<const float4*>(part + i);
    for (int c = 1; c < chunks; c++) {
        const float4 t = *reinterpret_cast<const float4*>(part + long(c) * count + i);
        s.x += t.x;
        s.y += t.y;
        s.z += t.z;
        s.w += t.w;
    }
    *reinterpret_cast<float4*>(out + i) = s;
}

int dense_head_chunks(int K) { return K / kHeadChunk; }

cudaError_t launch_dense_head(const float* in, int nrows, const float* w, int N, int K, float* part, float* out,
                              cudaStream_t stream) {
    if (nrows <= 0) return cudaSuccess;
    if (N % kHeadTile || K % kHeadChunk) return cudaErrorInvalidValue;
    const int chunks = K / kHeadChunk;
    const dim3 grid(N / kHeadTile, chunks, (nrows + kHeadTile - 1) / kHeadTile);
    CK_LAUNCH(launch_kernel(k_dense_head_part, grid, dim3(256), 0, stream, 1, in, nrows, w, N, K, part));
    const long count = long(nrows) * N;
    CK_LAUNCH(launch_kernel(k_dense_head_sum, dim3(unsigned((count / 4 + 255) / 256)), dim3(256), 0, stream, 1, part,
                            chunks, count, out));
    return cudaGetLastError();
}

cudaError_t launch_dense_f32(const float* in, int nrows, const float* w, int N, int K, float* out,
                             cudaStream_t stream) {
    if (nrows <= 0) return cudaSuccess;
    if (K % 128) return cudaErrorInvalidValue;
    if (K == 768) {
        CK_LAUNCH((launch_dense_rows<4, 6>(in, nrows, w, N, out, stream)));
        return cudaGetLastError();
    }
    const dim3 grid((N + kRowsPerBlock - 1) / kRowsPerBlock, (nrows + kDenseRows - 1) / kDenseRows);
    CK_LAUNCH(launch_kernel(k_dense_f32, grid, dim3(256), 0, stream, 1, in, nrows, w, N, K, out));
    return cudaGetLastError();
}

}  // namespace ge
