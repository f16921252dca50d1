// vision.cu -- row kernels of the gemma4v image encoder: patchify, position rows plus the first
// norm, per-head norm with 2-D RoPE, and the merge-window pool with its norm.  One warp per
// row, fp32 arithmetic in the reference's order, fp16 stores for every value that feeds a GEMM.
//
// Reference (Sources/GemmaEmbed):
//   PreparedImage.init (Image/ImagePreprocessor.swift:31-60)      -> k_patchify
//   add_position_rows + rmsnorm_rows (Shaders/Elementwise.metal:207-220, 38-75)
//                                                                  -> k_patch_position_norm
//   rmsnorm_rope_2d_64 + v norm (Elementwise.metal:167-205; Metal/VisionTower.swift:153-157)
//                                                                  -> k_vision_qkv_norm_rope
//   pool_patches + rmsnorm_rows (Elementwise.metal:223-240; VisionTower.swift:180-182)
//                                                                  -> k_pool_patches_norm
#include "kernels.hpp"
#include "ptx.cuh"

namespace ge {

#define CK_LAUNCH(expr)                   \
    do {                                  \
        const cudaError_t e_ = (expr);    \
        if (e_ != cudaSuccess) return e_; \
    } while (0)

namespace {
constexpr int kWarps = 8;  // rows per 256-thread block
}

// One block per (patch, image).  Thread t reads the patch's bytes in raster order (rows of
// 3p bytes) and writes element c * p^2 + ky * p + kx of the patch row: fp16(2 f - 1) with
// f = (byte / 255 - mean[c]) / std[c], the value PreparedImage rounds through Float16
// (2 f is exact, so a fused multiply-add rounds the same).  Columns past 3 p^2 (the GEMM's
// K padding) are zero.
__global__ void k_patchify(const uint8_t* __restrict__ rgb, const VisionImage* __restrict__ imgs, int p, int kpad,
                           NormParams np, __half* __restrict__ patches) {
    pdl_wait();
    const VisionImage im = imgs[blockIdx.y];
    const int pi = blockIdx.x;
    if (pi >= im.gx * im.gy) return;
    const int px = pi % im.gx, py = pi / im.gx;
    const int w = im.gx * p;
    __half* out = patches + (long(im.patch_start) + pi) * kpad;
    const int rowb = 3 * p, area = rowb * p;
    const uint8_t* src = rgb + im.rgb_offset + (long(py) * p * w + long(px) * p) * 3;
    for (int t = threadIdx.x; t < area; t += blockDim.x) {
        const int ky = t / rowb, rem = t - ky * rowb;
        const int kx = rem / 3, c = rem - kx * 3;
        const float byte = float(src[long(ky) * w * 3 + rem]);
        const float f = (byte / 255.0f - np.mean[c]) / np.std[c];
        out[c * p * p + ky * p + kx] = __float2half_rn(2.0f * f - 1.0f);
    }
    for (int t = area + threadIdx.x; t < kpad; t += blockDim.x) out[t] = __float2half_rn(0.f);
    pdl_launch_if_one_wave();
}

// x = (x + pos[px]) + pos[n + py] (the patch GEMM's fp32 output, updated in place), then
// h = fp16(rmsnorm(x) * w).  Rows at or past ntok get h = 0.
__global__ void k_patch_position_norm(float* __restrict__ x, const uint32_t* __restrict__ xy, int ntok, int rows, int d,
                                      const float* __restrict__ pos, int npos, const float* __restrict__ w, float eps,
                                      __half* __restrict__ h) {
    pdl_wait();
    pdl_launch_if_one_wave();
    const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    __half* hr = h + long(row) * d;
    if (row >= ntok) {
        for (int i = lane; i < d; i += 32) hr[i] = __float2half_rn(0.f);
        return;
    }
    float* xr = x + long(row) * d;
    const uint32_t c = xy[row];
    const float* tx = pos + long(c & 0xffffu) * d;
    const float* ty = pos + (long(npos) + (c >> 16)) * d;
    float ss = 0.f;
    for (int i = lane; i < d; i += 32) {
        const float v = (xr[i] + tx[i]) + ty[i];
        xr[i] = v;
        ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(d) + eps);
    for (int i = lane; i < d; i += 32) hr[i] = __float2half_rn(xr[i] * inv * w[i]);
}

// One warp per token over its 3 H heads of 64 (q | k | v in the fused projection row).  Lane l
// holds dims 2l and 2l + 1 of every head: lanes 0-15 the first half (rotated by the patch
// column), lanes 16-31 the second (by the patch row); a dim's NeoX partner 16 dims away sits
// in lane l ^ 8.  q and k: weighted RMSNorm then the rotation; v: unweighted RMSNorm.  The
// heads of q (then k, then v) are loaded together before the first is normalised.
template <int H>
__global__ void k_vision_qkv_norm_rope(const __half* __restrict__ qkv, int ntok, int rows,
                                       const float* __restrict__ qw, const float* __restrict__ kw,
                                       const uint32_t* __restrict__ xy, const float* __restrict__ rope, float eps,
                                       __half* __restrict__ q, __half* __restrict__ k, __half* __restrict__ v) {
    pdl_wait();
    pdl_launch_if_one_wave();
    constexpr int D = H * 64;
    const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const long base = long(row) * D + 2 * lane;
    uint32_t* q32 = reinterpret_cast<uint32_t*>(q);
    uint32_t* k32 = reinterpret_cast<uint32_t*>(k);
    uint32_t* v32 = reinterpret_cast<uint32_t*>(v);
    if (row >= ntok) {
#pragma unroll
        for (int hh = 0; hh < H; hh++) {
            q32[(base + hh * 64) / 2] = 0u;
            k32[(base + hh * 64) / 2] = 0u;
            v32[(base + hh * 64) / 2] = 0u;
        }
        return;
    }
    const uint32_t* src = reinterpret_cast<const uint32_t*>(qkv + long(row) * 3 * D) + lane;
    const uint32_t c = xy[row];
    const int axis = lane >> 4;
    const int posi = axis ? int(c >> 16) : int(c & 0xffffu);
    const int j0 = (2 * lane) & 31;  // dim within the half; 2 consecutive pairs i0, i0 + 1
    const bool first = j0 < 16;
    const float4 cs = *reinterpret_cast<const float4*>(rope + (long(posi) * 16 + (j0 & 15)) * 2);
    const float2 wq = *reinterpret_cast<const float2*>(qw + 2 * lane);
    const float2 wk = *reinterpret_cast<const float2*>(kw + 2 * lane);
    // q, then k, then v: the H heads of each loaded together (H independent loads in flight).
#pragma unroll 1
    for (int g = 0; g < 3; g++) {
        uint32_t raw[H];
#pragma unroll
        for (int hh = 0; hh < H; hh++) raw[hh] = src[(g * H + hh) * 32];
#pragma unroll
        for (int hh = 0; hh < H; hh++) {
            const int s = g * H + hh;
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&raw[hh]));
            const float ss = warp_sum(f.x * f.x + f.y * f.y);
            const float inv = 1.0f / sqrtf(ss / 64.0f + eps);
            uint32_t outw;
            if (s < 2 * H) {
                const float2 wv = s < H ? wq : wk;
                const float u0 = f.x * inv * wv.x, u1 = f.y * inv * wv.y;
                const float p0 = __shfl_xor_sync(0xffffffffu, u0, 8);
                const float p1 = __shfl_xor_sync(0xffffffffu, u1, 8);
                float r0, r1;
                if (first) {
                    r0 = u0 * cs.x - p0 * cs.y;
                    r1 = u1 * cs.z - p1 * cs.w;
                } else {
                    r0 = p0 * cs.y + u0 * cs.x;
                    r1 = p1 * cs.w + u1 * cs.z;
                }
                outw = pack_half2(r0, r1);
                uint32_t* dst = s < H ? q32 : k32;
                dst[(base + (s % H) * 64) / 2] = outw;
            } else {
                outw = pack_half2(f.x * inv, f.y * inv);
                v32[(base + (s - 2 * H) * 64) / 2] = outw;
            }
        }
    }
}

// One warp per token of an image: the merge x merge window of its patch rows summed in raster
// order, times `scale` (sqrt(d) / merge^2), then RMSNorm without a weight, stored fp16 (the
// projection's operand).
template <int D>
__global__ void k_pool_patches_norm(const float* __restrict__ x, const VisionImage* __restrict__ imgs, int merge,
                                    float scale, float eps, __half* __restrict__ out) {
    pdl_wait();
    pdl_launch_if_one_wave();
    constexpr int PER = D / 32;
    const VisionImage im = imgs[blockIdx.y];
    const int tx = im.gx / merge, tokens = tx * (im.gy / merge);
    const int tok = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (tok >= tokens) return;
    const int ox = tok % tx, oy = tok / tx;
    float acc[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) acc[i] = 0.f;
    for (int ky = 0; ky < merge; ky++)
        for (int kx = 0; kx < merge; kx++) {
            const float* src = x + (long(im.patch_start) + long(oy * merge + ky) * im.gx + ox * merge + kx) * D;
#pragma unroll
            for (int i = 0; i < PER; i++) acc[i] += src[lane + 32 * i];
        }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        acc[i] *= scale;
        ss += acc[i] * acc[i];
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(D) + eps);
    __half* dst = out + (long(im.token_start) + tok) * D;
#pragma unroll
    for (int i = 0; i < PER; i++) dst[lane + 32 * i] = __float2half_rn(acc[i] * inv);
}

cudaError_t launch_patchify(const uint8_t* rgb, const VisionImage* imgs, int nimg, int max_patches, int p, int kpad,
                            const NormParams& np, __half* patches, cudaStream_t stream) {
    if (nimg <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_patchify, dim3(unsigned(max_patches), unsigned(nimg)), dim3(256), 0, stream, 1, rgb, imgs,
                            p, kpad, np, patches));
    return cudaGetLastError();
}

cudaError_t launch_patch_position_norm(float* x, const uint32_t* xy, int ntok, int rows, int d, const float* pos,
                                       int npos, const float* w, float eps, __half* h, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    CK_LAUNCH(launch_kernel(k_patch_position_norm, dim3((rows + kWarps - 1) / kWarps), dim3(256), 0, stream, 1, x, xy,
                            ntok, rows, d, pos, npos, w, eps, h));
    return cudaGetLastError();
}

cudaError_t launch_vision_qkv_norm_rope(const __half* qkv, int ntok, int rows, int heads, const float* qw,
                                        const float* kw, const uint32_t* xy, const float* rope, float eps, __half* q,
                                        __half* k, __half* v, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const dim3 grid((rows + kWarps - 1) / kWarps);
    switch (heads) {
    case 12:
        CK_LAUNCH(launch_kernel(k_vision_qkv_norm_rope<12>, grid, dim3(256), 0, stream, 1, qkv, ntok, rows, qw, kw, xy,
                                rope, eps, q, k, v));
        break;
    case 8:
        CK_LAUNCH(launch_kernel(k_vision_qkv_norm_rope<8>, grid, dim3(256), 0, stream, 1, qkv, ntok, rows, qw, kw, xy,
                                rope, eps, q, k, v));
        break;
    case 16:
        CK_LAUNCH(launch_kernel(k_vision_qkv_norm_rope<16>, grid, dim3(256), 0, stream, 1, qkv, ntok, rows, qw, kw, xy,
                                rope, eps, q, k, v));
        break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_pool_patches_norm(const float* x, const VisionImage* imgs, int nimg, int max_tokens, int d, int merge,
                                     float scale, float eps, __half* out, cudaStream_t stream) {
    if (nimg <= 0) return cudaSuccess;
    const dim3 grid(unsigned((max_tokens + kWarps - 1) / kWarps), unsigned(nimg));
    switch (d) {
    case 768:
        CK_LAUNCH(launch_kernel(k_pool_patches_norm<768>, grid, dim3(256), 0, stream, 1, x, imgs, merge, scale, eps, out));
        break;
    case 1024:
        CK_LAUNCH(launch_kernel(k_pool_patches_norm<1024>, grid, dim3(256), 0, stream, 1, x, imgs, merge, scale, eps, out));
        break;
    case 512:
        CK_LAUNCH(launch_kernel(k_pool_patches_norm<512>, grid, dim3(256), 0, stream, 1, x, imgs, merge, scale, eps, out));
        break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace ge
