// noalloc.cu -- mean-pool and head over caller-provided device buffers, allocating nothing.
//
// Some callers cannot call cudaMalloc: a plugin inside a host runtime that owns all device
// memory through its own allocator and only hands kernels preallocated buffers, or a serving
// loop where an allocation could implicitly synchronise the device and stall other work on it.
// ge_pool_head_noalloc gives them the last stage of the forward (mean-pool, then the dense head
// or output projection) with its intermediates -- the pooled rows and the head's hidden rows --
// in one file-scope __device__ array instead of a workspace.  Every GPU that loads this library
// holds that array until the process exits.
#include <mutex>

#include "gemma_embed.h"
#include "model.hpp"

namespace {

constexpr int kMaxSeqs = GE_NOALLOC_MAX_SEQS;
constexpr int kMaxHidden = 1024;  // widest pooled row the scratch holds
constexpr int kMaxMid = 4096;     // widest dense-head hidden row the scratch holds

// pooled rows [kMaxSeqs][kMaxHidden], then head rows [kMaxSeqs][kMaxMid]: 2.5 MiB.
__device__ __align__(256) float g_head_scratch[kMaxSeqs * (kMaxHidden + kMaxMid)];

std::mutex g_setup_mu;
float* g_scratch_addr[64] = {};

// The device address of g_head_scratch on the current device, looked up once per device.  In
// host code the array's name is only a host-side stand-in, never a device pointer.
cudaError_t scratch_address(int device, float** out) {
    std::lock_guard<std::mutex> g(g_setup_mu);
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_head_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[device] = static_cast<float*>(p);
    }
    *out = g_scratch_addr[device];
    return cudaSuccess;
}

}  // namespace

namespace ge {
// One-time set-up for `device` (which must be current): ge_load calls it for each device it
// loads, so later calls of ge_pool_head_noalloc only read the cached address.
cudaError_t noalloc_setup(int device) {
    float* p = nullptr;
    return scratch_address(device, &p);
}
}  // namespace ge

namespace {
// Puts the calling thread's current device back on every return path: the caller's host
// runtime manages devices itself and must not see this call change them.
struct CurrentDeviceGuard {
    int saved = -1;
    CurrentDeviceGuard() {
        if (cudaGetDevice(&saved) != cudaSuccess) saved = -1;
    }
    ~CurrentDeviceGuard() {
        if (saved >= 0) cudaSetDevice(saved);
    }
};
}  // namespace

extern "C" int ge_pool_head_noalloc(ge_model* m, int32_t device_ordinal, const float* d_hidden, int32_t ntok,
                                    const uint32_t* d_seqs, int32_t nseq, float* d_out, void* stream) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    std::lock_guard<std::mutex> g(m->mu);
    const ge::Config& c = m->cfg;
    ge::Device* dev = nullptr;
    for (auto& d : m->devs)
        if (d.ordinal == device_ordinal) dev = &d;
    if (!dev) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: the model is not loaded on that device");
    if (nseq < 1 || nseq > kMaxSeqs)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS,
                             "invalid options: ge_pool_head_noalloc takes 1.." + std::to_string(kMaxSeqs) +
                                 " sequences per call, got " + std::to_string(nseq));
    if (ntok < 1 || !d_hidden || !d_seqs || !d_out)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: bad sizes or NULL device arrays");
    if (c.hidden > kMaxHidden || (c.has_dense && c.dense_head > kMaxMid))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: the model's head is wider than the scratch");
    // The pooling and head kernels work in 128-column groups; other widths are refused here
    // rather than reported later as a failed launch.
    if (c.hidden % 128 || (c.has_dense && c.dense_head % 128))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS,
                             "invalid options: ge_pool_head_noalloc needs hidden and dense-head widths that are "
                             "multiples of 128");
    CurrentDeviceGuard keep_current_device;
    cudaError_t e = cudaSetDevice(dev->ordinal);
    float* scratch = nullptr;
    if (e == cudaSuccess) e = scratch_address(dev->ordinal, &scratch);
    if (e != cudaSuccess)
        return ge::set_error(m, GE_ERR_GPU_FAILURE, std::string("GPU execution failed: scratch set-up: ") + cudaGetErrorString(e));
    float* pooled = scratch;
    float* mid = scratch + size_t(kMaxSeqs) * kMaxHidden;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
    // Each kernel writes every scratch element it later reads, so no call depends on what the
    // previous call left in the array and nothing needs clearing.  The pooling kernel reads only
    // rows [0, ntok) of d_hidden whatever the ranges say.
    e = ge::launch_mean_pool_seq(d_hidden, c.hidden, ntok, d_seqs, nseq, pooled, st);
    int launches = 1;
    if (e == cudaSuccess && c.has_dense) {
        e = ge::launch_dense_f32(pooled, nseq, dev->dense2, c.dense_head, c.hidden, mid, st);
        if (e == cudaSuccess) e = ge::launch_dense_f32(mid, nseq, dev->dense3, c.out_dim, c.dense_head, d_out, st);
        launches += 2;
    } else if (e == cudaSuccess) {
        e = ge::launch_dense_f32(pooled, nseq, dev->output, c.out_dim, c.hidden, d_out, st);
        launches += 1;
    }
    m->launches += launches;
    if (e != cudaSuccess)
        return ge::set_error(m, GE_ERR_GPU_FAILURE, std::string("GPU execution failed: ") + cudaGetErrorString(e));
    return GE_OK;
}
