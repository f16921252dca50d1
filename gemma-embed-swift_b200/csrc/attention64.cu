// attention64.cu -- tensor-core attention for head dim 64 without a mask inside each
// sequence: the vision tower's bidirectional attention over one image's patches
// (Sources/GemmaEmbed/Shaders/Attention.metal:190-312, CPUReference.attention with no window,
// Model/CPUReference.swift:117-174, scale 1).
//
// Persistent: one CTA per SM walks its list of work items, each item 128 query rows of one
// head.  Roles (352 threads):
//   warp 0      TMA producer: the item's Q tile, then K and V tiles of 128 keys through
//               3-stage rings that run on across items.
//   warp 1      S issuer: S_j = Q K_j^T (M 128, N 128, K 64) into one of two tensor-memory
//               buffers; a buffer takes block j + 2 once every softmax thread has loaded block j.
//   warp 10     PV issuer: O += P_j V_j (M 128, N 64, K 128) with P read from tensor memory.
//               (One thread issues a tcgen05.mma about every 90 cycles whatever its N, so the
//               eight PV products of a block, 32 tensor cycles each, get a thread of their own.)
//   warps 2-9   softmax, two threads per query row (64 keys each): running maximum with a
//               lazy rescale of O (only when the maximum grows by more than kRescaleRaw),
//               P = 2^(s log2e - m log2e) in fp16 into tensor memory, and at the end of an item
//               O / l stored as fp16.
// Tensor memory: S buffers in columns [0, 128) and [128, 256), O in [256, 320), P buffers in
// [320, 384) and [384, 448).
// Every wait is bounded (mbar_wait); after an error the kernel drains its loads and returns.
#include "kernels.hpp"
#include "ptx.cuh"

namespace ge {

namespace {
constexpr int kQ = 128, kKeys = 128, kHd = 64, kStages = 3;
constexpr float kLog2e = 1.4426950408889634f;
// O is rescaled only when a row's maximum grows by more than this (2^8 in probability); until
// then every term of the row shares the stale maximum, so the result is exact.
constexpr float kRescaleRaw = 8.0f / kLog2e;
constexpr int kTileBytes = kKeys * kHd * 2;       // 16 KB: [128 rows][64 dims] = [128][128 B]
constexpr int kOffK = kTileBytes;                 // Q at 0
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffRed = kOffV + kStages * kTileBytes;  // [2 halves][128 rows] floats
constexpr int kOffBar = kOffRed + 2 * kQ * 4;
constexpr int kSmem = kOffBar + 256 + 1024;
constexpr int kThreads = 352;
constexpr int kPVWarp = 10;
constexpr uint32_t kTmemS = 0, kTmemO = 256, kTmemP = 320;

struct Params {
    const uint4* work;       // (sequence start, sequence length, first query, head), grouped by CTA
    const uint32_t* offset;  // CTA c's items are [offset[c], offset[c + 1])
    __half* out;
    int dmodel;              // heads * 64
    int* err;
};

__device__ __forceinline__ void drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (!mbar_test(bar, parity) && globaltimer() - t0 < kWaitLimitNs) {
    }
}

__global__ void __launch_bounds__(kThreads, 1) k_attention64(const __grid_constant__ CUtensorMap mapQ,
                                                             const __grid_constant__ CUtensorMap mapK,
                                                             const __grid_constant__ CUtensorMap mapV, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* q_full = bars;
    uint64_t* q_empty = bars + 1;
    uint64_t* k_full = bars + 2;   // [3]
    uint64_t* k_empty = bars + 5;  // [3]
    uint64_t* v_full = bars + 8;   // [3]
    uint64_t* v_empty = bars + 11; // [3]
    uint64_t* s_full = bars + 14;  // [2]
    uint64_t* p_full = bars + 16;  // [2]
    uint64_t* pv_done = bars + 18; // [2]
    uint64_t* o_empty = bars + 20;
    uint64_t* s_free = bars + 21;  // [2] S buffer loaded by every softmax thread
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int it0 = int(p.offset[blockIdx.x]), it1 = int(p.offset[blockIdx.x + 1]);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int i = 0; i < kStages; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 256);
            mbar_init(&pv_done[i], 1);
        }
        mbar_init(o_empty, 256);
        for (int i = 0; i < 2; i++) mbar_init(&s_free[i], 256);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&mapQ);
        tma_prefetch(&mapK);
        tma_prefetch(&mapV);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // q, k, v come from the previous kernel

    if (warp == 0) {
        // ---------------------------------------------------------- TMA producer
        if (lane == 0) {
            bool ok = true;
            int gb = 0, issued_q = 0, issued_k = 0, issued_v = 0;
            for (int it = it0, li = 0; it < it1 && ok; it++, li++) {
                const uint4 w = p.work[it];
                const int nblk = (int(w.y) + kKeys - 1) / kKeys;
                const int x = int(w.w) * kHd;
                if (!mbar_wait(q_empty, uint32_t(li & 1) ^ 1u, p.err)) break;
                mbar_expect_tx(q_full, kTileBytes);
                tma_load_2d(smem, &mapQ, q_full, x, int(w.x + w.z));
                issued_q++;
                for (int j = 0; j < nblk; j++, gb++) {
                    const int s = gb % kStages;
                    const uint32_t ph = uint32_t((gb / kStages) & 1);
                    const int row = int(w.x) + j * kKeys;
                    if (!mbar_wait(&k_empty[s], ph ^ 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&k_full[s], kTileBytes);
                    tma_load_2d(smem + kOffK + s * kTileBytes, &mapK, &k_full[s], x, row);
                    issued_k++;
                    if (!mbar_wait(&v_empty[s], ph ^ 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&v_full[s], kTileBytes);
                    tma_load_2d(smem + kOffV + s * kTileBytes, &mapV, &v_full[s], x, row);
                    issued_v++;
                }
            }
            pdl_launch();
            // Every issued load lands before the CTA exits, also after an error.
            if (issued_q > 0) drain(q_full, uint32_t((issued_q - 1) & 1));
            for (int s = 0; s < kStages; s++) {
                const int ck = issued_k / kStages + (s < issued_k % kStages ? 1 : 0);
                const int cv = issued_v / kStages + (s < issued_v % kStages ? 1 : 0);
                if (ck > 0) drain(&k_full[s], uint32_t((ck - 1) & 1));
                if (cv > 0) drain(&v_full[s], uint32_t((cv - 1) & 1));
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- S issuer
        if (lane == 0) {
            const uint32_t id_s = idesc_f16(kQ, kKeys);  // K-major Q and K
            const uint32_t q_addr = smem_u32(smem);
            bool ok = true;
            int gb = 0;
            for (int it = it0, li = 0; it < it1 && ok; it++, li++) {
                const uint4 w = p.work[it];
                const int nblk = (int(w.y) + kKeys - 1) / kKeys;
                if (!mbar_wait(q_full, uint32_t(li & 1), p.err)) break;
                tc_fence_after();
                for (int j = 0; j < nblk; j++, gb++) {
                    const int b = gb & 1;
                    const int s = gb % kStages;
                    // S buffer b is free once every softmax thread holds block gb - 2's scores.
                    if ((gb >= 2 && !mbar_wait(&s_free[b], uint32_t(((gb - 2) >> 1) & 1), p.err)) ||
                        !mbar_wait(&k_full[s], uint32_t((gb / kStages) & 1), p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ka = smem_u32(smem + kOffK + s * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < kHd / 16; kk++) {
                        const uint64_t ad = sw128_desc(q_addr + kk * 32, 16, 1024);
                        const uint64_t bd = sw128_desc(ka + kk * 32, 16, 1024);
                        umma_f16(tmem + kTmemS + b * kKeys, ad, bd, id_s, kk != 0);
                    }
                    umma_commit(&k_empty[s]);
                    umma_commit(&s_full[b]);
                    if (j == nblk - 1) umma_commit(q_empty);  // every S of the item has read Q
                }
            }
        }
    } else if (warp == kPVWarp) {
        // ---------------------------------------------------------- PV issuer
        if (lane == 0) {
            const uint32_t id_o = idesc_f16(kQ, kHd, 0, 1);  // P from tensor memory, MN-major V
            bool ok = true;
            int gb = 0;
            for (int it = it0, li = 0; it < it1 && ok; it++, li++) {
                const uint4 w = p.work[it];
                const int nblk = (int(w.y) + kKeys - 1) / kKeys;
                for (int j = 0; j < nblk; j++, gb++) {
                    const int b = gb & 1;
                    const int s = gb % kStages;
                    // An item's first PV overwrites O once the previous item's O has been read.
                    if ((j == 0 && li > 0 && !mbar_wait(o_empty, uint32_t((li - 1) & 1), p.err)) ||
                        !mbar_wait(&p_full[b], uint32_t((gb >> 1) & 1), p.err) ||
                        !mbar_wait(&v_full[s], uint32_t((gb / kStages) & 1), p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t va = smem_u32(smem + kOffV + s * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < kKeys / 16; kk++) {
                        const uint64_t bd = sw128_desc(va + kk * 2048, kTileBytes, 1024);  // 16 keys = 2048 B
                        umma_f16_ta(tmem + kTmemO, tmem + kTmemP + uint32_t(b * (kKeys / 2) + kk * 8), bd, id_o,
                                    !(j == 0 && kk == 0));
                    }
                    umma_commit(&v_empty[s]);
                    umma_commit(&pv_done[b]);
                }
            }
        }
    } else {
        // ---------------------------------------------------------- softmax (two threads per row)
        const int quad = warp & 3;         // tensor-memory lane quarter of this warp
        const int half = (warp - 2) >> 2;  // which 64 keys of each block, and which 32 O columns
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
        float* red = reinterpret_cast<float*>(smem + kOffRed);
        auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory"); };
        // `ok` stays warp-uniform; after a failed wait the loops run on without work so both
        // warps of a quarter reach every named barrier and every tcgen05 load is warp-wide.
        bool ok = true;
        auto wait_all = [&](uint64_t* bar, uint32_t parity) {
            const bool w = ok && mbar_wait(bar, parity, p.err);
            ok = __all_sync(0xffffffffu, w);
        };
        int gb = 0;
        for (int it = it0; it < it1; it++) {
            const uint4 w = p.work[it];
            const int len = int(w.y);
            const int nblk = (len + kKeys - 1) / kKeys;
            float m_used = -INFINITY, l = 0.f;
            for (int j = 0; j < nblk; j++, gb++) {
                const int b = gb & 1;
                wait_all(&s_full[b], uint32_t((gb >> 1) & 1));
                // Raw scores; the maximum is kept in the same units and each probability is
                // 2^(s log2e - m log2e), one FFMA and one ex2 per key.
                uint32_t sr[64];
                float mh = -INFINITY;
                const int kb = j * kKeys + half * 64;
                if (ok) {
                    tc_fence_after();
                    tmem_ld32(lane_base + kTmemS + b * kKeys + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
                    tmem_ld32(lane_base + kTmemS + b * kKeys + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
                    tmem_wait_ld();
                    tc_fence_before();
                    mbar_arrive(&s_free[b]);  // the S buffer may take block gb + 2
                    if (kb + 64 > len) {
#pragma unroll
                        for (int i = 0; i < 64; i++)
                            if (kb + i >= len) sr[i] = __float_as_uint(-INFINITY);
                    }
                    // Eight independent partial maxima instead of one 64-long dependency chain.
                    float mp[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) mp[i] = __uint_as_float(sr[i]);
#pragma unroll
                    for (int i = 8; i < 64; i++) mp[i & 7] = fmaxf(mp[i & 7], __uint_as_float(sr[i]));
                    mh = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
                }
                red[half * kQ + r] = mh;
                pair_sync();
                const float mb = fmaxf(mh, red[(1 - half) * kQ + r]);
                pair_sync();
                if (!ok) continue;
                const bool grow = mb > m_used + kRescaleRaw && m_used != -INFINITY;
                if (__any_sync(0xffffffffu, grow)) {
                    const float alpha = grow ? ex2_approx((m_used - mb) * kLog2e) : 1.0f;
                    if (j > 0) wait_all(&pv_done[(gb - 1) & 1], uint32_t(((gb - 1) >> 1) & 1));
                    if (!ok) continue;
                    tc_fence_after();
                    uint32_t o[32];
                    const uint32_t col = kTmemO + uint32_t(half * 32);
                    tmem_ld32(lane_base + col, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(lane_base + col, o);
                    tmem_wait_st();
                    if (grow) {
                        l *= alpha;
                        m_used = mb;
                    }
                }
                if (m_used == -INFINITY) m_used = mb;
                // P goes to buffer b once the PV two blocks back, which read that buffer, is done.
                if (gb >= 2) wait_all(&pv_done[b], uint32_t(((gb - 2) >> 1) & 1));
                if (!ok) continue;
                float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // independent partial sums
                const float nmu = m_used == -INFINITY ? 0.f : -m_used * kLog2e;
                uint32_t pk[32];  // this half's 64 probabilities as fp16 pairs
#pragma unroll
                for (int c = 0; c < 8; c++) {  // 8 groups of 8 keys
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c * 8 + 2 * e]), kLog2e, nmu));
                        const float p1 = ex2_approx(fmaf(__uint_as_float(sr[c * 8 + 2 * e + 1]), kLog2e, nmu));
                        ps[2 * e] += p0;
                        ps[2 * e + 1] += p1;
                        pk[c * 4 + e] = pack_half2(p0, p1);
                    }
                }
                // This half's 32 columns of P buffer b in tensor memory (the PV product's A).
                tmem_st32(lane_base + kTmemP + uint32_t(b * (kKeys / 2) + half * 32), pk);
                l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&p_full[b]);
            }
            // ---- epilogue: O / l; each half stores its 32 columns, then O is handed back
            red[half * kQ + r] = l;
            pair_sync();
            const float lt = l + red[(1 - half) * kQ + r];
            pair_sync();
            if (ok) {
                wait_all(&pv_done[(gb - 1) & 1], uint32_t(((gb - 1) >> 1) & 1));
                if (ok) {
                    tc_fence_after();
                    uint32_t o[32];
                    tmem_ld32(lane_base + kTmemO + uint32_t(half * 32), o);
                    tmem_wait_ld();
                    tc_fence_before();
                    mbar_arrive(o_empty);
                    const float inv = lt > 0.f ? 1.0f / lt : 0.f;
                    const int qr = int(w.z) + r;
                    if (qr < len) {
                        uint4* dst = reinterpret_cast<uint4*>(p.out + (long(w.x) + qr) * p.dmodel + int(w.w) * kHd +
                                                              half * 32);
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            uint32_t pk[4];
#pragma unroll
                            for (int e = 0; e < 4; e++)
                                pk[e] = pack_half2(__uint_as_float(o[8 * c + 2 * e]) * inv,
                                                   __uint_as_float(o[8 * c + 2 * e + 1]) * inv);
                            dst[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

cudaError_t configure_attention64() {
    return cudaFuncSetAttribute(k_attention64, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
}

cudaError_t launch_attention64(const Attn64Launch& a, cudaStream_t stream) {
    if (a.ctas <= 0 || a.sched_items <= 0) return cudaSuccess;
    const int dm = a.heads * kHd;
    CUtensorMap mq, mk, mv;
    if (!encode_fp16_map(&mq, a.q, uint64_t(dm), uint64_t(a.rows), kHd, kQ) ||
        !encode_fp16_map(&mk, a.k, uint64_t(dm), uint64_t(a.rows), kHd, kKeys) ||
        !encode_fp16_map(&mv, a.v, uint64_t(dm), uint64_t(a.rows), kHd, kKeys))
        return cudaErrorInvalidValue;
    Params p;
    p.work = reinterpret_cast<const uint4*>(a.work);
    p.offset = a.work + 4 * size_t(a.sched_items);
    p.out = a.out;
    p.dmodel = dm;
    p.err = a.err;
    return launch_kernel(k_attention64, dim3(unsigned(a.ctas)), dim3(kThreads), size_t(kSmem), stream, 1, mq, mk, mv, p);
}

}  // namespace ge
