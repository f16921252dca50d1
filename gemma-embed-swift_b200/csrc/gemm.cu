// gemm.cu -- Y[M,N] = X[M,K] * W[N,K]^T on the sm_100a tensor cores (tcgen05, kind::f16).
//
// Replaces the reference's Q8_0 GEMM family (Sources/GemmaEmbed/Shaders/GEMM.metal:72-165,
// 219-412; dispatch in Metal/MetalForward.swift:513-612).  X is an fp16 activation, W a
// Q8_0 weight; both multiply as fp16 and accumulate in fp32 in tensor memory.
//
// Persistent, warp-specialised kernel, one CTA per SM, tiles of 128 x BN, K steps of 64:
//   warp 4      TMA producer (one elected thread): X tile, and either the fp16 W tile or
//               the Q8 W tile (int8 values + fp16 block scales)
//   warps 6-9   (Q8 only) dequantise the int8 tile into the 128-byte-swizzled fp16 operand:
//               q * scale rounded once to fp16, the same value the fp16-resident weights hold
//   warp 5      tcgen05.mma issuer (one elected thread) and tensor-memory owner
//   warps 0-3   epilogue: tensor memory -> registers -> global, with fused activations
// Two accumulators of BN columns let the epilogue of one tile overlap the next tile's MMAs.
// Every wait is bounded: on timeout the kernel records GE_ERR_TIMEOUT and returns.
//
// Split tiles (fp16 weights on single CTAs, GEMM_SPLIT): tiles can run as S pieces of BN/S columns each (a
// GeGLU piece: BN/2S gate rows and the BN/2S up rows they pair with) on S times as many CTAs.
// When the tiles do not divide evenly over the CTAs, the last, partial round runs as S = 2
// pieces per tile, so the kernel ends half a tile after the full rounds instead of a whole
// tile; when all tiles fit in one round with SMs to spare (small batches), every tile is split
// (S up to 8 for fp32 stores, 4 for fp16, 2 for GeGLU) to put more SMs on the batch.  A piece
// multiplies the same A rows by the same B rows over the same K steps as the whole tile; only
// the MMA's N differs, so every output element gets the same bits either way.  Measured on a
// B200, neither split is faster than whole tiles on the forward's shapes: in the last round the
// few busy CTAs already run faster than in a full one, and a small batch's time is the 12-step
// K loop's latency, which pieces do not shorten.  So the split runs only on request.
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <tuple>

#include "kernels.hpp"
#include "ptx.cuh"

namespace ge {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kBN = 256;

// PAIR: a 2-CTA cluster computes 256 x BN tiles with tcgen05.mma.cta_group::2; each CTA
// holds 128 rows of A and BN/2 rows of B per stage, so shared-memory traffic per MMA halves.
// RES (EPI_RESIDUAL): clusters of N / BN CTAs share row blocks; the epilogue also stages
// residual-stream tiles (kXin) and receives the cluster's per-row sums of squares (kXch).
// PAIR stages hold 128 K (two 64-wide swizzled chunks per operand): a stage's wait and commits
// then cover eight MMAs, and three 64 KB stages keep about two stages of loads in flight.
template <int BN, bool Q8, bool PAIR = false, bool RES = false>
struct GemmLayout {
    static constexpr int kBK = PAIR ? 2 * BK : BK;  // K per stage
    static constexpr int kStages = RES ? (Q8 ? 2 : 3) : Q8 ? 3 : PAIR ? 3 : (BN < 256 ? 6 : 4);
    static constexpr int kA = BM * kBK * 2;
    static constexpr int kB = (PAIR ? BN / 2 : BN) * kBK * 2;
    static constexpr int kB8 = Q8 ? BN * BK : 0;
    static constexpr int kSc = Q8 ? 2 * BN * 2 : 0;
    static constexpr int kStage = (kA + kB + kB8 + kSc + 1023) / 1024 * 1024;
    // Epilogue staging: per epilogue warp, kStgBufs tiles of 32 rows x 128 bytes that TMA
    // stores to global memory (one buffer on the Q8 path, whose stages are larger).  RES: four,
    // which also receive the residual-stream tiles and are rewritten in place.
    // RES on fp16 weights: eight epilogue warps, two per TMEM lane quarter, each owning half of
    // the tile's columns (warps 0-3 and 6-9; warp w reads TMEM lanes 32 * (w % 4) + [0, 32)).
    static constexpr int kEpiWarps = (RES && !Q8) ? 8 : 4;
    static constexpr int kStgBufs = RES ? (kEpiWarps == 8 ? 2 : 4) : Q8 ? 1 : 2;
    static constexpr int kStgOff = kStages * kStage;
    static constexpr int kXchOff = kStgOff + kEpiWarps * kStgBufs * 4096;
    static constexpr int kMaxCluster = 4;  // RES: [2 tile parities][2 rounds][kMaxCluster][128] floats
    static constexpr int kHsumOff = kXchOff + (RES ? 2 * 2 * kMaxCluster * 128 * 4 : 0);
    static constexpr int kBarOff = kHsumOff + (RES ? 2 * 2 * 2 * 128 * 4 : 0);  // [parity][round][half][128]
    static constexpr int kBytes = kBarOff + 512 + 1024;  // barriers, TMEM slot, alignment slack
    static constexpr int kThreads = (Q8 || kEpiWarps == 8) ? 320 : 192;
};

struct GemmParams {
    int M, N, K;
    void* out;
    int ldo;
    const float* aux;
    int ldaux;
    int* err;
    // EPI_RESIDUAL
    const float* w_post;
    const float* w_next;
    float scale, eps;
    int store_h, store_y;
    // clamp epilogues (aux holds the optional bias)
    float lo1, hi1, lo2, hi2;
    // Split tiles: tiles from split_from on run as `split` pieces of BN / split columns
    // (split_from == the tile count: no split)
    int split_from, split;
    // EPI_QKV (eps above)
    const int32_t* pos;
    const float* rope;
    const float* qw;
    const float* kw;
    int ntok, heads, kvh;
};

// EPI_RESIDUAL output maps: the next norm's fp16 (boxes of 32 rows x 64) and fp32 (32 x 32)
// results.  mapC is the residual stream's fp32 map, used to load and to store it.
struct EpiMaps {
    CUtensorMap h, y;
};

__device__ __forceinline__ float round_f16(uint32_t acc_bits) {
    return __half2float(__float2half_rn(__uint_as_float(acc_bits)));
}

// Waits without giving up on another role's error (used to drain in-flight TMA loads).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (!mbar_test(bar, parity) && globaltimer() - t0 < kWaitLimitNs) {
    }
}

// Dequantises 16 int8 values with one fp16 scale into 8 half2 words (exact q, one rounding).
__device__ __forceinline__ void dequant16(uint4 raw, __half2 s2, uint32_t (&o)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152 = 1024 + 128
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t u = w[i] ^ 0x80808080u;  // int8 -> uint8 biased by 128
        uint32_t lo = __byte_perm(u, 0x64646464u, 0x4140);  // halves 1024 + b0, 1024 + b1
        uint32_t hi = __byte_perm(u, 0x64646464u, 0x4342);  // halves 1024 + b2, 1024 + b3
        __half2 hl = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&lo), bias), s2);
        __half2 hh = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&hi), bias), s2);
        o[2 * i] = *reinterpret_cast<uint32_t*>(&hl);
        o[2 * i + 1] = *reinterpret_cast<uint32_t*>(&hh);
    }
}

template <int BN, int EPI, bool Q8, bool PAIR>
__global__ void __launch_bounds__(GemmLayout<BN, Q8, PAIR, EPI == EPI_RESIDUAL>::kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
           const __grid_constant__ CUtensorMap mapS, const __grid_constant__ CUtensorMap mapP,
           const __grid_constant__ CUtensorMap mapC, const __grid_constant__ EpiMaps emaps, GemmParams p) {
    constexpr bool RES = EPI == EPI_RESIDUAL;
    static_assert(!(PAIR && Q8), "the pair kernel reads fp16 weights");
    static_assert(!(PAIR && RES), "row clusters and CTA pairs are exclusive");
    using L = GemmLayout<BN, Q8, PAIR, RES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_tma = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
    uint64_t* full_b = full_tma + L::kStages;
    uint64_t* empty = full_b + L::kStages;
    uint64_t* tfull = empty + L::kStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* xin_bar = tempty + 2;   // RES: [epilogue warp][up to 4 buffers]
    uint64_t* xch_bar = xin_bar + 32;  // RES: [tile parity][round]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xch_bar + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = p.N / BN;
    const int kb_count = p.K / L::kBK;
    // Tiles in a fixed order: n fastest, so the CTAs working at one time share A rows in L2.
    // A pair's tile covers 256 rows: the pair leader (rank 0) the first 128, rank 1 the rest.
    // A row cluster (RES) walks row blocks; its CTA of rank r always takes columns r * BN.
    const uint32_t crank = (PAIR || RES) ? cluster_ctarank() : 0;
    const bool leader = !PAIR || crank == 0;  // issues the MMAs and drains the loads
    const uint32_t csize = RES ? cluster_nctarank() : PAIR ? 2u : 1u;
    const int tiles = RES ? p.M / BM : n_tiles * (PAIR ? (p.M + 2 * BM - 1) / (2 * BM) : p.M / BM);
    const int first = int(blockIdx.x / csize);
    const int step = int(gridDim.x / csize);
    auto tile_origin = [&](int t, int& m0, int& n0) {
        if (RES) {
            m0 = t * BM;
            n0 = int(crank) * BN;
        } else {
            m0 = (t / n_tiles) * (PAIR ? 2 * BM : BM) + int(crank) * BM;
            n0 = (t % n_tiles) * BN;
        }
    };
    // Work items: tiles [0, split_from) whole, then `split` pieces (sub 0 .. split - 1) of each
    // later tile.  Every role walks the same items in the same order.
    constexpr bool kSplit = !PAIR && !RES && !Q8 && EPI != EPI_QKV;
    const int split = kSplit ? p.split : 1;
    const int split_from = split > 1 ? min(p.split_from, tiles) : tiles;
    const int items = split_from + split * (tiles - split_from);
    auto item_origin = [&](int w, int& m0, int& n0, int& sub) {
        if (w < split_from) {
            tile_origin(w, m0, n0);
            sub = -1;
        } else {
            tile_origin(split_from + (w - split_from) / split, m0, n0);
            sub = (w - split_from) % split;
        }
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::kStages; s++) {
            mbar_init(&full_tma[s], 1);
            mbar_init(&full_b[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            // PAIR: one arrival per epilogue warp of both CTAs; otherwise one per epilogue thread
            mbar_init(&tempty[a], PAIR ? 8 : 32 * L::kEpiWarps);
        }
        if (RES) {
            for (int i = 0; i < 32; i++) mbar_init(&xin_bar[i], 1);
            // Each exchange barrier completes when every other CTA of the cluster has delivered
            // its 128 row sums; its single arrival is this CTA's own arming for the next use.
            for (int i = 0; i < 4; i++) {
                mbar_init(&xch_bar[i], 1);
                mbar_expect_tx(&xch_bar[i], (csize - 1) * 128 * 4);
            }
        }
        fence_mbar_init();
    }
    if (warp == 4 && lane == 0) {
        tma_prefetch(&mapA);
        tma_prefetch(&mapB);
        if (Q8) tma_prefetch(&mapS);
        if (kSplit && split_from < tiles) tma_prefetch(&mapP);
        tma_prefetch(&mapC);
        if (RES) {
            tma_prefetch(&emaps.h);
            tma_prefetch(&emaps.y);
        }
    }
    if (warp == 5) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, 2 * BN);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, 2 * BN);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR || RES) cluster_sync();  // the peers' barriers are initialised before any remote use
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The set-up above overlaps the previous kernel's tail; A and the output are its data.
    pdl_wait();

    if (warp == 4) {
        // ---------------------------------------------------------- TMA producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long issued = 0;
            bool ok = true;
            for (int w = first; w < items && ok; w += step) {
                int m0, n0, sub;
                item_origin(w, m0, n0, sub);
                for (int kb = 0; kb < kb_count; kb++) {
                    if (!mbar_wait(&empty[s], ph ^ 1, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * L::kStage;
                    if (PAIR) {
                        // Both CTAs' loads complete on the leader's barrier, which expects them all.
                        const uint32_t bar = mapa_shared(&full_tma[s], 0);
                        if (crank == 0) mbar_expect_tx(&full_tma[s], 2 * (L::kA + L::kB));
                        for (int c = 0; c < L::kBK / BK; c++) {  // 64-wide K chunks
                            tma_load_2d_pair(st + c * (L::kA / (L::kBK / BK)), &mapA, bar, kb * L::kBK + c * BK, m0);
                            tma_load_2d_pair(st + L::kA + c * (L::kB / (L::kBK / BK)), &mapB, bar, kb * L::kBK + c * BK,
                                             n0 + int(crank) * (BN / 2));
                        }
                    } else {
                        mbar_expect_tx(&full_tma[s], L::kA + (Q8 ? L::kB8 + L::kSc : sub < 0 ? L::kB : L::kB / split));
                        tma_load_2d(st, &mapA, &full_tma[s], kb * BK, m0);
                    }
                    if (PAIR) {
                    } else if (Q8) {
                        tma_load_2d(st + L::kA + L::kB, &mapB, &full_tma[s], kb * BK, n0);
                        tma_load_2d(st + L::kA + L::kB + L::kB8, &mapS, &full_tma[s], n0, kb * 2);
                    } else if (sub < 0) {
                        tma_load_2d(st + L::kA, &mapB, &full_tma[s], kb * BK, n0);
                    } else if (epi_is_geglu(EPI)) {
                        // BN/2S gate rows, then the BN/2S up rows they pair with (BN/2 further on)
                        const int hp = BN / (2 * split);
                        tma_load_2d(st + L::kA, &mapP, &full_tma[s], kb * BK, n0 + sub * hp);
                        tma_load_2d(st + L::kA + hp * BK * 2, &mapP, &full_tma[s], kb * BK, n0 + BN / 2 + sub * hp);
                    } else {
                        tma_load_2d(st + L::kA, &mapP, &full_tma[s], kb * BK, n0 + sub * (BN / split));
                    }
                    issued++;
                    if (++s == L::kStages) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            pdl_launch();  // this CTA's loads are all issued: the next kernel may be scheduled
            // Every issued load must land before the CTA exits, also after an error.  A pair's
            // loads complete on the leader's barriers, so the leader drains for both CTAs.
            if (leader)
                for (int j = 0; j < L::kStages; j++) {
                    const long c = issued / L::kStages + (j < issued % L::kStages ? 1 : 0);
                    if (c > 0) drain_wait(&full_tma[j], uint32_t((c - 1) & 1));
                }
        }
    } else if (warp == 5) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0 && leader) {  // a pair's MMAs are issued by its leader alone
            const uint32_t idesc_tile = idesc_f16(PAIR ? 2 * BM : BM, BN);
            const uint32_t idesc_piece = idesc_f16(BM, BN / (kSplit ? split : 1));
            int s = 0, acc = 0;
            uint32_t ph = 0, acc_ph = 0;
            bool ok = true;
            for (int w = first; w < items && ok; w += step) {
                const uint32_t idesc = w < split_from ? idesc_tile : idesc_piece;
                if (!mbar_wait(&tempty[acc], acc_ph ^ 1, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * BN);
                for (int kb = 0; kb < kb_count; kb++) {
                    if (!mbar_wait(&full_tma[s], ph, p.err) || (Q8 && !mbar_wait(&full_b[s], ph, p.err))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint8_t* st = smem + s * L::kStage;
                    const uint64_t ad = sw128_desc(smem_u32(st), 16, 1024);
                    const uint64_t bd = sw128_desc(smem_u32(st + L::kA), 16, 1024);
                    if (PAIR) {
                        // 16-wide K steps: chunk kk / 4 of each operand, 32 bytes apart inside it
#pragma unroll
                        for (int kk = 0; kk < L::kBK / 16; kk++) {
                            const uint64_t ca = uint64_t(((kk >> 2) * (L::kA / (L::kBK / BK))) >> 4);
                            const uint64_t cb = uint64_t(((kk >> 2) * (L::kB / (L::kBK / BK))) >> 4);
                            umma_f16_pair(d, ad + ca + uint64_t((kk & 3) * 2), bd + cb + uint64_t((kk & 3) * 2), idesc,
                                          (kb | kk) != 0);
                        }
                        umma_commit_pair(mapa_shared(&empty[s], 0));
                        umma_commit_pair(mapa_shared(&empty[s], 1));
                    } else {
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++)
                            umma_f16(d, ad + uint64_t(kk * 2), bd + uint64_t(kk * 2), idesc, (kb | kk) != 0);
                        umma_commit(&empty[s]);
                    }
                    if (++s == L::kStages) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
                if (PAIR) {
                    umma_commit_pair(mapa_shared(&tfull[acc], 0));
                    umma_commit_pair(mapa_shared(&tfull[acc], 1));
                } else {
                    umma_commit(&tfull[acc]);
                }
                if (++acc == 2) {
                    acc = 0;
                    acc_ph ^= 1;
                }
            }
        }
    } else if (warp < 4 || (L::kEpiWarps == 8 && warp >= 6)) {
        // ---------------------------------------------------------- epilogue
        // Each warp owns 32 accumulator rows (its TMEM lane quarter).  Per 128-byte column group
        // a thread packs its row's values, writes them 128-byte-swizzled into the warp's staging
        // buffer, and lane 0 TMA-stores the 32 x 128-byte box: full-line writes to global memory.
        const int epi = warp < 4 ? warp : warp - 2;  // epilogue warp index 0..7
        uint8_t* stg = smem + L::kStgOff + epi * L::kStgBufs * 4096;
        int sbuf = 0;
        auto emit = [&](const uint32_t (&v)[32], int x, int y, const CUtensorMap* map) {
            if (lane == 0) bulk_wait_read<L::kStgBufs - 1>();
            __syncwarp();
            uint8_t* buf = stg + sbuf * 4096 + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; j++)
                *reinterpret_cast<uint4*>(buf + ((j ^ (lane & 7)) * 16)) =
                    make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(map, stg + sbuf * 4096, x, y);
                bulk_commit();
            }
            sbuf = (sbuf + 1 == L::kStgBufs) ? 0 : sbuf + 1;
        };
        // The accumulator is handed back to the MMA warp as soon as its last columns are in
        // registers, before they are converted and stored.
        auto release = [&](int a) {
            tc_fence_before();
            if (PAIR) {  // the accumulator is released to the leader, which issues the MMAs
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(&tempty[a], 0));
            } else {
                mbar_arrive(&tempty[a]);
            }
        };
        int acc = 0;
        uint32_t acc_ph = 0;
        if constexpr (RES) {
            // Residual epilogue, per tile of 128 rows x BN columns (this CTA's share of the row
            // block).  A thread owns one row of HW columns: all BN with four epilogue warps, or
            // one half with eight (the two warps of a TMEM lane quarter split the columns).
            //   1. ss = sum of t^2 over the columns, t = fp16(acc); the halves of a row add
            //      through shared memory (a named barrier per lane quarter)
            //   2. exchange: the CTA's 128 row sums go to the other CTAs of the cluster
            //      (st.async completing on their exchange barrier); sums add in rank order
            //   3. x = (x + t * inv * w_post) * scale, 32 columns at a time: the x tile streams
            //      through the warp's staging buffers by TMA (kStgBufs chunks ahead), the new
            //      values go back to TMEM; ss2 = sum of the new x^2
            //   4. ss2 as in 1-2
            //   5. from TMEM: x stored back, y = x * inv2 * w_next stored as fp16 and/or fp32
            // The order of every sum is fixed, so a row's results do not depend on the batch.
            constexpr int NB = L::kStgBufs;
            constexpr int HALVES = L::kEpiWarps / 4;
            constexpr int HW = BN / HALVES;
            const int quarter = warp & 3;
            const int half = warp < 4 ? 0 : 1;
            float* xch = reinterpret_cast<float*>(smem + L::kXchOff);
            float* hsum = reinterpret_cast<float*>(smem + L::kHsumOff);
            const int row_local = quarter * 32 + lane;
            uint32_t xin_ph = 0u, xin_pending = 0u;  // bit b: phase parity / load in flight of buffer b
            auto load_x = [&](int b, int x, int y) {
                if (lane == 0) {
                    mbar_expect_tx(&xin_bar[epi * 4 + b], 4096);
                    tma_load_2d(stg + b * 4096, &mapC, &xin_bar[epi * 4 + b], x, y);
                }
                xin_pending |= 1u << b;
            };
            // Row sum over the CTA's columns, then over the cluster, in fixed order.
            auto row_total = [&](float part, int par, int rd, uint32_t ph, float& total) -> bool {
                if (HALVES == 2) {
                    float* hs = hsum + ((par * 2 + rd) * 2) * 128;
                    hs[half * 128 + row_local] = part;
                    asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
                    part = hs[row_local] + hs[128 + row_local];
                }
                const int slot_index = par * 2 + rd;
                float* slot = xch + slot_index * L::kMaxCluster * 128;
                uint64_t* bar = &xch_bar[slot_index];
                if (half == 0)
                    for (uint32_t q = 0; q < csize; q++)
                        if (q != crank)
                            st_async_b32(mapa_shared(slot + crank * 128 + row_local, q), __float_as_uint(part),
                                         mapa_shared(bar, q));
                if (!mbar_wait(bar, ph, p.err)) return false;
                float sum = 0.f;
                for (uint32_t q = 0; q < csize; q++) sum += q == crank ? part : slot[q * 128 + row_local];
                total = sum;
                // Armed again for its next use, two tiles on; no peer can deliver for that use
                // before this CTA has sent its sums of the tile in between.
                if (threadIdx.x == 0) mbar_expect_tx(bar, (csize - 1) * 128 * 4);
                return true;
            };
            constexpr int kchunks = HW / 32;
            int k = 0;
            bool ok = true;
            for (int t = first; t < tiles && ok; t += step, k++) {
                int m0, n0;
                tile_origin(t, m0, n0);
                const int c0 = n0 + half * HW;  // this warp's first column
                const int y = m0 + quarter * 32;
                // The first x chunks travel while the accumulator fills, once the previous
                // tile's stores have left the buffers.
                if (lane == 0) bulk_wait_read<0>();
                __syncwarp();
                for (int b = 0; b < NB; b++) load_x(b, c0 + 32 * b, y);
                if (!mbar_wait(&tfull[acc], acc_ph, p.err)) break;
                tc_fence_after();
                const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + half * HW);
                const int par = k & 1;
                const uint32_t xph = uint32_t(k >> 1) & 1u;
                // 1.-2. sum of squares of the fp16-rounded projection: one partial per 128
                // columns, added as (first + second) with four warps or eight alike
                float ssh[2] = {0.f, 0.f};
#pragma unroll
                for (int c = 0; c < HW / 128; c++) {
                    uint32_t r[128];
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        tmem_ld32(taddr + uint32_t(c * 128 + q * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32 * q]));
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 128; i++) {
                        const float tv = round_f16(r[i]);
                        ssh[c] += tv * tv;
                    }
                }
                float total;
                if (!row_total(HALVES == 2 ? ssh[0] : ssh[0] + ssh[1], par, 0, xph, total)) break;
                const float inv = 1.0f / sqrtf(total / float(p.N) + p.eps);
                // 3. the residual update (ss2 in per-128-column partials like ss)
                float ss2a = 0.f, ss2b = 0.f;
#pragma unroll 1
                for (int c = 0; c < kchunks; c++) {
                    const int b = c % NB;
                    if (!mbar_wait(&xin_bar[epi * 4 + b], (xin_ph >> b) & 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    xin_ph ^= 1u << b;
                    xin_pending &= ~(1u << b);
                    uint32_t r[32];
                    tmem_ld32(taddr + uint32_t(c * 32), r);
                    const uint8_t* xb = stg + b * 4096 + lane * 128;
                    float xv[32];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float4 q = *reinterpret_cast<const float4*>(xb + ((j ^ (lane & 7)) * 16));
                        xv[4 * j] = q.x;
                        xv[4 * j + 1] = q.y;
                        xv[4 * j + 2] = q.z;
                        xv[4 * j + 3] = q.w;
                    }
                    // The buffer is read: it takes chunk c + NB.
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (c + NB < kchunks) load_x(b, c0 + (c + NB) * 32, y);
                    tmem_wait_ld();
                    const float4* wp4 = reinterpret_cast<const float4*>(p.w_post + c0 + c * 32);
                    uint32_t vo[32];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float4 w = __ldg(wp4 + j);
                        const float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int i = 4 * j + e;
                            float v = xv[i] + round_f16(r[i]) * inv * ww[e];
                            if (p.scale != 1.0f) v *= p.scale;
                            vo[i] = __float_as_uint(v);
                        }
                    }
                    float s2 = c >= 4 ? ss2b : ss2a;
#pragma unroll
                    for (int i = 0; i < 32; i++) s2 += __uint_as_float(vo[i]) * __uint_as_float(vo[i]);
                    if (c >= 4)
                        ss2b = s2;
                    else
                        ss2a = s2;
                    tmem_st32(taddr + uint32_t(c * 32), vo);
                }
                if (!ok) break;
                tmem_wait_st();
                const bool next = p.store_h || p.store_y;
                float inv2 = 0.f;
                if (next) {
                    if (!row_total(HALVES == 2 ? ss2a : ss2a + ss2b, par, 1, xph, total)) break;
                    inv2 = 1.0f / sqrtf(total / float(p.N) + p.eps);
                }
                // 5. stores from TMEM, 64 columns at a time
                sbuf = 0;
#pragma unroll 1
                for (int c = 0; c < HW / 64; c++) {
                    uint32_t r[64];
                    tmem_ld32(taddr + uint32_t(c * 64), *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
                    tmem_ld32(taddr + uint32_t(c * 64 + 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
                    tmem_wait_ld();
                    if (c == HW / 64 - 1) release(acc);
                    emit(*reinterpret_cast<uint32_t(*)[32]>(&r[0]), c0 + c * 64, y, &mapC);
                    emit(*reinterpret_cast<uint32_t(*)[32]>(&r[32]), c0 + c * 64 + 32, y, &mapC);
                    if (!next) continue;
                    const float4* wn4 = reinterpret_cast<const float4*>(p.w_next + c0 + c * 64);
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const float4 w = __ldg(wn4 + j);
                        r[4 * j] = __float_as_uint(__uint_as_float(r[4 * j]) * inv2 * w.x);
                        r[4 * j + 1] = __float_as_uint(__uint_as_float(r[4 * j + 1]) * inv2 * w.y);
                        r[4 * j + 2] = __float_as_uint(__uint_as_float(r[4 * j + 2]) * inv2 * w.z);
                        r[4 * j + 3] = __float_as_uint(__uint_as_float(r[4 * j + 3]) * inv2 * w.w);
                    }
                    if (p.store_h) {
                        uint32_t packed[32];
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            packed[i] = pack_half2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
                        emit(packed, c0 + c * 64, y, &emaps.h);
                    }
                    if (p.store_y) {
                        emit(*reinterpret_cast<uint32_t(*)[32]>(&r[0]), c0 + c * 64, y, &emaps.y);
                        emit(*reinterpret_cast<uint32_t(*)[32]>(&r[32]), c0 + c * 64 + 32, y, &emaps.y);
                    }
                }
                if (++acc == 2) {
                    acc = 0;
                    acc_ph ^= 1;
                }
            }
            // x loads still in flight after an error land before the CTA exits.
            for (int b = 0; b < NB; b++)
                if ((xin_pending >> b) & 1u) drain_wait(&xin_bar[epi * 4 + b], (xin_ph >> b) & 1u);
        } else
        for (int w = first; w < items; w += step) {
            if (!mbar_wait(&tfull[acc], acc_ph, p.err)) break;
            tc_fence_after();
            int m0, n0, sub;
            item_origin(w, m0, n0, sub);
            // A piece holds BN/S accumulator columns: output columns n0 + sub * BN/S onward, or
            // for GeGLU BN/2S gate columns then BN/2S up columns (output n0/2 + sub * BN/2S on).
            const int width = sub < 0 ? BN : BN / split;
            const int nc = sub < 0 ? n0 : n0 + sub * width;
            const int ng = sub < 0 ? n0 / 2 : n0 / 2 + sub * (width / 2);
            const int y = m0 + warp * 32;
            const long row = y + lane;
            const uint32_t taddr = tmem + (uint32_t(warp * 32) << 16) + uint32_t(acc * BN);
            uint32_t packed[32];
            if constexpr (EPI == EPI_QKV) {
                // One tile is one head slot of 256 columns.  Pass 1: the sum of squares of the
                // fp16-rounded projection; pass 2: columns j and j + 128 (NeoX rotation partners)
                // together, 64 of each per step, normalised, weighted, rotated and stored.
                static_assert(BN == 256, "EPI_QKV tiles are one 256-wide head slot");
                const int slot = n0 / BN;
                const bool live = row < p.ntok;
                const float* w = slot < p.heads ? p.qw : (slot < p.heads + p.kvh ? p.kw : nullptr);
                float ss = 0.f;
#pragma unroll 1
                for (int c = 0; c < 2; c++) {
                    uint32_t r[128];
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        tmem_ld32(taddr + uint32_t(c * 128 + q * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32 * q]));
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 128; i++) {
                        const float v = round_f16(r[i]);
                        ss += v * v;
                    }
                }
                const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
                // This row's position's (cos, sin) pairs; read row-major, each thread's own
                // 1 KB row (a pair-major table, coalesced across the warp, measured slower).
                const float* cs = (w && live) ? p.rope + long(p.pos[row]) * 256 : nullptr;
#pragma unroll 1
                for (int c = 0; c < 2; c++) {
                    uint32_t r[128];
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        tmem_ld32(taddr + uint32_t(c * 64 + q * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32 * q]));
                        tmem_ld32(taddr + uint32_t(128 + c * 64 + q * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[64 + 32 * q]));
                    }
                    tmem_wait_ld();
                    if (c == 1) release(acc);
                    uint32_t pb[32];
#pragma unroll
                    for (int i = 0; i < 64; i += 2) {
                        const int j = c * 64 + i;  // pair index (column of the first half)
                        float a0 = round_f16(r[i]) * inv, a1 = round_f16(r[i + 1]) * inv;
                        float b0 = round_f16(r[64 + i]) * inv, b1 = round_f16(r[64 + i + 1]) * inv;
                        if (w) {
                            const float2 wa = *reinterpret_cast<const float2*>(w + j);
                            const float2 wb = *reinterpret_cast<const float2*>(w + 128 + j);
                            a0 = a0 * wa.x;
                            a1 = a1 * wa.y;
                            b0 = b0 * wb.x;
                            b1 = b1 * wb.y;
                        }
                        if (cs) {
                            const float4 f = *reinterpret_cast<const float4*>(cs + 2 * j);  // cos j, sin j, cos j+1, sin j+1
                            const float x0 = a0 * f.x - b0 * f.y, y0 = a0 * f.y + b0 * f.x;
                            const float x1 = a1 * f.z - b1 * f.w, y1 = a1 * f.w + b1 * f.z;
                            a0 = x0;
                            b0 = y0;
                            a1 = x1;
                            b1 = y1;
                        }
                        if (!live) a0 = a1 = b0 = b1 = 0.f;
                        packed[i / 2] = pack_half2(a0, a1);
                        pb[i / 2] = pack_half2(b0, b1);
                    }
                    emit(packed, n0 + c * 64, y, &mapC);
                    emit(pb, n0 + 128 + c * 64, y, &mapC);
                }
            } else if (EPI == EPI_F32 || EPI == EPI_CLAMP_F32) {
                uint32_t r[32];
#pragma unroll 1
                for (int c = 0; c < width / 32; c++) {
                    tmem_ld32(taddr + uint32_t(c * 32), r);
                    tmem_wait_ld();
                    if (c == width / 32 - 1) release(acc);
                    if (EPI == EPI_CLAMP_F32) {
                        const float* b = p.aux ? p.aux + nc + c * 32 : nullptr;
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            float v = fminf(fmaxf(__uint_as_float(r[i]), p.lo1), p.hi1);
                            if (b) v += b[i];
                            r[i] = __float_as_uint(v);
                        }
                    }
                    emit(r, nc + c * 32, y, &mapC);
                }
            } else if (epi_is_geglu(EPI)) {
                // Columns [0, BN/2) of the tile are gate rows, [BN/2, BN) the matching up rows.
                // Per 64 output columns: 64 gate and 64 up values in flight, one wait.
#pragma unroll 1
                for (int c = 0; c < width / 128; c++) {
                    uint32_t g[64], u[64];
                    tmem_ld32(taddr + uint32_t(c * 64), *reinterpret_cast<uint32_t(*)[32]>(&g[0]));
                    tmem_ld32(taddr + uint32_t(c * 64 + 32), *reinterpret_cast<uint32_t(*)[32]>(&g[32]));
                    tmem_ld32(taddr + uint32_t(width / 2 + c * 64), *reinterpret_cast<uint32_t(*)[32]>(&u[0]));
                    tmem_ld32(taddr + uint32_t(width / 2 + c * 64 + 32), *reinterpret_cast<uint32_t(*)[32]>(&u[32]));
                    tmem_wait_ld();
                    if (c == width / 128 - 1) release(acc);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float g0 = __uint_as_float(g[2 * i]), g1 = __uint_as_float(g[2 * i + 1]);
                        float u0 = __uint_as_float(u[2 * i]), u1 = __uint_as_float(u[2 * i + 1]);
                        float a0, a1;
                        if (EPI == EPI_GEGLU) {
                            a0 = gelu_fast(g0);
                            a1 = gelu_fast(g1);
                        } else if (EPI == EPI_GEGLU_QUICK) {
                            a0 = gelu_quick_fast(g0);
                            a1 = gelu_quick_fast(g1);
                        } else {
                            a0 = sigmoid_fast(fminf(fmaxf(g0, p.lo1), p.hi1));
                            a1 = sigmoid_fast(fminf(fmaxf(g1, p.lo1), p.hi1));
                            u0 = fminf(fmaxf(u0, p.lo1), p.hi1);
                            u1 = fminf(fmaxf(u1, p.lo1), p.hi1);
                        }
                        packed[i] = pack_half2(a0 * u0, a1 * u1);
                    }
                    emit(packed, ng + c * 64, y, &mapC);
                }
            } else if (EPI == EPI_F16 || EPI == EPI_GELU_MUL || EPI == EPI_CLAMP_F16 || EPI == EPI_CLAMP_SILU) {
                // 128 columns in flight per wait (64 for a 64-wide piece), stored as 64-column boxes.
                const int chunk = width < 128 ? 64 : 128;
#pragma unroll 1
                for (int c = 0; c < width / chunk; c++) {
                    uint32_t r[128];
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (q < chunk / 32)
                            tmem_ld32(taddr + uint32_t(c * 128 + q * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32 * q]));
                    tmem_wait_ld();
                    if (c == width / chunk - 1) release(acc);
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        if (half >= chunk / 64) break;
                        const uint32_t* rv = r + 64 * half;
                        if (EPI == EPI_GELU_MUL) {
                            const float4* ax =
                                reinterpret_cast<const float4*>(p.aux + row * p.ldaux + nc + c * 128 + half * 64);
#pragma unroll
                            for (int i = 0; i < 16; i++) {
                                const float4 a = ax[i];
                                packed[2 * i] = pack_half2(gelu_fast(__uint_as_float(rv[4 * i])) * a.x,
                                                           gelu_fast(__uint_as_float(rv[4 * i + 1])) * a.y);
                                packed[2 * i + 1] = pack_half2(gelu_fast(__uint_as_float(rv[4 * i + 2])) * a.z,
                                                               gelu_fast(__uint_as_float(rv[4 * i + 3])) * a.w);
                            }
                        } else if (EPI == EPI_CLAMP_F16 || EPI == EPI_CLAMP_SILU) {
                            const float* b = p.aux ? p.aux + nc + c * 128 + half * 64 : nullptr;
#pragma unroll
                            for (int i = 0; i < 32; i++) {
                                float v0 = fminf(fmaxf(__uint_as_float(rv[2 * i]), p.lo1), p.hi1);
                                float v1 = fminf(fmaxf(__uint_as_float(rv[2 * i + 1]), p.lo1), p.hi1);
                                if (b) {
                                    v0 += b[2 * i];
                                    v1 += b[2 * i + 1];
                                }
                                if (EPI == EPI_CLAMP_SILU) {
                                    v0 = fminf(fmaxf(silu_fast(v0), p.lo2), p.hi2);
                                    v1 = fminf(fmaxf(silu_fast(v1), p.lo2), p.hi2);
                                }
                                packed[i] = pack_half2(v0, v1);
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; i++)
                                packed[i] = pack_half2(__uint_as_float(rv[2 * i]), __uint_as_float(rv[2 * i + 1]));
                        }
                        emit(packed, nc + c * 128 + half * 64, y, &mapC);
                    }
                }
            }
            if (++acc == 2) {
                acc = 0;
                acc_ph ^= 1;
            }
        }
        // Every store has left shared memory and reached global memory before the CTA exits.
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    } else if (Q8) {
        // ---------------------------------------------------------- Q8 -> fp16 converters
        const int tid = threadIdx.x - 192;
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int t = first; t < tiles && ok; t += step) {
            for (int kb = 0; kb < kb_count; kb++) {
                if (!mbar_wait(&full_tma[s], ph, p.err)) {
                    ok = false;
                    break;
                }
                uint8_t* st = smem + s * L::kStage;
                uint8_t* b16 = st + L::kA;
                const uint8_t* b8 = b16 + L::kB;
                const __half* sc = reinterpret_cast<const __half*>(b8 + L::kB8);
#pragma unroll 2
                for (int i = 0; i < BN * 4 / 128; i++) {
                    const int idx = i * 128 + tid;
                    const int r = idx >> 2, c = idx & 3;
                    const uint4 raw = *reinterpret_cast<const uint4*>(b8 + r * BK + c * 16);
                    const __half2 s2 = __half2half2(sc[(c >> 1) * BN + r]);
                    uint32_t o[8];
                    dequant16(raw, s2, o);
                    uint8_t* rowp = b16 + r * 128;
                    const int j0 = (2 * c) ^ (r & 7), j1 = (2 * c + 1) ^ (r & 7);
                    *reinterpret_cast<uint4*>(rowp + j0 * 16) = make_uint4(o[0], o[1], o[2], o[3]);
                    *reinterpret_cast<uint4*>(rowp + j1 * 16) = make_uint4(o[4], o[5], o[6], o[7]);
                }
                fence_proxy_async_smem();
                mbar_arrive(&full_b[s]);
                if (++s == L::kStages) {
                    s = 0;
                    ph ^= 1;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (PAIR || RES) cluster_sync();  // no CTA leaves while another may still signal it
    if (warp == 5) {
        tc_fence_after();
        if (PAIR)
            tmem_dealloc_pair(tmem, 2 * BN);
        else
            tmem_dealloc(tmem, 2 * BN);
    }
}

// ---------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

static bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes, void* ptr, uint64_t inner,
                      uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz,
                      uint64_t row_stride = 0) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {(row_stride ? row_stride : inner) * uint64_t(elem_bytes)};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_weight_maps(DevWeight& w, int bn) {
    if (!w.q8 && !w.f16) return false;
    bool ok = true;
    if (w.q8)  // weights stored as F16/BF16/F32 in the GGUF have no Q8 planes
        ok = encode_2d(&w.map_q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.q8, w.K, w.N, BK, bn,
                       CU_TENSOR_MAP_SWIZZLE_NONE) &&
             encode_2d(&w.map_scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.scales_t, w.N, w.K / 32, bn, 2,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
    // A weight narrower than a full tile (N = bn / 2) gets a full-tile map of its own height.
    if (ok && w.f16)
        ok = encode_2d(&w.map_f16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.f16, w.K, w.N, BK,
                       uint32_t(w.N < bn ? w.N : bn), CU_TENSOR_MAP_SWIZZLE_128B) &&
             encode_2d(&w.map_f16_half, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.f16, w.K, w.N, BK, bn / 2,
                       CU_TENSOR_MAP_SWIZZLE_128B) &&
             encode_2d(&w.map_f16_quarter, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.f16, w.K, w.N, BK, bn / 4,
                       CU_TENSOR_MAP_SWIZZLE_128B) &&
             encode_2d(&w.map_f16_eighth, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.f16, w.K, w.N, BK, bn / 8,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    return ok;
}

bool encode_fp16_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint32_t box_inner,
                     uint32_t box_outer, uint64_t row_stride) {
    return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), inner, outer, box_inner, box_outer,
                     CU_TENSOR_MAP_SWIZZLE_128B, row_stride);
}

bool encode_fp16_map_3d(CUtensorMap* map, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0,
                        uint32_t b1, uint32_t b2, uint64_t stride2) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {d0 * 2, (stride2 ? stride2 : d0 * d1) * 2};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_activation_map(DevActivation& a) {
    return encode_2d(&a.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.ptr, a.cols, a.rows, BK, BM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int EPI, bool Q8, bool PAIR, int BN = kBN>
static cudaError_t configure_t() {
    using L = GemmLayout<BN, Q8, PAIR, EPI == EPI_RESIDUAL>;
    return cudaFuncSetAttribute(k_gemm<BN, EPI, Q8, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
}

template <int EPI>
static cudaError_t configure_epi() {
    cudaError_t e = configure_t<EPI, false, false>();
    if (e == cudaSuccess) e = configure_t<EPI, true, false>();
    if constexpr (EPI != EPI_RESIDUAL) {
        if (e == cudaSuccess) e = configure_t<EPI, false, true>();
        if constexpr (!epi_is_geglu(EPI) && EPI != EPI_QKV)
            if (e == cudaSuccess) e = configure_t<EPI, false, false, 128>();
    }
    return e;
}

// Sets the shared-memory limit of every GEMM variant on the current device; runs at load,
// before any stream capture.
cudaError_t configure_gemm_kernels() {
    cudaError_t e = configure_epi<EPI_F32>();
    if (e == cudaSuccess) e = configure_epi<EPI_F16>();
    if (e == cudaSuccess) e = configure_epi<EPI_GEGLU>();
    if (e == cudaSuccess) e = configure_epi<EPI_GELU_MUL>();
    if (e == cudaSuccess) e = configure_epi<EPI_RESIDUAL>();
    if (e == cudaSuccess) e = configure_epi<EPI_GEGLU_QUICK>();
    if (e == cudaSuccess) e = configure_epi<EPI_CLAMP_F32>();
    if (e == cudaSuccess) e = configure_epi<EPI_CLAMP_F16>();
    if (e == cudaSuccess) e = configure_epi<EPI_CLAMP_SILU>();
    if (e == cudaSuccess) e = configure_epi<EPI_GLU>();
    if (e == cudaSuccess) e = configure_epi<EPI_QKV>();
    return e;
}

// Co-resident clusters of `csize` CTAs per device and kernel, measured once (persistent
// cluster grids larger than this would run in waves).
static std::mutex g_cluster_mu;
static std::map<std::tuple<int, const void*, int>, int> g_cluster_cap;

static int max_clusters(const void* kern, int csize, int threads, int smem, int num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_tuple(dev, kern, csize);
    {
        std::lock_guard<std::mutex> g(g_cluster_mu);
        auto it = g_cluster_cap.find(key);
        if (it != g_cluster_cap.end()) return it->second;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(csize * (num_sms / csize)));
    cfg.blockDim = dim3(unsigned(threads));
    cfg.dynamicSmemBytes = size_t(smem);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = unsigned(csize);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = num_sms / csize;
    }
    std::lock_guard<std::mutex> g(g_cluster_mu);
    g_cluster_cap[key] = n;
    return n;
}

template <int EPI, bool Q8, bool PAIR, int BN = kBN>
static cudaError_t launch_t(const GemmLaunch& g, cudaStream_t stream) {
    constexpr bool RES = EPI == EPI_RESIDUAL;
    using L = GemmLayout<BN, Q8, PAIR, RES>;
    auto kern = k_gemm<BN, EPI, Q8, PAIR>;
    GemmParams p{};
    p.M = g.m_rows;
    p.N = g.w->N;
    p.K = g.w->K;
    p.out = g.out;
    p.ldo = g.ldo;
    p.aux = epi_is_clamp(EPI) ? g.bias : g.aux;
    p.ldaux = g.ldaux;
    p.err = g.err;
    p.lo1 = g.clamp_lo;
    p.hi1 = g.clamp_hi;
    p.lo2 = g.act_lo;
    p.hi2 = g.act_hi;
    if (EPI == EPI_QKV) {
        if (!g.positions || !g.rope || !g.q_norm || !g.k_norm || g.heads <= 0 || g.kv_heads <= 0 ||
            g.w->N != (g.heads + 2 * g.kv_heads) * BN || g.ntok > g.m_rows)
            return cudaErrorInvalidValue;
        p.pos = g.positions;
        p.rope = g.rope;
        p.qw = g.q_norm;
        p.kw = g.k_norm;
        p.ntok = g.ntok;
        p.heads = g.heads;
        p.kvh = g.kv_heads;
        p.eps = g.eps;
    }
    // Weight boxes: kBN rows (map_f16, map_q8) or kBN / 2 rows (CTA pairs, 128-wide tiles);
    // the pieces of split tail tiles use kBN / 2 rows, or kBN / 4 for the GeGLU gate and up halves.
    const CUtensorMap& mb = Q8 ? g.w->map_q8 : ((PAIR || BN != kBN) ? g.w->map_f16_half : g.w->map_f16);
    p.split_from = 1 << 30;
    p.split = 1;
    const CUtensorMap* mp = &g.w->map_f16_half;
    CUtensorMap mc;
    EpiMaps em;
    if (RES) {
        // mapC is the residual stream (fp32, boxes of 32 rows x 32 columns, loaded and stored).
        const int csize = g.w->N / BN;
        if (!g.x || !g.w_post || g.w->N % BN || csize > L::kMaxCluster) return cudaErrorInvalidValue;
        p.w_post = g.w_post;
        p.w_next = g.w_next;
        p.scale = g.scale;
        p.eps = g.eps;
        p.store_h = g.w_next && g.h16;
        p.store_y = g.w_next && g.y32;
        if (!encode_2d(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.x, uint64_t(g.w->N), uint64_t(g.m_rows), 32, 32,
                       CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        em.h = mc;
        em.y = mc;
        if (p.store_h && !encode_2d(&em.h, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, g.h16, uint64_t(g.w->N),
                                    uint64_t(g.m_rows), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        if (p.store_y && !encode_2d(&em.y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.y32, uint64_t(g.w->N),
                                    uint64_t(g.m_rows), 32, 32, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        const int row_blocks = g.m_rows / BM;
        const int cap = max_clusters(reinterpret_cast<const void*>(kern), csize, L::kThreads, L::kBytes, g.num_sms);
        const int clusters = row_blocks < cap ? row_blocks : cap;
        return launch_kernel(kern, dim3(csize * clusters), dim3(L::kThreads), L::kBytes, stream, csize, g.a->map, mb,
                             g.w->map_scales, *mp, mc, em, p);
    }
    // Output map: boxes of 32 rows x 128 bytes (32 fp32 or 64 fp16 columns), 128-byte swizzle.
    const bool f32 = EPI == EPI_F32 || EPI == EPI_CLAMP_F32;
    const int out_cols = epi_is_geglu(EPI) ? g.w->N / 2 : g.w->N;
    if (g.ldo < out_cols) return cudaErrorInvalidValue;
    if (!encode_2d(&mc, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, f32 ? 4 : 2, g.out,
                   uint64_t(g.ldo), uint64_t(g.m_rows), f32 ? 32 : 64, 32, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    em.h = mc;
    em.y = mc;
    if (!PAIR) {
        const int tiles = (g.m_rows / BM) * (g.w->N / BN);
        int grid = tiles < g.num_sms ? tiles : g.num_sms;
        // Split tiles (fp16 weights on 256-wide single-CTA tiles only).  With F full rounds of
        // `grid` tiles and R < grid tiles left, the R tiles run as 2R half-width pieces when those
        // fit in one round (2R <= grid), so the last round takes half a tile's time.  When every
        // tile fits in one round, each tile runs as S pieces, S the largest power of two with
        // S * tiles <= SMs, up to the narrowest piece the epilogue stores (32 fp32 columns, 64
        // fp16 columns, 64 GeGLU output columns).
        p.split_from = tiles;
        if (!Q8 && BN == kBN && EPI != EPI_QKV && g.mode == GEMM_SPLIT) {
            const bool f32 = EPI == EPI_F32 || EPI == EPI_CLAMP_F32;
            const int max_split = epi_is_geglu(EPI) ? 2 : f32 ? 8 : 4;
            if (tiles > grid) {
                const int full = tiles / grid * grid, rest = tiles - full;
                if (rest > 0 && 2 * rest <= grid) {
                    p.split_from = full;
                    p.split = 2;
                }
            } else {
                int sp = 1;
                while (sp < max_split && tiles * sp * 2 <= g.num_sms) sp *= 2;
                if (sp > 1) {
                    p.split_from = 0;
                    p.split = sp;
                    grid = tiles * sp;
                }
            }
            // the B box of one piece: BN / S rows, or BN / 2S for the GeGLU gate and up halves
            const int box = epi_is_geglu(EPI) ? BN / (2 * p.split) : BN / p.split;
            mp = box == BN / 2 ? &g.w->map_f16_half : box == BN / 4 ? &g.w->map_f16_quarter : &g.w->map_f16_eighth;
        }
        return launch_kernel(kern, dim3(grid), dim3(L::kThreads), L::kBytes, stream, 1, g.a->map, mb, g.w->map_scales,
                             *mp, mc, em, p);
    }
    // CTA pairs: clusters of 2, each pair looping over 256-row tiles.
    const int tiles = ((g.m_rows + 2 * BM - 1) / (2 * BM)) * (g.w->N / BN);
    const int cap = max_clusters(reinterpret_cast<const void*>(kern), 2, L::kThreads, L::kBytes, g.num_sms);
    const int pairs = tiles < cap ? tiles : cap;
    return launch_kernel(kern, dim3(2 * pairs), dim3(L::kThreads), L::kBytes, stream, 2, g.a->map, mb, g.w->map_scales,
                         *mp, mc, em, p);
}

template <int EPI>
static cudaError_t launch_epi(const GemmLaunch& g, cudaStream_t stream, bool q8, bool pair, bool narrow) {
    if (q8) return launch_t<EPI, true, false>(g, stream);
    if constexpr (EPI == EPI_RESIDUAL) {
        return launch_t<EPI, false, false>(g, stream);
    } else {
        if (pair) return launch_t<EPI, false, true>(g, stream);
        if constexpr (!epi_is_geglu(EPI) && EPI != EPI_QKV)
            if (narrow) return launch_t<EPI, false, false, 128>(g, stream);
        return launch_t<EPI, false, false>(g, stream);
    }
}

cudaError_t launch_gemm(const GemmLaunch& g, cudaStream_t stream) {
    if (g.m_rows <= 0) return cudaSuccess;
    // The Q8 path needs the Q8 planes; weights without them always take the fp16 path.
    if (!g.w->f16 && !g.w->q8) return cudaErrorInvalidValue;
    const bool q8 = g.w->q8 && (g.use_q8 || !g.w->f16);
    // CTA pairs run 128-deep K stages.  Under AUTO they take large batches: a pair streams half
    // the operand bytes per MMA of a single CTA and issues one instruction per 256 x 256 x 16
    // product, but below two rounds of pair tiles single CTAs spread the work over more SMs.
    const int pair_tiles = ((g.m_rows + 2 * BM - 1) / (2 * BM)) * (g.w->N / kBN);
    // The last pair tile's second CTA may lie wholly past m_rows (loads there read zeros and its
    // stores are clipped), so an epilogue that reads per-row inputs for every row (GELU_MUL's
    // aux) and the residual clusters stay on single CTAs.  QKV reads positions only for rows
    // below ntok <= m_rows.
    const bool pair_ok = !q8 && g.w->K % (2 * BK) == 0 && g.w->N % kBN == 0 && g.epilogue != EPI_RESIDUAL &&
                         g.epilogue != EPI_GELU_MUL;
    const bool pair = pair_ok && (g.mode == GEMM_PAIR || (g.mode == GEMM_AUTO && pair_tiles >= g.num_sms));
    // 128-wide tiles read each A tile twice as often; measured slower on every forward shape,
    // so they run only when asked for (or when N is a multiple of 128 but not of 256).
    const bool narrow = !q8 && !pair && !epi_is_geglu(g.epilogue) &&
                        (g.mode == GEMM_NARROW || (g.w->N % kBN && g.w->N % (kBN / 2) == 0 && g.mode == GEMM_AUTO));
    if (g.m_rows % BM || g.w->N % (narrow ? kBN / 2 : kBN) || g.w->K % BK || g.a->cols != g.w->K ||
        g.a->rows < g.m_rows)
        return cudaErrorInvalidValue;
    switch (g.epilogue) {
    case EPI_F32: return launch_epi<EPI_F32>(g, stream, q8, pair, narrow);
    case EPI_F16: return launch_epi<EPI_F16>(g, stream, q8, pair, narrow);
    case EPI_GEGLU: return launch_epi<EPI_GEGLU>(g, stream, q8, pair, narrow);
    case EPI_GELU_MUL: return launch_epi<EPI_GELU_MUL>(g, stream, q8, pair, narrow);
    case EPI_GEGLU_QUICK: return launch_epi<EPI_GEGLU_QUICK>(g, stream, q8, pair, narrow);
    case EPI_CLAMP_F32: return launch_epi<EPI_CLAMP_F32>(g, stream, q8, pair, narrow);
    case EPI_CLAMP_F16: return launch_epi<EPI_CLAMP_F16>(g, stream, q8, pair, narrow);
    case EPI_CLAMP_SILU: return launch_epi<EPI_CLAMP_SILU>(g, stream, q8, pair, narrow);
    case EPI_GLU: return launch_epi<EPI_GLU>(g, stream, q8, pair, narrow);
    case EPI_QKV:
        if (narrow || g.mode == GEMM_NARROW) return cudaErrorInvalidValue;
        return launch_epi<EPI_QKV>(g, stream, q8, pair, false);
    case EPI_RESIDUAL:
        if (g.mode == GEMM_PAIR || g.mode == GEMM_NARROW) return cudaErrorInvalidValue;
        return launch_epi<EPI_RESIDUAL>(g, stream, q8, false, false);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace ge
