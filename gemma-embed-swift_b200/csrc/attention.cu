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
#include <algorithm>
#include <vector>

#include "kernels.hpp"
#include "ptx.cuh"

namespace ge {

// ---------------------------------------------------------------------------------------
// Tensor-core kernel (head dim 256 or 512), persistent: CTA c walks its own range of work
// items, assigned on the host longest-processing-time first by key blocks.  An item is T tokens
// of one sequence with the G query heads that share one KV head (G = H / KV): row t * G + g of
// its Q tile is token t0 + t, head kh * G + g (one 3-D TMA box per 64 dims), so each K and V
// tile serves all G heads and a short sequence fills its tile with heads instead of padding.
// Head dim 256: T = 128 / G, and O is the whole head (256 fp32 columns of tensor memory).
// Head dim 512: O would need all 512 columns, so an item computes one half of the head's output
// dims (the item's `half`, two items per token block) with S over all 512 dims; T = 64 / G, so
// the Q tile (64 rows x 512 dims) fits the 64 KB that 128 x 256 takes.  Its eight 64-dim chunks
// lie 8 KB apart, and the 128-row MMA reads rows 64..127 of chunk c from chunk c + 1 (the last
// from the K ring): those S rows are masked and never stored.  A key block's K arrives as two
// 256-dim halves through the 2-slot K ring, so the next block's first half loads while the
// second half's MMAs run.
//   warp 0      TMA producer: per item the Q tile, once both S issuers have read the previous
//               one, then K and V tiles of 64 keys into 2-slot rings that run on from item to
//               item, K and V on independent cursors (each load as soon as its slot is free)
//   warps 1, 2  S issuers (warp 1 also owns tensor memory): S_j = Q K_j^T (128 x 64, fp32 in
//               TMEM, two buffers); head dim 256: warp 1 the even global key blocks and warp 2
//               the odd ones, each through its own K-ring slot (one thread issues a tcgen05.mma
//               about every 90 cycles, as long as a 128 x 64 x 16 product runs); head dim 512:
//               warp 1 alone.  A buffer takes block j + 2 once every softmax thread holds block
//               j's scores.
//   warp 3      PV issuer: O += P_j V_j (128 x 256, fp32 in TMEM, P read from TMEM); an
//               item's first PV runs as two 128-column halves, each once the epilogue warps
//               have read that half of the previous item's O
//   warps 4-11  softmax, two threads per row (one per 32-key half of a block; warps w and
//               w + 4 share a tensor-memory lane quarter): mask S_j, exchange the row's block
//               maximum through shared memory, keep running maximum and partial sums, write
//               their half of P_j (fp16 pairs) to tensor memory, and rescale their half of O in
//               tensor memory only when the row maximum grows by more than kRescale; until then
//               every term of the row uses the same stale maximum, so the result is exact.
//               At an item's end each thread leaves its half sum in shared memory and goes on
//               with the next item's first block.
//   warps 12-15 O epilogue, one warp per lane quarter: once an item's last PV has completed,
//               O / l of the live rows, staged through shared memory into coalesced stores, so
//               the next item's softmax overlaps the previous item's epilogue.
// Tensor memory: O in columns [0, 256), the S buffers in [256, 320) and [320, 384), the P
// buffers in [384, 416) and [416, 448).
constexpr int kTcQ = 128;
constexpr int kTcKeys = 64;
constexpr int kTcHd = 256;  // output dims per item (the head dim, or half of a 512-dim head) and K-ring slot width
constexpr float kRescale = 8.0f;  // log2 units: a stale maximum may leave P up to 2^8
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kQBytes = kTcQ * kTcHd * 2;     // 64 KB: 4 chunks of [128 rows][64 dims]
constexpr int kKVBytes = kTcKeys * kTcHd * 2; // 32 KB per stage: 4 chunks of [64 keys][64 dims]
constexpr int kPBytes = kTcQ * kTcKeys * 2;   // 16 KB: [128 rows][64 keys] fp16, two of them (see kOffStg)
constexpr int kOffK = kQBytes;
constexpr int kOffV = kOffK + 2 * kKVBytes;
constexpr int kOffP = kOffV + 2 * kKVBytes;
constexpr int kOffRed = kOffP + 2 * kPBytes;    // [2 halves][128 rows] floats: row maxima
constexpr int kOffBar = kOffRed + 2 * kTcQ * 4;
// The P region is free since P moved to tensor memory: the epilogue warps' staging tiles
// ([4 warps][32 rows][128 B]) and the row sums the softmax hands them ([2 item parities][2
// halves][128 rows] floats).
constexpr int kOffStg = kOffP;
constexpr int kOffL = kOffP + 4 * 32 * 128;
constexpr int kTcSmem = kOffBar + 256 + 1024;
constexpr int kTcThreads = 512;
constexpr int kSWarpB = 2;     // the second S issuer
constexpr int kPVWarp = 3;     // the PV issuer
constexpr int kSoftWarp0 = 4;  // softmax warps 4-11
constexpr int kEpiWarp0 = 12;  // O epilogue warps 12-15
constexpr uint32_t kPollNs = 64;  // producer and issuer poll interval
constexpr uint32_t kTmemO = 0, kTmemS = 256, kTmemP = 384;

struct TcAttnParams {
    const uint4* work;       // (sequence start, sequence length, first token, KV head), grouped by CTA
    const uint32_t* offset;  // CTA c's items are [offset[c], offset[c + 1])
    __half* out;
    int heads, group, tokens, hw;  // G = heads / KV heads, T = tokens per item = 128 / G
    int* err;
};

__device__ __forceinline__ void drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (!mbar_test(bar, parity) && globaltimer() - t0 < kWaitLimitNs) {
    }
}

// Key blocks of an item: the whole sequence, or the window of all its tokens
// (Attention.metal:66-74), starting on a multiple of kTcKeys from the sequence start.
__device__ __forceinline__ void item_keys(const uint4& w, const TcAttnParams& p, int& k_start, int& nblk) {
    const int len = int(w.y), t0 = int(w.z);
    int ks = 0, ke = len;
    if (p.hw > 0) {
        ks = max(t0 - p.hw, 0);
        ke = min(t0 + p.tokens - 1 + p.hw + 1, len);
    }
    k_start = ks / kTcKeys * kTcKeys;
    nblk = (ke - k_start + kTcKeys - 1) / kTcKeys;
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads, 1) k_attention_tc(const __grid_constant__ CUtensorMap mapQ,
                                                          const __grid_constant__ CUtensorMap mapK,
                                                          const __grid_constant__ CUtensorMap mapV, TcAttnParams p) {
    static_assert(HD == 256 || HD == 512, "head dim 256 or 512");
    constexpr int kChunks = HD / 64;              // 64-dim chunks of Q and K
    constexpr int kHalves = HD / kTcHd;           // K-ring slots per key block
    constexpr int kQChunk = kQBytes / kChunks;    // bytes between Q chunks: 128 or 64 rows x 128 bytes
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* q_full = bars;
    uint64_t* q_empty = bars + 1;
    uint64_t* k_full = bars + 2;
    uint64_t* k_empty = bars + 4;
    uint64_t* v_full = bars + 6;
    uint64_t* v_empty = bars + 8;
    uint64_t* s_full = bars + 10;
    uint64_t* p_full = bars + 12;
    uint64_t* pv_done = bars + 14;
    uint64_t* o_empty = bars + 16;  // columns [0, 128) of O read out (and bars + 25: [128, 256))
    uint64_t* s_free = bars + 17;  // S buffer read into registers by every softmax thread
    uint64_t* o_full = bars + 19;  // an item's last PV has completed
    uint64_t* l_full = bars + 20;  // an item's row sums are in shared memory (by item parity)
    uint64_t* l_empty = bars + 22; // and have been read by the epilogue warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
    uint64_t* o_empty_hi = bars + 25;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int live_rows = p.group * p.tokens;
    const uint32_t q_bytes = uint32_t(kChunks * 128 * live_rows);  // kChunks boxes of live_rows x 128 bytes

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 2);  // both S issuers sign off each Q tile
        for (int i = 0; i < 2; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 256);
            mbar_init(&pv_done[i], 1);
        }
        mbar_init(o_empty, 128);
        mbar_init(o_empty_hi, 128);
        mbar_init(o_full, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&s_free[i], 256);
            mbar_init(&l_full[i], 256);
            mbar_init(&l_empty[i], 128);
        }
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
    // Rows [live_rows, rows per chunk) of the Q chunks are never loaded: zeroed once, their
    // scores stay finite, so the softmax can treat them as unmasked rows (never stored).
    {
        constexpr int kChunkRows = kQChunk / 128;
        const int dead = kChunkRows - live_rows;
        for (int i = threadIdx.x; i < kChunks * dead * 8; i += kTcThreads) {
            const int c = i / (dead * 8), rr = live_rows + (i / 8) % dead, q = i % 8;
            *reinterpret_cast<uint4*>(smem + c * kQChunk + rr * 128 + q * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // q, k, v come from the previous kernel; the set-up above overlapped its tail

    if (warp == 0) {
        // ---------------------------------------------------------- TMA producer
        // Two cursors walk the CTA's items: Q and K tiles (each item's Q, then its K tiles), and
        // V tiles.  Each load is issued as soon as its ring slot is free, so a K tile never
        // waits behind a V tile whose slot is still being read, or the other way round.
        if (lane == 0) {
            const int it_end = int(p.offset[blockIdx.x + 1]);
            int issued_q = 0, issued_k = 0, issued_v = 0;
            // K cursor: item kit (local index kli), block kj of nk, half kh; global half gk.
            int kit = int(p.offset[blockIdx.x]), kli = 0, kj = 0, kh = 0, gk = 0, nk = 0, ks = 0;
            bool q_done = false;
            // V cursor: item vit, block vj of nv; global block gv.
            int vit = int(p.offset[blockIdx.x]), vj = 0, gv = 0, nv = 0, vs = 0;
            if (vit < it_end) item_keys(p.work[vit], p, vs, nv);
            uint64_t idle_since = globaltimer();
            bool ok = true;
            while (ok && (kit < it_end || vit < it_end)) {
                bool moved = false;
                if (kit < it_end) {
                    const uint4 w = p.work[kit];
                    const int kvh = int(w.w & 0xffffu);
                    if (!q_done) {
                        if (mbar_poll(q_empty, uint32_t(kli & 1) ^ 1u)) {
                            mbar_expect_tx(q_full, q_bytes);
                            for (int c = 0; c < kChunks; c++)
                                tma_load_3d(smem + c * kQChunk, &mapQ, q_full, c * 64, kvh * p.group, int(w.x + w.z));
                            issued_q++;
                            q_done = true;
                            item_keys(w, p, ks, nk);
                            moved = true;
                        }
                    } else {
                        const int bk = gk & 1;
                        if (mbar_poll(&k_empty[bk], uint32_t((gk >> 1) & 1) ^ 1u)) {
                            mbar_expect_tx(&k_full[bk], kKVBytes);
                            const int row = int(w.x) + ks + kj * kTcKeys;
                            for (int c = 0; c < 4; c++)
                                tma_load_2d(smem + kOffK + bk * kKVBytes + c * (kKVBytes / 4), &mapK, &k_full[bk],
                                            kvh * HD + kh * kTcHd + c * 64, row);
                            issued_k++;
                            gk++;
                            moved = true;
                            if (++kh == kHalves) {
                                kh = 0;
                                if (++kj == nk) {
                                    kj = 0;
                                    kit++;
                                    kli++;
                                    q_done = false;
                                }
                            }
                        }
                    }
                }
                if (vit < it_end) {
                    const int b = gv & 1;
                    if (mbar_poll(&v_empty[b], uint32_t((gv >> 1) & 1) ^ 1u)) {
                        const uint4 w = p.work[vit];
                        const int kvh = int(w.w & 0xffffu), hv = int(w.w >> 16);  // KV head, output half
                        mbar_expect_tx(&v_full[b], kKVBytes);
                        const int row = int(w.x) + vs + vj * kTcKeys;
                        for (int c = 0; c < 4; c++)
                            tma_load_2d(smem + kOffV + b * kKVBytes + c * (kKVBytes / 4), &mapV, &v_full[b],
                                        kvh * HD + hv * kTcHd + c * 64, row);
                        issued_v++;
                        gv++;
                        moved = true;
                        if (++vj == nv) {
                            vj = 0;
                            if (++vit < it_end) item_keys(p.work[vit], p, vs, nv);
                        }
                    }
                }
                if (moved) {
                    idle_since = globaltimer();
                } else {
                    // Nothing to issue yet: back off, and give up like a bounded wait would.
                    __nanosleep(kPollNs);
                    if (*reinterpret_cast<volatile int*>(p.err) != 0) {
                        ok = false;
                    } else if (globaltimer() - idle_since > kWaitLimitNs) {
                        atomicCAS(p.err, 0, kErrTimeout);
                        ok = false;
                    }
                }
            }
            pdl_launch();  // this CTA's loads are all issued: the next kernel may be scheduled
            // Every issued load lands before the CTA exits, also after an error.
            if (issued_q > 0) drain(q_full, uint32_t((issued_q - 1) & 1));
            for (int b = 0; b < 2; b++) {
                const int ck = issued_k / 2 + (b < issued_k % 2 ? 1 : 0);
                const int cv = issued_v / 2 + (b < issued_v % 2 ? 1 : 0);
                if (ck > 0) drain(&k_full[b], uint32_t((ck - 1) & 1));
                if (cv > 0) drain(&v_full[b], uint32_t((cv - 1) & 1));
            }
        }
    } else if (warp == 1 || warp == kSWarpB) {
        // ---------------------------------------------------------- S issuers
        // A tcgen05.mma takes its issuing thread about as long to issue as a 128 x 64 x 16
        // product takes the tensor core to run, so one thread cannot keep up with the S products
        // of 64-key blocks.  Head dim 256: warp 1 issues S for the even global blocks and warp
        // kSWarpB for the odd ones, each through its own K-ring slot (block g into S buffer
        // g & 1, the same chain of MMAs one issuer would run).  Head dim 512 takes both K-ring
        // slots per block, so warp 1 issues every block and warp kSWarpB only signs off Q tiles.
        if (lane == 0) {
            const int par = warp == 1 ? 0 : 1;
            const uint32_t id_s = idesc_f16(kTcQ, kTcKeys);  // K-major Q and K
            const uint32_t q_addr = smem_u32(smem);
            bool ok = true;
            int gb = 0;
            for (int it = int(p.offset[blockIdx.x]), li = 0; it < int(p.offset[blockIdx.x + 1]) && ok; it++, li++) {
                const uint4 w = p.work[it];
                int k_start, nblk;
                item_keys(w, p, k_start, nblk);
                // Every issuer waits for every Q tile, so neither runs a phase ahead of the other.
                if (!mbar_wait_sleep(q_full, uint32_t(li & 1), p.err, kPollNs)) break;
                bool used_q = false;
                for (int j = 0; j < nblk; j++, gb++) {
                    if (kHalves == 1 ? (gb & 1) != par : par != 0) continue;
                    const int b = gb & 1;
                    // S buffer b is free once every softmax thread holds block gb - 2's scores.
                    if (gb >= 2 && !mbar_wait_sleep(&s_free[b], uint32_t(((gb - 2) >> 1) & 1), p.err, kPollNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    used_q = true;
                    // S_gb = Q K_gb^T over every dim, one K-ring slot (256 dims) at a time
                    for (int hk = 0; hk < kHalves && ok; hk++) {
                        const int gk = gb * kHalves + hk, bk = gk & 1;
                        if (!mbar_wait_sleep(&k_full[bk], uint32_t((gk >> 1) & 1), p.err, kPollNs)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t ka = smem_u32(smem + kOffK + bk * kKVBytes);
#pragma unroll
                        for (int kk = 0; kk < kTcHd / 16; kk++) {
                            const int c = kk >> 2, wq = kk & 3;  // 64-dim chunk of the slot, 16-dim step inside it
                            const uint64_t ad = sw128_desc(q_addr + (hk * 4 + c) * kQChunk + wq * 32, 16, 1024);
                            const uint64_t bd = sw128_desc(ka + c * (kKVBytes / 4) + wq * 32, 16, 1024);
                            umma_f16(tmem + kTmemS + b * kTcKeys, ad, bd, id_s, (hk | kk) != 0);
                        }
                        umma_commit(&k_empty[bk]);
                    }
                    if (!ok) break;
                    umma_commit(&s_full[b]);
                }
                if (!ok) break;
                // Both issuers sign off each item's Q: after their S products have read it, or
                // at once when this issuer ran no block of the item.
                if (used_q)
                    umma_commit(q_empty);
                else
                    mbar_arrive(q_empty);
            }
        }
    } else if (warp == kPVWarp) {
        // ---------------------------------------------------------- PV issuer
        if (lane == 0) {
            const uint32_t id_o = idesc_f16(kTcQ, kTcHd, 0, 1);          // K-major P, MN-major V
            const uint32_t id_oh = idesc_f16(kTcQ, kTcHd / 2, 0, 1);     // one 128-column half of O
            bool ok = true;
            int gb = 0;
            for (int it = int(p.offset[blockIdx.x]), li = 0; it < int(p.offset[blockIdx.x + 1]) && ok; it++, li++) {
                const uint4 w = p.work[it];
                int k_start, nblk;
                item_keys(w, p, k_start, nblk);
                for (int j = 0; j < nblk; j++, gb++) {
                    const int b = gb & 1;
                    const uint32_t ph = uint32_t((gb >> 1) & 1);
                    if (!mbar_wait_sleep(&p_full[b], ph, p.err, kPollNs) || !mbar_wait_sleep(&v_full[b], ph, p.err, kPollNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t va = smem_u32(smem + kOffV + b * kKVBytes);
                    if (j == 0 && li > 0) {
                        // An item's first PV overwrites O in two 128-column halves, each once the
                        // epilogue warps have read that half of the previous item's O.
                        for (int hh = 0; hh < 2 && ok; hh++) {
                            if (!mbar_wait_sleep(hh ? o_empty_hi : o_empty, uint32_t((li - 1) & 1), p.err, kPollNs)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
#pragma unroll
                            for (int kk = 0; kk < kTcKeys / 16; kk++) {
                                const uint32_t pa = tmem + kTmemP + uint32_t(b * (kTcKeys / 2) + kk * 8);
                                // dims 128 hh .. 128 hh + 127: two 64-dim chunks of V on
                                const uint64_t bd = sw128_desc(va + hh * 2 * (kKVBytes / 4) + kk * 2048, kKVBytes / 4, 1024);
                                umma_f16_ta(tmem + kTmemO + uint32_t(hh * (kTcHd / 2)), pa, bd, id_oh, kk != 0);
                            }
                        }
                        if (!ok) break;
                    } else {
#pragma unroll
                        for (int kk = 0; kk < kTcKeys / 16; kk++) {
                            // P_b's keys 16 kk .. 16 kk + 15 from tensor memory
                            const uint32_t pa = tmem + kTmemP + uint32_t(b * (kTcKeys / 2) + kk * 8);
                            // V chunk of 64 dims = one [64 keys][128 B] box; 16 keys advance 2048 B.
                            const uint64_t bd = sw128_desc(va + kk * 2048, kKVBytes / 4, 1024);
                            umma_f16_ta(tmem + kTmemO, pa, bd, id_o, !(j == 0 && kk == 0));
                        }
                    }
                    umma_commit(&v_empty[b]);
                    umma_commit(&pv_done[b]);
                    if (j == nblk - 1) umma_commit(o_full);  // O of the item is complete
                }
            }
        }
    } else if (warp < kEpiWarp0) {
        // ---------------------------------------------------------- softmax (two threads per row)
        const int quad = warp & 3;                  // tensor-memory lane quarter of this warp
        const int half = (warp - kSoftWarp0) >> 2;  // which 32 keys of each block
        const int r = quad * 32 + lane;
        const int rt = r / p.group;  // token of this row within a tile (rows are token * G + head)
        const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
        float* red = reinterpret_cast<float*>(smem + kOffRed);
        // The two warps of a quarter meet on named barrier 1 + quad (64 threads).
        auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory"); };
        // `ok` stays warp-uniform, and after a failed wait the loops keep running without work,
        // so both warps of a quarter reach every named barrier and every tcgen05 load or store
        // is executed by a whole warp.
        bool ok = true;
        auto wait_all = [&](uint64_t* bar, uint32_t parity) {
            const bool w = ok && mbar_wait(bar, parity, p.err);
            ok = __all_sync(0xffffffffu, w);
        };
        float* lbuf = reinterpret_cast<float*>(smem + kOffL);
        int gb = 0;
        for (int it = int(p.offset[blockIdx.x]), li = 0; it < int(p.offset[blockIdx.x + 1]); it++, li++) {
            const uint4 w = p.work[it];
            int k_start, nblk;
            item_keys(w, p, k_start, nblk);
            const int len = int(w.y);
            const int qi = int(w.z) + rt;  // this row's token within its sequence
            // Keys this row sees: [row_lo, row_hi) of its sequence.  Rows past the item's G x T
            // see every key (their Q rows are zero and they are never stored): no per-key mask,
            // which would hold up their warps on every block.
            const bool dead = r >= live_rows;
            const int row_lo = dead ? 0 : p.hw > 0 ? max(qi - p.hw, 0) : 0;
            const int row_hi = dead ? (1 << 30) : p.hw > 0 ? min(qi + p.hw + 1, len) : len;
            float m_used = -INFINITY, l = 0.f;  // running maximum (log2 units) and this half's sum
            for (int j = 0; j < nblk; j++, gb++) {
                const int b = gb & 1;
                const uint32_t ph = uint32_t((gb >> 1) & 1);
                wait_all(&s_full[b], ph);
                uint32_t sr[32];
                float mh = -INFINITY;
                const int kb = k_start + j * kTcKeys + half * 32;
                if (ok) {
                    tc_fence_after();
                    tmem_ld32(lane_base + kTmemS + b * kTcKeys + half * 32, sr);
                    tmem_wait_ld();
                    tc_fence_before();
                    mbar_arrive(&s_free[b]);  // the S buffer may take block gb + 2
                    // Raw scores, masked keys at -inf; the maximum is taken on them and scaled once
                    // (x -> x log2e rounds monotonically), and p = 2^(s log2e - m) is one FFMA and
                    // one ex2 per key.
                    if (!(kb >= row_lo && kb + 32 <= row_hi)) {  // some key of this half is masked
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            const int kj = kb + i;
                            if (!(kj >= row_lo && kj < row_hi)) sr[i] = __float_as_uint(-INFINITY);
                        }
                    }
                    // Eight independent partial maxima instead of one 32-long dependency chain.
                    float mp[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) mp[i] = __uint_as_float(sr[i]);
#pragma unroll
                    for (int i = 8; i < 32; i++) mp[i & 7] = fmaxf(mp[i & 7], __uint_as_float(sr[i]));
                    mh = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
                    mh *= kLog2e;
                }
                // Row maximum of the block from both halves (the slot is rewritten only after the
                // next pair_sync, by which time the partner has read it).
                red[half * kTcQ + r] = mh;
                pair_sync();
                const float mb = fmaxf(mh, red[(1 - half) * kTcQ + r]);
                pair_sync();
                if (!ok) continue;
                // Rescale this half of O when the row's maximum grew past the threshold (both
                // halves decide alike; tensor-memory loads and stores are warp-collective).
                const bool grow = mb > m_used + kRescale && m_used != -INFINITY;
                if (__any_sync(0xffffffffu, grow)) {
                    const float alpha = grow ? ex2_approx(m_used - mb) : 1.0f;
                    if (j > 0) wait_all(&pv_done[(gb - 1) & 1], uint32_t(((gb - 1) >> 1) & 1));
                    if (!ok) continue;
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < kTcHd / 64; c++) {
                        uint32_t o[32];
                        const uint32_t col = kTmemO + uint32_t(half * (kTcHd / 2) + c * 32);
                        tmem_ld32(lane_base + col, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(lane_base + col, o);
                    }
                    tmem_wait_st();
                    if (grow) {
                        l *= alpha;
                        m_used = mb;
                    }
                }
                if (m_used == -INFINITY) m_used = mb;  // first block with a visible key (O and l are still 0)
                float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // independent partial sums
                const float mu = m_used == -INFINITY ? 0.f : m_used;
                uint32_t pk[16];  // this half's 32 probabilities as fp16 pairs
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * e]), kLog2e, -mu));  // 2^-inf = 0
                    const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * e + 1]), kLog2e, -mu));
                    ps[(2 * e) & 7] += p0;
                    ps[(2 * e + 1) & 7] += p1;
                    pk[e] = pack_half2(p0, p1);
                }
                // P goes to buffer b once the PV two blocks back, which read that buffer, has
                // completed (waited for after the exponentials, which do not need the buffer).
                if (gb >= 2) wait_all(&pv_done[b], uint32_t(((gb - 2) >> 1) & 1));
                if (!ok) continue;
                // This half's 16 columns of P buffer b in tensor memory (the PV product's A).
                tmem_st16(lane_base + kTmemP + uint32_t(b * (kTcKeys / 2) + half * 16), pk);
                l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&p_full[b]);
            }
            // ---- the row's half sum goes to the epilogue warps, which read O once the item's last
            // PV has completed; this warp goes on with the next item's first block.
            if (ok && li >= 2) wait_all(&l_empty[li & 1], uint32_t(((li - 2) >> 1) & 1));
            lbuf[(li & 1) * 2 * kTcQ + half * kTcQ + r] = l;
            mbar_arrive(&l_full[li & 1]);
        }
    } else {
        // ---------------------------------------------------------- O epilogue (one warp per lane quarter)
        // Per item: both halves' row sums, then O / l of the live rows once the item's last PV
        // has completed, 64 columns at a time: each thread writes its row's 128 bytes to the
        // warp's staging tile, then the warp stores 4 rows of 128 bytes per instruction.  O is
        // handed back for the next item's first PV after its last columns are in registers.
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
        const float* lbuf = reinterpret_cast<const float*>(smem + kOffL);
        uint8_t* stg = smem + kOffStg + quad * 32 * 128;
        bool ok = true;
        auto wait_all = [&](uint64_t* bar, uint32_t parity) {
            const bool w = ok && mbar_wait(bar, parity, p.err);
            ok = __all_sync(0xffffffffu, w);
        };
        for (int it = int(p.offset[blockIdx.x]), li = 0; it < int(p.offset[blockIdx.x + 1]); it++, li++) {
            const uint4 w = p.work[it];
            const int len = int(w.y);
            wait_all(&l_full[li & 1], uint32_t((li >> 1) & 1));
            // Half 0's sum plus half 1's (the order the two halves added them in before).
            const float lt = ok ? lbuf[(li & 1) * 2 * kTcQ + r] + lbuf[(li & 1) * 2 * kTcQ + kTcQ + r] : 0.f;
            mbar_arrive(&l_empty[li & 1]);
            wait_all(o_full, uint32_t(li & 1));
            if (!ok) {
                mbar_arrive(o_empty);
                mbar_arrive(o_empty_hi);
                continue;
            }
            tc_fence_after();
            const float inv = lt > 0.f ? 1.0f / lt : 0.f;
            // The output row (token x heads + head) of each of this lane's eight store slots (row
            // i * 4 + lane / 8 of the warp's 32), or -1 for a row past the item's tokens; the
            // lane stores 16 bytes at column 8 * (lane % 8) of each 64-column round.  The row
            // index fits 32 bits: the output holds tokens x heads x head-dim fp16 values, and
            // a batch's int32 token count times the heads stays far below 2^31 for any
            // workspace that fits a device.
            int orow[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int rr = quad * 32 + i * 4 + (lane >> 3);
                const int rrt = rr / p.group, rrg = rr - rrt * p.group;
                const int qr = int(w.z) + rrt;
                orow[i] = (rr < live_rows && qr < len) ? (int(w.x) + qr) * p.heads + int(w.w & 0xffffu) * p.group + rrg : -1;
            }
            __half* const ocol = p.out + int(w.w >> 16) * kTcHd + (lane & 7) * 8;
#pragma unroll 1
            for (int rd = 0; rd < kTcHd / 64; rd++) {
                uint32_t o[64];
                const uint32_t col = kTmemO + uint32_t(rd * 64);
                tmem_ld32(lane_base + col, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
                tmem_ld32(lane_base + col + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
                tmem_wait_ld();
                if (rd % 2 == 1) {  // a half of O is read: the next item's first PV may overwrite it
                    tc_fence_before();
                    mbar_arrive(rd == 1 ? o_empty : o_empty_hi);
                }
                uint8_t* srow = stg + lane * 128;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        __half2 hv = __floats2half2_rn(__uint_as_float(o[8 * j + 2 * e]) * inv,
                                                       __uint_as_float(o[8 * j + 2 * e + 1]) * inv);
                        pk[e] = *reinterpret_cast<uint32_t*>(&hv);
                    }
                    *reinterpret_cast<uint4*>(srow + ((j ^ (lane & 7)) * 16)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int lr = i * 4 + (lane >> 3), ch = lane & 7;
                    const uint4 val = *reinterpret_cast<const uint4*>(stg + lr * 128 + ((ch ^ (lr & 7)) * 16));
                    if (orow[i] >= 0) *reinterpret_cast<uint4*>(ocol + long(orow[i]) * HD + rd * 64) = val;
                }
                __syncwarp();
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

int build_attention_work(const uint32_t* sl, int nseq, int kvh, int group, int hw, int max_ctas, uint32_t* out,
                         int* ctas, int hd) {
    const int T = attention_tokens_per_item(group, hd);
    const int halves = hd == 512 ? 2 : 1;  // a 512-dim head's output dims in two items
    // The item count alone answers the size query the forward makes before filling.
    long count_items = 0;
    for (int s = 0; s < nseq; s++) count_items += (long(sl[2 * s + 1]) + T - 1) / T * (kvh * halves);
    const int n = int(count_items);
    const int grid = std::max(1, std::min(n, max_ctas));
    if (ctas) *ctas = n ? grid : 0;
    if (n == 0) return 0;
    const int words = 4 * n + grid + 1;
    if (!out) return words;
    // Built on every forward from the host, so the buffers are kept per thread.
    struct Item {
        uint32_t start, len, t0, kh;
        int cost;
    };
    struct Buffers {
        std::vector<Item> items;
        std::vector<int> order, owner, count, first;
        std::vector<long> load;       // per CTA, the sum of its items' costs
        std::vector<uint64_t> mask;   // per load value, the CTAs at that load
    };
    thread_local Buffers tls;
    Buffers& B = tls;  // one thread-local lookup
    auto& items = B.items;
    auto& order = B.order;
    auto& owner = B.owner;
    auto& count = B.count;
    auto& first = B.first;
    auto& load = B.load;
    auto& mask = B.mask;
    items.clear();
    int max_cost = 0;
    for (int s = 0; s < nseq; s++)
        for (uint32_t t0 = 0; t0 < sl[2 * s + 1]; t0 += uint32_t(T))
            for (int kh = 0; kh < kvh * halves; kh++) {
                const int len = int(sl[2 * s + 1]);
                int ks = 0, ke = len;
                if (hw > 0) {
                    ks = std::max(int(t0) - hw, 0);
                    ke = std::min(int(t0) + T - 1 + hw + 1, len);
                }
                ks = ks / kTcKeys * kTcKeys;
                // An item costs its key blocks plus about two blocks of set-up and epilogue.
                // KV head in the low 16 bits, output half of a 512-dim head in the high 16
                const uint32_t tag = uint32_t(kh / halves) | (uint32_t(kh % halves) << 16);
                const int cost = (ke - ks + kTcKeys - 1) / kTcKeys + 2;
                max_cost = std::max(max_cost, cost);
                items.push_back({sl[2 * s], sl[2 * s + 1], t0, tag, cost});
            }
    // Longest first, items of equal cost in the order they were made (a stable counting sort).
    first.assign(size_t(max_cost) + 2, 0);
    for (const Item& it : items) first[size_t(max_cost - it.cost) + 1]++;
    for (size_t c = 1; c < first.size(); c++) first[c] += first[c - 1];
    order.resize(size_t(n));
    for (int i = 0; i < n; i++) order[size_t(first[size_t(max_cost - items[size_t(i)].cost)]++)] = i;
    // Each item goes to the least-loaded CTA so far (lowest index on ties): deterministic.  The
    // loads are small integers that only grow, so the CTAs sit in buckets by load, a bitmask of
    // CTA indices each: the next CTA is the lowest bit of the lowest non-empty bucket.  No load
    // exceeds the total cost / grid + the largest cost (a CTA is chosen only while it is the
    // least loaded).
    long total = 0;
    for (const Item& it : items) total += it.cost;
    const int mw = (grid + 63) / 64;  // mask words per bucket
    const long nbuckets = total / grid + max_cost + 2;
    mask.assign(size_t(nbuckets) * size_t(mw), 0ull);
    for (int c = 0; c < grid; c++) mask[size_t(c >> 6)] |= 1ull << (c & 63);
    load.assign(size_t(grid), 0);
    owner.resize(size_t(n));
    count.assign(size_t(grid), 0);
    long lo = 0;  // the lowest bucket that may hold a CTA
    for (int i = 0; i < n; i++) {
        int c = -1;
        while (c < 0) {
            const uint64_t* m = &mask[size_t(lo) * size_t(mw)];
            for (int q = 0; q < mw && c < 0; q++)
                if (m[q]) c = q * 64 + __builtin_ctzll(m[q]);
            if (c < 0) lo++;
        }
        const int cost = items[size_t(order[size_t(i)])].cost;
        mask[size_t(lo) * size_t(mw) + size_t(c >> 6)] &= ~(1ull << (c & 63));
        load[size_t(c)] += cost;
        mask[size_t(load[size_t(c)]) * size_t(mw) + size_t(c >> 6)] |= 1ull << (c & 63);
        owner[size_t(i)] = c;
        count[size_t(c)]++;
    }
    uint32_t* off = out + 4 * size_t(n);
    off[0] = 0;
    for (int c = 0; c < grid; c++) off[c + 1] = off[c] + uint32_t(count[size_t(c)]);
    for (int c = 0; c < grid; c++) count[size_t(c)] = int(off[c]);  // next free slot of each CTA
    for (int i = 0; i < n; i++) {
        const Item& it = items[size_t(order[size_t(i)])];
        uint32_t* w = out + 4 * size_t(count[size_t(owner[size_t(i)])]++);
        w[0] = it.start;
        w[1] = it.len;
        w[2] = it.t0;
        w[3] = it.kh;
    }
    return words;
}

// Sets the shared-memory limits of the attention kernels on the current device; runs at
// load, before any stream capture.
cudaError_t configure_attention_kernels() {
    cudaError_t e = cudaFuncSetAttribute(k_attention_tc<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_attention_tc<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e == cudaSuccess) e = configure_attention64();
    return e;
}

template <int HD>
static cudaError_t launch_tc(const AttnLaunch& a, cudaStream_t stream) {
    const int group = a.heads / a.kv_heads;
    if (attention_tokens_per_item(group, HD) < 1) return cudaErrorInvalidValue;
    TcAttnParams p{reinterpret_cast<const uint4*>(a.work), a.work + 4 * size_t(a.sched_items), a.out, a.heads, group,
                   attention_tokens_per_item(group, HD), a.half_window, a.err};
    return launch_kernel(k_attention_tc<HD>, dim3(a.work_items), dim3(kTcThreads), kTcSmem, stream, 1, a.maps->q,
                         a.maps->k, a.maps->v, p);
}

// Q as [rows][heads][hd] with boxes of 64 dims x G heads x T tokens (one work item's tile,
// row t * G + g); K and V as [rows][kv_heads * hd] with boxes of 64 dims x 64 keys.
bool encode_attention_maps(AttnMaps& m, const __half* q, const __half* k, const __half* v, int rows, int heads, int kvh,
                           int hd, int row_stride) {
    if ((hd != 256 && hd != 512) || heads % kvh) return false;
    const int group = heads / kvh;
    if (attention_tokens_per_item(group, hd) < 1) return false;
    const uint64_t qs = row_stride ? uint64_t(row_stride) : uint64_t(heads) * hd;
    const uint64_t kvs = row_stride ? uint64_t(row_stride) : uint64_t(kvh) * hd;
    return encode_fp16_map_3d(&m.q, q, uint64_t(hd), uint64_t(heads), uint64_t(rows), 64, uint32_t(group),
                              uint32_t(attention_tokens_per_item(group, hd)), qs) &&
           encode_fp16_map(&m.k, k, uint64_t(kvh) * hd, rows, 64, kTcKeys, kvs) &&
           encode_fp16_map(&m.v, v, uint64_t(kvh) * hd, rows, 64, kTcKeys, kvs);
}

cudaError_t launch_attention(const AttnLaunch& a, cudaStream_t stream) {
    if (a.work_items <= 0) return cudaSuccess;
    if (a.heads % a.kv_heads) return cudaErrorInvalidValue;
    if (!a.maps) return cudaErrorInvalidValue;
    if (a.hd == 256) return launch_tc<256>(a, stream);
    if (a.hd == 512) return launch_tc<512>(a, stream);
    return cudaErrorInvalidValue;
}

}  // namespace ge
