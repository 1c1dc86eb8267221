// hf_gemm.cu -- tcgen05 grouped GEMM over expert segments (prefill path).
//
// Replaces, for segments with many tokens, the per-token GEMVs of expertFFNRaw
// (model/glm_forward.cpp:434-449); the reference has no batched or
// tensor-core code at all.
//
// Orientation ("swap AB"): the MMA's M = 128 rows of an expert weight matrix,
// N = the segment's tokens (up to BN per tile, rounded up to 16 at run time),
// K = hidden (gate/up) or intermediate (down). Both operands are K-major, so
// the reference's [gate | up | down] row-major weights feed the tensor cores
// unchanged: one TMA box of 64 elements x 128 rows per weight matrix and
// k-block, and boxes of 64 x 16 token rows for the activations.
//
//   GEMM1  acc_g = Wg x^T, acc_u = Wu x^T (two TMEM accumulators, BF16 x
//          BF16); epilogue mid = g / (1 + exp(-g)) * u in fp32, stored as one
//          FP16 plane holding mid * 2^-6 when the layer's down blocks are FP16
//          (hf_weights.cu), else as a BF16 hi + lo pair (hi = bf16(mid),
//          lo = bf16(mid - hi)), so the next GEMM sees 11 or ~16 mantissa
//          bits instead of BF16's 8.
//   GEMM2  acc = Wd mid^T: one FP16 x FP16 pass (the accumulator scaled back
//          by the powers of two), or Wd mid_hi^T + Wd mid_lo^T with BF16;
//          epilogue stores the expert outputs y[position][h] -- one FP16
//          plane holding y * 2^-4 on a forward with no GEMV segment, else
//          fp32 -- for the deterministic combine (or, for an expert-parallel
//          receiver, into the row of its source's output slab).
//
// CTA = 10 warps, one CTA (or one CTA of a pair) per SM, persistent over the
// tile list: warp 0 issues TMA loads into a STAGES-deep shared-memory ring,
// warp 1 owns TMEM and issues tcgen05.mma from one thread, warps 2-9 drain the
// TMEM accumulators (two warps per lane quadrant). Every wait is bounded (see
// hf_sm100.cuh): on timeout the CTA drains its TMA loads and MMAs, frees TMEM
// and reports HF_ERR_TIMEOUT through the error word instead of hanging.
#include <algorithm>
#include <map>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "hf_internal.cuh"
#include "hf_sm100.cuh"

namespace hf {

using namespace sm100;

// warp 0: TMA producer, warp 1: MMA issuer and TMEM owner, warps 2-9: epilogue
// (two per TMEM lane quadrant, alternating 32-column chunks: the SwiGLU of a
// 256-token tile kept four warps busy long enough to stall the next tile's MMAs)
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kBoxRowsB = 16;
constexpr uint32_t kTileABytes = 128 * 64 * 2;  // 128 rows x 64 bf16
constexpr uint64_t kDrainNs = 500ull * 1000 * 1000;
constexpr int kTileQ = 8;        // tile ids in flight from the producer to the MMA / epilogue
constexpr int kBarBytes = 512;   // barriers, tile queue, TMEM slot, abort flag

// PAIR: a cluster of two CTAs computes a 256-row tile with cta_group::2 MMAs;
// each CTA then holds its own 128 weight rows per A tile and half of the BN
// token rows, so it loads half the activation bytes of a one-CTA tile.
template <int NUM_A, int NUM_B, int BN, bool PAIR = false>
struct GemmCfg {
    static constexpr int kBRows = PAIR ? BN / 2 : BN;  // token rows of B per CTA
    static constexpr int kStageBytes = NUM_A * kTileABytes + NUM_B * kBRows * 128;
    static constexpr int kStages0 = (220 * 1024) / kStageBytes;
    static constexpr int kStages = kStages0 > 12 ? 12 : kStages0;
    static constexpr int kAccCols = NUM_A * BN;
    // two accumulator buffers (epilogue of tile i overlaps MMAs of tile i+1)
    // when they fit in the 512 TMEM columns, else one
    static constexpr int kBufs = 2 * kAccCols <= 512 ? 2 : 1;
    static constexpr int kCols0 = kBufs * kAccCols;
    static constexpr uint32_t kTmemCols = kCols0 <= 32 ? 32 : kCols0 <= 64 ? 64 : kCols0 <= 128 ? 128
                                          : kCols0 <= 256 ? 256 : 512;
    static constexpr int kBarOff = kStages * kStageBytes;
    static constexpr int kSmem = 1024 + kBarOff + kBarBytes;
    static_assert(kCols0 <= 512, "TMEM holds 512 columns");
    static_assert(kStages >= 3, "pipeline needs at least 3 stages");
    static_assert((2 * kStages + 6 + 2 * kTileQ) * 8 + kTileQ * 4 + 8 <= kBarBytes,
                  "barrier area overflow");
    static_assert(kStageBytes % 1024 == 0, "stage must keep 1024-byte alignment");
    static_assert(!PAIR || BN % 32 == 0, "pair tiles: BN/2 in 16-row boxes");
};

struct TileInfo {
    int g;             // group (expert) of the tile
    int seg, n0, n, m0, mvalid;
    int kb0, kb1;      // K blocks [kb0, kb1) of this tile (split-K runs)
    int rowA0, rowA1;
    long long yoff;    // split-K partial plane of the output
    bool shared;
};

// The three plan arrays a tile decode reads (tile prefix, counts, offsets),
// staged in shared memory at kernel start when they fit, else read in place.
struct PlanView {
    const int32_t* pref;
    const int32_t* cnt;
    const int32_t* off;
};

// PAIR: the kernel runs on CTA pairs (a down tile then spans 512 rows). This is
// the kernel's own shape, not GemmArgs::pair, which marks the pass.
template <bool PAIR>
__device__ __forceinline__ void decode_tile(const GemmArgs& a, const PlanView& p, int u,
                                            TileInfo& t) {
    int ks = 0;
    if (a.nsplit > 1) {  // K-split runs of one output tile are adjacent tile ids
        ks = u % a.nsplit;
        u /= a.nsplit;
    }
    const int G = a.pl.G;
    const int g = find_group(p.pref, G, u);
    const int c = p.cnt[g];
    const int nt = (c + a.bn - 1) / a.bn;
    const int local = u - p.pref[g];
    const int mi = local / nt, ni = local % nt;
    t.g = g;
    t.shared = (g == G - 1);
    const int Ig = t.shared ? a.Is : a.I;
    t.seg = p.off[g];
    // the segment's nt token tiles get equal widths (ceil(c / nt) <= bn), so
    // the CTAs that stream the same weight rows for them progress at the same
    // rate and the later reads of those rows hit L2
    const int nw = (c + nt - 1) / nt;
    t.n0 = ni * nw;
    t.n = min(nw, c - t.n0);
    t.m0 = mi * a.mrows;
    // routed experts: one [gate|up|down] block per expert in one view; the
    // shared expert: separate gate, up and down views
    if (a.which == 1) {
        const int base = g * 3 * a.I;
        t.rowA0 = t.shared ? t.m0 : base + t.m0;
        t.rowA1 = t.shared ? t.m0 : base + Ig + t.m0;
        t.mvalid = Ig - t.m0;
        t.kb1 = (a.H + 63) / 64;
    } else {  // down rows; a second accumulator takes the next 128 rows (256 on a pair)
        t.rowA0 = t.shared ? t.m0 : g * 3 * a.H + 2 * a.H + t.m0;
        t.rowA1 = t.rowA0 + (PAIR ? 256 : 128);
        t.mvalid = a.H - t.m0;
        t.kb1 = (Ig + 63) / 64;
    }
    t.kb0 = 0;
    t.yoff = 0;
    if (a.nsplit > 1) {  // the launcher sizes nsplit so that no run is empty
        t.kb0 = ks * a.kbper;
        t.kb1 = min(t.kb1, t.kb0 + a.kbper);
        t.yoff = ks * a.split_stride;
    }
}

__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity) {
    const uint64_t dl = globaltimer() + kDrainNs;
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() > dl) return false;
    return true;
}

// Kernel body. One CTA (PAIR = false) or one CTA of a pair (PAIR = true; rank
// 0 is the leader: it takes tile ids, arms the stage barriers and issues the
// MMAs for both; both CTAs load their halves and run their own epilogue).
template <int NUM_A, int NUM_B, int BN, bool PAIR>
__device__ __forceinline__ void gemm_body(const CUtensorMap& tmA, const CUtensorMap& tmA_sh,
                                          const CUtensorMap& tmA_sh2, const CUtensorMap& tmB0,
                                          const CUtensorMap& tmB1, const CUtensorMap& tmB0_sh,
                                          const CUtensorMap& tmB1_sh, const GemmArgs& a) {
    using C = GemmCfg<NUM_A, NUM_B, BN, PAIR>;
    constexpr int S = C::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;
    uint64_t* tempty = tfull + 2;
    uint64_t* final_bar = tempty + 2;
    uint64_t* stall_bar = final_bar + 1;  // never signalled (test hook)
    uint64_t* tq_full = stall_bar + 1;    // tile queue: producer -> MMA + epilogue
    uint64_t* tq_empty = tq_full + kTileQ;
    int* tile_q = reinterpret_cast<int*>(tq_empty + kTileQ);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_q + kTileQ);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    const bool leader = rank == 0;
    const int row_off = int(rank) * 128;  // this CTA's weight rows inside a pair tile
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    const int G = a.pl.G;
    int total;
    PlanView pv;
    if (!a.plan) {  // one group of dense_T rows: tile prefix, count and offset in shared memory
        int32_t* sp = reinterpret_cast<int32_t*>(smem + C::kBarOff + kBarBytes);
        const int rows_out = a.which == 1 ? a.Is : a.H;
        total = ((a.dense_T + a.bn - 1) / a.bn) * ((rows_out + a.mrows - 1) / a.mrows);
        if (threadIdx.x == 0) {
            sp[0] = 0;
            sp[1] = total;
            sp[2] = a.dense_T;
            sp[3] = 0;
        }
        pv = PlanView{sp, sp + 2, sp + 3};
    } else {
        const int32_t* pref_g = a.plan + (a.which == 1 ? a.pl.g1 : a.pl.g2);
        total = pref_g[G];
        pv = PlanView{pref_g, a.plan + a.pl.counts, a.plan + a.pl.offsets};
        if (a.plan_smem) {
            int32_t* sp = reinterpret_cast<int32_t*>(smem + C::kBarOff + kBarBytes);
            for (int i = threadIdx.x; i <= G; i += blockDim.x) sp[i] = pref_g[i];
            for (int i = threadIdx.x; i < G; i += blockDim.x) {
                sp[G + 1 + i] = a.plan[a.pl.counts + i];
                sp[2 * G + 1 + i] = a.plan[a.pl.offsets + i];
            }
            pv = PlanView{sp, sp + G + 1, sp + 2 * G + 1};
        }
    }
    if (a.nsplit > 1) total *= a.nsplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            // epilogue warps of this CTA (and the peer)
            mbar_init(&tempty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);
        }
        mbar_init(final_bar, 1);
        mbar_init(stall_bar, 1);
        for (int q = 0; q < kTileQ; ++q) {
            mbar_init(&tq_full[q], 1);
            // MMA thread + 4 epilogue warps (+ the peer's producer and 4 epilogue warps)
            mbar_init(&tq_empty[q], PAIR ? 2 * (1 + kEpiWarps) : 1 + kEpiWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, C::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, C::kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // waits: barriers that the peer CTA (or its TMA / MMA completions) arrive
    // on are waited on with cluster-scope acquire
    auto wait = [&](uint64_t* bar, uint32_t parity) {
        return PAIR ? mbar_wait_cl(bar, parity, abort_flag, deadline)
                    : mbar_wait(bar, parity, abort_flag, deadline);
    };

    if (warp == 0 && lane == 0) {
        // ---------------------------------------------------------- TMA producer
        // Tiles are taken from a global counter in launch order, so tiles that
        // share weight rows (a segment's token tiles, adjacent ids) start
        // together on different SMs; each id goes to the MMA thread and the
        // epilogue (and the peer CTA) through the shared-memory tile queue.
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB0);
        uint32_t it = 0, qi = 0;
        bool ok = true;
        int u = leader ? atomicAdd(a.sched, 1) : 0;
        while (true) {
            const uint32_t q = qi % kTileQ;
            if (leader) {
                if (!wait(&tq_empty[q], ((qi / kTileQ) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                tile_q[q] = u;
                mbar_arrive(&tq_full[q]);
                if constexpr (PAIR) {
                    st_cluster_u32(cluster_addr(&tile_q[q], 1), uint32_t(u));
                    mbar_arrive_remote(cluster_addr(&tq_full[q], 1));
                }
            } else {
                if (!wait(&tq_full[q], (qi / kTileQ) & 1)) {
                    ok = false;
                    break;
                }
                u = tile_q[q];
                mbar_arrive_remote(cluster_addr(&tq_empty[q], 0));
            }
            ++qi;
            if (u >= total) break;
            const int u_next = leader ? atomicAdd(a.sched, 1) : 0;
            TileInfo t;
            decode_tile<PAIR>(a, pv, u, t);
            u = u_next;
            // token rows of B this CTA loads: all of the tile (one CTA) or its
            // half of the MMA's N (pair; N rounded up to 32)
            const int half = PAIR ? ((t.n + 31) & ~31) / 2 : 0;
            // rows of one activation box (the launcher checks box <= kBRows);
            // a last box may reach past the tile: those rows are loaded (or
            // zero-filled past the tensor) but not read by the MMA
            const int box = a.box_b > 0 ? a.box_b : kBoxRowsB;
            const int nb = PAIR ? (half + box - 1) / box : (t.n + box - 1) / box;
            const int brow0 = t.seg + t.n0 + (PAIR ? int(rank) * half : 0);
            const uint32_t bytes = (NUM_A * kTileABytes + NUM_B * nb * (box * 128)) * (PAIR ? 2 : 1);
            const CUtensorMap* mA = t.shared ? &tmA_sh : &tmA;
            const CUtensorMap* mA1 = (t.shared && a.which == 1) ? &tmA_sh2 : mA;
            const CUtensorMap* mB0 = (a.which == 2 && t.shared) ? &tmB0_sh : &tmB0;
            const CUtensorMap* mB1 = (a.which == 2 && t.shared) ? &tmB1_sh : &tmB1;
            const int rA0 = t.rowA0 + (PAIR ? row_off : 0);
            const int rA1 = PAIR ? t.rowA1 + row_off : t.rowA1;
            for (int kb = t.kb0; kb < t.kb1; ++kb, ++it) {
                const uint32_t s = it % S, ph = (it / S) & 1;
                if (!wait(&empty[s], ph ^ 1)) {
                    ok = false;
                    break;
                }
                uint8_t* st = smem + s * C::kStageBytes;
                uint8_t* sb = st + NUM_A * kTileABytes;
                if constexpr (PAIR) {
                    const uint32_t fb = cluster_addr(&full[s], 0);
                    if (leader) mbar_arrive_expect_tx(&full[s], bytes);
                    tma_load_2d_pair(st, mA, fb, kb * 64, rA0);
                    if (NUM_A == 2) tma_load_2d_pair(st + kTileABytes, mA1, fb, kb * 64, rA1);
                    for (int j = 0; j < nb; ++j) {
                        const int row = brow0 + j * box;
                        tma_load_2d_pair(sb + j * (box * 128), mB0, fb, kb * 64, row);
                        if (NUM_B == 2)
                            tma_load_2d_pair(sb + C::kBRows * 128 + j * (box * 128), mB1, fb,
                                             kb * 64, row);
                    }
                } else {
                    mbar_arrive_expect_tx(&full[s], bytes);
                    tma_load_2d(st, mA, &full[s], kb * 64, rA0);
                    if (NUM_A == 2) tma_load_2d(st + kTileABytes, mA1, &full[s], kb * 64, rA1);
                    for (int j = 0; j < nb; ++j) {
                        const int row = brow0 + j * box;
                        tma_load_2d(sb + j * (box * 128), mB0, &full[s], kb * 64, row);
                        if (NUM_B == 2)
                            tma_load_2d(sb + BN * 128 + j * (box * 128), mB1, &full[s],
                                        kb * 64, row);
                    }
                }
            }
            if (!ok) break;
        }
        if (!ok && leader) {  // drain: let every issued load land before the CTA exits
            const uint32_t first = it > uint32_t(S) ? it - S : 0;
            for (uint32_t i = first; i < it; ++i) drain_wait(&full[i % S], (i / S) & 1);
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ---------------------------------------------------------- MMA issuer
        uint32_t it = 0, lt = 0, qi = 0;
        bool ok = true;
        if (a.test_stall) ok = mbar_wait(stall_bar, 0, abort_flag, deadline);
        for (; ok; ++lt) {
            const uint32_t q = qi % kTileQ;
            if (!mbar_wait(&tq_full[q], (qi / kTileQ) & 1, abort_flag, deadline)) {
                ok = false;
                break;
            }
            const int u = tile_q[q];
            mbar_arrive(&tq_empty[q]);
            ++qi;
            if (u >= total) break;
            TileInfo t;
            decode_tile<PAIR>(a, pv, u, t);
            const uint32_t acc = lt % C::kBufs, aph = (lt / C::kBufs) & 1;
            if (!wait(&tempty[acc], aph ^ 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t nmma = PAIR ? uint32_t((t.n + 31) & ~31) : uint32_t((t.n + 15) & ~15);
            const bool f16 = a.down_f16 && a.which == 2;  // FP16 down rows x FP16 mid
            const uint32_t idesc = PAIR ? (f16 ? idesc_f16_m256(nmma) : idesc_bf16_m256(nmma))
                                        : (f16 ? idesc_f16_m128(nmma) : idesc_bf16_m128(nmma));
            const uint32_t d0 = tmem_base + acc * C::kAccCols;
            for (int kb = t.kb0; kb < t.kb1; ++kb, ++it) {
                const uint32_t s = it % S, ph = (it / S) & 1;
                if (!wait(&full[s], ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_u32(smem + s * C::kStageBytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                    for (int ai = 0; ai < NUM_A; ++ai) {
                        const uint64_t ad = desc_k_sw128(st + ai * kTileABytes) + 2 * kk;
#pragma unroll
                        for (int bi = 0; bi < NUM_B; ++bi) {
                            const uint64_t bd = desc_k_sw128(st + NUM_A * kTileABytes +
                                                             bi * C::kBRows * 128) +
                                                2 * kk;
                            const uint32_t accum = (kb != t.kb0 || kk || bi);
                            if constexpr (PAIR) mma_bf16_pair(d0 + ai * BN, ad, bd, idesc, accum);
                            else mma_bf16(d0 + ai * BN, ad, bd, idesc, accum);
                        }
                    }
                }
                if constexpr (PAIR) {  // the stage is free in both CTAs
                    mma_commit_pair(smem_u32(&empty[s]));
                    mma_commit_pair(cluster_addr(&empty[s], 1));
                } else {
                    mma_commit(&empty[s]);
                }
            }
            if (!ok) break;
            if constexpr (PAIR) {
                mma_commit_pair(smem_u32(&tfull[acc]));
                mma_commit_pair(cluster_addr(&tfull[acc], 1));
            } else {
                mma_commit(&tfull[acc]);
            }
        }
        // completes once every MMA issued above is done
        if constexpr (PAIR) mma_commit_pair(smem_u32(final_bar));
        else mma_commit(final_bar);
        drain_wait(final_bar, 0);
    } else if (warp >= 2) {
        // ---------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int r = q * 32 + lane;
        uint32_t lt = 0, qi = 0;
        for (;; ++lt) {
            const uint32_t qs = qi % kTileQ;
            if (!wait(&tq_full[qs], (qi / kTileQ) & 1)) break;
            const int u = tile_q[qs];
            __syncwarp();
            if (lane == 0) {
                if (leader) mbar_arrive(&tq_empty[qs]);
                else mbar_arrive_remote(cluster_addr(&tq_empty[qs], 0));
            }
            ++qi;
            if (u >= total) break;
            TileInfo t;
            decode_tile<PAIR>(a, pv, u, t);
            const uint32_t acc = lt % C::kBufs, aph = (lt / C::kBufs) & 1;
            if (!wait(&tfull[acc], aph)) break;
            tc_fence_after();
            const uint32_t ta = tmem_base + (uint32_t(q * 32) << 16) + acc * C::kAccCols;
            const int rr = r + (PAIR ? row_off : 0);  // weight row inside the tile
            const bool rv = rr < t.mvalid;
            // second down row block: the next 128 rows on one CTA; on a pair (a
            // 512-row tile) the second 256-row MMA block, this CTA's half of it
            constexpr int kRow1 = PAIR ? 256 : 128;
            const bool rv1 = rr + kRow1 < t.mvalid;
            // TMEM is read 16 columns at a time, one load in flight while the
            // previous one is processed (a load's latency, not its bandwidth,
            // bounds a drain that waits for each load before using it); the two
            // warps of a quadrant take alternate 16-column chunks
            constexpr int CW = 16;
            auto process = [&](int c0, const uint32_t (&v0)[CW], const uint32_t (&v1)[CW]) {
                if (NUM_A == 2 && a.which == 1) {  // gate/up pair -> SwiGLU -> mid planes
                    if (rv && a.down_f16) {
                        // one FP16 plane: mid * 2^-kMidF16Shift (exact scaling, one
                        // rounding); columns j and j + 1 share one packed conversion
                        // (a conversion per value bounded the epilogue)
                        const size_t o0 = size_t(t.seg + t.n0 + c0) * a.Imax + t.m0 + rr;
                        __half* ph = reinterpret_cast<__half*>(a.mid_hi) + o0;
                        constexpr float kDown = 1.0f / float(1 << kMidF16Shift);
                        float mx = 0.0f;
#pragma unroll
                        for (int j = 0; j < CW; j += 2) {
                            if (c0 + j < t.n) {
                                const bool two = c0 + j + 1 < t.n;
                                const float m0 = __fmul_rn(
                                    swiglu_fast(__uint_as_float(v0[j]), __uint_as_float(v1[j])), kDown);
                                const float m1 =
                                    two ? __fmul_rn(swiglu_fast(__uint_as_float(v0[j + 1]),
                                                                __uint_as_float(v1[j + 1])),
                                                    kDown)
                                        : 0.0f;
                                mx = fmaxf(mx, fmaxf(fabsf(m0), fabsf(m1)));
                                const __half2 h = __floats2half2_rn(m0, m1);
                                ph[size_t(j) * a.Imax] = __low2half(h);
                                if (two) ph[size_t(j + 1) * a.Imax] = __high2half(h);
                            }
                        }
                        // beyond the FP16 range (Inf included): HF_ERR_RANGE
                        if (mx > 65504.0f) atomicOr(a.err, 8);
                    } else if (rv) {
                        // column c0 of this row in both planes; one row of mid per column
                        const size_t o0 = size_t(t.seg + t.n0 + c0) * a.Imax + t.m0 + rr;
                        __nv_bfloat16* ph = reinterpret_cast<__nv_bfloat16*>(a.mid_hi) + o0;
                        __nv_bfloat16* pl = reinterpret_cast<__nv_bfloat16*>(a.mid_lo) + o0;
#pragma unroll
                        for (int j = 0; j < CW; ++j) {
                            if (c0 + j < t.n) {
                                const float m =
                                    swiglu_fast(__uint_as_float(v0[j]), __uint_as_float(v1[j]));
                                const __nv_bfloat16 hi = __float2bfloat16_rn(m);
                                ph[size_t(j) * a.Imax] = hi;
                                pl[size_t(j) * a.Imax] =
                                    __float2bfloat16_rn(__fsub_rn(m, __bfloat162float(hi)));
                            }
                        }
                    }
                } else if (!a.resid) {  // down rows m0 + r (and m0 + 128 + r) -> fp32 outputs
                    // FP16 pass: the product carries 2^S (weights) and 2^-6 (mid); both
                    // powers of two, so undoing them is exact
                    const float sc = (a.which == 2 && a.down_f16)
                                         ? a.groups[t.g].down_scale * float(1 << kMidF16Shift)
                                         : 1.0f;
                    if (a.y16) {
                        // one FP16 plane: y * 2^-kYF16Shift (folded into the exact
                        // power-of-two scale, so one rounding). Columns j and j + 1
                        // convert together (one packed conversion for two values);
                        // an output beyond the plane's range is HF_ERR_RANGE
                        const float sc16 = sc * (1.0f / float(1 << kYF16Shift));
                        float mx = 0.0f;
                        auto row = [&](int col) {
                            const size_t pos = size_t(t.seg + t.n0 + col);
                            return (a.yrow ? reinterpret_cast<__half*>(a.yrow[pos])
                                           : reinterpret_cast<__half*>(a.y) + t.yoff + pos * a.H) +
                                   t.m0 + rr;
                        };
#pragma unroll
                        for (int j = 0; j < CW; j += 2) {
                            const int col = c0 + j;
                            if (col < t.n) {
                                const bool two = col + 1 < t.n;
                                __half* y0 = row(col);
                                __half* y1 = two ? row(col + 1) : y0;
#pragma unroll
                                for (int b = 0; b < NUM_A; ++b) {
                                    if (b == 0 ? !rv : !rv1) continue;
                                    const uint32_t(&v)[CW] = b == 0 ? v0 : v1;
                                    const float m0 = __fmul_rn(__uint_as_float(v[j]), sc16);
                                    const float m1 =
                                        two ? __fmul_rn(__uint_as_float(v[j + 1]), sc16) : 0.0f;
                                    mx = fmaxf(mx, fmaxf(fabsf(m0), fabsf(m1)));
                                    const __half2 h = __floats2half2_rn(m0, m1);
                                    const int ro = b == 0 ? 0 : kRow1;
                                    y0[ro] = __low2half(h);
                                    if (two) y1[ro] = __high2half(h);
                                }
                            }
                        }
                        if (mx > 65504.0f) atomicOr(a.err, 8);
                    } else {
#pragma unroll
                        for (int j = 0; j < CW; ++j) {
                            const int col = c0 + j;
                            if (col < t.n) {
                                const size_t pos = size_t(t.seg + t.n0 + col);
                                float* yr =
                                    (a.yrow ? a.yrow[pos] : a.y + t.yoff + pos * a.H) + t.m0 + rr;
                                if (rv) yr[0] = __fmul_rn(__uint_as_float(v0[j]), sc);
                                if (NUM_A == 2 && rv1)
                                    yr[kRow1] = __fmul_rn(__uint_as_float(v1[j]), sc);
                            }
                        }
                    }
                } else {  // residual block (dense MLP): y = resid + down row; the thread
                          // reads, then writes, its own elements, 8 columns of loads in flight
#pragma unroll
                    for (int j0 = 0; j0 < CW; j0 += 8) {
                        float q0[8], q1[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int col = c0 + j0 + j;
                            const size_t yi = size_t(t.seg + t.n0 + col) * a.H + t.m0 + rr;
                            q0[j] = (col < t.n && rv) ? a.resid[yi] : 0.f;
                            q1[j] = (NUM_A == 2 && col < t.n && rv1) ? a.resid[yi + kRow1] : 0.f;
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int col = c0 + j0 + j;
                            if (col < t.n) {
                                float* yr = a.y + size_t(t.seg + t.n0 + col) * a.H + t.m0 + rr;
                                if (rv) yr[0] = __fadd_rn(q0[j], __uint_as_float(v0[j0 + j]));
                                if (NUM_A == 2 && rv1)
                                    yr[kRow1] = __fadd_rn(q1[j], __uint_as_float(v1[j0 + j]));
                            }
                        }
                    }
                }
            };
            uint32_t a0[CW], a1[CW], b0[CW], b1[CW];
#pragma unroll
            for (int j = 0; j < CW; ++j) a1[j] = b1[j] = 0u;  // untouched when NUM_A == 1
            int c0 = ((warp - 2) / 4) * CW;
            if (c0 < t.n) {
                tmem_ld16(ta + c0, a0);
                if constexpr (NUM_A == 2) tmem_ld16(ta + BN + c0, a1);
            }
            tmem_ld_wait_regs(a0, a1);
            while (c0 < t.n) {
                const int c1 = c0 + 2 * CW;
                if (c1 < t.n) {
                    tmem_ld16(ta + c1, b0);
                    if constexpr (NUM_A == 2) tmem_ld16(ta + BN + c1, b1);
                }
                process(c0, a0, a1);
                tmem_ld_wait_regs(b0, b1);
                if (c1 >= t.n) break;
                const int c2 = c1 + 2 * CW;
                if (c2 < t.n) {
                    tmem_ld16(ta + c2, a0);
                    if constexpr (NUM_A == 2) tmem_ld16(ta + BN + c2, a1);
                }
                process(c1, b0, b1);
                tmem_ld_wait_regs(a0, a1);
                c0 = c2;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) mbar_arrive(&tempty[acc]);
                else mbar_arrive_remote(cluster_addr(&tempty[acc], 0));
            }
        }
    }
    __syncwarp();  // reconverge warps 0 and 1 (one lane of each ran a role loop)
    if (a.sig_flags) __threadfence_system();  // this thread's output stores, system-wide
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // no remote arrive or TMEM write targets a finished CTA
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::kTmemCols);
        else tmem_dealloc(tmem_base, C::kTmemCols);
    }
    if (threadIdx.x == 0) {
        if (*abort_flag) atomicOr(a.err, 1);
        // the last CTA out resets the tile counter for the next launch (every
        // producer has taken its final id before its CTA gets here)
        __threadfence();
        if (atomicAdd(a.sched + 1, 1) == int(gridDim.x) - 1) {
            a.sched[0] = 0;
            a.sched[1] = 0;
            __threadfence();
            if (a.sig_flags) {  // every CTA's outputs are out: tell their owners
                __threadfence_system();
                for (int d = 0; d < a.sig_n; ++d) st_release_sys(a.sig_flags[d] + a.sig_slot, a.sig_seq);
            }
        }
    }
}

template <int NUM_A, int NUM_B, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_moe_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA_sh,
               const __grid_constant__ CUtensorMap tmA_sh2,
               const __grid_constant__ CUtensorMap tmB0, const __grid_constant__ CUtensorMap tmB1,
               const __grid_constant__ CUtensorMap tmB0_sh,
               const __grid_constant__ CUtensorMap tmB1_sh, GemmArgs a) {
    gemm_body<NUM_A, NUM_B, BN, false>(tmA, tmA_sh, tmA_sh2, tmB0, tmB1, tmB0_sh, tmB1_sh, a);
}

template <int NUM_A, int NUM_B, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    k_moe_gemm_pair(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmA_sh,
                    const __grid_constant__ CUtensorMap tmA_sh2,
                    const __grid_constant__ CUtensorMap tmB0,
                    const __grid_constant__ CUtensorMap tmB1,
                    const __grid_constant__ CUtensorMap tmB0_sh,
                    const __grid_constant__ CUtensorMap tmB1_sh, GemmArgs a) {
    gemm_body<NUM_A, NUM_B, BN, true>(tmA, tmA_sh, tmA_sh2, tmB0, tmB1, tmB0_sh, tmB1_sh, a);
}

// ============================================================ activation gather
// xp[pos] = x[token(perm[pos])] for every position of a GEMM segment, as BF16
// (hi plane) plus, for fp32 activations, the residual BF16 lo plane.
template <bool XF32>
__global__ void __launch_bounds__(256) k_gather_x(GatherArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int G = a.pl.G;
    const int total = a.plan[a.pl.offsets + G];
    const int32_t* g1 = a.plan + a.pl.g1;
    for (int p = warp; p < total; p += nw) {
        const int g = find_group(a.plan + a.pl.offsets, G, p);
        if (g1[g + 1] == g1[g]) continue;  // GEMV segment
        const int t = token_of_slot(a.perm[p], a.T, a.k);
        uint4* dh = reinterpret_cast<uint4*>(a.xp_hi + size_t(p) * a.H);
        if constexpr (XF32) {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) +
                                                                size_t(t) * a.H);
            uint4* dl = reinterpret_cast<uint4*>(a.xp_lo + size_t(p) * a.H);
            for (int c = lane; c < a.H / 8; c += 32) {
                const float4 u0 = __ldg(src + 2 * c), u1 = __ldg(src + 2 * c + 1);
                const float f[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                uint32_t h[4], l[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint16_t h0 = f32_to_bf16_rne(f[2 * q]), h1 = f32_to_bf16_rne(f[2 * q + 1]);
                    const uint16_t l0 = f32_to_bf16_rne(__fsub_rn(f[2 * q], bf16_to_f32(h0)));
                    const uint16_t l1 = f32_to_bf16_rne(__fsub_rn(f[2 * q + 1], bf16_to_f32(h1)));
                    h[q] = uint32_t(h0) | (uint32_t(h1) << 16);
                    l[q] = uint32_t(l0) | (uint32_t(l1) << 16);
                }
                dh[c] = make_uint4(h[0], h[1], h[2], h[3]);
                dl[c] = make_uint4(l[0], l[1], l[2], l[3]);
            }
        } else {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) +
                                                              size_t(t) * a.H);
            for (int c = lane; c < a.H / 8; c += 32) dh[c] = ld_nc_u4(src + c);
        }
    }
}

// Token-major form of the bf16 gather: a warp reads token t's row once and
// writes it to the positions of all of the token's slots (its k routed slots
// and its shared-expert slot) that belong to GEMM segments. Each row is read
// once instead of k + 1 times.
__global__ void __launch_bounds__(256) k_gather_tokens(GatherArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int G = a.pl.G;
    const int32_t* offs = a.plan + a.pl.offsets;
    const int32_t* g1 = a.plan + a.pl.g1;
    const int ns = a.k + (a.has_shared ? 1 : 0);  // <= 9
    const int row_vec = a.H / 8;
    for (int t = warp; t < a.T; t += nw) {
        // lane i < ns: the position of slot i of token t, or -1 (GEMV segment)
        int pos = -1;
        if (lane < ns) {
            const int slot = lane < a.k ? t * a.k + lane : a.T * a.k + t;
            const int p = a.slot_pos[slot];
            const int g = find_group(offs, G, p);
            pos = g1[g + 1] != g1[g] ? p : -1;
        }
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) +
                                                          size_t(t) * a.H);
        for (int c0 = lane; c0 < row_vec; c0 += 32 * 8) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c0 + 32 * u < row_vec) v[u] = ld_nc_u4(src + c0 + 32 * u);
            for (int i = 0; i < ns; ++i) {
                const int p = __shfl_sync(0xffffffffu, pos, i);
                if (p < 0) continue;
                uint4* dst = reinterpret_cast<uint4*>(a.xp_hi + size_t(p) * a.H);
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (c0 + 32 * u < row_vec) dst[c0 + 32 * u] = v[u];
            }
        }
    }
}

// ============================================================ host launchers
// Grid of a pair kernel: two CTAs per cluster that can be resident at once
// (an odd SM left in a GPC cannot host a pair), at most `want`.
static int pair_grid(const void* kern, int smem, int want) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> cache;  // (kernel, device) -> CTAs
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({kern, dev});
    if (it == cache.end()) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(unsigned(want & ~1));
        cfg.blockDim = dim3(kGemmThreads);
        cfg.dynamicSmemBytes = size_t(smem);
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
            cudaGetLastError();
            clusters = want / 2;
        }
        it = cache.emplace(std::make_pair(kern, dev), 2 * clusters).first;
    }
    return std::max(2, std::min(want & ~1, it->second));
}

template <int NUM_A, int NUM_B, int BN, bool PAIR = false>
static hf_status launch_one(const GemmMaps& m, const GemmArgs& a, int grid, cudaStream_t st) {
    using C = GemmCfg<NUM_A, NUM_B, BN, PAIR>;
    auto kern = [] {
        if constexpr (PAIR) return k_moe_gemm_pair<NUM_A, NUM_B, BN>;
        else return k_moe_gemm<NUM_A, NUM_B, BN>;
    }();
    GemmArgs args = a;
    const int plan_bytes = ((3 * a.pl.G + 1) * 4 + 15) & ~15;
    int smem = C::kSmem;
    args.plan_smem = (C::kSmem + plan_bytes) <= 227 * 1024;
    if (args.plan_smem) smem += plan_bytes;
    else if (!a.plan) return fail(HF_ERR_ARG, "plan-free GEMM needs its shared-memory plan slot");
    if (!a.sched) return fail(HF_ERR_ARG, "GEMM launch without a tile-scheduler counter");
    // an activation box must fit this CTA's B region of a stage, and the wide
    // boxes only come with the pair tiles' wide maps
    if (a.box_b != 0 && a.box_b != kBoxRowsB &&
        !(PAIR && a.box_b == kPairBoxB && C::kBRows >= kPairBoxB))
        return fail(HF_ERR_ARG, "GEMM activation box does not fit the tile");
    HF_CUDA(ensure_smem(reinterpret_cast<const void*>(kern), smem));
    if (PAIR) grid = pair_grid(reinterpret_cast<const void*>(kern), smem, grid);
    kern<<<grid, kGemmThreads, smem, st>>>(m.A, m.A_sh, m.A_sh2, m.B0, m.B1, m.B0_sh, m.B1_sh, args);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

hf_status launch_gemm(const GemmMaps& m, const GemmArgs& a, int num_b, int grid, cudaStream_t st) {
    if (a.pair && a.which == 2 && a.mrows == 512) {
        // prefill down: 512-row tiles on CTA pairs (two 256-row MMA blocks);
        // one mid plane on the FP16 pass, hi + lo on the BF16 one
        if (num_b == 2) {
            if (a.bn == 128) return launch_one<2, 2, 128, true>(m, a, grid, st);
            if (a.bn == 256) return launch_one<2, 2, 256, true>(m, a, grid, st);
        } else {
            if (a.bn == 128) return launch_one<2, 1, 128, true>(m, a, grid, st);
            if (a.bn == 256) return launch_one<2, 1, 256, true>(m, a, grid, st);
        }
    }
    if (a.pair && a.which == 1) {  // prefill gate/up: 256-row tiles on CTA pairs
        if (a.bn == 128 && a.mrows == 256)
            return num_b == 1 ? launch_one<2, 1, 128, true>(m, a, grid, st)
                              : launch_one<2, 2, 128, true>(m, a, grid, st);
        if (a.bn == 256 && a.mrows == 256)  // 128 tokens per CTA; one TMEM buffer
            return num_b == 1 ? launch_one<2, 1, 256, true>(m, a, grid, st)
                              : launch_one<2, 2, 256, true>(m, a, grid, st);
        return fail(HF_ERR_ARG, "unsupported pair GEMM tile");
    }
    if (a.which == 1) {
        if (a.bn == 32) return num_b == 1 ? launch_one<2, 1, 32>(m, a, grid, st)
                                          : launch_one<2, 2, 32>(m, a, grid, st);
        if (a.bn == 64) return num_b == 1 ? launch_one<2, 1, 64>(m, a, grid, st)
                                          : launch_one<2, 2, 64>(m, a, grid, st);
        if (a.bn == 128) return num_b == 1 ? launch_one<2, 1, 128>(m, a, grid, st)
                                           : launch_one<2, 2, 128>(m, a, grid, st);
    } else if (num_b == 1) {  // single-plane B: router logits (bf16) or the FP16 down pass
        if (a.mrows == 256) {
            if (a.bn == 16) return launch_one<2, 1, 16>(m, a, grid, st);
            if (a.bn == 32) return launch_one<2, 1, 32>(m, a, grid, st);
            if (a.bn == 64) return launch_one<2, 1, 64>(m, a, grid, st);
            if (a.bn == 128) return launch_one<2, 1, 128>(m, a, grid, st);
        } else if (a.mrows == 128) {
            if (a.bn == 16) return launch_one<1, 1, 16>(m, a, grid, st);
            if (a.bn == 32) return launch_one<1, 1, 32>(m, a, grid, st);
            if (a.bn == 64) return launch_one<1, 1, 64>(m, a, grid, st);
            if (a.bn == 128) return launch_one<1, 1, 128>(m, a, grid, st);
        }
    } else if (a.mrows == 256) {
        if (a.bn == 16) return launch_one<2, 2, 16>(m, a, grid, st);
        if (a.bn == 128) return launch_one<2, 2, 128>(m, a, grid, st);
    } else if (a.mrows == 128) {
        if (a.bn == 16) return launch_one<1, 2, 16>(m, a, grid, st);
        if (a.bn == 32) return launch_one<1, 2, 32>(m, a, grid, st);
        if (a.bn == 64) return launch_one<1, 2, 64>(m, a, grid, st);
        if (a.bn == 128) return launch_one<1, 2, 128>(m, a, grid, st);
    }
    return fail(HF_ERR_ARG, "unsupported GEMM token tile");
}

hf_status launch_gather(const GatherArgs& a, int x_f32, cudaStream_t st) {
    const int grid = num_sms(a.device) * 4;
    if (x_f32) k_gather_x<true><<<grid, 256, 0, st>>>(a);
    else if (a.slot_pos && a.k > 1 && a.k <= kMaxTopK) k_gather_tokens<<<grid, 256, 0, st>>>(a);
    else k_gather_x<false><<<grid, 256, 0, st>>>(a);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

// ------------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D BF16 view: `rows` rows of `cols` elements, `pitch` elements apart;
// box of 64 elements x box_rows rows, 128-byte swizzle, OOB reads as zero.
hf_status make_map_bf16(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                        uint64_t pitch, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(HF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch * 2) % 16)
        return fail(HF_ERR_ARG, "tensor map base/pitch not 16-byte aligned");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {pitch * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(HF_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return HF_OK;
}


}  // namespace hf
