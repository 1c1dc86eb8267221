// hf_route.cu -- router logits, noaux_tc top-k, canonical permutation, work plan.
//
// Reference: GLMForward::moeLayer router section (model/glm_forward.cpp:517-541)
// and topKScores (compute/moe_router.h:29-57). The permutation into per-expert
// segments and the work plan have no reference counterpart (the reference runs
// one token at a time and loops its 8 experts, glm_forward.cpp:581).
//
// Permutation: positions are ordered (group asc, token asc). Each block of 128
// tokens builds, per expert, a 128-bit mask of the tokens that picked it
// (atomicOr: order-independent). A slot's rank inside its segment is the
// popcount of the mask bits below its token, so the result is deterministic
// without sorting.
#include "hf_internal.cuh"
#include "hf_sm100.cuh"

#include <math.h>

namespace hf {

// ============================================================ router logits
// Small T: one block per router row, its 8 warps each own one K-slice. A lane
// keeps up to 4 16-byte chunks of its slice in registers and applies them to
// the tokens 8 at a time (24-32 activation loads in flight per lane), so the
// 3 MB router weight is read from HBM once and token latency overlaps.
constexpr int kRouterRowsPerBlock = 1;
constexpr int kRouterSlices = 8;
constexpr int kRouterMaxT = 64;
constexpr int kRouterRegChunks = 4;
constexpr int kRouterTokBatch = 8;

template <bool XF32>
__device__ __forceinline__ void load_x8(const void* x, size_t elem, float (&o)[8]) {
    if constexpr (XF32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + elem);
        float4 a = __ldg(p), b = __ldg(p + 1);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    } else {
        uint4 v = ld_nc_u4(static_cast<const uint16_t*>(x) + elem);
        unpack8(v, o);
    }
}

template <bool XF32>
__device__ __forceinline__ void router_rows(const RouteArgs& a) {
    __shared__ float part[kRouterSlices][kRouterRowsPerBlock][kRouterMaxT];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rloc = warp / kRouterSlices, slice = warp % kRouterSlices;
    const int row = blockIdx.x * kRouterRowsPerBlock + rloc;
    const int H = a.H, T = a.T;
    float* P = &part[slice][rloc][0];
    for (int t = lane; t < T; t += 32) P[t] = 0.0f;
    __syncwarp();
    if (row < a.E) {
        const int nchunk = H / 8;
        const int per = (nchunk + kRouterSlices - 1) / kRouterSlices;
        const int c0 = slice * per, c1 = min(nchunk, c0 + per);
        const uint16_t* wrow = a.router + size_t(row) * H;
        for (int cb = c0; cb < c1; cb += 32 * kRouterRegChunks) {
            uint4 wv[kRouterRegChunks];
#pragma unroll
            for (int j = 0; j < kRouterRegChunks; ++j) {
                const int c = cb + lane + 32 * j;
                wv[j] = (c < c1) ? ld_stream_u4(wrow + size_t(c) * 8) : make_uint4(0, 0, 0, 0);
            }
            // blocks start at different tokens so they do not all request the
            // same activation lines from L2 at the same time
            const int nbatch = (T + kRouterTokBatch - 1) / kRouterTokBatch;
            const int rot = int(blockIdx.x % unsigned(nbatch));
            for (int bi = 0; bi < nbatch; ++bi) {
                const int t0 = ((bi + rot) % nbatch) * kRouterTokBatch;
                float acc[kRouterTokBatch];
#pragma unroll
                for (int b = 0; b < kRouterTokBatch; ++b) acc[b] = 0.0f;
#pragma unroll
                for (int j = 0; j < kRouterRegChunks; ++j) {
                    const int c = cb + lane + 32 * j;
                    if (c < c1) {
                        float wf[8];
                        unpack8(wv[j], wf);
#pragma unroll
                        for (int b = 0; b < kRouterTokBatch; ++b) {
                            if (t0 + b < T) {
                                float xf[8];
                                load_x8<XF32>(a.x, size_t(t0 + b) * H + size_t(c) * 8, xf);
#pragma unroll
                                for (int q = 0; q < 8; ++q) acc[b] = fmaf(wf[q], xf[q], acc[b]);
                            }
                        }
                    }
                }
#pragma unroll
                for (int b = 0; b < kRouterTokBatch; ++b) {
                    const float s = warp_sum(acc[b]);
                    if (lane == 0 && t0 + b < T) P[t0 + b] += s;
                }
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kRouterRowsPerBlock * T; i += blockDim.x) {
        const int rl = i / T, t = i % T;
        const int r = blockIdx.x * kRouterRowsPerBlock + rl;
        if (r < a.E) {
            float s = part[0][rl][t];
#pragma unroll
            for (int q = 1; q < kRouterSlices; ++q) s += part[q][rl][t];
            a.logits[size_t(t) * a.E + r] = s;
        }
    }
}

template <bool XF32>
__global__ void __launch_bounds__(256) k_router_gemv(RouteArgs a) {
    router_rows<XF32>(a);
}

// Large T: 64 tokens x 64 experts per block, K in steps of 32, 4x4 per thread.
template <bool XF32>
__global__ void __launch_bounds__(256) k_router_tile(RouteArgs a) {
    __shared__ __align__(16) float xs[32][68];
    __shared__ __align__(16) float ws[32][68];
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * 64, e0 = blockIdx.y * 64;
    const int ty = tid / 16, tx = tid % 16;
    const int lr = tid / 4, lk = (tid % 4) * 8;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < a.H; k0 += 32) {
        float xv[8], wv[8];
        const int t = t0 + lr, e = e0 + lr, kk = k0 + lk;
        if (t < a.T && kk < a.H) load_x8<XF32>(a.x, size_t(t) * a.H + kk, xv);
        else
#pragma unroll
            for (int q = 0; q < 8; ++q) xv[q] = 0.0f;
        if (e < a.E && kk < a.H) unpack8(ld_nc_u4(a.router + size_t(e) * a.H + kk), wv);
        else
#pragma unroll
            for (int q = 0; q < 8; ++q) wv[q] = 0.0f;
        __syncthreads();
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            xs[lk + q][lr] = xv[q];
            ws[lk + q][lr] = wv[q];
        }
        __syncthreads();
#pragma unroll 8
        for (int q = 0; q < 32; ++q) {
            const float4 xa = *reinterpret_cast<const float4*>(&xs[q][ty * 4]);
            const float4 wb = *reinterpret_cast<const float4*>(&ws[q][tx * 4]);
            const float xr[4] = {xa.x, xa.y, xa.z, xa.w};
            const float wr[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xr[i], wr[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= a.T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + tx * 4 + j;
            if (e < a.E) a.logits[size_t(t) * a.E + e] = acc[i][j];
        }
    }
}

// ============================================================ top-k (one warp per token)
// compute/moe_router.h:29-57: rank by score + bias, descending; weights are
// the unbiased scores, divided by their rank-order fp32 sum when normTopkProb
// and that sum > 0, then multiplied by routedScalingFactor. Sigmoid as
// glm_forward.cpp:522-524. Ties go to the lower expert id.
template <int NPL>
__device__ __forceinline__ void topk_warp(const float* row, int planes, size_t pstride,
                                          int apply_sigmoid, const float* bias,
                                          int E, int k, float scale, int norm, int lane,
                                          int32_t* ids_out, float* w_out, float* margin_out,
                                          int32_t* ids_smem) {
    float v[NPL], s[NPL], lg[NPL];
#pragma unroll
    for (int j = 0; j < NPL; ++j) lg[j] = (j * 32 + lane < E) ? row[j * 32 + lane] : 0.0f;
    // split-K partial planes, summed in plane order (deterministic); four
    // planes x NPL experts of loads are issued before each group of adds
    for (int p = 1; p < planes; p += 4) {
        float b[4][NPL];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < NPL; ++j)
                b[i][j] = (p + i < planes && j * 32 + lane < E)
                              ? row[size_t(p + i) * pstride + j * 32 + lane] : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (p + i < planes)
#pragma unroll
                for (int j = 0; j < NPL; ++j) lg[j] = __fadd_rn(lg[j], b[i][j]);
    }
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = j * 32 + lane;
        if (e < E) {
            const float l = lg[j];
            const float sc = apply_sigmoid ? __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-l))) : l;
            s[j] = sc;
            v[j] = __fadd_rn(sc, bias ? bias[e] : 0.0f);
        } else {
            s[j] = 0.0f;
            v[j] = -INFINITY;
        }
    }
    // k (+1 for the margin) rounds of a warp argmax; lane r keeps the r-th
    // pick. Scores become order-preserving 32-bit keys (-0 as +0; NaN and
    // absent experts 0, below every real score), so a round is one local
    // scan, one redux.sync max and a ballot; equal scores on several lanes
    // (rare) take the lowest expert id with a redux.sync min. A picked key is
    // cleared to 0. The round loop stays rolled: this code runs once per
    // token, so its instruction footprint (cold at every launch) costs more
    // than the loop overhead.
    uint32_t key[NPL];
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        uint32_t b = __float_as_uint(v[j]);
        if (b == 0x80000000u) b = 0u;
        key[j] = (j * 32 + lane < E && v[j] == v[j]) ? ((b & 0x80000000u) ? ~b : (b | 0x80000000u))
                                                      : 0u;
    }
    int my_i = 0;
    float my_s = 0.0f;
    float kth = 0.0f, next = -INFINITY;
    const int rounds = (k < E) ? k + 1 : k;
#pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
        uint32_t bk = 0u;
        int bj = 0;
        float bs = 0.0f;
#pragma unroll
        for (int j = 0; j < NPL; ++j)
            if (key[j] > bk) {  // strict: the lowest expert id of this lane on equal keys
                bk = key[j];
                bj = j;
                bs = s[j];
            }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
        const unsigned cand = __ballot_sync(0xffffffffu, bk == mk);
        int win;
        if ((cand & (cand - 1u)) == 0u) {
            win = __ffs(cand) - 1;
        } else {
            const int id = ((cand >> lane) & 1u) ? bj * 32 + lane : 0x7fffffff;
            win = __reduce_min_sync(0xffffffffu, id) & 31;
        }
        const int wj = __shfl_sync(0xffffffffu, bj, win);
        const float ws = __shfl_sync(0xffffffffu, bs, win);
        const float bv = __uint_as_float((mk & 0x80000000u) ? (mk & 0x7fffffffu) : ~mk);
        if (r < k) {
            if (lane == r) {
                my_i = wj * 32 + win;
                my_s = ws;
            }
            kth = bv;
            if (lane == win)
#pragma unroll
                for (int j = 0; j < NPL; ++j)
                    if (j == wj) key[j] = 0u;
        } else {
            next = bv;
        }
    }
    float sum = 0.0f;  // rank order, as the reference sums
#pragma unroll 1
    for (int i = 0; i < k; ++i) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, my_s, i));
    if (lane < k) {
        float wi = my_s;
        if (norm && sum > 0.0f) wi = __fdiv_rn(wi, sum);
        wi = __fmul_rn(wi, scale);
        ids_out[lane] = my_i;
        w_out[lane] = wi;
        if (ids_smem) ids_smem[lane] = my_i;
    }
    if (lane == 0 && margin_out) *margin_out = (k < E) ? __fsub_rn(kth, next) : INFINITY;
}

template <int NPL>
__global__ void __launch_bounds__(256) k_topk(const float* scores, int planes, int T, int E,
                                              const float* bias, int k, float scale, int norm,
                                              int apply_sigmoid, int32_t* ids, float* w,
                                              float* margins) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    topk_warp<NPL>(scores + size_t(t) * E, planes, size_t(T) * E, apply_sigmoid, bias, E, k,
                   scale, norm, lane,
                   ids + size_t(t) * k, w + size_t(t) * k, margins ? margins + t : nullptr,
                   nullptr);
}

// ============================================================ work plan (one block)
// Path of one expert segment: the grouped GEMV for short segments (AUTO) or
// always (GEMV, or shapes the tcgen05 tiles do not cover); else the GEMM.
__device__ __forceinline__ bool segment_uses_gemv(const RouteArgs& a, int c, int I) {
    if (c <= 0 || I <= 0) return false;
    if (!a.gemm_ok || a.path == HF_PATH_GEMV) return true;
    if (a.path == HF_PATH_GEMM) return false;
    return c <= a.gemv_max;
}

constexpr int kPlanVals = 8;  // per group: count, GEMV1/GEMV2 units, GEMM1/GEMM2 tiles, 3 stats
constexpr int kPlanScratch = 33 * kPlanVals;  // ints of warp_tot

// From per-group counts (shared memory s_cnt[G], G <= 2 * blockDim.x) write
// counts, offsets, the GEMV unit and GEMM tile prefixes and the stats into the
// plan buffer, and the offsets also into s_off[G+1]. One fused block scan of
// eight values per group: two barriers.
__device__ void plan_from_counts(const RouteArgs& a, const int* s_cnt, int* s_off, int* warp_tot) {
    const int G = a.pl.G, H = a.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = int(blockDim.x >> 5);
    int v[2][kPlanVals];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int g = 2 * tid + q;
        const int c = g < G ? s_cnt[g] : 0;
        const int I = (g == G - 1) ? a.shared_inter : a.inter;
        const bool gemv = g < G && segment_uses_gemv(a, c, I);
        const bool gemm = g < G && c > 0 && I > 0 && !gemv;
        const int nch = (c + kGemvTE - 1) / kGemvTE;
        const int nt1 = gemm ? (c + a.gemm_bn1 - 1) / a.gemm_bn1 : 0;
        const int nt2 = gemm ? (c + a.gemm_bn2 - 1) / a.gemm_bn2 : 0;
        v[q][0] = c;
        v[q][1] = gemv ? nch * ((I + kGemv1Rows - 1) / kGemv1Rows) : 0;
        v[q][2] = gemv ? nch * ((H + kGemv2Rows - 1) / kGemv2Rows) : 0;
        v[q][3] = nt1 * ((I + a.gemm_m1 - 1) / a.gemm_m1);
        v[q][4] = nt2 * ((H + a.gemm_m2 - 1) / a.gemm_m2);
        v[q][5] = (g < G - 1 && c > 0) ? 1 : 0;
        v[q][6] = gemv ? 1 : 0;
        v[q][7] = gemm ? 1 : 0;
    }
    int sum[kPlanVals], incl[kPlanVals];
#pragma unroll
    for (int i = 0; i < kPlanVals; ++i) {
        sum[i] = v[0][i] + v[1][i];
        incl[i] = sum[i];
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
#pragma unroll
        for (int i = 0; i < kPlanVals; ++i) {
            const int y = __shfl_up_sync(0xffffffffu, incl[i], o);
            if (lane >= o) incl[i] += y;
        }
    if (lane == 31)
#pragma unroll
        for (int i = 0; i < kPlanVals; ++i) warp_tot[warp * kPlanVals + i] = incl[i];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int i = 0; i < kPlanVals; ++i) {
            const int wv = lane < nwarps ? warp_tot[lane * kPlanVals + i] : 0;
            int wi = wv;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += y;
            }
            warp_tot[lane * kPlanVals + i] = wi - wv;  // exclusive prefix of warps
            if (lane == 31) warp_tot[32 * kPlanVals + i] = wi;
        }
    }
    __syncthreads();
    int32_t* plan = a.plan;
    const int dst[5] = {a.pl.offsets, a.pl.u1, a.pl.u2, a.pl.g1, a.pl.g2};
    int base[kPlanVals];
#pragma unroll
    for (int i = 0; i < kPlanVals; ++i) base[i] = warp_tot[warp * kPlanVals + i] + incl[i] - sum[i];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int g = 2 * tid + q;
        if (g < G) {
            plan[a.pl.counts + g] = v[q][0];
            s_off[g] = base[0];
#pragma unroll
            for (int i = 0; i < 5; ++i) plan[dst[i] + g] = base[i];
        }
#pragma unroll
        for (int i = 0; i < kPlanVals; ++i) base[i] += v[q][i];
    }
    if (tid == 0) {
        const int* tot = warp_tot + 32 * kPlanVals;
        s_off[G] = tot[0];
#pragma unroll
        for (int i = 0; i < 5; ++i) plan[dst[i] + G] = tot[i];
        plan[a.pl.stats + 0] = tot[5];
        plan[a.pl.stats + 1] = tot[6];
        plan[a.pl.stats + 2] = tot[7];
    }
    __syncthreads();
}

// Rank of token tl (0..127) among the set bits of a 128-bit mask.
__device__ __forceinline__ int mask_rank(const uint32_t* m, int tl) {
    int r = 0;
    const int w = tl >> 5;
    for (int q = 0; q < w; ++q) r += __popc(m[q]);
    return r + __popc(m[w] & ((1u << (tl & 31)) - 1u));
}

// ============================================================ T <= 128: one block
// One block builds the masks, counts, plan and permutation of up to 128
// tokens. With TOPK it first runs their top-k itself (one warp per token;
// used for a handful of tokens, where a separate launch costs more than it
// saves); otherwise the top-k already ran one warp per token on many SMs.
constexpr int kFusedTopkMaxT = 16;

template <int NPL, bool TOPK>
__device__ void route_block_body(const RouteArgs& a, uint32_t* sm) {
    const int E = a.E, T = a.T, k = a.k, G = a.pl.G;
    uint32_t* masks = sm;                                   // [E][4]
    int* s_cnt = reinterpret_cast<int*>(masks + 4 * E);     // [G]
    int* s_off = s_cnt + G;                                  // [G+1]
    int* s_ids = s_off + G + 1;                              // [128 * 8]
    int* warp_tot = s_ids + kSmallRouteT * kMaxTopK;         // [kPlanScratch]

    for (int i = threadIdx.x; i < 4 * E; i += blockDim.x) masks[i] = 0u;
    if constexpr (TOPK) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int t = warp; t < T; t += int(blockDim.x >> 5))
            topk_warp<NPL>(a.logits + size_t(t) * E, a.lsplit, size_t(T) * E, 1, a.bias, E, k,
                           a.scale, a.norm, lane,
                           a.ids + size_t(t) * k, a.w + size_t(t) * k,
                           a.margins ? a.margins + t : nullptr, s_ids + t * kMaxTopK);
    } else {
        for (int i = threadIdx.x; i < T * k; i += blockDim.x)
            s_ids[(i / k) * kMaxTopK + i % k] = a.ids[i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * k; i += blockDim.x) {
        const int t = i / k, e = s_ids[t * kMaxTopK + i % k];
        atomicOr(&masks[4 * e + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        int c = 0;
        if (g < E) c = __popc(masks[4 * g]) + __popc(masks[4 * g + 1]) + __popc(masks[4 * g + 2]) +
                       __popc(masks[4 * g + 3]);
        else c = a.has_shared ? T : 0;
        s_cnt[g] = c;
    }
    __syncthreads();
    plan_from_counts(a, s_cnt, s_off, warp_tot);
    for (int i = threadIdx.x; i < T * k; i += blockDim.x) {
        const int t = i / k, e = s_ids[t * kMaxTopK + i % k];
        const int pos = s_off[e] + mask_rank(&masks[4 * e], t);
        a.perm[pos] = i;
        a.slot_pos[i] = pos;
    }
    if (a.has_shared)
        for (int t = threadIdx.x; t < T; t += blockDim.x) {
            const int pos = s_off[G - 1] + t, slot = T * k + t;
            a.perm[pos] = slot;
            a.slot_pos[slot] = pos;
        }
}

template <int NPL, bool TOPK>
__global__ void __launch_bounds__(1024) k_route_block(RouteArgs a) {
    extern __shared__ __align__(16) uint32_t sm[];
    route_block_body<NPL, TOPK>(a, sm);
}

// Decode (T <= kFusedTopkMaxT): router rows, then the last block to finish
// (a device counter, reset by that block) runs top-k, counts, plan and
// permutation over all logits -- one launch instead of two. Every block
// fences its logits before it counts itself in, the last one after it has
// seen the full count.
template <bool XF32, int NPL>
__global__ void __launch_bounds__(256) k_router_route(RouteArgs a) {
    extern __shared__ __align__(16) uint32_t sm[];
    __shared__ int s_last;
    griddep_launch_dependents();  // the expert kernel may take its place in the queue now
    router_rows<XF32>(a);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.route_counter, 1) == int(gridDim.x) - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    route_block_body<NPL, true>(a, sm);
    if (threadIdx.x == 0) *a.route_counter = 0;
}


// ============================================================ T > 128: four launches
// (1) k_topk, (2) masks + per-block counts, (3) scan + plan + per-block bases,
// (4) scatter.
__global__ void __launch_bounds__(256) k_perm_masks(RouteArgs a) {
    __shared__ uint32_t masks[4 * kMaxExperts];
    const int b = blockIdx.x, E = a.E, k = a.k;
    const int t0 = b * kSmallRouteT;
    const int nt = min(kSmallRouteT, a.T - t0);
    for (int i = threadIdx.x; i < 4 * E; i += blockDim.x) masks[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < nt * k; i += blockDim.x) {
        const int tl = i / k, e = a.ids[size_t(t0 + tl) * k + i % k];
        atomicOr(&masks[4 * e + (tl >> 5)], 1u << (tl & 31));
    }
    __syncthreads();
    uint32_t* gm = a.masks + size_t(b) * 4 * E;
    for (int i = threadIdx.x; i < 4 * E; i += blockDim.x) gm[i] = masks[i];
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        a.blk_counts[size_t(b) * E + e] = __popc(masks[4 * e]) + __popc(masks[4 * e + 1]) +
                                          __popc(masks[4 * e + 2]) + __popc(masks[4 * e + 3]);
}

__global__ void __launch_bounds__(1024) k_perm_plan(RouteArgs a, int nb) {
    extern __shared__ __align__(16) uint32_t sm[];
    const int E = a.E, G = a.pl.G;
    int* s_cnt = reinterpret_cast<int*>(sm);
    int* s_tmp = s_cnt + G;
    int* warp_tot = s_tmp + G + 1;
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        int c = 0;
        if (g < E) for (int b = 0; b < nb; ++b) c += a.blk_counts[size_t(b) * E + g];
        else c = a.has_shared ? a.T : 0;
        s_cnt[g] = c;
    }
    __syncthreads();
    plan_from_counts(a, s_cnt, s_tmp, warp_tot);
    // per-block bases (in place over blk_counts)
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = a.plan[a.pl.offsets + e];
        for (int b = 0; b < nb; ++b) {
            const int c = a.blk_counts[size_t(b) * E + e];
            a.blk_counts[size_t(b) * E + e] = run;
            run += c;
        }
    }
}

__global__ void __launch_bounds__(1024) k_plan_counts(RouteArgs a, const int32_t* counts) {
    extern __shared__ __align__(16) uint32_t sm[];
    const int G = a.pl.G;
    int* s_cnt = reinterpret_cast<int*>(sm);
    int* s_tmp = s_cnt + G;
    int* warp_tot = s_tmp + G + 1;
    for (int g = threadIdx.x; g < G; g += blockDim.x) s_cnt[g] = counts[g];
    __syncthreads();
    plan_from_counts(a, s_cnt, s_tmp, warp_tot);
}

hf_status launch_plan_from_counts(const RouteArgs& a, const int32_t* counts, cudaStream_t st) {
    const int G = a.pl.G;
    const size_t smem = sizeof(int) * (G + G + 1 + kPlanScratch);
    k_plan_counts<<<1, 1024, smem, st>>>(a, counts);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

// Expert-parallel receiver plan from counts already on the device (the
// decode exchange, no host round trip). Source s sent its rows for local
// expert j (cnt[s * El + j] of them) in expert order at the start of its
// slab of `cap` rows. Local positions are expert-major, then source, then
// arrival -- the order the host plan of the large-batch exchange uses -- and
// the shared expert's T_loc local tokens come last (rows W * cap + t). Also
// writes row_pos (slab row -> local position) and recv_tot[s] (rows from s).
// With yrow set it also writes each position's output row (rows of ro.esz * H
// bytes): received row i from source s goes back to row rank * cap + i of s's
// output slab
// (peer_y[s], mapped here), a local token t to row W * cap + t of this rank's
// own slab (peer_y[rank]).
__global__ void __launch_bounds__(1024) k_ep_plan(RouteArgs a, const int32_t* cnt,
                                                  const int32_t* rmap, int W, int El,
                                                  int cap, int T_loc, int32_t* perm,
                                                  int32_t* row_pos, int32_t* recv_tot,
                                                  const unsigned long long* flags,
                                                  unsigned long long seq,
                                                  unsigned long long timeout_ns, int* err,
                                                  EpRowOut ro) {
    extern __shared__ __align__(16) uint32_t sm[];
    // peer-memory exchange: counts and rows are in place once every source's
    // flag shows this forward's sequence number
    if (flags) {
        if (threadIdx.x == 0) sm100::wait_flags_sys(flags, W, seq, timeout_ns, err);
        __syncthreads();
    }
    const int G = a.pl.G;  // El + 1
    int* s_cnt = reinterpret_cast<int*>(sm);  // [G]
    int* s_off = s_cnt + G;                   // [G + 1]
    int* warp_tot = s_off + G + 1;            // [kPlanScratch]
    int* s_src = warp_tot + kPlanScratch;     // [W x El] row of (s, j) inside s's slab
    int* s_pos = s_src + W * El;              // [W x El] position of (s, j) inside expert j
    for (int j = threadIdx.x; j < El; j += blockDim.x) {
        int acc = 0;
        for (int s = 0; s < W; ++s) {
            s_pos[s * El + j] = acc;
            acc += cnt[s * El + j];
        }
        s_cnt[j] = acc;
    }
    for (int s = threadIdx.x; s < W; s += blockDim.x) {
        int acc = 0;
        for (int j = 0; j < El; ++j) {
            s_src[s * El + j] = acc;
            acc += cnt[s * El + j];
        }
        recv_tot[s] = acc;
    }
    if (threadIdx.x == 0) s_cnt[El] = a.has_shared ? T_loc : 0;
    __syncthreads();
    plan_from_counts(a, s_cnt, s_off, warp_tot);  // ends with a barrier: s_off is complete
    const int rows = W * cap;
    for (int sj = threadIdx.x; sj < W * El; sj += blockDim.x) {
        const int n = cnt[sj];
        const int pos0 = s_off[sj % El] + s_pos[sj];
        const int row0 = (sj / El) * cap + s_src[sj];
        const int s = sj / El;
        // output rows are ro.esz * H bytes (fp32 or the FP16 plane)
        const size_t rowb = size_t(ro.esz) * ro.H;
        char* yb = ro.yrow ? reinterpret_cast<char*>(ro.peer_y[s]) +
                                 (size_t(ro.rank) * cap + s_src[sj]) * rowb
                           : nullptr;
        const int32_t* rm = rmap ? rmap + row0 : nullptr;
        for (int i = 0; i < n; ++i) {
            // slot id = row of [slabs | local tokens] (k = 1): the arrival row,
            // or the row the source stored the token's activations in
            perm[pos0 + i] = rm ? (sj / El) * cap + rm[i] : row0 + i;
            row_pos[row0 + i] = pos0 + i;
            if (yb) ro.yrow[pos0 + i] = reinterpret_cast<float*>(yb + size_t(i) * rowb);
        }
    }
    if (a.has_shared)  // slot ids past all rows name the local tokens (token_of_slot)
        for (int t = threadIdx.x; t < T_loc; t += blockDim.x) {
            perm[s_off[El] + t] = (rows + T_loc) + (rows + t);
            if (ro.yrow)
                ro.yrow[s_off[El] + t] = reinterpret_cast<float*>(
                    reinterpret_cast<char*>(ro.peer_y[ro.rank]) +
                    size_t(rows + t) * ro.esz * ro.H);
        }
}

hf_status launch_ep_plan(const RouteArgs& a, const int32_t* cnt, const int32_t* rmap, int W,
                         int El, int cap, int T_loc, int32_t* perm, int32_t* row_pos,
                         int32_t* recv_tot,
                         const unsigned long long* flags, unsigned long long seq,
                         unsigned long long timeout_ns, int* err, const EpRowOut& ro,
                         cudaStream_t st) {
    const int G = a.pl.G;
    if (G != El + 1 || G > 2 * 1024) return fail(HF_ERR_ARG, "expert-parallel plan: bad group count");
    const size_t smem = sizeof(int) * (G + G + 1 + kPlanScratch + 2 * W * El);
    HF_CUDA(ensure_smem(reinterpret_cast<const void*>(k_ep_plan), int(smem)));
    k_ep_plan<<<1, 1024, smem, st>>>(a, cnt, rmap, W, El, cap, T_loc, perm, row_pos, recv_tot,
                                     flags, seq, timeout_ns, err, ro);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

// Plan of a dense MLP pass: a single group (the shared-expert slot, G = 1)
// holding all T tokens in order (perm = identity, slot id = token with k = 0).
// Block 0 also writes the group's weight pointers and clears the error word.
__global__ void __launch_bounds__(1024) k_dense_plan(RouteArgs a, GroupW w, GroupW* groups,
                                                     int32_t* perm, int* sched) {
    __shared__ int s_cnt[1], s_off[2];
    __shared__ int warp_tot[kPlanScratch];
    if (blockIdx.x == 0) {
        if (threadIdx.x == 0) {
            groups[0] = w;
            s_cnt[0] = a.T;
            a.plan[a.pl.stats + 3] = 0;
            sched[0] = sched[1] = 0;  // the workspace may be fresh memory
        }
        __syncthreads();
        plan_from_counts(a, s_cnt, s_off, warp_tot);
    }
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < a.T; p += gridDim.x * blockDim.x)
        perm[p] = p;
}

hf_status launch_dense_plan(const RouteArgs& a, const GroupW& w, GroupW* groups, int32_t* perm,
                            int* sched, cudaStream_t st) {
    const int blocks = std::max(1, std::min(64, (a.T + 1023) / 1024));
    k_dense_plan<<<blocks, 1024, 0, st>>>(a, w, groups, perm, sched);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

__global__ void __launch_bounds__(256) k_gather_rows(uint4* dst, const uint4* src, int row_vec, int n,
                                                     const int32_t* idx, int div) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int i = warp; i < n; i += nw) {
        const int s = idx[i] / div;
        const uint4* sr = src + size_t(s) * row_vec;
        uint4* dr = dst + size_t(i) * row_vec;
        for (int c = lane; c < row_vec; c += 32) dr[c] = ld_nc_u4(sr + c);
    }
}

hf_status launch_gather_rows(void* dst, const void* src, size_t row_bytes, int n,
                             const int32_t* idx, int div, cudaStream_t st) {
    if (n <= 0) return HF_OK;
    if (row_bytes % 16) return fail(HF_ERR_ARG, "row gather needs 16-byte rows");
    const int blocks = std::min(num_sms(0) * 8, (n + 7) / 8);
    k_gather_rows<<<blocks, 256, 0, st>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src),
                                          int(row_bytes / 16), n, idx, div);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

__global__ void __launch_bounds__(256) k_perm_scatter(RouteArgs a) {
    const int b = blockIdx.x, E = a.E, k = a.k, T = a.T;
    const int t0 = b * kSmallRouteT;
    const int nt = min(kSmallRouteT, T - t0);
    const uint32_t* gm = a.masks + size_t(b) * 4 * E;
    const int32_t* base = a.blk_counts + size_t(b) * E;
    for (int i = threadIdx.x; i < nt * k; i += blockDim.x) {
        const int tl = i / k;
        const int slot = (t0 + tl) * k + i % k;
        const int e = a.ids[slot];
        const int pos = base[e] + mask_rank(gm + 4 * e, tl);
        a.perm[pos] = slot;
        a.slot_pos[slot] = pos;
    }
    if (a.has_shared) {
        const int off = a.plan[a.pl.offsets + a.pl.G - 1];
        for (int tl = threadIdx.x; tl < nt; tl += blockDim.x) {
            const int t = t0 + tl, pos = off + t, slot = T * k + t;
            a.perm[pos] = slot;
            a.slot_pos[slot] = pos;
        }
    }
}

// ============================================================ launchers
// Runs the statement with NPL = scores per lane (E/32 rounded up to a power of 2).
#define HF_NPL_SWITCH(E, ...)                                      \
    do {                                                           \
        const int _n = ((E) + 31) / 32;                            \
        if (_n <= 1) { constexpr int NPL = 1; __VA_ARGS__; }        \
        else if (_n <= 2) { constexpr int NPL = 2; __VA_ARGS__; }   \
        else if (_n <= 4) { constexpr int NPL = 4; __VA_ARGS__; }   \
        else if (_n <= 8) { constexpr int NPL = 8; __VA_ARGS__; }   \
        else if (_n <= 16) { constexpr int NPL = 16; __VA_ARGS__; } \
        else { constexpr int NPL = 32; __VA_ARGS__; }              \
    } while (0)

size_t route_block_smem(const RouteArgs& a) {
    const int G = a.pl.G;
    return sizeof(uint32_t) * (4 * a.E + G + G + 1 + kSmallRouteT * kMaxTopK + kPlanScratch);
}

hf_status launch_router_logits(const RouteArgs& a, cudaStream_t st, bool* routed) {
    if (routed) *routed = false;
    if (a.T == 0) return HF_OK;
    const int grid = (a.E + kRouterRowsPerBlock - 1) / kRouterRowsPerBlock;
    if (routed && a.route_counter && a.T <= kFusedTopkMaxT && a.lsplit == 1 && a.pl.G <= 2 * 256) {
        const size_t smem = route_block_smem(a);
        HF_NPL_SWITCH(a.E, {
            if (a.x_f32) k_router_route<true, NPL><<<grid, 256, smem, st>>>(a);
            else k_router_route<false, NPL><<<grid, 256, smem, st>>>(a);
        });
        HF_CUDA(cudaGetLastError());
        *routed = true;
        return HF_OK;
    }
    if (a.T <= kRouterMaxT) {
        if (a.x_f32) k_router_gemv<true><<<grid, 256, 0, st>>>(a);
        else k_router_gemv<false><<<grid, 256, 0, st>>>(a);
    } else {
        dim3 grid((a.T + 63) / 64, (a.E + 63) / 64);
        if (a.x_f32) k_router_tile<true><<<grid, 256, 0, st>>>(a);
        else k_router_tile<false><<<grid, 256, 0, st>>>(a);
    }
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

hf_status launch_route(const RouteArgs& a, cudaStream_t st, int* launches) {
    *launches = 0;
    if (a.T == 0) return HF_OK;
    const int G = a.pl.G;
    if (a.T <= kSmallRouteT) {
        const size_t smem = route_block_smem(a);
        if (a.T <= kFusedTopkMaxT) {
            *launches = 1;
            HF_NPL_SWITCH(a.E, { k_route_block<NPL, true><<<1, 1024, smem, st>>>(a); });
        } else {
            *launches = 2;
            HF_NPL_SWITCH(a.E, {
                k_topk<NPL><<<(a.T + 7) / 8, 256, 0, st>>>(a.logits, a.lsplit, a.T, a.E,
                                                           a.bias, a.k, a.scale, a.norm, 1,
                                                           a.ids, a.w, a.margins);
            });
            HF_CUDA(cudaGetLastError());
            k_route_block<1, false><<<1, 1024, smem, st>>>(a);
        }
        HF_CUDA(cudaGetLastError());
        return HF_OK;
    }
    *launches = 4;
    const int nb = (a.T + kSmallRouteT - 1) / kSmallRouteT;
    HF_NPL_SWITCH(a.E, {
        k_topk<NPL><<<(a.T + 7) / 8, 256, 0, st>>>(a.logits, a.lsplit, a.T, a.E, a.bias, a.k,
                                                   a.scale, a.norm, 1, a.ids, a.w, a.margins);
    });
    HF_CUDA(cudaGetLastError());
    k_perm_masks<<<nb, 256, 0, st>>>(a);
    HF_CUDA(cudaGetLastError());
    const size_t smem = sizeof(int) * (G + G + 1 + kPlanScratch);
    k_perm_plan<<<1, 1024, smem, st>>>(a, nb);
    HF_CUDA(cudaGetLastError());
    k_perm_scatter<<<nb, 256, 0, st>>>(a);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

hf_status launch_topk(const float* scores, int T, int E, const float* bias, int k, float scale,
                      int norm, int32_t* idx, float* w, int apply_sigmoid, float* margins,
                      cudaStream_t st) {
    if (T == 0) return HF_OK;
    HF_NPL_SWITCH(E, {
        k_topk<NPL><<<(T + 7) / 8, 256, 0, st>>>(scores, 1, T, E, bias, k, scale, norm,
                                                 apply_sigmoid, idx, w, margins);
    });
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

}  // namespace hf
