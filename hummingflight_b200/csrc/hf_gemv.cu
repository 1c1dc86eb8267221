// hf_gemv.cu -- decode grouped GEMV over expert segments, weighted combine,
// and the device twin of gemv_bf16_f32.
//
// Reference: expertFFNRaw (model/glm_forward.cpp:434-449): g = G x, u = U x,
// mid = g / (1 + exp(-g)) * u in fp32, y = D mid; the sm_86 offload replaced
// here is matvecStreamKernel + siluScaleKernel (compute/cuda_kernels.cu:125-153,
// one block per row, 2-byte loads, x and y crossing PCIe per expert).
//
// B200 design: a segment (the tokens routed to one expert) is cut into chunks
// of up to kGemvTE tokens. A unit of work is (expert, row block, chunk); units
// of one expert are adjacent with the chunk index fastest, so a weight row is
// fetched from HBM once and re-served from L2 to the other chunks. Persistent
// CTAs (a multiple of the SM count) stride over the unit list the routing
// kernel wrote. Each warp streams 2 gate + 2 up rows (GEMV1) or 4 down rows
// (GEMV2) with 16-byte L1-bypassing loads, 8 loads in flight per lane, the
// chunk's activations sitting in shared memory; fp32 accumulation, butterfly
// shuffles, SwiGLU in the GEMV1 epilogue, mid kept fp32.
#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include <cuda_fp16.h>

#include "hf_internal.cuh"

namespace hf {

constexpr int kUnroll = 2;

template <bool XF32>
__device__ __forceinline__ void lds_x8(const void* xs, int j, int H, int c, float (&o)[8]) {
    if constexpr (XF32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(xs) +
                                                          size_t(j) * H + c * 8);
        const float4 a = p[0], b = p[1];
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    } else {
        const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xs) +
                                                        size_t(j) * H + c * 8);
        unpack8(v, o);
    }
}

// Two gate rows and two up rows (r0, r0+1) against NT tokens held in shared memory.
template <bool XF32, int NT>
__device__ __forceinline__ void gemv1_rows(const GroupW& W, int H, int r0, const void* xs,
                                           int lane, float* mid, int p0, int mid_stride) {
    const int I = W.inter;
    if (r0 >= I) return;
    const bool v1 = (r0 + 1) < I;
    const uint16_t* pr[4] = {W.gate + size_t(r0) * H, W.gate + size_t(v1 ? r0 + 1 : r0) * H,
                             W.up + size_t(r0) * H, W.up + size_t(v1 ? r0 + 1 : r0) * H};
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[r][j] = 0.0f;
    const int nc = H >> 3;
    int c = lane;
    for (; c + 32 * (kUnroll - 1) < nc; c += 32 * kUnroll) {
        uint4 wv[kUnroll][4];
#pragma unroll
        for (int q = 0; q < kUnroll; ++q)
#pragma unroll
            for (int r = 0; r < 4; ++r) wv[q][r] = ld_stream_u4(pr[r] + size_t(c + 32 * q) * 8);
#pragma unroll
        for (int q = 0; q < kUnroll; ++q) {
            float wf[4][8];
#pragma unroll
            for (int r = 0; r < 4; ++r) unpack8(wv[q][r], wf[r]);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                float xf[8];
                lds_x8<XF32>(xs, j, H, c + 32 * q, xf);
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[r][j] = fmaf(wf[r][e], xf[e], acc[r][j]);
            }
        }
    }
    for (; c < nc; c += 32) {
        uint4 wv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) wv[r] = ld_stream_u4(pr[r] + size_t(c) * 8);
        float wf[4][8];
#pragma unroll
        for (int r = 0; r < 4; ++r) unpack8(wv[r], wf[r]);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            float xf[8];
            lds_x8<XF32>(xs, j, H, c, xf);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[r][j] = fmaf(wf[r][e], xf[e], acc[r][j]);
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[r][j] = warp_sum(acc[r][j]);
    // lane q < 2*NT writes (row r0 + (q & 1), token q >> 1)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            if (lane == 2 * j + rr && (rr == 0 || v1)) {
                const float g = acc[rr][j], u = acc[2 + rr][j];
                mid[size_t(p0 + j) * mid_stride + r0 + rr] = swiglu(g, u);
            }
        }
    }
}

template <bool XF32>
__global__ void __launch_bounds__(256) k_gemv1(GemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    void* xs = smem_raw;
    const int G = a.pl.G;
    const int H = a.H;
    if (a.prefetch_shared) {
        // the shared expert's weights do not depend on the routing: stream them
        // into L2 while the routing kernel still runs (HBM is idle then); its
        // units run first below, the down rows stay for GEMV2 (evict_last)
        const GroupW S = a.groups[G - 1];
        const size_t n = size_t(S.inter) * H * 2;
        prefetch_l2<false>(S.gate, n);
        prefetch_l2<false>(S.up, n);
        prefetch_l2<true>(S.down, n);
    }
    griddep_wait();  // the plan and permutation come from the routing kernel
    griddep_launch_dependents();
    int32_t* sp = reinterpret_cast<int32_t*>(smem_raw + size_t(a.te_cap) * H * (XF32 ? 4 : 2));
    stage_plan(sp, a.plan + a.pl.u1, a.plan, a.pl);
    __syncthreads();
    const int32_t* u1 = sp;
    const int32_t* cnts = sp + G + 1;
    const int32_t* offs = sp + 2 * G + 1;
    const int total = u1[G];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int ui = blockIdx.x; ui < total; ui += gridDim.x) {
        const int u = a.prefetch_shared ? total - 1 - ui : ui;  // shared expert first
        const int g = find_group(u1, G, u);
        const int cnt = cnts[g];
        const int nch = (cnt + kGemvTE - 1) / kGemvTE;
        const int local = u - u1[g];
        const int rb = local / nch, ch = local % nch;
        const int p0 = offs[g] + ch * kGemvTE;
        const int te = min(kGemvTE, cnt - ch * kGemvTE);
        __syncthreads();
        // stage the chunk's activation rows: te x H elements, 16 bytes per thread-step
        const int vec = XF32 ? 4 : 8;
        const int per_row = H / vec;
        for (int i = threadIdx.x; i < te * per_row; i += blockDim.x) {
            const int j = i / per_row, c = i % per_row;
            const int t = token_of_slot(a.perm[p0 + j], a.T, a.k);
            const uint4 v = ld_nc_u4(static_cast<const char*>(a.x) +
                                     (size_t(t) * H + size_t(c) * vec) * (XF32 ? 4 : 2));
            reinterpret_cast<uint4*>(xs)[size_t(j) * per_row + c] = v;
        }
        __syncthreads();
        const GroupW W = a.groups[g];
        const int r0 = rb * kGemv1Rows + warp * 2;
        switch (te) {
            case 1: gemv1_rows<XF32, 1>(W, H, r0, xs, lane, a.mid, p0, a.inter_max); break;
            case 2: gemv1_rows<XF32, 2>(W, H, r0, xs, lane, a.mid, p0, a.inter_max); break;
            case 3: gemv1_rows<XF32, 3>(W, H, r0, xs, lane, a.mid, p0, a.inter_max); break;
            default: gemv1_rows<XF32, 4>(W, H, r0, xs, lane, a.mid, p0, a.inter_max); break;
        }
    }
}

// Four down rows (h0..h0+3) against NT mid vectors (fp32, shared memory).
// Eight FP16 weights (a down block in the FP16 resident format, w * 2^S).
__device__ __forceinline__ void unpack8_f16(const uint4& v, float (&o)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
        o[2 * q] = f.x;
        o[2 * q + 1] = f.y;
    }
}

// F16: the down block holds FP16 w * 2^S; the sums carry 2^S exactly and
// are multiplied by W.down_scale = 2^-S at the end (the same bits as the
// BF16 block would give).
template <int NT, bool F16>
__device__ __forceinline__ void gemv2_rows(const GroupW& W, int H, int h0, const float* ms,
                                           int lane, float* y, int p0, const float* resid) {
    const int I = W.inter;
    if (h0 >= H) return;
    const uint16_t* pr[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) pr[r] = W.down + size_t(min(h0 + r, H - 1)) * I;
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[r][j] = 0.0f;
    const int nc = I >> 3;
    int c = lane;
    for (; c + 32 * (kUnroll - 1) < nc; c += 32 * kUnroll) {
        uint4 wv[kUnroll][4];
#pragma unroll
        for (int q = 0; q < kUnroll; ++q)
#pragma unroll
            for (int r = 0; r < 4; ++r) wv[q][r] = ld_stream_u4(pr[r] + size_t(c + 32 * q) * 8);
#pragma unroll
        for (int q = 0; q < kUnroll; ++q) {
            float wf[4][8];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if constexpr (F16) unpack8_f16(wv[q][r], wf[r]);
                else unpack8(wv[q][r], wf[r]);
            }
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                float xf[8];
                lds_x8<true>(ms, j, I, c + 32 * q, xf);
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[r][j] = fmaf(wf[r][e], xf[e], acc[r][j]);
            }
        }
    }
    for (; c < nc; c += 32) {
        uint4 wv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) wv[r] = ld_stream_u4(pr[r] + size_t(c) * 8);
        float wf[4][8];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            if constexpr (F16) unpack8_f16(wv[r], wf[r]);
            else unpack8(wv[r], wf[r]);
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            float xf[8];
            lds_x8<true>(ms, j, I, c, xf);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[r][j] = fmaf(wf[r][e], xf[e], acc[r][j]);
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            acc[r][j] = warp_sum(acc[r][j]);
            if constexpr (F16) acc[r][j] = __fmul_rn(acc[r][j], W.down_scale);
        }
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (lane == 4 * j + r && h0 + r < H) {
                const size_t yi = size_t(p0 + j) * H + h0 + r;
                // residual block (dense MLP, positions are tokens): read, then write, yi
                y[yi] = resid ? __fadd_rn(resid[yi], acc[r][j]) : acc[r][j];
            }
}

__global__ void __launch_bounds__(256) k_gemv2(GemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* ms = reinterpret_cast<float*>(smem_raw);
    const int G = a.pl.G;
    griddep_wait();  // mid comes from GEMV1
    griddep_launch_dependents();
    int32_t* sp = reinterpret_cast<int32_t*>(smem_raw + size_t(a.te_cap) * a.inter_max * 4);
    stage_plan(sp, a.plan + a.pl.u2, a.plan, a.pl);
    __syncthreads();
    const int32_t* u2 = sp;
    const int32_t* cnts = sp + G + 1;
    const int32_t* offs = sp + 2 * G + 1;
    const int total = u2[G];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H;
    for (int ui = blockIdx.x; ui < total; ui += gridDim.x) {
        const int u = a.prefetch_shared ? total - 1 - ui : ui;  // shared expert first
        const int g = find_group(u2, G, u);
        const int cnt = cnts[g];
        const int nch = (cnt + kGemvTE - 1) / kGemvTE;
        const int local = u - u2[g];
        const int rb = local / nch, ch = local % nch;
        const int p0 = offs[g] + ch * kGemvTE;
        const int te = min(kGemvTE, cnt - ch * kGemvTE);
        const GroupW W = a.groups[g];
        const int I = W.inter;
        __syncthreads();
        const int per_row = I / 4;
        for (int i = threadIdx.x; i < te * per_row; i += blockDim.x) {
            const int j = i / per_row, c = i % per_row;
            reinterpret_cast<float4*>(ms)[size_t(j) * per_row + c] =
                *reinterpret_cast<const float4*>(a.mid + size_t(p0 + j) * a.inter_max + c * 4);
        }
        __syncthreads();
        const int h0 = rb * kGemv2Rows + warp * 4;
        if (W.down_f16) {
            switch (te) {
                case 1: gemv2_rows<1, true>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
                case 2: gemv2_rows<2, true>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
                case 3: gemv2_rows<3, true>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
                default: gemv2_rows<4, true>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
            }
        } else {
            switch (te) {
                case 1: gemv2_rows<1, false>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
                case 2: gemv2_rows<2, false>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
                case 3: gemv2_rows<3, false>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
                default: gemv2_rows<4, false>(W, H, h0, ms, lane, a.y, p0, a.resid); break;
            }
        }
        if (a.prefetch_shared && g == G - 1 && ch == nch - 1 && h0 < H) {
            // last use of these shared down rows: back to normal L2 priority
            const int nr = min(4, H - h0);
            const char* base = reinterpret_cast<const char*>(W.down + size_t(h0) * I);
            for (int l = lane; l < nr * I * 2 / 128; l += 32)
                asm volatile("applypriority.global.L2::evict_normal [%0], 128;" ::"l"(base + l * 128));
        }
    }
}

size_t gemv1_smem(int H, bool xf32, int G, int te) {
    return size_t(te) * H * (xf32 ? 4 : 2) + plan_smem_bytes(G);
}
size_t gemv2_smem(int inter_max, int G, int te) {
    return size_t(te) * inter_max * 4 + plan_smem_bytes(G);
}

hf_status launch_gemv1(const GemvArgs& a, cudaStream_t st) {
    const size_t s1 = gemv1_smem(a.H, a.x_f32 != 0, a.pl.G, a.te_cap);
    if (a.x_f32) {
        HF_CUDA(ensure_smem(reinterpret_cast<const void*>(k_gemv1<true>), (int)s1));
        HF_CUDA(launch_pdl(k_gemv1<true>, dim3(a.grid1), dim3(256), s1, st, a));
    } else {
        HF_CUDA(ensure_smem(reinterpret_cast<const void*>(k_gemv1<false>), (int)s1));
        HF_CUDA(launch_pdl(k_gemv1<false>, dim3(a.grid1), dim3(256), s1, st, a));
    }
    return HF_OK;
}

hf_status launch_gemv2(const GemvArgs& a, cudaStream_t st) {
    const size_t s2 = gemv2_smem(a.inter_max, a.pl.G, a.te_cap);
    HF_CUDA(ensure_smem(reinterpret_cast<const void*>(k_gemv2), (int)s2));
    HF_CUDA(launch_pdl(k_gemv2, dim3(a.grid2), dim3(256), s2, st, a));
    return HF_OK;
}

// Persistent grid: SMs x resident blocks at the shared memory a launch with
// chunks of up to `te` tokens stages (cached per shape).
int gemv_grid(int device, bool first, bool xf32, int H, int inter_max, int G, int te) {
    static std::mutex mu;
    static std::map<std::tuple<int, bool, bool, int, int, int, int>, int> cache;
    const auto key = std::make_tuple(device, first, xf32, H, inter_max, G, te);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int per_sm = 1;
    if (first) {
        const size_t s = gemv1_smem(H, xf32, G, te);
        auto kern = xf32 ? k_gemv1<true> : k_gemv1<false>;
        // raise-only (another launch may already need a larger opt-in)
        ensure_smem(reinterpret_cast<const void*>(kern), (int)s);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, s);
    } else {
        const size_t s = gemv2_smem(inter_max, G, te);
        ensure_smem(reinterpret_cast<const void*>(k_gemv2), (int)s);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_gemv2, 256, s);
    }
    if (per_sm < 1) per_sm = 1;
    const int grid = per_sm * num_sms(device);
    cache.emplace(key, grid);
    return grid;
}

// ============================================================ combine
// glm_forward.cpp:555-556, 639-640, 658-660: moeOut = 0; moeOut += w_i * y_i in
// top-k rank order (separate multiply and add); output = moeOut + sharedOut.
// With a residual (the MLP block, glm_forward.cpp:795-796): output = residual +
// (moeOut + sharedOut); each thread reads its residual elements before it
// writes the same elements, so the residual may be the output buffer.
// A thread owns V consecutive elements of one token: 4 of fp32 outputs, 8 of
// the FP16 plane -- one 16-byte load a slot either way. The loads of all
// slots are issued first, as raw 16-byte vectors; FP16 values are widened
// (times 2^kYF16Shift, exact) only where the accumulation uses them.
template <bool Y16>
struct CombineVec {
    static constexpr int V = Y16 ? 8 : 4;
    uint4 q;
    __device__ __forceinline__ void load(const float* y, size_t row, int H, int h) {
        q = Y16 ? *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(y) + row * H + h)
                : *reinterpret_cast<const uint4*>(y + row * H + h);
    }
    __device__ __forceinline__ void zero() { q = make_uint4(0u, 0u, 0u, 0u); }
    __device__ __forceinline__ void get(float (&v)[V]) const {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        if constexpr (Y16) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                v[2 * i] = __fmul_rn(f.x, float(1 << kYF16Shift));
                v[2 * i + 1] = __fmul_rn(f.y, float(1 << kYF16Shift));
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(w[i]);
        }
    }
};

template <int V>
__device__ __forceinline__ void store_f32(float* p, const float (&v)[V]) {
#pragma unroll
    for (int i = 0; i < V; i += 4)
        *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}

template <bool Y16>
__global__ void __launch_bounds__(256) k_combine(CombineArgs a) {
    griddep_wait();  // expert outputs of the previous kernel
    using Vec = CombineVec<Y16>;
    constexpr int V = Vec::V;
    const int HV = a.H / V;
    const size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= size_t(a.T) * HV) return;
    const int t = int(idx / HV), h = int(idx % HV) * V;
    // all loads first (independent), then the accumulation in rank order
    int pos[kMaxTopK];
    float wt[kMaxTopK];
    Vec yv[kMaxTopK];
#pragma unroll
    for (int i = 0; i < kMaxTopK; ++i)
        if (i < a.k) {
            pos[i] = a.slot_pos[t * a.k + i];
            wt[i] = a.w[t * a.k + i];
        }
#pragma unroll
    for (int i = 0; i < kMaxTopK; ++i)
        if (i < a.k) yv[i].load(a.y, size_t(pos[i]), a.H, h);
    Vec sv;
    sv.zero();
    const int sslot = a.T * a.k + t;
    if (a.has_shared) sv.load(a.y, size_t(a.slot_pos[sslot]), a.H, h);
    float acc[V];
#pragma unroll
    for (int e = 0; e < V; ++e) acc[e] = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxTopK; ++i) {
        if (i >= a.k) break;
        const float wi = wt[i];
        float y[V];
        yv[i].get(y);
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(wi, y[e]));
        if (a.slot_out) store_f32<V>(a.slot_out + size_t(t * a.k + i) * a.H + h, y);
    }
    {
        float s[V];
        sv.get(s);
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = __fadd_rn(acc[e], s[e]);
        if (a.has_shared && a.slot_out) store_f32<V>(a.slot_out + size_t(sslot) * a.H + h, s);
    }
    if (a.resid) {
#pragma unroll
        for (int e = 0; e < V; e += 4) {
            const float4 rs = *reinterpret_cast<const float4*>(a.resid + size_t(t) * a.H + h + e);
            acc[e] = __fadd_rn(rs.x, acc[e]);
            acc[e + 1] = __fadd_rn(rs.y, acc[e + 1]);
            acc[e + 2] = __fadd_rn(rs.z, acc[e + 2]);
            acc[e + 3] = __fadd_rn(rs.w, acc[e + 3]);
        }
    }
    store_f32<V>(a.out + size_t(t) * a.H + h, acc);
}

hf_status launch_combine(const CombineArgs& a, cudaStream_t st) {
    if (a.y16 && a.H % 8) return fail(HF_ERR_ARG, "combine: FP16 outputs need H % 8 == 0");
    const size_t n = size_t(a.T) * (a.H / (a.y16 ? 8 : 4));
    if (n == 0) return HF_OK;
    if (a.y16)
        HF_CUDA(launch_pdl(k_combine<true>, dim3(unsigned((n + 255) / 256)), dim3(256), 0, st, a));
    else
        HF_CUDA(launch_pdl(k_combine<false>, dim3(unsigned((n + 255) / 256)), dim3(256), 0, st, a));
    return HF_OK;
}

// ============================================================ gemv_bf16_f32 twin
// compute/cpu_kernels.cpp:43-94: y[i] = alpha * dot(A[i,:], x) + beta * y[i],
// y read even when beta == 0. The call sites (the attention projections,
// glm_forward.cpp:314-408, and the router) are single vectors, so the kernel is
// a pure weight stream. A block of 256 threads is cut into 256 / TPR groups;
// a group owns R rows and its TPR threads walk them together in 16-byte chunks
// (contiguous spans of TPR * 16 bytes per row), 8 / R chunks of each row in
// flight per thread (eight 16-byte loads), x from L1; the partial sums of each
// row are added across the group. TPR follows K (short rows: small groups, so
// no thread idles) and R the row-block size; the grid is persistent (the
// resident blocks of all SMs walk the row blocks), so no wave tail or block
// turnover leaves an SM without loads in flight.
template <int R, int TPR>
__global__ void __launch_bounds__(256) k_gemv_rows(const uint16_t* __restrict__ A,
                                                   const float* __restrict__ x, float* y, int M,
                                                   int K, float alpha, float beta) {
    constexpr int G = 256 / TPR, WPG = TPR / 32, U = 8 / R;
    const int grp = threadIdx.x / TPR, t = threadIdx.x % TPR;
    const int nc = K >> 3;  // 16-byte chunks per row
    const int nblk = (M + G * R - 1) / (G * R);
    __shared__ float part[8][R];
    // persistent: the grid fills the SMs once and walks the row blocks
    for (int bi = blockIdx.x; bi < nblk; bi += gridDim.x) {
    const int r0 = (bi * G + grp) * R;
    const uint16_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = A + size_t(min(r0 + r, M - 1)) * K;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    const float4* xv = reinterpret_cast<const float4*>(x);
    int c = t;
    // U chunks of each of the R rows per thread in flight (R * U = 8 loads)
    for (; c + (U - 1) * TPR < nc; c += U * TPR) {
        uint4 w[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int r = 0; r < R; ++r) w[u][r] = ld_stream_u4(rows[r] + size_t(c + u * TPR) * 8);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int cu = c + u * TPR;
            const float4 a0 = __ldg(xv + 2 * cu), a1 = __ldg(xv + 2 * cu + 1);
            const float xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float f[8];
                unpack8(w[u][r], f);
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[r] = fmaf(f[e], xa[e], acc[r]);
            }
        }
    }
    for (; c < nc; c += TPR) {
        const float4 a0 = __ldg(xv + 2 * c), a1 = __ldg(xv + 2 * c + 1);
        const float xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float f[8];
            unpack8(ld_stream_u4(rows[r] + size_t(c) * 8), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r] = fmaf(f[e], xa[e], acc[r]);
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float v = warp_sum(acc[r]);
        if (lane == 0) part[warp][r] = v;
    }
    __syncthreads();
    if (threadIdx.x < G * R) {
        const int g = threadIdx.x / R, r = threadIdx.x % R;
        const int row = (bi * G + g) * R + r;
        if (row < M) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < WPG; ++w) v += part[g * WPG + w][r];
            y[row] = __fadd_rn(__fmul_rn(alpha, v), __fmul_rn(beta, y[row]));
        }
    }
    __syncthreads();  // part[] is rewritten by the next row block
    }
}

// Launches one persistent grid: at most the resident blocks of all SMs.
template <int R, int TPR>
cudaError_t launch_rows(unsigned nblk, int dev, const uint16_t* A, const float* x, float* y,
                        int M, int K, float alpha, float beta, cudaStream_t st) {
    static std::atomic<int> per_sm{0};
    int b = per_sm.load(std::memory_order_relaxed);
    if (b == 0) {
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_gemv_rows<R, TPR>,
                                                                      256, 0);
        if (e != cudaSuccess || b <= 0) b = 1;
        per_sm.store(b, std::memory_order_relaxed);
    }
    const unsigned grid = std::min<unsigned>(nblk, unsigned(b * num_sms(dev)));
    k_gemv_rows<R, TPR><<<grid, 256, 0, st>>>(A, x, y, M, K, alpha, beta);
    return cudaGetLastError();
}

template <int TPR>
cudaError_t launch_gemv_tpr(int R, unsigned nblk, int dev, const uint16_t* A, const float* x,
                            float* y, int M, int K, float alpha, float beta, cudaStream_t st) {
    switch (R) {
        case 8: return launch_rows<8, TPR>(nblk, dev, A, x, y, M, K, alpha, beta, st);
        case 4: return launch_rows<4, TPR>(nblk, dev, A, x, y, M, K, alpha, beta, st);
        case 2: return launch_rows<2, TPR>(nblk, dev, A, x, y, M, K, alpha, beta, st);
        default: return launch_rows<1, TPR>(nblk, dev, A, x, y, M, K, alpha, beta, st);
    }
}

// Any K or alignment: one warp per row, scalar loads.
__global__ void __launch_bounds__(256) k_gemv_plain(const uint16_t* A, const float* x, float* y,
                                                    int M, int K, float alpha, float beta) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= M) return;
    const uint16_t* ar = A + size_t(row) * K;
    float acc = 0.0f;
    for (int j = lane; j < K; j += 32) acc = fmaf(bf16_to_f32(ar[j]), __ldg(x + j), acc);
    acc = warp_sum(acc);
    if (lane == 0) y[row] = __fadd_rn(__fmul_rn(alpha, acc), __fmul_rn(beta, y[row]));
}

hf_status launch_gemv_plain(const uint16_t* A, const float* x, float* y, int M, int K,
                            float alpha, float beta, cudaStream_t st) {
    if (M == 0) return HF_OK;
    const bool vec = (K % 8 == 0) && (reinterpret_cast<uintptr_t>(A) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    if (!vec) {
        k_gemv_plain<<<(M + 7) / 8, 256, 0, st>>>(A, x, y, M, K, alpha, beta);
    } else {
        // threads per row group: two or more chunks each. Rows per group: 4
        // while there are as many row blocks as SMs (a sweep of 1, 2, 4 and 8
        // rows and of 2, 4 and 8 chunks per thread on the attention shapes:
        // 4 rows and 2 chunks fastest or within 5 % everywhere but q_b, where
        // 8 chunks gain 15 %), else 2, else 1.
        const int nc = K / 8;
        const int tpr = nc >= 512 ? 256 : nc >= 256 ? 128 : nc >= 128 ? 64 : 32;
        const int G = 256 / tpr;
        int dev = 0;
        HF_CUDA(cudaGetDevice(&dev));
        const long long nsm = num_sms(dev);
        int R = 1;
        for (int r : {4, 2})
            if ((M + G * r - 1) / (G * r) >= nsm) {
                R = r;
                break;
            }

        const unsigned g = unsigned((M + G * R - 1) / (G * R));
        cudaError_t e;
        switch (tpr) {
            case 256: e = launch_gemv_tpr<256>(R, g, dev, A, x, y, M, K, alpha, beta, st); break;
            case 128: e = launch_gemv_tpr<128>(R, g, dev, A, x, y, M, K, alpha, beta, st); break;
            case 64: e = launch_gemv_tpr<64>(R, g, dev, A, x, y, M, K, alpha, beta, st); break;
            default: e = launch_gemv_tpr<32>(R, g, dev, A, x, y, M, K, alpha, beta, st); break;
        }
        HF_CUDA(e);
    }
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

}  // namespace hf
