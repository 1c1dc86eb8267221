// hf_norm.cu -- RMSNorm of the hidden states in front of the MLP block and
// its hand-off to the MoE / dense kernels (GLMForward::rmsNorm,
// glm_forward.cpp:185-197, called at :785-786 on postAttentionLayernorm).
//
// The reference, per token of n = H values:
//   sq  = sum_i x_i * x_i               (fp32, i ascending)
//   rms = 1 / sqrt(sq / n + eps)        (fp32, IEEE divide and sqrt)
//   x_i = x_i * rms * w_i               (w BF16 widened; x_i * rms when the
//                                        weight pointer is missing, :194-195)
// Here one block per token holds the row in registers (1024 threads while
// the tokens are fewer than two per SM, else 256; rows too long for 8 float4
// per thread take a two-pass kernel that re-reads them), sums the squares per
// thread (fma) and across the block, and writes the normalised values in the
// form the next kernel consumes:
//   kNormF32   fp32 [T x H]                    (the reference's hand-off)
//   kNormBf16  bf16 [T x H], RNE               (tensor-core router and GEMM read it in place)
//   kNormHiLo  bf16 hi [T x H] + lo [T x H]     (v = hi + lo to 16 mantissa bits: the
//                                                operand pair of the fp32 GEMM path)
// Only the squares' summation order differs from the reference (a relative
// difference of ~1e-7 in rms); the products and the rms itself are the
// reference's correctly rounded fp32 operations.
#include "hf_internal.cuh"

namespace hf {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint2 pack_bf16x4(float a, float b, float c, float d) {
    uint2 r;
    r.x = uint32_t(f32_to_bf16_rne(a)) | (uint32_t(f32_to_bf16_rne(b)) << 16);
    r.y = uint32_t(f32_to_bf16_rne(c)) | (uint32_t(f32_to_bf16_rne(d)) << 16);
    return r;
}

__device__ __forceinline__ float lo_part(float v) {
    return __fsub_rn(v, bf16_to_f32(f32_to_bf16_rne(v)));
}

template <int MODE>
__device__ __forceinline__ void store_row(float4 y, size_t o, void* out, uint16_t* out_lo) {
    if constexpr (MODE == kNormF32) {
        reinterpret_cast<float4*>(out)[o] = y;
    } else {
        reinterpret_cast<uint2*>(out)[o] = pack_bf16x4(y.x, y.y, y.z, y.w);
        if constexpr (MODE == kNormHiLo)
            reinterpret_cast<uint2*>(out_lo)[o] =
                pack_bf16x4(lo_part(y.x), lo_part(y.y), lo_part(y.z), lo_part(y.w));
    }
}

// x * rms, then * w (glm_forward.cpp:193, left to right)
__device__ __forceinline__ float4 scale_row(float4 v, float rms, const uint16_t* w, int i) {
    float4 y = make_float4(__fmul_rn(v.x, rms), __fmul_rn(v.y, rms), __fmul_rn(v.z, rms),
                           __fmul_rn(v.w, rms));
    if (w) {
        const uint2 wb = reinterpret_cast<const uint2*>(w)[i];
        y.x = __fmul_rn(y.x, __uint_as_float(wb.x << 16));
        y.y = __fmul_rn(y.y, __uint_as_float(wb.x & 0xffff0000u));
        y.z = __fmul_rn(y.z, __uint_as_float(wb.y << 16));
        y.w = __fmul_rn(y.w, __uint_as_float(wb.y & 0xffff0000u));
    }
    return y;
}

// Sum over the block (<= 1024 threads); every thread gets rms.
__device__ __forceinline__ float block_rms(float sq, int H, float eps) {
    __shared__ float red[32];
    __shared__ float rms_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    if (warp == 0) {
        float v = lane < nw ? red[lane] : 0.f;
        v = warp_sum(v);
        if (lane == 0) rms_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, float(H)), eps)));
    }
    __syncthreads();
    return rms_s;
}

// Row held in registers: V float4 per thread, all loads in flight at once
// (decode: one block of 1024 threads per token; batches: 256).
template <int MODE, int V>
__global__ void __launch_bounds__(1024) k_rmsnorm_reg(const float* __restrict__ x,
                                                      const uint16_t* __restrict__ w, float eps,
                                                      int H, void* out, uint16_t* out_lo) {
    const int t = blockIdx.x, H4 = H >> 2, nt = blockDim.x;
    const float4* xr = reinterpret_cast<const float4*>(x + size_t(t) * H);
    float4 v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * nt;
        v[j] = i < H4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
        sq = fmaf(v[j].x, v[j].x, sq);
        sq = fmaf(v[j].y, v[j].y, sq);
        sq = fmaf(v[j].z, v[j].z, sq);
        sq = fmaf(v[j].w, v[j].w, sq);
    }
    const float rms = block_rms(sq, H, eps);
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * nt;
        if (i < H4) store_row<MODE>(scale_row(v[j], rms, w, i), size_t(t) * H4 + i, out, out_lo);
    }
}

// Any H: pass 2 re-reads the row (an L1 / L2 hit).
template <int MODE>
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm(const float* __restrict__ x,
                                                          const uint16_t* __restrict__ w,
                                                          float eps, int H, void* out,
                                                          uint16_t* out_lo) {
    const int t = blockIdx.x;
    const int H4 = H >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + size_t(t) * H);
    float sq = 0.f;
    for (int i = threadIdx.x; i < H4; i += kNormThreads) {
        const float4 v = xr[i];
        sq = fmaf(v.x, v.x, sq);
        sq = fmaf(v.y, v.y, sq);
        sq = fmaf(v.z, v.z, sq);
        sq = fmaf(v.w, v.w, sq);
    }
    const float rms = block_rms(sq, H, eps);
    for (int i = threadIdx.x; i < H4; i += kNormThreads)
        store_row<MODE>(scale_row(xr[i], rms, w, i), size_t(t) * H4 + i, out, out_lo);
}

template <int MODE>
void launch_mode(const float* x, const uint16_t* w, float eps, int T, int H, void* out,
                 uint16_t* out_lo, cudaStream_t st) {
    const int H4 = H >> 2;
    // few tokens: wide blocks so each row's loads are issued together
    const int nt = T < 2 * 148 ? 1024 : kNormThreads;
    const int v = (H4 + nt - 1) / nt;
    const unsigned grid = unsigned(T);
    if (v <= 1) k_rmsnorm_reg<MODE, 1><<<grid, nt, 0, st>>>(x, w, eps, H, out, out_lo);
    else if (v <= 2) k_rmsnorm_reg<MODE, 2><<<grid, nt, 0, st>>>(x, w, eps, H, out, out_lo);
    else if (v <= 4) k_rmsnorm_reg<MODE, 4><<<grid, nt, 0, st>>>(x, w, eps, H, out, out_lo);
    else if (v <= 8) k_rmsnorm_reg<MODE, 8><<<grid, nt, 0, st>>>(x, w, eps, H, out, out_lo);
    else k_rmsnorm<MODE><<<grid, kNormThreads, 0, st>>>(x, w, eps, H, out, out_lo);
}

}  // namespace

hf_status launch_rmsnorm(const float* x, const uint16_t* w, float eps, int T, int H, int mode,
                         void* out, uint16_t* out_lo, cudaStream_t st) {
    if (T <= 0) return HF_OK;
    switch (mode) {
        case kNormF32: launch_mode<kNormF32>(x, w, eps, T, H, out, out_lo, st); break;
        case kNormBf16: launch_mode<kNormBf16>(x, w, eps, T, H, out, out_lo, st); break;
        case kNormHiLo: launch_mode<kNormHiLo>(x, w, eps, T, H, out, out_lo, st); break;
        default: return fail(HF_ERR_ARG, "launch_rmsnorm: bad output mode");
    }
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

}  // namespace hf

using namespace hf;

extern "C" {

hf_status hf_rmsnorm(const float* x, const uint16_t* weight, float eps, int T, int H, void* out,
                     hf_dtype out_dtype, hf_stream stream) {
    if (T < 0 || H <= 0 || H % 4) return fail(HF_ERR_ARG, "hf_rmsnorm: T >= 0 and H a multiple of 4");
    if (T == 0) return HF_OK;
    if (!x || !out) return fail(HF_ERR_ARG, "hf_rmsnorm: null pointer");
    if (out_dtype != HF_F32 && out_dtype != HF_BF16)
        return fail(HF_ERR_ARG, "hf_rmsnorm: out_dtype must be HF_F32 or HF_BF16");
    const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!a16(x) || !a16(out) || (weight && !a16(weight)))
        return fail(HF_ERR_ARG, "hf_rmsnorm: pointers must be 16-byte aligned");
    return launch_rmsnorm(x, weight, eps, T, H, out_dtype == HF_F32 ? kNormF32 : kNormBf16, out,
                          nullptr, as_cuda(stream));
}

}  // extern "C"
