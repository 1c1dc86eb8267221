// hf_synth.cu -- seeded synthetic tensors written directly into HBM.
//
// No reference counterpart (the reference loads the GLM-5.2 checkpoint,
// model/weight_index.cpp). Formulas: splitmix64 mixing of (key + (i+1) *
// golden), Irwin-Hall(4) normal from the four 16-bit lanes (integer sum, one
// fp32 multiply), RNE to BF16 as BFloat16::fromF32 (compute/dtype_bf16.h:27-33);
// uniform = lo + (hi - lo) * u24 * 2^-24 with explicit round-to-nearest fp32
// operations. A host implementation of the same formulas gives the same bits.
#include <math.h>

#include "hf_internal.cuh"
#include "hf_synth.h"

namespace hf {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ULL;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBULL;
    z ^= z >> 31;
    return z;
}

uint64_t synth_key(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert) {
    const uint64_t k = mix64(seed + kGolden);
    return mix64(k ^ ((uint64_t(layer) << 40) | (uint64_t(kind) << 32) | uint64_t(expert)));
}

float synth_normal_scale(double sigma) { return float(sigma / sqrt(1431655765.0)); }

__device__ __forceinline__ uint16_t normal_bf16(uint64_t key, uint64_t i, float scale) {
    const uint64_t b = mix64(key + (i + 1) * kGolden);
    const int32_t s = int32_t(b & 0xFFFFu) + int32_t((b >> 16) & 0xFFFFu) +
                      int32_t((b >> 32) & 0xFFFFu) + int32_t(b >> 48);
    return f32_to_bf16_rne(__fmul_rn(__int2float_rn(s - 131070), scale));
}

__global__ void k_synth_bf16(uint16_t* dst, uint64_t n, uint64_t key, float scale) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x * 8;
    for (uint64_t i0 = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i0 < n;
         i0 += stride) {
        if (i0 + 8 <= n && (reinterpret_cast<uintptr_t>(dst + i0) & 15) == 0) {
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                w[q] = uint32_t(normal_bf16(key, i0 + 2 * q, scale)) |
                       (uint32_t(normal_bf16(key, i0 + 2 * q + 1, scale)) << 16);
            *reinterpret_cast<uint4*>(dst + i0) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
            for (uint64_t i = i0; i < n && i < i0 + 8; ++i) dst[i] = normal_bf16(key, i, scale);
        }
    }
}

__global__ void k_synth_f32u(float* dst, uint64_t n, uint64_t key, float lo, float hi) {
    const float w = __fsub_rn(hi, lo);
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t b = mix64(key + (i + 1) * kGolden);
        const float t = __fmul_rn(__uint2float_rn(uint32_t(b >> 40)), 5.9604644775390625e-08f);
        dst[i] = __fadd_rn(lo, __fmul_rn(w, t));
    }
}

hf_status synth_bf16(uint16_t* dst, uint64_t n, uint64_t key, float scale, cudaStream_t st) {
    if (n == 0) return HF_OK;
    const uint64_t blocks = (n + 8 * 256 - 1) / (8 * 256);
    const unsigned grid = unsigned(blocks < 148ull * 64 ? blocks : 148ull * 64);
    k_synth_bf16<<<grid, 256, 0, st>>>(dst, n, key, scale);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

hf_status synth_f32u(float* dst, uint64_t n, uint64_t key, float lo, float hi, cudaStream_t st) {
    if (n == 0) return HF_OK;
    const uint64_t blocks = (n + 255) / 256;
    const unsigned grid = unsigned(blocks < 148ull * 16 ? blocks : 148ull * 16);
    k_synth_f32u<<<grid, 256, 0, st>>>(dst, n, key, lo, hi);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

}  // namespace hf

extern "C" hf_status hf_synth_bf16_normal(uint16_t* dst, uint64_t n, uint64_t seed,
                                          uint32_t layer, uint32_t kind, uint32_t expert,
                                          double sigma, hf_stream stream) {
    if (!dst && n) return hf::fail(HF_ERR_ARG, "hf_synth_bf16_normal: null dst");
    return hf::synth_bf16(dst, n, hf::synth_key(seed, layer, kind, expert),
                          hf::synth_normal_scale(sigma), hf::as_cuda(stream));
}

extern "C" hf_status hf_synth_f32_uniform(float* dst, uint64_t n, uint64_t seed, uint32_t layer,
                                          uint32_t kind, uint32_t expert, float lo, float hi,
                                          hf_stream stream) {
    if (!dst && n) return hf::fail(HF_ERR_ARG, "hf_synth_f32_uniform: null dst");
    return hf::synth_f32u(dst, n, hf::synth_key(seed, layer, kind, expert), lo, hi,
                          hf::as_cuda(stream));
}
