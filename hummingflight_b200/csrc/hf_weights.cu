// hf_weights.cu -- resident format of the down projections (FP16 down pass).
//
// The down GEMM multiplies the expert's down rows [H x I] by the SwiGLU
// intermediate mid. With BF16 operands mid must be split into a BF16 hi + lo
// pair (BF16 alone rounds mid to 8 bits: rel-L2 1.65e-3 against the
// reference's fp32 mid, above the 1e-3 bar), which doubles the down GEMM's
// MMAs. Stored as FP16, the weights keep every bit of their BF16 values and
// mid gets 11 bits, so one MMA pass suffices (rel-L2 ~2e-4):
//
//   * each down block is scaled by a power of two 2^S chosen from its largest
//     |w| (max * 2^S in [2^14, 2^15)), so every BF16 value whose magnitude is
//     at least max * 2^-29 converts exactly (smaller ones round to FP16's
//     subnormal step, an absolute error below max * 2^-40);
//   * the conversion runs on the device when a forward finds blocks written
//     since the last one (the weight setters, the generator and the
//     checkpoint loader write the reference's BF16 layout), and runs back to
//     BF16 -- exactly -- when a caller asks for a block's address to read or
//     write it in place (hf_moe_expert_device_ptr), so the API only ever shows
//     the [gate | up | down] BF16 layout of Scheduler::getExpertPtr
//     (engine/scheduler.h:80-84);
//   * a layer whose down weights hold Inf or NaN keeps BF16 (the hi + lo pass).
// The reference has no counterpart: its expertFFNRaw (model/glm_forward.cpp:
// 434-449) multiplies the BF16 rows by the fp32 mid on the CPU.
#include <cuda_fp16.h>

#include <cstdlib>
#include <vector>

#include "hf_ctx.cuh"

namespace hf {

constexpr unsigned kBf16NonFinite = 0x7f80u;  // |bits| from here on: Inf or NaN

// Largest |w| of each listed block, as BF16 magnitude bits (ordered like the
// values for finite numbers). Grid: x strides the block, y = list entry.
__global__ void __launch_bounds__(256) k_down_absmax(uint16_t* const* blocks, const int* list,
                                                     size_t n_routed, size_t n_shared, int G,
                                                     unsigned* absmax) {
    const int g = list[blockIdx.y];
    const size_t n = g == G - 1 ? n_shared : n_routed;
    const uint4* p = reinterpret_cast<const uint4*>(blocks[g]);
    unsigned m = 0;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n / 8;
         i += size_t(gridDim.x) * blockDim.x) {
        const uint4 v = p[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            m = max(m, w[q] & 0x7fffu);
            m = max(m, (w[q] >> 16) & 0x7fffu);
        }
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0) atomicMax(absmax + g, m);
}

// 2^S for a block whose largest magnitude has BF16 bits `m`: max * 2^S lands
// in [2^14, 2^15) (S = 141 - biased exponent), clamped so 2^S stays a normal
// fp32; 0 for an all-zero block.
__device__ __forceinline__ int down_shift(unsigned m) {
    if (m == 0) return 0;
    const int e = int(m >> 7);
    return max(-100, min(100, 141 - e));
}
__device__ __forceinline__ float pow2(int s) { return __int_as_float((s + 127) << 23); }

__global__ void __launch_bounds__(256) k_down_to_f16(uint16_t* const* blocks, const int* list,
                                                     size_t n_routed, size_t n_shared, int G,
                                                     const unsigned* absmax, float* scale) {
    const int g = list[blockIdx.y];
    const size_t n = g == G - 1 ? n_shared : n_routed;
    const int S = down_shift(absmax[g]);
    const float up = pow2(S);
    uint4* p = reinterpret_cast<uint4*>(blocks[g]);
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n / 8;
         i += size_t(gridDim.x) * blockDim.x) {
        const uint4 v = p[i];
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float lo = __fmul_rn(__uint_as_float(w[q] << 16), up);
            const float hi = __fmul_rn(__uint_as_float(w[q] & 0xffff0000u), up);
            const __half2 h = __floats2half2_rn(lo, hi);
            w[q] = *reinterpret_cast<const uint32_t*>(&h);
        }
        p[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) scale[g] = pow2(-S);
}

// Back to BF16 (exact for every value the forward conversion kept exact).
__global__ void __launch_bounds__(256) k_down_to_bf16(uint16_t* const* blocks, const int* list,
                                                      size_t n_routed, size_t n_shared, int G,
                                                      const float* scale) {
    const int g = list[blockIdx.y];
    const size_t n = g == G - 1 ? n_shared : n_routed;
    const float down = scale[g];
    uint4* p = reinterpret_cast<uint4*>(blocks[g]);
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n / 8;
         i += size_t(gridDim.x) * blockDim.x) {
        const uint4 v = p[i];
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[q]);
            const float2 f = __half22float2(h);
            const uint32_t lo = f32_to_bf16_rne(__fmul_rn(f.x, down));
            const uint32_t hi = f32_to_bf16_rne(__fmul_rn(f.y, down));
            w[q] = lo | (hi << 16);
        }
        p[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// The format flags and scales of the listed groups in the device table the
// GEMV and GEMM read (after the conversion kernels, stream-ordered).
__global__ void k_down_flags(GroupW* groups, const int* list, int n, int f16, const float* scale) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int g = list[i];
        groups[g].down_f16 = f16;
        groups[g].down_scale = f16 ? scale[g] : 1.0f;
    }
}

static bool down_f16_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("HF_DOWN_F16");  // tuning knob: 0 keeps the BF16 hi + lo pass
        return !(e && std::atoi(e) == 0);
    }();
    return on;
}

static hf_status convert(hf_moe_ctx* c, LayerBuf& L, const std::vector<int>& list, bool to_f16,
                         cudaStream_t st) {
    if (list.empty()) return HF_OK;
    const int G = c->G;
    HF_CUDA(cudaMemcpyAsync(L.d_list, list.data(), sizeof(int) * list.size(),
                            cudaMemcpyHostToDevice, st));
    const size_t nr = size_t(c->H) * c->I, ns = size_t(c->H) * c->Is;
    const dim3 grid(unsigned(std::max(1, c->nsm * 4 / int(list.size()))), unsigned(list.size()));
    if (to_f16) {
        k_down_to_f16<<<grid, 256, 0, st>>>(L.d_blocks, L.d_list, nr, ns, G, L.d_absmax,
                                            L.d_scale);
    } else {
        k_down_to_bf16<<<grid, 256, 0, st>>>(L.d_blocks, L.d_list, nr, ns, G, L.d_scale);
    }
    HF_CUDA(cudaGetLastError());
    k_down_flags<<<1, 256, 0, st>>>(L.groups, L.d_list, int(list.size()), to_f16 ? 1 : 0, L.d_scale);
    HF_CUDA(cudaGetLastError());
    HF_CUDA(cudaStreamSynchronize(st));  // the host list is reused; this runs after weight changes only
    for (int g : list) L.dfmt[size_t(g)] = to_f16 ? 1 : 0;
    return HF_OK;
}

static hf_status down_tables(hf_moe_ctx* c, LayerBuf& L) {
    if (L.d_blocks) return HF_OK;
    const int G = c->G;
    std::vector<uint16_t*> b(static_cast<size_t>(G), nullptr);
    for (int g = 0; g < G; ++g) {
        if (g < c->E_local) b[size_t(g)] = L.experts + size_t(g) * c->expert_elems + size_t(2) * c->I * c->H;
        else if (g == G - 1 && c->Is > 0) b[size_t(g)] = L.shared + size_t(2) * c->Is * c->H;
    }
    HF_TRY(dalloc(&L.d_blocks, size_t(G)));
    HF_TRY(dalloc(&L.d_list, size_t(G)));
    HF_TRY(dalloc(&L.d_absmax, size_t(G)));
    HF_TRY(dalloc(&L.d_scale, size_t(G)));
    HF_CUDA(cudaMemcpy(L.d_blocks, b.data(), sizeof(uint16_t*) * G, cudaMemcpyHostToDevice));
    L.dfmt.assign(size_t(G), 0);
    return HF_OK;
}

// Before a forward: every down block of the layer in FP16 (L.down_f16), or
// every one in BF16 when a block holds a non-finite weight or the FP16 pass
// is switched off.
hf_status ensure_down_format(hf_moe_ctx* c, LayerBuf& L, cudaStream_t st) {
    if (L.down_ready) return HF_OK;
    HF_TRY(down_tables(c, L));
    const int G = c->G;
    std::vector<int> raw, f16;
    for (int g = 0; g < G; ++g) {
        if (g == G - 1 && c->Is == 0) continue;
        (L.dfmt[size_t(g)] ? f16 : raw).push_back(g);
    }
    bool want = down_f16_enabled() && c->gemm_ok;
    if (want && !raw.empty()) {
        HF_CUDA(cudaMemsetAsync(L.d_absmax, 0, sizeof(unsigned) * G, st));
        HF_CUDA(cudaMemcpyAsync(L.d_list, raw.data(), sizeof(int) * raw.size(),
                                cudaMemcpyHostToDevice, st));
        const size_t nr = size_t(c->H) * c->I, ns = size_t(c->H) * c->Is;
        const dim3 grid(unsigned(std::max(1, c->nsm * 4 / int(raw.size()))), unsigned(raw.size()));
        k_down_absmax<<<grid, 256, 0, st>>>(L.d_blocks, L.d_list, nr, ns, G, L.d_absmax);
        HF_CUDA(cudaGetLastError());
        std::vector<unsigned> m(static_cast<size_t>(G));
        HF_CUDA(cudaMemcpyAsync(m.data(), L.d_absmax, sizeof(unsigned) * G, cudaMemcpyDeviceToHost, st));
        HF_CUDA(cudaStreamSynchronize(st));
        for (int g : raw) want = want && m[size_t(g)] < kBf16NonFinite;
    }
    if (want) {
        HF_TRY(convert(c, L, raw, true, st));
    } else {
        HF_TRY(convert(c, L, f16, false, st));
    }
    L.down_f16 = want;
    L.down_ready = true;
    return HF_OK;
}

// A block about to be read or written in place through its device address
// (or overwritten by a weight setter) goes back to the BF16 layout.
hf_status down_to_bf16(hf_moe_ctx* c, LayerBuf& L, int g) {
    L.down_ready = false;
    if (!L.d_blocks || g < 0 || g >= c->G || !L.dfmt[size_t(g)]) return HF_OK;
    return convert(c, L, std::vector<int>{g}, false, nullptr);
}

// Weights written over (BF16 again, in the reference layout).
void down_written(LayerBuf& L, int g) {
    L.down_ready = false;
    if (L.dfmt.empty()) return;
    if (g < 0) L.dfmt.assign(L.dfmt.size(), 0);
    else if (size_t(g) < L.dfmt.size()) L.dfmt[size_t(g)] = 0;
}

}  // namespace hf
