// hf_noalloc.cu -- routing for callers that cannot allocate device memory.
//
// hf_moe_route_noalloc runs the same router-logits and single-block routing
// kernels as hf_moe_route, but its scratch (router logits, the work plan and
// the slot -> position table) lives in the file-scope array below instead of
// memory from cudaMalloc. It exists for callers that cannot allocate: an
// engine that has handed all device memory to its resident expert weights up
// front, or code on a latency-critical decode path that must not take the
// device-wide synchronization cudaMalloc/cudaFree can imply.
//
// Rules of use:
// * Sizes: T <= 128 tokens, E <= 256 experts, k <= 8 (the array holds
//   128 x 256 fp32 logits plus the plan); larger calls get HF_ERR_ARG.
// * The array is one per device and lives until the process exits.
// * The first call on a device looks up the array's device address
//   (cudaGetSymbolAddress, with that device current); make that first call
//   before any stream capture.
// * Every call on a device shares the array: calls whose kernels can overlap
//   on the GPU (different streams, no ordering) race and corrupt each other.
//   Calls ordered on one stream are safe. Nothing in the array has to start at
//   zero: each call writes every word it later reads.
#include <mutex>

#include "hf_internal.cuh"

namespace hf {
namespace {

constexpr int kNaMaxT = kSmallRouteT;  // single-block routing limit
constexpr int kNaMaxE = 256;
constexpr int kNaMaxG = kNaMaxE + 1;
constexpr size_t kNaLogitsBytes = size_t(kNaMaxT) * kNaMaxE * sizeof(float);
constexpr size_t kNaPlanWords = size_t(kNaMaxG) + 5 * size_t(kNaMaxG + 1) + 4;
constexpr size_t kNaSlotWords = size_t(kNaMaxT) * (kMaxTopK + 1);
constexpr size_t kNaBytes =
    kNaLogitsBytes + 256 * ((kNaPlanWords * 4 + 255) / 256) + 256 * ((kNaSlotWords * 4 + 255) / 256);

static __device__ __align__(256) unsigned char g_route_scratch[kNaBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the array on the current device (looked up once).
hf_status scratch_for_current_device(unsigned char** out) {
    int dev = -1;
    HF_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(HF_ERR_ARG, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_route_scratch)");
        g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_scratch_ptr[dev];
    return HF_OK;
}

}  // namespace
}  // namespace hf

using namespace hf;

extern "C" hf_status hf_moe_route_noalloc(const uint16_t* router_bf16, const float* bias,
                                          const void* x, hf_dtype x_dtype, int T, int H, int E,
                                          int top_k, float routed_scaling_factor,
                                          int norm_topk_prob, int has_shared, int32_t* topk_ids,
                                          float* topk_weights, int32_t* counts, int32_t* offsets,
                                          int32_t* perm, hf_stream stream) {
    if (T < 0 || T > kNaMaxT)
        return fail(HF_ERR_ARG, "hf_moe_route_noalloc: T must be in 0..128 (static scratch limit)");
    if (E <= 0 || E > kNaMaxE)
        return fail(HF_ERR_ARG, "hf_moe_route_noalloc: E must be in 1..256 (static scratch limit)");
    if (top_k <= 0 || top_k > kMaxTopK)
        return fail(HF_ERR_ARG, "hf_moe_route_noalloc: top_k must be in 1..8");
    if (H <= 0 || H % 8) return fail(HF_ERR_ARG, "hf_moe_route_noalloc: H must be a positive multiple of 8");
    if (x_dtype != HF_BF16 && x_dtype != HF_F32)
        return fail(HF_ERR_ARG, "hf_moe_route_noalloc: x_dtype must be HF_BF16 or HF_F32");
    if (T > 0 && (!router_bf16 || !x || !topk_ids || !topk_weights || !counts || !offsets || !perm))
        return fail(HF_ERR_ARG, "hf_moe_route_noalloc: null pointer");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_bf16)) & 15)
        return fail(HF_ERR_ARG, "hf_moe_route_noalloc: x and router must be 16-byte aligned");
    unsigned char* base = nullptr;
    HF_TRY(scratch_for_current_device(&base));
    cudaStream_t st = as_cuda(stream);
    const int k = top_k < E ? top_k : E;
    const int G = E + 1;
    if (T == 0) {  // an empty batch: every count and offset is zero (as hf_moe_route reports)
        if (counts) HF_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * G, st));
        if (offsets) HF_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (G + 1), st));
        return HF_OK;
    }
    RouteArgs a{};
    a.x = x;
    a.x_f32 = x_dtype == HF_F32;
    a.T = T;
    a.H = H;
    a.E = E;
    a.k = k;
    a.router = router_bf16;
    a.bias = bias;
    a.scale = routed_scaling_factor;
    a.norm = norm_topk_prob;
    a.logits = reinterpret_cast<float*>(base);
    a.plan = reinterpret_cast<int32_t*>(base + kNaLogitsBytes);
    a.pl = PlanLayout::make(G);
    a.slot_pos = reinterpret_cast<int32_t*>(base + kNaLogitsBytes +
                                            256 * ((kNaPlanWords * 4 + 255) / 256));
    a.ids = topk_ids;
    a.w = topk_weights;
    a.margins = nullptr;
    a.has_shared = has_shared != 0;
    a.inter = 64;  // the work plan's unit counts are not returned by this entry
    a.shared_inter = has_shared ? 64 : 0;
    a.perm = perm;
    a.masks = nullptr;
    a.blk_counts = nullptr;
    a.path = HF_PATH_GEMV;
    a.gemv_max = 1 << 30;
    a.gemm_ok = 0;
    a.gemm_bn1 = a.gemm_bn2 = 64;
    a.lsplit = 1;
    a.gemm_m1 = a.gemm_m2 = 128;
    a.gemm_pair = 0;
    HF_TRY(launch_router_logits(a, st));
    int n = 0;
    HF_TRY(launch_route(a, st, &n));
    HF_CUDA(cudaMemcpyAsync(counts, a.plan + a.pl.counts, sizeof(int32_t) * G,
                            cudaMemcpyDeviceToDevice, st));
    HF_CUDA(cudaMemcpyAsync(offsets, a.plan + a.pl.offsets, sizeof(int32_t) * (G + 1),
                            cudaMemcpyDeviceToDevice, st));
    return HF_OK;
}
