// ref_harness.cpp -- drives the reference's own CPU MoE math (test infrastructure).
//
// Built by oracle/Makefile into oracle/_ref/ together with the UNMODIFIED
// reference translation unit compute/cpu_kernels.cpp and header
// compute/moe_router.h, compiled from the reference source tree. Two builds:
//   libhfref_avx2.so   cpu_kernels.cpp with -mavx2 -mfma -D_MSC_VER=1930, which
//                      selects its AVX2 branch (cpu_kernels.cpp:47-81; that
//                      branch is compiled only under _MSC_VER)
//   libhfref_scalar.so cpu_kernels.cpp as GCC builds it on Linux (:82-93)
//
// The glue of GLMForward::moeLayer (model/glm_forward.cpp:509-661) and
// expertFFNRaw (:434-449) is restated here in the same order, calling the
// reference's glm::gemv_bf16_f32 and glm::topKScores. Weights come from the
// seeded generator in oracle/hf_gen.h, so the GPU run and this harness see the
// same bytes. Used to validate oracle/hf_oracle.c, to write tests/golden/, and
// as bench.py's timed CPU baseline.
#include "compute/cpu_kernels.h"
#include "compute/dtype_bf16.h"
#include "compute/moe_router.h"

#include "hf_gen.h"

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <thread>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

using glm::BFloat16;

namespace {

struct Layer {
    int H = 0, E = 0, K = 0, I = 0, Is = 0;
    float scale = 2.5f;
    bool norm = true;
    uint64_t seed = 0;
    uint32_t layer = 0;
    std::vector<BFloat16> router;
    std::vector<float> bias;
    std::map<int, std::vector<BFloat16>> experts;  // eid (E = shared) -> [g|u|d]
    // per-call workspace, as GLMForward::ws_ (glm_forward.h)
    std::vector<float> scores, gate, up, mid, expertOut, moeOut, sharedOut;
};

void genExpert(Layer& L, int e) {
    if (L.experts.count(e)) return;
    const int I = (e == L.E) ? L.Is : L.I;
    const uint64_t n = uint64_t(L.H) * uint64_t(I);
    std::vector<BFloat16> w(3 * n);
    const float sc = hfg_normal_scale(0.02);
    const uint32_t kinds[3] = {HFG_KIND_GATE, HFG_KIND_UP, HFG_KIND_DOWN};
    for (int m = 0; m < 3; ++m) {
        const uint64_t key = hfg_key(L.seed, L.layer, kinds[m], uint32_t(e));
        BFloat16* dst = w.data() + m * n;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < int64_t(n); ++i)
            dst[i] = BFloat16(hfg_f32_to_bf16(hfg_normal(key, uint64_t(i), sc)));
    }
    L.experts.emplace(e, std::move(w));
}

// GLMForward::expertFFNRaw (glm_forward.cpp:434-449)
void expertFFNRaw(Layer& L, const BFloat16* gateW, const BFloat16* upW, const BFloat16* downW,
                  const float* x, float* out, int hidden, int inter) {
    L.gate.resize(inter);
    L.up.resize(inter);
    L.mid.resize(inter);
    glm::gemv_bf16_f32(gateW, x, L.gate.data(), inter, hidden);
    glm::gemv_bf16_f32(upW, x, L.up.data(), inter, hidden);
    for (int i = 0; i < inter; ++i) L.mid[i] = L.gate[i] / (1.0f + std::exp(-L.gate[i])) * L.up[i];
    glm::gemv_bf16_f32(downW, L.mid.data(), out, hidden, inter);
}

// GLMForward::moeLayer (glm_forward.cpp:509-661), CPU branch, no scheduler.
void moeLayer(Layer& L, const float* input, float* output, int* idxOut, float* wOut,
              float* slotOut) {
    const int hidden = L.H, inter = L.I, numExperts = L.E;
    L.scores.resize(numExperts);
    glm::gemv_bf16_f32(L.router.data(), input, L.scores.data(), numExperts, hidden);
    for (int i = 0; i < numExperts; ++i) L.scores[i] = 1.0f / (1.0f + std::exp(-L.scores[i]));
    auto topk = glm::topKScores(L.scores.data(), numExperts, L.bias.data(), L.K, L.scale, L.norm);
    L.moeOut.assign(hidden, 0.0f);
    L.expertOut.resize(hidden);
    for (int i = 0; i < topk.k; ++i) {
        std::fill(L.expertOut.begin(), L.expertOut.end(), 0.0f);
        const int eid = topk.indices[i];
        genExpert(L, eid);
        const BFloat16* eG = L.experts[eid].data();
        const BFloat16* eU = eG + int64_t(inter) * hidden;
        const BFloat16* eD = eU + int64_t(inter) * hidden;
        expertFFNRaw(L, eG, eU, eD, input, L.expertOut.data(), hidden, inter);
        if (slotOut) std::memcpy(slotOut + size_t(i) * hidden, L.expertOut.data(), sizeof(float) * hidden);
        const float w = topk.weights[i];
        for (int j = 0; j < hidden; ++j) L.moeOut[j] += w * L.expertOut[j];
    }
    L.sharedOut.assign(hidden, 0.0f);
    if (L.Is > 0) {  // sharedExpertFFNRaw (glm_forward.cpp:459-479)
        genExpert(L, L.E);
        const BFloat16* g = L.experts[L.E].data();
        const BFloat16* u = g + int64_t(L.Is) * hidden;
        const BFloat16* d = u + int64_t(L.Is) * hidden;
        expertFFNRaw(L, g, u, d, input, L.sharedOut.data(), hidden, L.Is);
        if (slotOut) std::memcpy(slotOut + size_t(L.K) * hidden, L.sharedOut.data(), sizeof(float) * hidden);
    }
    for (int j = 0; j < hidden; ++j) output[j] = L.moeOut[j] + L.sharedOut[j];
    for (int i = 0; i < topk.k; ++i) {
        if (idxOut) idxOut[i] = topk.indices[i];
        if (wOut) wOut[i] = topk.weights[i];
    }
}

}  // namespace

extern "C" {

// glm::gemv_bf16_f32 (compute/cpu_kernels.h:16-17), as built in this library.
void hfr_gemv_bf16_f32(const uint16_t* A, const float* x, float* y, int M, int K, float alpha,
                       float beta) {
    glm::gemv_bf16_f32(reinterpret_cast<const BFloat16*>(A), x, y, M, K, alpha, beta);
}

// glm::topKScores (compute/moe_router.h:29-57). Returns k.
int hfr_topk_scores(const float* scores, int E, const float* bias, int topK, float scale, int norm,
                    int32_t* idx, float* w) {
    auto r = glm::topKScores(scores, E, bias, topK, scale, norm != 0);
    for (int i = 0; i < r.k; ++i) {
        idx[i] = r.indices[i];
        w[i] = r.weights[i];
    }
    return r.k;
}

int hfr_threads(void) { return glm::cpuThreadCount(); }

void* hfr_layer_create(int H, int E, int K, int I, int Is, float scale, int norm, uint64_t seed,
                       uint32_t layer, const float* bias_override) {
    if (H <= 0 || E <= 0 || K <= 0 || K > 8 || I <= 0 || Is < 0) return nullptr;
    auto* L = new Layer();
    L->H = H; L->E = E; L->K = K; L->I = I; L->Is = Is;
    L->scale = scale; L->norm = norm != 0; L->seed = seed; L->layer = layer;
    L->router.resize(size_t(E) * H);
    const uint64_t rk = hfg_key(seed, layer, HFG_KIND_ROUTER, 0);
    const float sc = hfg_normal_scale(0.02);
    for (size_t i = 0; i < L->router.size(); ++i)
        L->router[i] = BFloat16(hfg_f32_to_bf16(hfg_normal(rk, i, sc)));
    L->bias.resize(E);
    const uint64_t bk = hfg_key(seed, layer, HFG_KIND_BIAS, 0);
    for (int i = 0; i < E; ++i)
        L->bias[i] = bias_override ? bias_override[i] : hfg_uniform(bk, uint64_t(i), -0.1f, 0.1f);
    return L;
}

void hfr_layer_destroy(void* h) { delete static_cast<Layer*>(h); }

// Generate (outside any timed region) every expert the given tokens select.
void hfr_layer_prepare(void* h, const float* x, int T) {
    auto& L = *static_cast<Layer*>(h);
    std::vector<float> sc(L.E);
    for (int t = 0; t < T; ++t) {
        glm::gemv_bf16_f32(L.router.data(), x + size_t(t) * L.H, sc.data(), L.E, L.H);
        for (int i = 0; i < L.E; ++i) sc[i] = 1.0f / (1.0f + std::exp(-sc[i]));
        auto r = glm::topKScores(sc.data(), L.E, L.bias.data(), L.K, L.scale, L.norm);
        for (int i = 0; i < r.k; ++i) genExpert(L, r.indices[i]);
    }
    if (L.Is > 0) genExpert(L, L.E);
}

// moeLayer for tokens [0, T): out [T x H]; idx/w [T x K]; slot_out (optional)
// [T x (K+1) x H] per-slot expert outputs (shared last). Returns seconds spent
// inside the per-token loop (steady_clock).
double hfr_layer_forward(void* h, const float* x, int T, float* out, int32_t* idx, float* w,
                         float* slot_out) {
    auto& L = *static_cast<Layer*>(h);
    std::vector<int> ibuf(L.K);
    std::vector<float> wbuf(L.K);
    const auto t0 = std::chrono::steady_clock::now();
    for (int t = 0; t < T; ++t) {
        moeLayer(L, x + size_t(t) * L.H, out + size_t(t) * L.H, ibuf.data(), wbuf.data(),
                 slot_out ? slot_out + size_t(t) * (L.K + 1) * L.H : nullptr);
        for (int i = 0; i < L.K; ++i) {
            if (idx) idx[size_t(t) * L.K + i] = ibuf[i];
            if (w) w[size_t(t) * L.K + i] = wbuf[i];
        }
    }
    const auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
}

}  // extern "C"
