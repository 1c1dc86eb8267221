// ref_kat.cpp -- known-answer vectors from the reference's own code.
//
// Compiled by tests/golden/make_golden.py together with the reference's
// unmodified compute/cpu_kernels.cpp (output binary in oracle/_ref/). It
// rebuilds the inputs of the reference's self-tests exactly (same std::mt19937
// seeds and distributions) and records what the reference's functions return:
//   gemv    src/self_test.cpp:73-103     (M=8, K=33, mt19937(42), alpha/beta)
//   topk    src/self_test.cpp:180-200    (8 scores, k=3, bias -10 on expert 2)
//   bf16    src/self_test.cpp:53-70      (its values and rounding edges, BFloat16::fromF32)
//   rmsnorm src/self_test.cpp:125-138    (n=128, mt19937(3), eps 1e-5, no weight)
//   expert  compute/cuda_backend.cpp:497-520 (64x32 case, mt19937(1)); the
//           expected output is the CPU forward's math (expertFFNRaw,
//           model/glm_forward.cpp:434-449) on gemv_bf16_f32
// Floats are written as their uint32 bit patterns so the JSON is exact.
#include "compute/cpu_kernels.h"
#include "compute/dtype_bf16.h"
#include "compute/moe_router.h"

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

using glm::BFloat16;

static uint32_t bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}

static void put_f32(const char* name, const float* v, size_t n, bool last = false) {
    std::printf("\"%s\": [", name);
    for (size_t i = 0; i < n; ++i) std::printf("%s%u", i ? "," : "", bits(v[i]));
    std::printf("]%s\n", last ? "" : ",");
}

static void put_u16(const char* name, const BFloat16* v, size_t n) {
    std::printf("\"%s\": [", name);
    for (size_t i = 0; i < n; ++i) std::printf("%s%u", i ? "," : "", unsigned(v[i].bits_));
    std::printf("],\n");
}

static void put_i32(const char* name, const int* v, size_t n) {
    std::printf("\"%s\": [", name);
    for (size_t i = 0; i < n; ++i) std::printf("%s%d", i ? "," : "", v[i]);
    std::printf("],\n");
}

int main() {
    std::printf("{\n");
    {  // self_test.cpp:73-103
        const int M = 8, K = 33;
        std::vector<BFloat16> A(M * K);
        std::vector<float> x(K), y_naive(M), y(M), y2(M, 7.0f);
        std::mt19937 rng(42);
        std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
        for (auto& v : A) v = BFloat16::fromF32(dist(rng));
        for (auto& v : x) v = 1.5f * dist(rng);
        for (int i = 0; i < M; ++i) {
            float dot = 0.0f;
            for (int j = 0; j < K; ++j) dot += A[i * K + j].toF32() * x[j];
            y_naive[i] = dot;
        }
        glm::gemv_bf16_f32(A.data(), x.data(), y.data(), M, K);
        glm::gemv_bf16_f32(A.data(), x.data(), y2.data(), M, K, 2.0f, 0.5f);
        put_u16("gemv_A", A.data(), A.size());
        put_f32("gemv_x", x.data(), x.size());
        put_f32("gemv_y_naive", y_naive.data(), M);
        put_f32("gemv_y", y.data(), M);
        put_f32("gemv_y_alpha2_beta05_y7", y2.data(), M);
    }
    {  // self_test.cpp:180-200
        const float scores[8] = {0.1f, 0.6f, 0.9f, 0.4f, 0.7f, 0.2f, 0.8f, 0.3f};
        const float bias[8] = {0, 0, -10, 0, 0, 0, 0, 0};
        struct Case { const char* name; const float* bias; int k; float scale; bool norm; };
        const Case cases[] = {{"topk_plain", nullptr, 3, 1.0f, false},
                              {"topk_norm", nullptr, 3, 1.0f, true},
                              {"topk_scaled", nullptr, 3, 2.5f, false},
                              {"topk_bias", bias, 3, 1.0f, false},
                              {"topk_k8_norm_scaled", nullptr, 8, 2.5f, true}};
        put_f32("topk_scores", scores, 8);
        put_f32("topk_bias_vec", bias, 8);
        for (const auto& c : cases) {
            auto r = glm::topKScores(scores, 8, c.bias, c.k, c.scale, c.norm);
            char nm[96];
            std::snprintf(nm, sizeof nm, "%s_idx", c.name);
            put_i32(nm, r.indices, r.k);
            std::snprintf(nm, sizeof nm, "%s_w", c.name);
            put_f32(nm, r.weights, r.k);
        }
    }
    {  // self_test.cpp:53-70 (BFloat16): its values plus rounding edges (ties to
       // even both ways, carries into the exponent, subnormals, the largest
       // finite, infinities), through the reference's BFloat16::fromF32
        const uint32_t edge[] = {0x3F800000u, 0x40000000u, 0xBFC00000u, 0x3F000000u, 0x00000000u,
                                 0x80000000u, 0x3DCCCCCDu, 0x3E99999Au, 0x3EAAAAABu, 0x42F6E979u,
                                 0xC476E9DBu, 0x3A83126Fu, 0x447A0000u, 0x3F808000u, 0x3F818000u,
                                 0x3F80C000u, 0x3F7FFFFFu, 0x7F7FFFFFu, 0x00000001u, 0x00008000u,
                                 0x00018000u, 0x807FFFFFu, 0x7F800000u, 0xFF800000u, 0x477FFFFFu,
                                 0xBF808001u};
        const size_t n = sizeof(edge) / sizeof(edge[0]);
        std::vector<float> in(n);
        std::vector<BFloat16> out(n);
        for (size_t i = 0; i < n; ++i) {
            std::memcpy(&in[i], &edge[i], 4);
            out[i] = BFloat16::fromF32(in[i]);
        }
        put_f32("bf16_in", in.data(), n);
        put_u16("bf16_out", out.data(), n);
    }
    {  // self_test.cpp:125-138: the RMSNorm the reference checks GLMForward::rmsNorm's
       // math with (n = 128, mt19937(3), U(-1, 1), eps = 1e-5, no weight)
        const int n = 128;
        const float eps = 1e-5f;
        std::vector<float> x(n);
        std::mt19937 rng(3);
        std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
        for (auto& v : x) v = dist(rng);
        float sqSum = 0.0f;
        for (int i = 0; i < n; ++i) sqSum += x[i] * x[i];
        float rms = 1.0f / std::sqrt(sqSum / float(n) + eps);
        std::vector<float> ref = x;
        for (int i = 0; i < n; ++i) ref[i] *= rms;
        put_f32("rmsnorm_x", x.data(), n);
        put_f32("rmsnorm_y", ref.data(), n);
    }
    {  // cuda_backend.cpp:497-520, case {64, 32}
        const int h = 64, i = 32;
        const size_t half = size_t(h) * size_t(i);
        std::vector<BFloat16> w(3 * half);
        std::mt19937 rng(1);
        std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
        for (auto& v : w) v = BFloat16::fromF32(dist(rng));
        std::vector<float> x(h), g(i), u(i), m(i), y(h);
        for (auto& v : x) v = 0.7f * dist(rng);
        glm::gemv_bf16_f32(w.data(), x.data(), g.data(), i, h);
        glm::gemv_bf16_f32(w.data() + half, x.data(), u.data(), i, h);
        for (int r = 0; r < i; ++r) m[r] = g[r] / (1.0f + std::exp(-g[r])) * u[r];
        glm::gemv_bf16_f32(w.data() + 2 * half, m.data(), y.data(), h, i);
        put_u16("expert_w", w.data(), w.size());
        put_f32("expert_x", x.data(), x.size());
        put_f32("expert_y", y.data(), y.size(), true);
    }
    std::printf("}\n");
    return 0;
}
