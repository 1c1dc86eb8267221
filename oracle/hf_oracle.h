/*
 * hf_oracle.h -- CPU restatement of HummingFlight's MoE layer (parity oracle).
 *
 * TEST INFRASTRUCTURE, never the product: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg may load oracle/liboracle.so. The product
 * path (hummingflight_b200/libhf_moe.so) never links or calls it.
 *
 * Each function restates one piece of the reference (file:line into the
 * HummingFlight source tree) in plain C, with the reference's arithmetic order:
 * sequential fp32 dot products (compute/cpu_kernels.cpp:82-93, the scalar loop
 * every GCC/Clang build compiles), expf-based sigmoid/SiLU, separate fp32
 * multiply and add (the reference is built -std=c++20, so no FP contraction;
 * this file is built with -ffp-contract=off). Pinned against the reference's
 * own code: tests/golden/ holds vectors produced by oracle/_ref (the
 * reference's cpu_kernels.cpp and moe_router.h, compiled unmodified) and the
 * known-answer tests of src/self_test.cpp.
 */
#ifndef HF_ORACLE_H
#define HF_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Shapes of one MoE layer (model/config.h MoE keys, config.cpp:108-117). */
typedef struct hfo_dims {
    int hidden;          /* hiddenSize                                   */
    int num_experts;     /* numLocalExperts                              */
    int top_k;           /* numExpertsPerTok (<= 8)                      */
    int inter;           /* moeIntermediateSize                          */
    int shared_inter;    /* nSharedExperts * moeIntermediateSize, 0=none */
    float scale;         /* routedScalingFactor                          */
    int norm_topk;       /* normTopkProb                                 */
} hfo_dims;

/* gemv_bf16_f32 (compute/cpu_kernels.cpp:43-94, scalar branch :82-93):
 * y[i] = alpha * dot(A[i,:], x) + beta * y[i]; dot summed j = 0..K-1. */
void hfo_gemv_bf16_f32(const uint16_t* A, const float* x, float* y, int M, int K,
                       float alpha, float beta);

/* Router logits -> sigmoid (model/glm_forward.cpp:519-524). */
void hfo_router_scores(const uint16_t* router_w, const float* x, int E, int H, float* scores);

/* topKScores (compute/moe_router.h:29-57). Ties in score+bias are broken by
 * the lower expert id (the reference's partial_sort leaves them unspecified).
 * Returns k = min(top_k, E) (0 when either is <= 0). margin_out, if given,
 * receives biased[k-1] - biased[k] (the 8th/9th gap; +inf when k == E). */
int hfo_topk_scores(const float* scores, int E, const float* bias, int top_k, float scale,
                    int norm, int32_t* idx, float* w, float* margin_out);

/* expertFFNRaw (model/glm_forward.cpp:434-449): g = G x, u = U x,
 * mid = g / (1 + exp(-g)) * u in fp32, y = D mid. */
void hfo_expert_ffn(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                    const float* x, float* y, int H, int I);

/* hfo_expert_ffn for n tokens of one expert in one pass over its weights:
 * x [n x H] -> y [n x H] (y is read for the beta * y term of the down GEMV,
 * like hfo_expert_ffn's zero-filled output). Each token's result is
 * bit-identical to hfo_expert_ffn on that token alone. */
void hfo_expert_ffn_multi(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                          const float* x, float* y, int n, int H, int I);

/* GLMForward::rmsNorm (model/glm_forward.cpp:185-197) on one row of n:
 * sq = sum x_i^2 (i ascending), rms = 1 / sqrt(sq / n + eps),
 * out_i = x_i * rms * w_i (w BF16; x_i * rms when w is NULL). out may be x. */
void hfo_rmsnorm(const float* x, const uint16_t* w, float eps, int n, float* out);

/* The MLP residual block (model/glm_forward.cpp:785-796) of one token:
 * out = x + mlp(rmsNorm(x)), mlp_out given: out_i = x_i + mlp_out_i. */
void hfo_residual_add(const float* x, const float* mlp_out, int n, float* out);

/* Canonical permutation of the batched build (no reference counterpart; the
 * reference loops experts per token, glm_forward.cpp:581): order (expert asc,
 * token asc). counts[E+1], offsets[E+2], perm[T*k + T]; slot id t*k+i for
 * routed slots, T*k+t for the shared expert (group E), which holds every
 * token when has_shared. */
void hfo_permute(const int32_t* ids, int T, int k, int E, int has_shared, int32_t* counts,
                 int32_t* offsets, int32_t* perm);

/* One MoE layer over T tokens (model/glm_forward.cpp:509-661), weights
 * generated from the seeded generator (oracle/hf_gen.h) one expert at a time.
 * x: [T x H] fp32. out: [T x H]. ids/w: [T x k]. margins: [T] (optional).
 * slot_out (optional): [(T*k + T) x H] per-slot expert outputs, routed slot
 * t*k+i then the shared expert at T*k+t. Returns 0 on success. */
int hfo_moe_layer_synth(const hfo_dims* d, uint64_t wseed, uint32_t layer,
                        const float* bias_override, const float* x, int T, float* out,
                        int32_t* ids, float* w, float* margins, float* slot_out);

/* Same layer with caller-provided weights: router [E x H] bf16, bias [E] f32
 * (may be NULL), experts[e] -> [gate | up | down] bf16 as returned by
 * Scheduler::getExpertPtr (engine/scheduler.h:80-84), shared -> the same
 * layout (may be NULL when shared_inter == 0). */
int hfo_moe_layer(const hfo_dims* d, const uint16_t* router_w, const float* bias,
                  const uint16_t* const* experts, const uint16_t* shared, const float* x,
                  int T, float* out, int32_t* ids, float* w, float* margins, float* slot_out);

/* Generator entry points (oracle/hf_gen.h), for tests and fixtures. */
void hfo_gen_bf16_normal(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert,
                         double sigma, uint64_t n, uint16_t* out);
void hfo_gen_f32_uniform(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert,
                         float lo, float hi, uint64_t n, float* out);
/* One expert in getExpertPtr layout [gate I*H | up I*H | down H*I]. */
void hfo_gen_expert(uint64_t seed, uint32_t layer, uint32_t expert, int H, int I, uint16_t* out);

int hfo_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
