/*
 * hf_gen.h -- seeded synthetic tensors for the MoE-layer parity oracle.
 *
 * TEST INFRASTRUCTURE. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may use anything under oracle/. The product library has its
 * own device generator (hummingflight_b200/csrc/hf_synth.cu) with the same
 * formulas; tests/test_synth_gpu.py checks that both give identical bits.
 *
 * The reference has no generator: its weights come from the GLM-5.2 checkpoint
 * (model/weight_index.cpp:222-236). The configs ask for N(0, 0.02) BF16
 * weights, N(0, 1) BF16 activations and U(-0.1, 0.1) fp32 correction bias.
 * Every element is a pure function of (seed, layer, kind, expert, index), so
 * the CPU and the GPU produce the same bytes without copying them:
 *
 *   bits   = mix64(key + (index + 1) * GOLDEN)              (splitmix64 mixer)
 *   normal = (sum of the four 16-bit lanes of bits - 131070) * scale
 *            (Irwin-Hall with 4 terms: mean 0, variance 1 after scaling,
 *             support +-3.46 sigma; integer sum, then ONE fp32 multiply)
 *   uniform= lo + (hi - lo) * ((bits >> 40) * 2^-24)        (fp32 mul, fp32 add)
 *   bf16   = round-to-nearest-even of the fp32 value, exactly as
 *            BFloat16::fromF32 (compute/dtype_bf16.h:27-33)
 *
 * Integer arithmetic is exact and each fp32 step is a single IEEE-rounded
 * operation, so C (built with -ffp-contract=off), numpy and CUDA (__fmul_rn,
 * __fadd_rn) agree bit for bit.
 */
#ifndef HF_GEN_H
#define HF_GEN_H

#include <stdint.h>
#include <string.h>
#include <math.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    HFG_KIND_X = 0,       /* activations [T x H]              */
    HFG_KIND_ROUTER = 1,  /* mlp.gate.weight [E x H]          */
    HFG_KIND_BIAS = 2,    /* e_score_correction_bias [E] f32  */
    HFG_KIND_GATE = 3,    /* gate_proj [I x H]                */
    HFG_KIND_UP = 4,      /* up_proj   [I x H]                */
    HFG_KIND_DOWN = 5     /* down_proj [H x I]                */
};

#define HFG_GOLDEN 0x9E3779B97F4A7C15ULL

static inline uint64_t hfg_mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ULL;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBULL;
    z ^= z >> 31;
    return z;
}

/* Stream key of one tensor. The shared expert uses expert = num_experts. */
static inline uint64_t hfg_key(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert) {
    uint64_t k = hfg_mix64(seed + HFG_GOLDEN);
    return hfg_mix64(k ^ (((uint64_t)layer << 40) | ((uint64_t)kind << 32) | (uint64_t)expert));
}

static inline uint64_t hfg_bits(uint64_t key, uint64_t index) {
    return hfg_mix64(key + (index + 1) * HFG_GOLDEN);
}

/* fp32 multiplier turning the centred 4-lane sum into sigma * N(0,1). */
static inline float hfg_normal_scale(double sigma) {
    return (float)(sigma / sqrt(1431655765.0)); /* sqrt((65536^2 - 1) / 3) */
}

static inline float hfg_normal(uint64_t key, uint64_t index, float scale) {
    uint64_t b = hfg_bits(key, index);
    int32_t s = (int32_t)(b & 0xFFFFu) + (int32_t)((b >> 16) & 0xFFFFu) +
                (int32_t)((b >> 32) & 0xFFFFu) + (int32_t)(b >> 48);
    return (float)(s - 131070) * scale;
}

static inline float hfg_uniform(uint64_t key, uint64_t index, float lo, float hi) {
    uint64_t b = hfg_bits(key, index);
    float t = (float)(uint32_t)(b >> 40) * 5.9604644775390625e-08f; /* exact: 2^-24 */
    float w = hi - lo;
    float p = w * t;
    return lo + p;
}

/* BFloat16::fromF32 (compute/dtype_bf16.h:27-33): RNE, no NaN special case. */
static inline uint16_t hfg_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof(u));
    uint32_t rounding_bias = 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)((u + rounding_bias) >> 16);
}

/* BFloat16::toF32 (compute/dtype_bf16.h:19-24): exact widening. */
static inline float hfg_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof(f));
    return f;
}

#ifdef __cplusplus
}
#endif
#endif /* HF_GEN_H */
