/*
 * hf_synth.h -- seeded synthetic layers on the device (benchmarks and tests).
 *
 * No counterpart in the reference, whose weights come from the GLM-5.2
 * checkpoint (model/weight_index.cpp). Each element is a pure function of
 * (seed, layer, kind, expert, index): 64-bit splitmix hashing, an
 * Irwin-Hall(4) normal from the four 16-bit lanes (one integer sum, one fp32
 * multiply) and round-to-nearest-even to BF16 (BFloat16::fromF32,
 * compute/dtype_bf16.h:27-33). Integer work is exact and every fp32 step is a
 * single rounded operation, so a host implementation of the same formulas
 * yields the same bytes; weights are never copied from the host.
 */
#ifndef HF_SYNTH_H
#define HF_SYNTH_H

#include "hf_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    HF_SYNTH_X = 0,       /* activations                        */
    HF_SYNTH_ROUTER = 1,  /* mlp.gate.weight                    */
    HF_SYNTH_BIAS = 2,    /* e_score_correction_bias            */
    HF_SYNTH_GATE = 3,    /* experts.*.gate_proj / shared gate  */
    HF_SYNTH_UP = 4,
    HF_SYNTH_DOWN = 5
};

/* dst[i] = bf16(sigma * normal(seed, layer, kind, expert, i)), i < n. */
HF_API hf_status hf_synth_bf16_normal(uint16_t* dst, uint64_t n, uint64_t seed, uint32_t layer,
                               uint32_t kind, uint32_t expert, double sigma, hf_stream stream);
/* dst[i] = lo + (hi - lo) * u24(seed, layer, kind, expert, i) * 2^-24 (fp32). */
HF_API hf_status hf_synth_f32_uniform(float* dst, uint64_t n, uint64_t seed, uint32_t layer,
                               uint32_t kind, uint32_t expert, float lo, float hi,
                               hf_stream stream);
/* Fills every weight of `layer` the context holds: router ~N(0, 0.02) BF16,
 * bias ~U(-0.1, 0.1) (or the host array bias_override [E]), each local routed
 * expert and the shared expert ~N(0, 0.02) BF16 (expert id E for the shared
 * one), generator layer index `gen_layer`. Marks the layer loaded. */
HF_API hf_status hf_moe_synth_layer(hf_moe_ctx* ctx, int layer, uint64_t seed, uint32_t gen_layer,
                             const float* bias_override, hf_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* HF_SYNTH_H */
