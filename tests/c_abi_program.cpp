// c_abi_program.cpp -- the MoE layer driven from plain C++ through the C ABI
// (include/hf_moe.h), the way the reference engine would call it: no PyTorch,
// no CUDA headers, host buffers only. Weights come from the seeded generator
// on the host and go in through hf_moe_set_router / hf_moe_set_expert_parts /
// hf_moe_set_shared (the checkpoint's per-projection tensors); the per-token
// drop-in hf_moe_layer (GLMForward::moeLayer's signature) and the batched
// hf_moe_forward_host are checked against the oracle's restatement of the
// reference (oracle/hf_oracle.h, test infrastructure) at the north-star bars.
//
// Built by tests/test_c_abi_program.py (g++, linked with libhf_moe.so and
// oracle/liboracle.so); run there on a GPU. Prints one line and exits 0 when
// every check holds.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "hf_moe.h"
#include "hf_ingest.h"
#include "hf_oracle.h"

namespace {

constexpr uint64_t kSeed = 91;
constexpr uint32_t kRouter = 1, kBias = 2, kGate = 3, kUp = 4, kDown = 5;

bool check(hf_status s, const char* what) {
    if (s != HF_OK) {
        std::printf("FAIL %s: %s (%s)\n", what, hf_status_string(s), hf_last_error());
        return false;
    }
    return true;
}

// max-abs <= 2e-2 and rel-L2 <= 1e-3 over a vector
bool close(const std::vector<float>& got, const std::vector<float>& ref, const char* what) {
    double num = 0, den = 0, mx = 0;
    for (size_t i = 0; i < got.size(); ++i) {
        const double d = double(got[i]) - double(ref[i]);
        num += d * d;
        den += double(ref[i]) * double(ref[i]);
        mx = std::fmax(mx, std::fabs(d));
    }
    const double rel = std::sqrt(num / (den > 0 ? den : 1e-30));
    if (mx > 2e-2 || rel > 1e-3) {
        std::printf("FAIL %s: max-abs %.3e rel-L2 %.3e\n", what, mx, rel);
        return false;
    }
    return true;
}

}  // namespace

int main() {
    const int H = 256, E = 16, K = 4, I = 128, Is = 192, T = 5;
    hf_moe_config c{};
    c.hidden_size = H;
    c.num_experts = E;
    c.num_experts_per_tok = K;
    c.moe_intermediate_size = I;
    c.shared_intermediate_size = Is;
    c.routed_scaling_factor = 2.5f;
    c.norm_topk_prob = 1;
    c.num_layers = 1;
    c.max_tokens = T;
    c.device = 0;
    c.path = HF_PATH_AUTO;
    c.ep_world = 1;
    hf_moe_ctx* ctx = nullptr;
    if (!check(hf_moe_create(&ctx, &c), "hf_moe_create")) return 1;

    // weights on the host, in the checkpoint's per-projection form
    std::vector<uint16_t> router(size_t(E) * H);
    std::vector<float> bias(E);
    hfo_gen_bf16_normal(kSeed, 0, kRouter, 0, 0.02, router.size(), router.data());
    hfo_gen_f32_uniform(kSeed, 0, kBias, 0, -0.1f, 0.1f, bias.size(), bias.data());
    bool ok = check(hf_moe_set_router(ctx, 0, router.data(), bias.data(), HF_MEM_HOST),
                    "hf_moe_set_router");
    std::vector<std::vector<uint16_t>> blocks(E);
    std::vector<const uint16_t*> block_ptrs(E);
    const size_t n = size_t(I) * H;
    for (int e = 0; e < E && ok; ++e) {
        std::vector<uint16_t> g(n), u(n), d(n);
        hfo_gen_bf16_normal(kSeed, 0, kGate, e, 0.02, n, g.data());
        hfo_gen_bf16_normal(kSeed, 0, kUp, e, 0.02, n, u.data());
        hfo_gen_bf16_normal(kSeed, 0, kDown, e, 0.02, n, d.data());
        ok = check(hf_moe_set_expert_parts(ctx, 0, e, g.data(), u.data(), d.data(), HF_MEM_HOST),
                   "hf_moe_set_expert_parts");
        blocks[e].reserve(3 * n);  // the [gate|up|down] block the oracle reads
        blocks[e].insert(blocks[e].end(), g.begin(), g.end());
        blocks[e].insert(blocks[e].end(), u.begin(), u.end());
        blocks[e].insert(blocks[e].end(), d.begin(), d.end());
        block_ptrs[e] = blocks[e].data();
    }
    const size_t ns = size_t(Is) * H;
    std::vector<uint16_t> sg(ns), su(ns), sd(ns), shared;
    hfo_gen_bf16_normal(kSeed, 0, kGate, E, 0.02, ns, sg.data());
    hfo_gen_bf16_normal(kSeed, 0, kUp, E, 0.02, ns, su.data());
    hfo_gen_bf16_normal(kSeed, 0, kDown, E, 0.02, ns, sd.data());
    ok = ok && check(hf_moe_set_shared(ctx, 0, sg.data(), su.data(), sd.data(), HF_MEM_HOST),
                     "hf_moe_set_shared");
    shared.insert(shared.end(), sg.begin(), sg.end());
    shared.insert(shared.end(), su.begin(), su.end());
    shared.insert(shared.end(), sd.begin(), sd.end());
    if (!ok) return 1;

    // activations: bf16-exact fp32 values (the reference's hiddenStates are fp32)
    std::vector<uint16_t> xb(size_t(T) * H);
    hfo_gen_bf16_normal(kSeed + 1, 0, 0, 0, 1.0, xb.size(), xb.data());
    std::vector<float> x(xb.size());
    for (size_t i = 0; i < xb.size(); ++i) {
        const uint32_t b = uint32_t(xb[i]) << 16;
        float f;
        __builtin_memcpy(&f, &b, 4);
        x[i] = f;
    }

    hfo_dims d{H, E, K, I, Is, 2.5f, 1};
    std::vector<float> ref(size_t(T) * H);
    std::vector<int32_t> ids(size_t(T) * K);
    std::vector<float> w(size_t(T) * K), margins(T);
    if (hfo_moe_layer(&d, router.data(), bias.data(), block_ptrs.data(), shared.data(), x.data(),
                      T, ref.data(), ids.data(), w.data(), margins.data(), nullptr) != 0) {
        std::printf("FAIL oracle rejected the shape\n");
        return 1;
    }

    // the per-token drop-in: GLMForward::moeLayer(layer, input, output)
    std::vector<float> out1(H);
    for (int t = 0; t < T && ok; ++t) {
        ok = check(hf_moe_layer(ctx, 0, x.data() + size_t(t) * H, out1.data()), "hf_moe_layer");
        std::vector<float> r(ref.begin() + size_t(t) * H, ref.begin() + size_t(t + 1) * H);
        ok = ok && close(out1, r, "hf_moe_layer");
    }
    // the batched host-buffer entry
    std::vector<float> outT(size_t(T) * H);
    ok = ok && check(hf_moe_forward_host(ctx, 0, x.data(), HF_F32, T, outT.data(), nullptr),
                     "hf_moe_forward_host");
    ok = ok && close(outT, ref, "hf_moe_forward_host");
    ok = ok && check(hf_moe_destroy(ctx), "hf_moe_destroy");
    std::printf("%s c_abi_program: %d tokens through hf_moe_layer and hf_moe_forward_host\n",
                ok ? "OK" : "FAIL", T);
    return ok ? 0 : 1;
}
