// hf_ctx.cuh -- the MoE context shared by hf_moe.cu (single device) and
// hf_ep.cu (expert parallelism over NCCL).
#pragma once

#include <string>
#include <vector>

#include "hf_internal.cuh"

struct ncclComm;

namespace hf {

// Makes the context's device current for one API call and restores the
// caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = (prev == dev) || (cudaSetDevice(dev) == cudaSuccess);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

struct LayerBuf {
    uint16_t* router = nullptr;  // [E x H] (global router on every rank)
    float* bias = nullptr;       // [E]
    bool has_bias = false;
    uint16_t* experts = nullptr; // [E_local][gate|up|down]
    uint16_t* shared = nullptr;  // [gate|up|down] of the shared expert
    GroupW* groups = nullptr;    // [G] device table: local experts, then shared
    bool loaded = false;
    // TMA views of the weights for the tcgen05 GEMM (built with the buffers)
    CUtensorMap gu{}, dn{};      // routed: H-wide / I-wide rows of the [gate|up|down] blocks
    CUtensorMap sh_gate{}, sh_up{}, sh_down{};  // shared expert: one view per matrix
    CUtensorMap rt{};            // router rows (the router GEMM's weight operand)
    bool maps = false;
    // Expert placement (expert parallelism): placed position j holds global
    // expert order[j], rank r owns positions [r*El, (r+1)*El); inv is the
    // inverse. The router rows and bias are stored in placed order, so routing
    // produces placed ids and the exchange sends each rank one contiguous
    // range; routing outputs are mapped back to global ids. Empty: identity.
    std::vector<int32_t> order, inv;
    int32_t* d_order = nullptr;  // [E] device copy of order
    // Resident format of the down blocks (hf_weights.cu): dfmt[g] = 1 when
    // group g's block holds FP16 (w * 2^S), 0 for the BF16 layout; down_ready
    // once a forward has put every block in one format, down_f16 which one.
    std::vector<uint8_t> dfmt;
    bool down_ready = false, down_f16 = false;
    uint16_t** d_blocks = nullptr;  // [G] down block of each group
    int* d_list = nullptr;          // [G] groups a conversion touches
    unsigned* d_absmax = nullptr;   // [G] largest |w| (BF16 bits)
    float* d_scale = nullptr;       // [G] 2^-S
};

template <typename T>
inline hf_status dalloc(T** p, size_t count) {
    *p = nullptr;
    if (count == 0) return HF_OK;
    HF_CUDA(cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)));
    return HF_OK;
}

// Expert-parallel state (hf_ep.cu). Absent when ep_world == 1.
struct EpState;

}  // namespace hf

struct hf_moe_ctx {
    hf_moe_config cfg{};
    int H = 0, E = 0, K = 0, k = 0, I = 0, Is = 0;
    int world = 1, rank = 0;
    int E_local = 0, e_begin = 0;
    int G = 0;        // expert groups run here: local experts + shared
    int G_src = 0;    // routing groups: all experts + shared
    int inter_max = 0;
    size_t expert_elems = 0;
    size_t slots_cap = 0;  // rows of the expert-side scratch
    std::vector<hf::LayerBuf> layers;
    hf::PlanLayout pl{};      // expert-side plan layout (G groups)
    hf::PlanLayout pl_src{};  // routing plan layout (G_src groups)
    int T_max = 0;
    // routing scratch
    float* logits = nullptr;
    int32_t* ids = nullptr;
    float* w = nullptr;
    float* margins = nullptr;
    int32_t* plan_src = nullptr;   // == plan on a single device
    int32_t* perm_src = nullptr;   // == perm on a single device
    int32_t* slot_pos = nullptr;
    uint32_t* masks = nullptr;
    int32_t* blk_counts = nullptr;
    // expert-side scratch
    int32_t* plan = nullptr;
    int32_t* perm = nullptr;
    float* mid = nullptr;
    float* y = nullptr;
    uint16_t* mid_hi = nullptr;  // GEMM path: SwiGLU output as bf16 hi + lo
    uint16_t* mid_lo = nullptr;
    uint16_t* xp_hi = nullptr;   // GEMM path: activations gathered by position
    uint16_t* xp_lo = nullptr;
    hf::GemmMaps maps1{}, maps2{};  // activation-side tensor maps (GEMM1, GEMM2)
    // the same with kPairBoxB-row activation boxes, for the CTA-pair passes
    hf::GemmMaps maps1w{}, maps2w{};
    // host-buffer API staging
    void* x_dev = nullptr;
    float* out_dev = nullptr;
    bool gemm_ok = false;
    unsigned long long timeout_ns = 2000ull * 1000 * 1000;
    int stall = 0;               // test hook: GEMM kernels wait on a dead barrier
    int gemm_bn = 0;             // GEMM token tile override (HF_GEMM_BN: 32, 64, 128)
    int router_mode = 0;         // 0: by batch size, 1: SIMT kernels, 2: tcgen05 (HF_ROUTER)
    int nsm = 148;
    int* err_host = nullptr;     // pinned copy of the device error word
    int* sched = nullptr;        // GEMM tile-scheduler counters (zero between launches)
    int grid1_bf16 = 0, grid1_f32 = 0, grid2 = 0;
    cudaStream_t last_stream = nullptr;
    hf::EpState* ep = nullptr;
    // profiling: event pairs per phase, launch counters
    bool profiling = false;
    std::vector<cudaEvent_t> ev_pool;
    struct Mark { int phase; cudaEvent_t a, b; };
    std::vector<Mark> marks;
    long long launches[HF_MOE_PHASES] = {};
};

namespace hf {

// Local slot of global expert `eid` on this rank (-1: not owned here), and
// the global id of local slot l, under the layer's placement.
inline int local_slot(const hf_moe_ctx* c, const LayerBuf& L, int eid) {
    if (eid < 0 || eid >= c->E) return -1;
    const int l = (L.inv.empty() ? eid : L.inv[size_t(eid)]) - c->e_begin;
    return (l >= 0 && l < c->E_local) ? l : -1;
}
inline int slot_expert(const hf_moe_ctx* c, const LayerBuf& L, int l) {
    const int pos = c->e_begin + l;
    return L.order.empty() ? pos : L.order[size_t(pos)];
}
// Down-block format (hf_weights.cu): before a forward, before handing out a
// block's address, and after a weight setter wrote group g (-1: all).
hf_status ensure_down_format(hf_moe_ctx* c, LayerBuf& L, cudaStream_t st);
hf_status down_to_bf16(hf_moe_ctx* c, LayerBuf& L, int g);
void down_written(LayerBuf& L, int g);
// Router rows and bias (written in global order) into the placed order.
hf_status place_router(hf_moe_ctx* c, LayerBuf& L, cudaStream_t st);
// Routing outputs of a forward in global expert ids (placed layers only).
hf_status unplace_routing(hf_moe_ctx* c, const LayerBuf& L, const hf_moe_routing* r, int T,
                          cudaStream_t st);

// Brackets one phase of a forward with events (when profiling) and counts its
// kernel launches.
struct PhaseTimer {
    hf_moe_ctx* c;
    cudaStream_t st;
    int phase;
    cudaEvent_t a = nullptr;
    PhaseTimer(hf_moe_ctx* ctx, cudaStream_t s, int p) : c(ctx), st(s), phase(p) {
        if (c->profiling) {
            a = take();
            if (a) cudaEventRecord(a, st);
        }
    }
    cudaEvent_t take() {
        cudaEvent_t e = nullptr;
        if (!c->ev_pool.empty()) {
            e = c->ev_pool.back();
            c->ev_pool.pop_back();
        } else if (cudaEventCreate(&e) != cudaSuccess) {
            e = nullptr;
        }
        return e;
    }
    void done(int nlaunch) {
        c->launches[phase] += nlaunch;
        if (!a) return;
        cudaEvent_t b = take();
        if (!b) return;
        cudaEventRecord(b, st);
        c->marks.push_back({phase, a, b});
        a = nullptr;
    }
    ~PhaseTimer() {
        if (a) c->ev_pool.push_back(a);
    }
};

// One expert pass: which plan, which activation rows, where outputs go. On a
// single device the slots are the routed slots (t*k + i) and the shared ones;
// on an expert-parallel receiver they are the received rows (k = 1) and the
// shared slots of the local tokens.
struct ExpertWork {
    const int32_t* plan;
    PlanLayout pl;
    const int32_t* perm;
    const void* x;     // activation rows addressed by token_of_slot(perm[p], T, k)
    int x_f32;
    int T, k;
    float* y;          // [positions x H]
    int bn1, bn2, m1, m2;  // GEMM tiles the plan's tile prefixes were built with
    int pair;              // the GEMM tiles run on CTA pairs
    bool maybe_gemm;   // some segment may take the GEMM / the GEMV (else skip the launches)
    bool maybe_gemv;
    int down_f16 = 0;  // the layer's down blocks are FP16 (GemmArgs::down_f16)
    int y16 = 0;       // outputs as the FP16 plane (GemmArgs::y16); GEMM-only passes
    int groups_base = 0;  // the plan's group g is the layer's group groups_base + g
    // GEMM2 outputs through per-position row pointers and the end-of-kernel
    // flag release (GemmArgs::yrow / sig_*); GEMM path only
    float* const* yrow = nullptr;
    unsigned long long* const* sig_flags = nullptr;
    int sig_n = 0, sig_slot = 0;
    unsigned long long sig_seq = 0;
};

// Routing arguments of a forward on the given (source) plan.
RouteArgs route_args(hf_moe_ctx* c, LayerBuf& L, const void* x, hf_dtype xd, int T);
hf_status run_route(hf_moe_ctx* c, LayerBuf& L, const RouteArgs& ra, cudaStream_t st);
// AUTO GEMV threshold (segments of up to this many tokens) of a pass over `rows` rows.
int gemv_threshold(const hf_moe_ctx* c, int rows);

// Router logits on the tensor cores: [E x H] router rows against the token
// rows, split over K into `nsplit` runs of `kbper` 64-wide blocks whose
// partial planes [T x E] the top-k sums in order.
struct RouterTiles {
    int bn, mrows, kbper, nsplit;
};
RouterTiles router_tiles(int T, int E, int H, int nsm);
bool use_tc_router(const hf_moe_ctx* c, const LayerBuf& L, const void* x, hf_dtype xd, int T);
hf_status run_experts(hf_moe_ctx* c, LayerBuf& L, const ExpertWork& w, cudaStream_t st);
// slot_pos: the row of y each slot reads (default: the context's slot -> position table);
// y16: y holds the FP16 plane (GemmArgs::y16)
hf_status run_combine(hf_moe_ctx* c, const float* y, int y16, int T, float* out,
                      const float* resid, float* slot_out, cudaStream_t st,
                      const int32_t* slot_pos = nullptr);
// Expert outputs of a forward whose every segment takes the GEMM go through
// the FP16 plane (HF_Y_F16=0 keeps fp32); the same answer on every rank.
bool y16_wanted(const hf_moe_ctx* c, bool maybe_gemv);

// Allocates a layer's weight buffers and tensor maps on first use (hf_moe.cu).
hf_status ctx_layer_alloc(hf_moe_ctx* c, int layer);

// hf_ep.cu
hf_status ep_create(hf_moe_ctx* c, const unsigned char* unique_id);
void ep_destroy(hf_moe_ctx* c);
hf_status ep_forward(hf_moe_ctx* c, LayerBuf& L, const void* x, hf_dtype xd, int T, float* out,
                     const float* resid, const hf_moe_routing* r, cudaStream_t st);
size_t ep_recv_cap(const hf_moe_ctx* c);

}  // namespace hf
