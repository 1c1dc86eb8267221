// hf_moe.cu -- C ABI of the MoE layer: context, weights, forward orchestration.
//
// Host side of the drop-in for GLMForward::moeLayer (model/glm_forward.cpp:
// 509-661) and the sm_86 expert cache it offloaded to (compute/cuda_backend.cpp:
// 196-492). Differences by design: all weights of a layer stay resident in HBM
// (no per-token staging over PCIe), a forward covers T tokens at once, every
// error is returned (no CPU fallback), and kernels run asynchronously on the
// caller's stream. A forward is three phases -- routing, experts, combine --
// that the expert-parallel path (hf_ep.cu) reuses around its exchanges.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "hf_ctx.cuh"
#include "hf_ingest.h"
#include "hf_synth.h"

namespace hf {

// ------------------------------------------------------------------ errors
static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

hf_status fail(hf_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

hf_status cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    return e == cudaErrorMemoryAllocation ? HF_ERR_OOM : HF_ERR_CUDA;
}

int num_sms(int device) {
    static std::atomic<int> cache[64];
    if (device >= 0 && device < 64) {
        const int c = cache[device].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
        n = 148;
    if (device >= 0 && device < 64) cache[device].store(n, std::memory_order_relaxed);
    return n;
}

cudaError_t ensure_smem(const void* kernel, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes set
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    int& have = done[{kernel, dev}];
    if (have >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

// ------------------------------------------------------------------ phases
RouteArgs route_args(hf_moe_ctx* c, LayerBuf& L, const void* x, hf_dtype xd, int T) {
    RouteArgs ra{};
    ra.x = x;
    ra.x_f32 = xd == HF_F32;
    ra.T = T;
    ra.H = c->H;
    ra.E = c->E;
    ra.k = c->k;
    ra.router = L.router;
    ra.bias = L.has_bias ? L.bias : nullptr;
    ra.scale = c->cfg.routed_scaling_factor;
    ra.norm = c->cfg.norm_topk_prob;
    ra.logits = c->logits;
    ra.ids = c->ids;
    ra.w = c->w;
    ra.margins = c->margins;
    ra.plan = c->plan_src;
    ra.pl = c->pl_src;
    ra.has_shared = c->Is > 0;
    ra.shared_inter = c->Is;
    ra.inter = c->I;
    ra.perm = c->perm_src;
    ra.slot_pos = c->slot_pos;
    ra.masks = c->masks;
    ra.blk_counts = c->blk_counts;
    ra.path = c->cfg.path;
    ra.gemv_max = gemv_threshold(c, T);
    ra.gemm_ok = c->gemm_ok && L.maps;
    set_gemm_tiles(c->gemm_bn, T, ra);
    ra.lsplit = use_tc_router(c, L, x, xd, T) ? router_tiles(T, c->E, c->H, c->nsm).nsplit : 1;
    ra.route_counter = c->sched + 4;
    return ra;
}

// Token tile 32/64/128 by batch; 128 router rows a tile for small batches
// (more CTAs), 256 (two accumulators) from 512 tokens when E > 128. K is
// split into at most kMaxRouterSplit runs so the grid covers more SMs while
// the top-k's in-order sum of the partial planes stays short (T = 64,
// E = 256, H = 6144: 2 x 12 CTAs of 8 K blocks).
constexpr int kMaxRouterSplit = 12;

RouterTiles router_tiles(int T, int E, int H, int nsm) {
    RouterTiles r{};
    r.bn = T <= 32 ? 32 : T <= 64 ? 64 : 128;
    r.mrows = (E > 128 && T >= 512) ? 256 : 128;
    const int kb = (H + 63) / 64;
    const int tiles = ((T + r.bn - 1) / r.bn) * ((E + r.mrows - 1) / r.mrows);
    const int ns = std::max(1, std::min(kMaxRouterSplit, (nsm + tiles - 1) / tiles));
    r.kbper = (kb + ns - 1) / ns;
    r.nsplit = (kb + r.kbper - 1) / r.kbper;  // no empty run
    return r;
}

// The SIMT kernels read fp32 activations exactly and serve single tokens
// (then also running the routing in the same launch); bf16 batches from
// kTcRouterMinT tokens take the tensor cores (measured: 8 tokens 31 us SIMT
// router + routing vs 13 us tensor-core logits).
constexpr int kTcRouterMinT = 2;

bool use_tc_router(const hf_moe_ctx* c, const LayerBuf& L, const void* x, hf_dtype xd, int T) {
    if (!L.maps || xd != HF_BF16 || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
    if (c->router_mode == 1) return false;
    if (c->router_mode == 2) return T > 0;
    return T >= kTcRouterMinT;
}

static hf_status launch_tc_router(hf_moe_ctx* c, LayerBuf& L, const RouteArgs& ra,
                                  cudaStream_t st) {
    const RouterTiles rt = router_tiles(ra.T, c->E, c->H, c->nsm);
    GemmMaps m{};
    m.A = m.A_sh = m.A_sh2 = L.rt;
    HF_TRY(make_map_bf16(&m.B0, ra.x, c->H, ra.T, c->H, 16));
    m.B1 = m.B0_sh = m.B1_sh = m.B0;
    GemmArgs g{};
    g.plan = nullptr;  // one group of T rows
    g.pl = PlanLayout::make(1);
    g.dense_T = ra.T;
    g.which = 2;       // y[t][e] = sum_k router[e][k] x[t][k]
    g.H = c->E;        // output rows
    g.I = g.Is = c->H; // K
    g.Imax = c->H;
    g.bn = rt.bn;
    g.mrows = rt.mrows;
    g.y = ra.logits;
    g.err = c->plan + c->pl.stats + 3;
    g.timeout_ns = c->timeout_ns;
    g.sched = c->sched;
    g.nsplit = rt.nsplit;
    g.kbper = rt.kbper;
    g.split_stride = (long long)ra.T * c->E;
    return launch_gemm(m, g, 1, c->nsm, st);
}

int gemv_threshold(const hf_moe_ctx* c, int rows) {
    if (c->cfg.gemv_max_tokens > 0) return c->cfg.gemv_max_tokens;
    return rows <= kGemvAutoBatch ? kGemvAutoMax : 0;
}

// Tiles of the two grouped GEMMs for a pass over `rows` activation rows.
// Decode (<= 64 rows, a few tokens per expert): narrow token tiles leave the
// shared memory to the weight ring -- gate/up 32-token tiles (two 16 KB
// weight boxes + 4 KB of tokens a stage, 6 stages), down 256 weight rows x
// 16 tokens (32 KB + 4 KB, 6 stages: as many weight bytes in flight as
// gate/up, against 9 x 16 KB for 128 x 32 tiles). Prefill (>= 1024 rows):
// 256 weight rows a tile. Gate/up runs on CTA pairs (cta_group::2, 256
// intermediate rows x 256 tokens, 128 of them loaded by each CTA; 7 % faster
// than one CTA's 128 x 128 tile on config 2 at 128 tokens per pair). The
// 256-token pair tile fills TMEM with one accumulator buffer, but each weight
// stage feeds twice the tokens, so segments and the shared expert with more
// than 128 tokens re-read their weight tiles half as often (config 2 gate/up
// 2.80 -> 2.64 ms against 128-token pair tiles). Down runs on CTA pairs too:
// two 256-row MMA blocks x 256 tokens (512 x 256 a pair, one TMEM buffer; the
// down epilogue only stores): each MMA instruction does four times the work of
// a one-CTA 128 x 128 one, and the down kernel spends most of its time issuing
// MMAs (the hi + lo pass doubles them) -- config 2 down 2.41 -> 2.01 ms. One
// CTA with two 128-row accumulators x 128 tokens (HF_GEMM_PAIR_DOWN=0) and the
// pair with 128 tokens (=1) measured the same as each other.
void set_gemm_tiles(int bn_override, int rows, RouteArgs& ra) {
    ra.gemm_m1 = 128;
    ra.gemm_pair = 0;
    if (bn_override) {
        ra.gemm_bn1 = ra.gemm_bn2 = bn_override;
        ra.gemm_m2 = 128;
    } else if (rows <= 64) {
        ra.gemm_bn1 = 32;
        ra.gemm_bn2 = 16;
        ra.gemm_m2 = 256;
    } else if (rows < 1024) {
        ra.gemm_bn1 = ra.gemm_bn2 = 128;
        ra.gemm_m2 = 128;
    } else {  // prefill: 256 weight rows per tile
        static const int pair_bn = [] {  // tuning knob: HF_GEMM_PAIR_BN = 128 or 256
            const char* e = std::getenv("HF_GEMM_PAIR_BN");
            return (e && std::atoi(e) == 128) ? 128 : 256;
        }();
        static const int pair_down = [] {  // tuning knob: HF_GEMM_PAIR_DOWN = 0, 1 or 2
            const char* e = std::getenv("HF_GEMM_PAIR_DOWN");
            const int v = e ? std::atoi(e) : 2;
            return (v == 0 || v == 1) ? v : 2;
        }();
        ra.gemm_pair = 1;  // gate/up on CTA pairs
        ra.gemm_bn1 = pair_bn;
        ra.gemm_m1 = 256;
        // down: 512 rows x 256 tokens on a CTA pair (or x 128 tokens; or 256 rows
        // x 128 tokens on one CTA)
        ra.gemm_bn2 = pair_down == 2 ? 256 : 128;
        ra.gemm_m2 = pair_down ? 512 : 256;
    }
}

hf_status run_route(hf_moe_ctx* c, LayerBuf& L, const RouteArgs& ra, cudaStream_t st) {
    bool routed = false;
    {
        PhaseTimer p0(c, st, 0);
        if (ra.lsplit > 1 || use_tc_router(c, L, ra.x, ra.x_f32 ? HF_F32 : HF_BF16, ra.T))
            HF_TRY(launch_tc_router(c, L, ra, st));
        else
            HF_TRY(launch_router_logits(ra, st, &routed));
        p0.done(1);
    }
    if (routed) return HF_OK;
    PhaseTimer p1(c, st, 1);
    int n = 0;
    HF_TRY(launch_route(ra, st, &n));
    p1.done(n);
    return HF_OK;
}

static bool gemm_wide_b() {
    static const bool on = [] {
        const char* e = std::getenv("HF_GEMM_WIDE_B");
        return !(e && std::atoi(e) == 0);
    }();
    return on;
}

hf_status run_experts(hf_moe_ctx* c, LayerBuf& L, const ExpertWork& w, cudaStream_t st) {
    if (w.maybe_gemm) {
        GatherArgs gx{};
        gx.plan = w.plan;
        gx.pl = w.pl;
        gx.perm = w.perm;
        gx.x = w.x;
        gx.T = w.T;
        gx.k = w.k;
        gx.H = c->H;
        gx.device = c->cfg.device;
        gx.xp_hi = c->xp_hi;
        gx.xp_lo = c->xp_lo;
        // single device: slot -> position of the routing (token-major gather)
        gx.slot_pos = w.k > 1 && w.perm == c->perm_src ? c->slot_pos : nullptr;
        gx.has_shared = c->Is > 0;
        PhaseTimer p1(c, st, 1);
        HF_TRY(launch_gather(gx, w.x_f32, st));
        p1.done(1);
    }
    GemvArgs ga{};
    ga.groups = L.groups;
    ga.plan = w.plan;
    ga.pl = w.pl;
    ga.perm = w.perm;
    ga.x = w.x;
    ga.x_f32 = w.x_f32;
    ga.T = w.T;
    ga.H = c->H;
    ga.k = w.k;
    ga.inter_max = c->inter_max;
    ga.mid = c->mid;
    ga.y = w.y;
    // chunks hold at most min(T, kGemvTE) tokens (a segment has at most T
    // slots): stage that many rows, and fit more blocks per SM when T is small
    ga.te_cap = std::max(1, std::min(w.k == 1 ? kGemvTE : w.T, kGemvTE));
    // every segment on the GEMV (so the shared expert too) and its three
    // matrices well inside L2: GEMV1 prefetches them during the routing kernel
    ga.prefetch_shared = !w.maybe_gemm && c->Is > 0 &&
                         size_t(3) * c->Is * c->H * 2 <= (size_t(96) << 20);
    ga.grid1 = gemv_grid(c->cfg.device, true, w.x_f32 != 0, c->H, c->inter_max, c->G, ga.te_cap);
    ga.grid2 = gemv_grid(c->cfg.device, false, false, c->H, c->inter_max, c->G, ga.te_cap);
    const bool gemv_possible = w.maybe_gemv;
    if (gemv_possible) {
        PhaseTimer p2(c, st, 2);
        HF_TRY(launch_gemv1(ga, st));
        p2.done(1);
    }
    GemmArgs gm{};
    // CTA-pair passes load their activations in kPairBoxB-row boxes (tuning
    // knob HF_GEMM_WIDE_B=0 keeps 16-row boxes)
    const bool wide = w.pair && gemm_wide_b();
    if (w.maybe_gemm) {
        gm.plan = w.plan;
        gm.pl = w.pl;
        gm.which = 1;
        gm.H = c->H;
        gm.I = c->I;
        gm.Is = c->Is;
        gm.Imax = c->inter_max;
        gm.bn = w.bn1;
        gm.mrows = w.m1;
        gm.pair = w.pair;
        gm.mid_hi = c->mid_hi;
        gm.mid_lo = c->mid_lo;
        gm.y = w.y;
        gm.err = c->plan + c->pl.stats + 3;
        gm.timeout_ns = c->timeout_ns;
        gm.test_stall = c->stall;
        gm.sched = c->sched;
        gm.down_f16 = w.down_f16;
        gm.groups = L.groups + w.groups_base;
        gm.box_b = wide ? kPairBoxB : 0;
        GemmMaps m1 = wide ? c->maps1w : c->maps1;
        m1.A = L.gu;
        m1.A_sh = L.sh_gate;
        m1.A_sh2 = L.sh_up;
        PhaseTimer p4(c, st, 4);
        HF_TRY(launch_gemm(m1, gm, w.x_f32 ? 2 : 1, c->nsm, st));
        p4.done(1);
    }
    if (gemv_possible) {
        PhaseTimer p3(c, st, 3);
        HF_TRY(launch_gemv2(ga, st));
        p3.done(1);
    }
    if (w.maybe_gemm) {
        gm.which = 2;
        gm.bn = w.bn2;
        gm.mrows = w.m2;
        gm.yrow = w.yrow;
        gm.sig_flags = w.sig_flags;
        gm.sig_n = w.sig_n;
        gm.sig_slot = w.sig_slot;
        gm.sig_seq = w.sig_seq;
        gm.y16 = w.y16;
        // the down pass runs on pairs only with its 512-row tiles
        const bool wide2 = wide && w.m2 == 512;
        gm.box_b = wide2 ? kPairBoxB : 0;
        GemmMaps m2 = wide2 ? c->maps2w : c->maps2;
        m2.A = L.dn;
        m2.A_sh = L.sh_down;
        m2.A_sh2 = L.sh_down;
        PhaseTimer p5(c, st, 5);
        HF_TRY(launch_gemm(m2, gm, w.down_f16 ? 1 : 2, c->nsm, st));
        p5.done(1);
    }
    return HF_OK;
}

bool y16_wanted(const hf_moe_ctx* c, bool maybe_gemv) {
    static const bool on = [] {
        const char* e = std::getenv("HF_Y_F16");  // tuning knob: 0 keeps fp32 expert outputs
        return !(e && std::atoi(e) == 0);
    }();
    return on && c->gemm_ok && !maybe_gemv && c->H % 8 == 0;
}

hf_status run_combine(hf_moe_ctx* c, const float* y, int y16, int T, float* out,
                      const float* resid, float* slot_out, cudaStream_t st,
                      const int32_t* slot_pos) {
    CombineArgs ca{};
    ca.resid = resid;
    ca.y = y;
    ca.y16 = y16;
    ca.slot_pos = slot_pos ? slot_pos : c->slot_pos;
    ca.w = c->w;
    ca.T = T;
    ca.H = c->H;
    ca.k = c->k;
    ca.has_shared = c->Is > 0;
    ca.out = out;
    ca.slot_out = slot_out;
    PhaseTimer p6(c, st, 6);
    HF_TRY(launch_combine(ca, st));
    p6.done(1);
    return HF_OK;
}

}  // namespace hf

using namespace hf;

extern "C" {

int hf_abi_version(void) { return HF_MOE_ABI_VERSION; }

const char* hf_status_string(hf_status s) {
    switch (s) {
        case HF_OK: return "HF_OK";
        case HF_ERR_ARG: return "HF_ERR_ARG";
        case HF_ERR_CUDA: return "HF_ERR_CUDA";
        case HF_ERR_NCCL: return "HF_ERR_NCCL";
        case HF_ERR_TIMEOUT: return "HF_ERR_TIMEOUT";
        case HF_ERR_OOM: return "HF_ERR_OOM";
        case HF_ERR_STATE: return "HF_ERR_STATE";
        case HF_ERR_UNSUPPORTED: return "HF_ERR_UNSUPPORTED";
        case HF_ERR_RANGE: return "HF_ERR_RANGE";
    }
    return "HF_ERR_UNKNOWN";
}

const char* hf_last_error(void) { return g_last_error.c_str(); }

static void free_ctx(hf_moe_ctx* c) {
    ep_destroy(c);
    for (auto& L : c->layers) {
        cudaFree(L.router);
        cudaFree(L.bias);
        cudaFree(L.experts);
        cudaFree(L.shared);
        cudaFree(L.groups);
        cudaFree(L.d_order);
        cudaFree(L.d_blocks);
        cudaFree(L.d_list);
        cudaFree(L.d_absmax);
        cudaFree(L.d_scale);
    }
    for (auto& m : c->marks) {
        cudaEventDestroy(m.a);
        cudaEventDestroy(m.b);
    }
    for (auto e : c->ev_pool) cudaEventDestroy(e);
    if (c->plan_src != c->plan) cudaFree(c->plan_src);
    if (c->perm_src != c->perm) cudaFree(c->perm_src);
    void* bufs[] = {c->logits, c->ids,    c->w,      c->margins, c->plan,  c->perm,
                    c->slot_pos, c->masks, c->blk_counts, c->mid, c->y,     c->x_dev,
                    c->out_dev, c->mid_hi, c->mid_lo, c->xp_hi,   c->xp_lo, c->sched};
    for (void* p : bufs) cudaFree(p);
    if (c->err_host) cudaFreeHost(c->err_host);
    delete c;
}

// Device error word (plan stats[3]) -> status; clears it.
static hf_status take_error_word(hf_moe_ctx* c, int word) {
    if (word == 0) return HF_OK;
    HF_CUDA(cudaMemset(c->plan + c->pl.stats + 3, 0, sizeof(int)));
    if (word == 8)
        return fail(HF_ERR_RANGE,
                    "a SwiGLU intermediate exceeded the FP16 down pass's range (|mid| > 4.2e6); "
                    "outputs of that forward are invalid (HF_DOWN_F16=0 keeps the BF16 hi + lo pass)");
    return fail(HF_ERR_TIMEOUT,
                "a bounded device wait in the tcgen05 GEMM gave up; the kernel drained and "
                "returned, outputs of that forward are invalid");
}

hf_status hf_moe_create(hf_moe_ctx** out, const hf_moe_config* cfg) {
    if (!out || !cfg) return fail(HF_ERR_ARG, "hf_moe_create: null argument");
    *out = nullptr;
    const hf_moe_config& c = *cfg;
    if (c.hidden_size <= 0 || c.hidden_size % 8)
        return fail(HF_ERR_ARG, "hidden_size must be a positive multiple of 8");
    if (c.num_experts <= 0 || c.num_experts > kMaxExperts)
        return fail(HF_ERR_ARG, "num_experts must be in 1..1024");
    if (c.num_experts_per_tok <= 0 || c.num_experts_per_tok > kMaxTopK)
        return fail(HF_ERR_ARG, "num_experts_per_tok must be in 1..8 (TopKResult holds 8)");
    if (c.moe_intermediate_size <= 0 || c.moe_intermediate_size % 8)
        return fail(HF_ERR_ARG, "moe_intermediate_size must be a positive multiple of 8");
    if (c.shared_intermediate_size < 0 || c.shared_intermediate_size % 8)
        return fail(HF_ERR_ARG, "shared_intermediate_size must be a non-negative multiple of 8");
    if (c.num_layers <= 0) return fail(HF_ERR_ARG, "num_layers must be positive");
    if (c.max_tokens < 0) return fail(HF_ERR_ARG, "max_tokens must be >= 0");
    if (c.path < HF_PATH_AUTO || c.path > HF_PATH_GEMM) return fail(HF_ERR_ARG, "bad path");
    const int world = c.ep_world <= 0 ? 1 : c.ep_world;
    if (world > 1) {
        if (c.num_experts % world)
            return fail(HF_ERR_ARG, "expert parallelism needs num_experts divisible by ep_world");
        if (c.ep_rank < 0 || c.ep_rank >= world) return fail(HF_ERR_ARG, "ep_rank out of range");
        if (!c.ep_unique_id) return fail(HF_ERR_ARG, "ep_unique_id is required when ep_world > 1");
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(HF_ERR_UNSUPPORTED, "no CUDA device");
    if (c.device < 0 || c.device >= ndev) return fail(HF_ERR_ARG, "device ordinal out of range");
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, c.device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, c.device);
    if (major != 10 || minor != 0)
        return fail(HF_ERR_UNSUPPORTED, "libhf_moe is built for sm_100a (B200) only");
    DeviceGuard dg(c.device);
    if (!dg.ok) return fail(HF_ERR_CUDA, "cudaSetDevice failed");

    auto* x = new hf_moe_ctx();
    x->cfg = c;
    x->cfg.ep_world = world;
    x->world = world;
    x->rank = world > 1 ? c.ep_rank : 0;
    x->H = c.hidden_size;
    x->E = c.num_experts;
    x->K = c.num_experts_per_tok;
    x->k = std::min(x->K, x->E);
    x->I = c.moe_intermediate_size;
    x->Is = c.shared_intermediate_size;
    x->E_local = x->E / world;
    x->e_begin = x->rank * x->E_local;
    x->G = x->E_local + 1;
    x->G_src = x->E + 1;
    x->inter_max = std::max(x->I, x->Is);
    x->expert_elems = size_t(3) * x->I * x->H;
    x->pl = PlanLayout::make(x->G);
    x->pl_src = PlanLayout::make(x->G_src);
    x->T_max = c.max_tokens;
    if (x->cfg.gemv_max_tokens < 0) x->cfg.gemv_max_tokens = 0;
    if (const char* bn = std::getenv("HF_GEMM_BN")) {  // tuning knob
        const int v = std::atoi(bn);
        x->gemm_bn = (v == 32 || v == 64 || v == 128) ? v : 0;
    }
    if (const char* rm = std::getenv("HF_ROUTER"))  // "simt" / "tc": force one router kernel
        x->router_mode = std::string(rm) == "simt" ? 1 : std::string(rm) == "tc" ? 2 : 0;
    x->nsm = num_sms(c.device);
    if (gemv1_smem(x->H, true, x->G) > 227 * 1024 || gemv2_smem(x->inter_max, x->G) > 227 * 1024) {
        free_ctx(x);
        return fail(HF_ERR_ARG, "hidden/intermediate size too large for the GEMV staging");
    }
    x->layers.resize(c.num_layers);
    const size_t T = size_t(std::max(1, c.max_tokens));
    const size_t src_slots = T * x->k + T;
    x->slots_cap = world > 1 ? ep_recv_cap(x) + T : src_slots;
    const size_t slots = x->slots_cap;
    const size_t nb = (T + kSmallRouteT - 1) / kSmallRouteT;
    hf_status s = HF_OK;
    auto A = [&](hf_status r) { if (s == HF_OK) s = r; };
    size_t lrows = T;  // logits: nsplit partial planes when the router GEMM splits K
    for (size_t t = 1; t <= T; ++t)
        lrows = std::max(lrows, t * size_t(router_tiles(int(t), x->E, x->H, x->nsm).nsplit));
    A(dalloc(&x->logits, lrows * x->E));
    A(dalloc(&x->ids, T * x->k));
    A(dalloc(&x->w, T * x->k));
    A(dalloc(&x->margins, T));
    A(dalloc(&x->plan, size_t(x->pl.words)));
    A(dalloc(&x->perm, slots));
    if (world > 1) {
        A(dalloc(&x->plan_src, size_t(x->pl_src.words)));
        A(dalloc(&x->perm_src, src_slots));
    } else {
        x->plan_src = x->plan;
        x->perm_src = x->perm;
    }
    A(dalloc(&x->slot_pos, src_slots));
    A(dalloc(&x->sched, 8));
    A(dalloc(&x->masks, nb * 4 * x->E));
    A(dalloc(&x->blk_counts, nb * x->E));
    A(dalloc(&x->mid, slots * x->inter_max));
    A(dalloc(&x->y, slots * x->H));
    A(dalloc(reinterpret_cast<float**>(&x->x_dev), T * x->H));
    A(dalloc(&x->out_dev, T * x->H));
    x->gemm_ok = (x->H % 64 == 0) && (x->I % 64 == 0) && (x->Is % 64 == 0) &&
                 x->cfg.path != HF_PATH_GEMV;
    if (x->gemm_ok) {
        A(dalloc(&x->mid_hi, slots * x->inter_max));
        A(dalloc(&x->mid_lo, slots * x->inter_max));
        A(dalloc(&x->xp_hi, slots * x->H));
        A(dalloc(&x->xp_lo, slots * x->H));
    }
    if (s != HF_OK) {
        std::string m = g_last_error;
        free_ctx(x);
        return fail(s, "hf_moe_create scratch: " + m);
    }
    if (x->gemm_ok) {
        // GEMM1 reads gathered activations (K = H); GEMM2 reads mid (K = I or Is).
        auto M = [&](CUtensorMap* m, const void* b, int cols, int pitch) {
            if (s == HF_OK) s = make_map_bf16(m, b, cols, slots, pitch, 16);
        };
        M(&x->maps1.B0, x->xp_hi, x->H, x->H);
        M(&x->maps1.B1, x->xp_lo, x->H, x->H);
        x->maps1.B0_sh = x->maps1.B0;
        x->maps1.B1_sh = x->maps1.B1;
        M(&x->maps2.B0, x->mid_hi, x->I, x->inter_max);
        M(&x->maps2.B1, x->mid_lo, x->I, x->inter_max);
        M(&x->maps2.B0_sh, x->mid_hi, x->Is > 0 ? x->Is : x->I, x->inter_max);
        M(&x->maps2.B1_sh, x->mid_lo, x->Is > 0 ? x->Is : x->I, x->inter_max);
        // the same views with kPairBoxB-row boxes (CTA-pair passes)
        auto W = [&](CUtensorMap* m, const void* b, int cols, int pitch) {
            if (s == HF_OK) s = make_map_bf16(m, b, cols, slots, pitch, kPairBoxB);
        };
        W(&x->maps1w.B0, x->xp_hi, x->H, x->H);
        W(&x->maps1w.B1, x->xp_lo, x->H, x->H);
        x->maps1w.B0_sh = x->maps1w.B0;
        x->maps1w.B1_sh = x->maps1w.B1;
        W(&x->maps2w.B0, x->mid_hi, x->I, x->inter_max);
        W(&x->maps2w.B1, x->mid_lo, x->I, x->inter_max);
        W(&x->maps2w.B0_sh, x->mid_hi, x->Is > 0 ? x->Is : x->I, x->inter_max);
        W(&x->maps2w.B1_sh, x->mid_lo, x->Is > 0 ? x->Is : x->I, x->inter_max);
        if (s != HF_OK) {
            std::string m = g_last_error;
            free_ctx(x);
            return fail(s, "hf_moe_create tensor maps: " + m);
        }
    }
    if (cudaMemset(x->plan, 0, sizeof(int32_t) * x->pl.words) != cudaSuccess ||
        cudaMemset(x->sched, 0, sizeof(int) * 8) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&x->err_host), 64) != cudaSuccess) {
        free_ctx(x);
        return fail(HF_ERR_CUDA, "hf_moe_create: plan/err buffer init failed");
    }
    *x->err_host = 0;
    x->grid1_bf16 = gemv_grid(c.device, true, false, x->H, x->inter_max, x->G);
    x->grid1_f32 = gemv_grid(c.device, true, true, x->H, x->inter_max, x->G);
    x->grid2 = gemv_grid(c.device, false, false, x->H, x->inter_max, x->G);
    if (world > 1) {
        s = ep_create(x, c.ep_unique_id);
        if (s != HF_OK) {
            std::string m = g_last_error;
            free_ctx(x);
            return fail(s, m);
        }
    }
    *out = x;
    return HF_OK;
}

hf_status hf_moe_destroy(hf_moe_ctx* ctx) {
    if (!ctx) return HF_OK;
    DeviceGuard dg(ctx->cfg.device);
    cudaDeviceSynchronize();
    free_ctx(ctx);
    return HF_OK;
}

static hf_status layer_alloc(hf_moe_ctx* c, int layer) {
    LayerBuf& L = c->layers[layer];
    if (L.router) return HF_OK;
    HF_TRY(dalloc(&L.router, size_t(c->E) * c->H));
    HF_TRY(dalloc(&L.bias, size_t(c->E)));
    HF_CUDA(cudaMemset(L.bias, 0, sizeof(float) * c->E));
    HF_TRY(dalloc(&L.experts, size_t(c->E_local) * c->expert_elems));
    if (c->Is > 0) HF_TRY(dalloc(&L.shared, size_t(3) * c->Is * c->H));
    HF_TRY(dalloc(&L.groups, size_t(c->G)));
    std::vector<GroupW> tab(c->G);
    for (int g = 0; g < c->G; ++g) {
        GroupW& w = tab[g];
        if (g < c->E_local) {
            const uint16_t* b = L.experts + size_t(g) * c->expert_elems;
            w.gate = b;
            w.up = b + size_t(c->I) * c->H;
            w.down = b + size_t(2) * c->I * c->H;
            w.inter = c->I;
        } else if (g == c->G - 1 && c->Is > 0) {
            w.gate = L.shared;
            w.up = L.shared + size_t(c->Is) * c->H;
            w.down = L.shared + size_t(2) * c->Is * c->H;
            w.inter = c->Is;
        } else {
            w.gate = w.up = w.down = nullptr;
            w.inter = 0;
        }
        w.down_f16 = 0;
        w.down_scale = 1.0f;
        w.pad = 0;
    }
    HF_CUDA(cudaMemcpy(L.groups, tab.data(), sizeof(GroupW) * c->G, cudaMemcpyHostToDevice));
    if (c->gemm_ok) {
        // one 2-D view per operand family covers every expert of the layer
        const uint64_t el = uint64_t(c->E_local);
        HF_TRY(make_map_bf16(&L.gu, L.experts, c->H, el * 3 * c->I, c->H, 128));
        HF_TRY(make_map_bf16(&L.dn, L.experts, c->I, el * 3 * c->H, c->I, 128));
        if (c->Is > 0) {
            const size_t n = size_t(c->Is) * c->H;
            HF_TRY(make_map_bf16(&L.sh_gate, L.shared, c->H, c->Is, c->H, 128));
            HF_TRY(make_map_bf16(&L.sh_up, L.shared + n, c->H, c->Is, c->H, 128));
            HF_TRY(make_map_bf16(&L.sh_down, L.shared + 2 * n, c->Is, c->H, c->Is, 128));
        } else {
            L.sh_gate = L.sh_up = L.gu;
            L.sh_down = L.dn;
        }
        HF_TRY(make_map_bf16(&L.rt, L.router, c->H, c->E, c->H, 128));
        L.maps = true;
    }
    return HF_OK;
}

static hf_status check_layer(hf_moe_ctx* c, int layer, const char* fn) {
    if (!c) return fail(HF_ERR_ARG, std::string(fn) + ": null context");
    if (layer < 0 || layer >= (int)c->layers.size())
        return fail(HF_ERR_ARG, std::string(fn) + ": layer out of range");
    return HF_OK;
}

static cudaMemcpyKind kind_of(hf_mem_kind k) {
    return k == HF_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
}

hf_status hf_moe_set_router(hf_moe_ctx* ctx, int layer, const uint16_t* router_bf16,
                            const float* bias, hf_mem_kind kind) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_set_router"));
    if (!router_bf16) return fail(HF_ERR_ARG, "hf_moe_set_router: null router weight");
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    HF_CUDA(cudaMemcpy(L.router, router_bf16, sizeof(uint16_t) * ctx->E * ctx->H, kind_of(kind)));
    if (bias) HF_CUDA(cudaMemcpy(L.bias, bias, sizeof(float) * ctx->E, kind_of(kind)));
    else HF_CUDA(cudaMemset(L.bias, 0, sizeof(float) * ctx->E));
    HF_TRY(place_router(ctx, L, nullptr));
    L.has_bias = bias != nullptr;
    L.loaded = true;
    return HF_OK;
}

hf_status hf_moe_set_expert(hf_moe_ctx* ctx, int layer, int eid, const uint16_t* gud,
                            hf_mem_kind kind) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_set_expert"));
    if (!gud) return fail(HF_ERR_ARG, "hf_moe_set_expert: null weights");
    const int l = local_slot(ctx, ctx->layers[layer], eid);
    if (l < 0) return fail(HF_ERR_ARG, "hf_moe_set_expert: expert id not owned by this context");
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    HF_CUDA(cudaMemcpy(L.experts + size_t(l) * ctx->expert_elems, gud,
                       sizeof(uint16_t) * ctx->expert_elems, kind_of(kind)));
    down_written(L, l);
    return HF_OK;
}

hf_status hf_moe_set_expert_parts(hf_moe_ctx* ctx, int layer, int eid, const uint16_t* gate,
                                  const uint16_t* up, const uint16_t* down, hf_mem_kind kind) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_set_expert_parts"));
    if (!gate || !up || !down) return fail(HF_ERR_ARG, "hf_moe_set_expert_parts: null projection");
    const int l = local_slot(ctx, ctx->layers[layer], eid);
    if (l < 0)
        return fail(HF_ERR_ARG, "hf_moe_set_expert_parts: expert id not owned by this context");
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    uint16_t* b = L.experts + size_t(l) * ctx->expert_elems;
    const size_t n = size_t(ctx->I) * ctx->H;
    HF_CUDA(cudaMemcpy(b, gate, sizeof(uint16_t) * n, kind_of(kind)));
    HF_CUDA(cudaMemcpy(b + n, up, sizeof(uint16_t) * n, kind_of(kind)));
    HF_CUDA(cudaMemcpy(b + 2 * n, down, sizeof(uint16_t) * n, kind_of(kind)));
    down_written(L, l);
    return HF_OK;
}

hf_status hf_moe_set_shared(hf_moe_ctx* ctx, int layer, const uint16_t* gate, const uint16_t* up,
                            const uint16_t* down, hf_mem_kind kind) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_set_shared"));
    if (ctx->Is == 0) return fail(HF_ERR_STATE, "hf_moe_set_shared: config has no shared expert");
    if (!gate || !up || !down) return fail(HF_ERR_ARG, "hf_moe_set_shared: null projection");
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    const size_t n = size_t(ctx->Is) * ctx->H;
    HF_CUDA(cudaMemcpy(L.shared, gate, sizeof(uint16_t) * n, kind_of(kind)));
    HF_CUDA(cudaMemcpy(L.shared + n, up, sizeof(uint16_t) * n, kind_of(kind)));
    HF_CUDA(cudaMemcpy(L.shared + 2 * n, down, sizeof(uint16_t) * n, kind_of(kind)));
    down_written(L, ctx->G - 1);
    return HF_OK;
}

hf_status hf_moe_expert_device_ptr(hf_moe_ctx* ctx, int layer, int eid, uint16_t** dev_ptr) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_expert_device_ptr"));
    if (!dev_ptr) return fail(HF_ERR_ARG, "hf_moe_expert_device_ptr: null output");
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    if (eid == ctx->E) {
        if (!L.shared) return fail(HF_ERR_STATE, "no shared expert in this config");
        HF_TRY(down_to_bf16(ctx, L, ctx->G - 1));  // the BF16 layout while the caller holds it
        *dev_ptr = L.shared;
        return HF_OK;
    }
    const int l = local_slot(ctx, L, eid);
    if (l < 0)
        return fail(HF_ERR_ARG, "hf_moe_expert_device_ptr: expert id not owned by this context");
    HF_TRY(down_to_bf16(ctx, L, l));
    *dev_ptr = L.experts + size_t(l) * ctx->expert_elems;
    return HF_OK;
}

hf_status hf_moe_router_device_ptr(hf_moe_ctx* ctx, int layer, uint16_t** router, float** bias) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_router_device_ptr"));
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    if (router) *router = L.router;
    if (bias) *bias = L.bias;
    L.has_bias = true;
    return HF_OK;
}

hf_status hf_moe_mark_loaded(hf_moe_ctx* ctx, int layer) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_mark_loaded"));
    if (!ctx->layers[layer].router) return fail(HF_ERR_STATE, "layer has no weights");
    ctx->layers[layer].loaded = true;
    ctx->layers[layer].down_ready = false;  // the next forward checks the down blocks again
    return HF_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static hf_status copy_routing(hf_moe_ctx* c, const LayerBuf& L, const hf_moe_routing* r, int T,
                              cudaStream_t st) {
    if (!r) return HF_OK;
    if (T == 0) {  // an empty batch routes nothing: zero counts and offsets
        if (r->counts) HF_CUDA(cudaMemsetAsync(r->counts, 0, sizeof(int32_t) * c->G_src, st));
        if (r->offsets)
            HF_CUDA(cudaMemsetAsync(r->offsets, 0, sizeof(int32_t) * (c->G_src + 1), st));
        return HF_OK;
    }
    if (!L.order.empty()) {  // placed expert ids: outputs in global ids
        const cudaMemcpyKind d2d = cudaMemcpyDeviceToDevice;
        if (r->topk_weights)
            HF_CUDA(cudaMemcpyAsync(r->topk_weights, c->w, sizeof(float) * T * c->k, d2d, st));
        if (r->margins) HF_CUDA(cudaMemcpyAsync(r->margins, c->margins, sizeof(float) * T, d2d, st));
        return unplace_routing(c, L, r, T, st);
    }
    const int k = c->k, G = c->G_src;
    const size_t nslots = size_t(T) * k + (c->Is > 0 ? T : 0);
    const cudaMemcpyKind d2d = cudaMemcpyDeviceToDevice;
    if (r->topk_ids) HF_CUDA(cudaMemcpyAsync(r->topk_ids, c->ids, sizeof(int32_t) * T * k, d2d, st));
    if (r->topk_weights) HF_CUDA(cudaMemcpyAsync(r->topk_weights, c->w, sizeof(float) * T * k, d2d, st));
    if (r->margins) HF_CUDA(cudaMemcpyAsync(r->margins, c->margins, sizeof(float) * T, d2d, st));
    if (r->counts)
        HF_CUDA(cudaMemcpyAsync(r->counts, c->plan_src + c->pl_src.counts, sizeof(int32_t) * G, d2d, st));
    if (r->offsets)
        HF_CUDA(cudaMemcpyAsync(r->offsets, c->plan_src + c->pl_src.offsets, sizeof(int32_t) * (G + 1),
                                d2d, st));
    if (r->perm) HF_CUDA(cudaMemcpyAsync(r->perm, c->perm_src, sizeof(int32_t) * nslots, d2d, st));
    return HF_OK;
}

static hf_status run_forward(hf_moe_ctx* c, int layer, const void* x, hf_dtype xd, int T,
                             float* out, const float* resid, const hf_moe_routing* r,
                             cudaStream_t st, bool route_only) {
    LayerBuf& L = c->layers[layer];
    if (!L.loaded) return fail(HF_ERR_STATE, "layer weights not set (hf_moe_set_router first)");
    if (T < 0 || T > c->T_max) return fail(HF_ERR_ARG, "T out of range (0..max_tokens)");
    if (xd != HF_BF16 && xd != HF_F32) return fail(HF_ERR_ARG, "x_dtype must be HF_BF16 or HF_F32");
    if (T > 0 && (!x || !aligned16(x))) return fail(HF_ERR_ARG, "x must be a 16-byte aligned device pointer");
    if (!route_only && T > 0 && (!out || !aligned16(out)))
        return fail(HF_ERR_ARG, "out must be a 16-byte aligned device pointer");
    c->last_stream = st;
    if (c->world > 1 && !route_only) {
        // every rank takes part in the exchanges, even with no tokens of its own
        HF_TRY(ensure_down_format(c, L, st));
        HF_TRY(ep_forward(c, L, x, xd, T, out, resid, r, st));
        return copy_routing(c, L, r, T, st);
    }
    if (T == 0) return copy_routing(c, L, r, T, st);  // zero counts and offsets
    if (!route_only) HF_TRY(ensure_down_format(c, L, st));
    const RouteArgs ra = route_args(c, L, x, xd, T);
    HF_TRY(run_route(c, L, ra, st));
    if (!route_only) {
        ExpertWork w{};
        w.down_f16 = L.down_f16;
        w.plan = c->plan;
        w.pl = c->pl;
        w.perm = c->perm;
        w.x = x;
        w.x_f32 = xd == HF_F32;
        w.T = T;
        w.k = c->k;
        w.y = c->y;
        w.bn1 = ra.gemm_bn1;
        w.bn2 = ra.gemm_bn2;
        w.m1 = ra.gemm_m1;
        w.m2 = ra.gemm_m2;
        w.pair = ra.gemm_pair;
        // segments can only exceed the GEMV threshold when T does
        w.maybe_gemm = ra.gemm_ok && (c->cfg.path == HF_PATH_GEMM || T > ra.gemv_max);
        w.maybe_gemv = !ra.gemm_ok || c->cfg.path == HF_PATH_GEMV ||
                       (c->cfg.path == HF_PATH_AUTO && ra.gemv_max > 0);
        w.y16 = y16_wanted(c, w.maybe_gemv);
        HF_TRY(run_experts(c, L, w, st));
        HF_TRY(run_combine(c, c->y, w.y16, T, out, resid, r ? r->slot_out : nullptr, st));
    }
    return copy_routing(c, L, r, T, st);
}

hf_status hf_moe_forward(hf_moe_ctx* ctx, int layer, const void* x, hf_dtype x_dtype, int T,
                         float* out, const hf_moe_routing* routing, hf_stream stream) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_forward"));
    DeviceGuard dg(ctx->cfg.device);
    return run_forward(ctx, layer, x, x_dtype, T, out, nullptr, routing, as_cuda(stream), false);
}

hf_status hf_moe_route(hf_moe_ctx* ctx, int layer, const void* x, hf_dtype x_dtype, int T,
                       const hf_moe_routing* routing, hf_stream stream) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_route"));
    DeviceGuard dg(ctx->cfg.device);
    return run_forward(ctx, layer, x, x_dtype, T, nullptr, nullptr, routing, as_cuda(stream), true);
}

hf_status hf_moe_forward_host(hf_moe_ctx* ctx, int layer, const void* x_host, hf_dtype x_dtype,
                              int T, float* out_host, hf_stream stream) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_forward_host"));
    if (T < 0 || T > ctx->T_max) return fail(HF_ERR_ARG, "T out of range (0..max_tokens)");
    if (T > 0 && (!x_host || !out_host)) return fail(HF_ERR_ARG, "null host buffer");
    DeviceGuard dg(ctx->cfg.device);
    cudaStream_t st = as_cuda(stream);
    const size_t xb = size_t(T) * ctx->H * (x_dtype == HF_F32 ? 4 : 2);
    if (T > 0) HF_CUDA(cudaMemcpyAsync(ctx->x_dev, x_host, xb, cudaMemcpyHostToDevice, st));
    HF_TRY(run_forward(ctx, layer, ctx->x_dev, x_dtype, T, ctx->out_dev, nullptr, nullptr, st,
                       false));
    if (T > 0)
        HF_CUDA(cudaMemcpyAsync(out_host, ctx->out_dev, sizeof(float) * T * ctx->H,
                                cudaMemcpyDeviceToHost, st));
    HF_CUDA(cudaMemcpyAsync(ctx->err_host, ctx->plan + ctx->pl.stats + 3, sizeof(int),
                            cudaMemcpyDeviceToHost, st));
    HF_CUDA(cudaStreamSynchronize(st));
    return take_error_word(ctx, *ctx->err_host);
}

hf_status hf_moe_synchronize(hf_moe_ctx* ctx) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_synchronize: null context");
    DeviceGuard dg(ctx->cfg.device);
    HF_CUDA(cudaStreamSynchronize(ctx->last_stream));
    int word = 0;
    HF_CUDA(cudaMemcpy(&word, ctx->plan + ctx->pl.stats + 3, sizeof(int), cudaMemcpyDeviceToHost));
    return take_error_word(ctx, word);
}

hf_status hf_moe_set_wait_timeout(hf_moe_ctx* ctx, uint64_t ns) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_set_wait_timeout: null context");
    ctx->timeout_ns = ns ? ns : 2000ull * 1000 * 1000;
    return HF_OK;
}

hf_status hf_moe_debug_stall(hf_moe_ctx* ctx, int enable) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_debug_stall: null context");
    ctx->stall = enable != 0;
    return HF_OK;
}

hf_status hf_moe_layer(hf_moe_ctx* ctx, int layer, const float* input, float* output) {
    return hf_moe_forward_host(ctx, layer, input, HF_F32, 1, output, nullptr);
}

// glm_forward.cpp:785-796: residual = hidden; hidden = rmsNorm(hidden);
// mlpOut = moeLayer(hidden); hidden = residual + mlpOut. The normalised rows
// go to the input staging buffer (fp32 or bf16), the layer runs on them, and
// the combine writes residual + (routed + shared) into hidden_out.
hf_status hf_moe_block_forward(hf_moe_ctx* ctx, int layer, const float* hidden_in,
                               float* hidden_out, const uint16_t* norm_weight, float eps,
                               hf_dtype act_dtype, int T, const hf_moe_routing* routing,
                               hf_stream stream) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_block_forward"));
    if (T < 0 || T > ctx->T_max) return fail(HF_ERR_ARG, "T out of range (0..max_tokens)");
    if (act_dtype != HF_F32 && act_dtype != HF_BF16)
        return fail(HF_ERR_ARG, "hf_moe_block_forward: act_dtype must be HF_F32 or HF_BF16");
    if (T > 0 && (!hidden_in || !hidden_out || !aligned16(hidden_in) || !aligned16(hidden_out)))
        return fail(HF_ERR_ARG, "hf_moe_block_forward: hidden must be 16-byte aligned device memory");
    if (norm_weight && !aligned16(norm_weight))
        return fail(HF_ERR_ARG, "hf_moe_block_forward: norm_weight must be 16-byte aligned");
    if (hidden_in != hidden_out && T > 0) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(hidden_in);
        const uintptr_t b = reinterpret_cast<uintptr_t>(hidden_out);
        const uintptr_t n = sizeof(float) * size_t(T) * ctx->H;
        if (a < b + n && b < a + n)
            return fail(HF_ERR_ARG, "hf_moe_block_forward: hidden_in and hidden_out overlap "
                                    "without being the same buffer");
    }
    DeviceGuard dg(ctx->cfg.device);
    cudaStream_t st = as_cuda(stream);
    if (T > 0) {
        PhaseTimer p9(ctx, st, 9);
        HF_TRY(launch_rmsnorm(hidden_in, norm_weight, eps, T, ctx->H,
                              act_dtype == HF_F32 ? kNormF32 : kNormBf16, ctx->x_dev, nullptr, st));
        p9.done(1);
    }
    return run_forward(ctx, layer, ctx->x_dev, act_dtype, T, hidden_out, hidden_in, routing, st,
                       false);
}

hf_status hf_moe_last_stats(hf_moe_ctx* ctx, int* active, int* gemv_segments, int* gemm_segments) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_last_stats: null context");
    DeviceGuard dg(ctx->cfg.device);
    int st[4] = {0, 0, 0, 0};
    HF_CUDA(cudaStreamSynchronize(ctx->last_stream));
    HF_CUDA(cudaMemcpy(st, ctx->plan + ctx->pl.stats, sizeof(st), cudaMemcpyDeviceToHost));
    if (active) *active = st[0];
    if (gemv_segments) *gemv_segments = st[1];
    if (gemm_segments) *gemm_segments = st[2];
    return HF_OK;
}

hf_status hf_moe_profile(hf_moe_ctx* ctx, int enable) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_profile: null context");
    ctx->profiling = enable != 0;
    return HF_OK;
}

hf_status hf_moe_profile_read(hf_moe_ctx* ctx, double* phase_ms, long long* launches) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_profile_read: null context");
    DeviceGuard dg(ctx->cfg.device);
    double ms[HF_MOE_PHASES] = {};
    hf_status s = HF_OK;
    for (auto& m : ctx->marks) {
        float t = 0.f;
        cudaError_t e = cudaEventSynchronize(m.b);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t, m.a, m.b);
        if (e != cudaSuccess && s == HF_OK) s = cuda_fail(e, "cudaEventElapsedTime");
        ms[m.phase] += t;
        ctx->ev_pool.push_back(m.a);
        ctx->ev_pool.push_back(m.b);
    }
    ctx->marks.clear();
    for (int i = 0; i < HF_MOE_PHASES; ++i) {
        if (phase_ms) phase_ms[i] = ms[i];
        if (launches) launches[i] = ctx->launches[i];
        ctx->launches[i] = 0;
    }
    return s;
}

hf_status hf_gemv_bf16_f32(const uint16_t* A, const float* x, float* y, int M, int K, float alpha,
                           float beta, hf_stream stream) {
    if (M < 0 || K < 0) return fail(HF_ERR_ARG, "hf_gemv_bf16_f32: negative size");
    if (M > 0 && (!y || (K > 0 && (!A || !x)))) return fail(HF_ERR_ARG, "hf_gemv_bf16_f32: null pointer");
    return launch_gemv_plain(A, x, y, M, K, alpha, beta, as_cuda(stream));
}

hf_status hf_topk_scores(const float* scores, int T, int E, const float* bias, int k, float scale,
                         int norm, int32_t* idx, float* weights, hf_stream stream) {
    if (T < 0 || E <= 0 || E > kMaxExperts || k <= 0 || k > kMaxTopK)
        return fail(HF_ERR_ARG, "hf_topk_scores: need T >= 0, 1 <= E <= 1024, 1 <= k <= 8");
    if (T > 0 && (!scores || !idx || !weights)) return fail(HF_ERR_ARG, "hf_topk_scores: null pointer");
    return launch_topk(scores, T, E, bias, std::min(k, E), scale, norm, idx, weights, 0, nullptr,
                       as_cuda(stream));
}

hf_status hf_moe_synth_layer(hf_moe_ctx* ctx, int layer, uint64_t seed, uint32_t gen_layer,
                             const float* bias_override, hf_stream stream) {
    HF_TRY(check_layer(ctx, layer, "hf_moe_synth_layer"));
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    cudaStream_t st = as_cuda(stream);
    const float sc = synth_normal_scale(0.02);
    HF_TRY(synth_bf16(L.router, size_t(ctx->E) * ctx->H,
                      synth_key(seed, gen_layer, HF_SYNTH_ROUTER, 0), sc, st));
    if (bias_override)
        HF_CUDA(cudaMemcpyAsync(L.bias, bias_override, sizeof(float) * ctx->E,
                                cudaMemcpyHostToDevice, st));
    else
        HF_TRY(synth_f32u(L.bias, size_t(ctx->E), synth_key(seed, gen_layer, HF_SYNTH_BIAS, 0),
                          -0.1f, 0.1f, st));
    L.has_bias = true;
    HF_TRY(place_router(ctx, L, st));
    const size_t n = size_t(ctx->I) * ctx->H;
    for (int e = 0; e < ctx->E_local; ++e) {
        uint16_t* b = L.experts + size_t(e) * ctx->expert_elems;
        const uint32_t eid = uint32_t(slot_expert(ctx, L, e));
        HF_TRY(synth_bf16(b, n, synth_key(seed, gen_layer, HF_SYNTH_GATE, eid), sc, st));
        HF_TRY(synth_bf16(b + n, n, synth_key(seed, gen_layer, HF_SYNTH_UP, eid), sc, st));
        HF_TRY(synth_bf16(b + 2 * n, n, synth_key(seed, gen_layer, HF_SYNTH_DOWN, eid), sc, st));
    }
    if (ctx->Is > 0) {
        const size_t ns = size_t(ctx->Is) * ctx->H;
        const uint32_t eid = uint32_t(ctx->E);
        HF_TRY(synth_bf16(L.shared, ns, synth_key(seed, gen_layer, HF_SYNTH_GATE, eid), sc, st));
        HF_TRY(synth_bf16(L.shared + ns, ns, synth_key(seed, gen_layer, HF_SYNTH_UP, eid), sc, st));
        HF_TRY(synth_bf16(L.shared + 2 * ns, ns, synth_key(seed, gen_layer, HF_SYNTH_DOWN, eid), sc, st));
    }
    if (bias_override) HF_CUDA(cudaStreamSynchronize(st));  // host array may go away
    down_written(L, -1);
    L.loaded = true;
    return HF_OK;
}

}  // extern "C"

namespace hf {
hf_status ctx_layer_alloc(hf_moe_ctx* c, int layer) { return layer_alloc(c, layer); }
}  // namespace hf
