// hf_dense.cu -- dense SwiGLU MLP (GLMForward::denseMlp, glm_forward.cpp:411-432).
//
// The reference runs three GEMVs per token: g = Wg x, u = Wu x (I x H each),
// mid = g / (1 + exp(-g)) * u in fp32, out = Wd mid (H x I). The math is the
// one of a routed expert, so this entry reuses the expert kernels unchanged:
// a plan with one group -- the shared-expert slot (G = 1) -- that holds all T
// tokens in order, with the three weight matrices given as separate pointers
// (the kernels read the shared expert through separate gate / up / down
// views). One token (decode) takes the GEMV pair; two or more take the tcgen05
// grouped GEMM, whose down-projection epilogue writes the fp32 output rows in
// place (positions are tokens; no combine step).
//
// Stateless: every buffer lives in the caller's workspace, so any number of
// dense layers can share one. Asynchronous on the stream; a bounded-wait
// timeout inside the GEMM is reported by hf_dense_mlp_status.
#include <algorithm>
#include <cstring>

#include "hf_internal.cuh"

namespace hf {
namespace {

constexpr size_t kAlign = 256;
constexpr int kDenseGemvMax = 1;  // tokens up to which the GEMV pair runs

size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

struct DenseWs {
    size_t plan, groups, sched, perm, scratch, total;
    // scratch: GEMV path mid fp32 [T x I]; GEMM path xp_hi, xp_lo [T x H] and
    // mid_hi, mid_lo [T x I] (bf16)
    size_t xp_lo, mid_hi, mid_lo;
    // GEMV path only: the residual block's normalised rows [T x H] (fp32 or bf16)
    size_t xn;
};

bool takes_gemm(int T, int H, int I) { return T > kDenseGemvMax && H % 64 == 0 && I % 64 == 0; }

DenseWs layout(int T, int H, int I) {
    DenseWs w{};
    const PlanLayout pl = PlanLayout::make(1);
    size_t o = 0;
    w.plan = o;
    o += up(sizeof(int32_t) * pl.words);
    w.groups = o;
    o += up(sizeof(GroupW));
    w.sched = o;
    o += up(sizeof(int) * 2);
    w.perm = o;
    o += up(sizeof(int32_t) * size_t(T));
    w.scratch = o;
    const size_t xp = up(size_t(T) * H * 2), mh = up(size_t(T) * I * 2);
    w.xp_lo = o + xp;
    w.mid_hi = o + 2 * xp;
    w.mid_lo = o + 2 * xp + mh;
    const size_t gemm = 2 * xp + 2 * mh;
    const size_t gemv = up(size_t(T) * I * 4);
    w.xn = o + std::max(gemm, gemv);
    w.total = w.xn + (takes_gemm(T, H, I) ? 0 : up(size_t(T) * H * 4));
    return w;
}

// The residual block around the MLP (glm_forward.cpp:785-796): the rows of
// `hidden` are normalised into the layer's input and added back by the down
// projection's store.
struct DenseNorm {
    const float* hidden;
    const uint16_t* w;
    float eps;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// x / x_dtype: the layer input (norm == nullptr), or the form the normalised
// rows take (norm != nullptr; x unused). resid: added by the down store.
hf_status dense_run(const char* fn, const uint16_t* gate, const uint16_t* upw,
                    const uint16_t* down, const void* x, hf_dtype x_dtype, const DenseNorm* norm,
                    int T, int H, int I, float* out, void* workspace, size_t workspace_bytes,
                    cudaStream_t st) {
    const std::string f(fn);
    if (T < 0 || H <= 0 || I <= 0) return fail(HF_ERR_ARG, f + ": bad shape");
    if (T == 0) return HF_OK;
    if (!gate || !upw || !down || !(norm ? (const void*)norm->hidden : x) || !out || !workspace)
        return fail(HF_ERR_ARG, f + ": null pointer");
    if (x_dtype != HF_BF16 && x_dtype != HF_F32)
        return fail(HF_ERR_ARG, f + ": activations must be bf16 or f32");
    if (H % 8 || I % 8) return fail(HF_ERR_ARG, f + ": H and I must be multiples of 8");
    if (!aligned16(gate) || !aligned16(upw) || !aligned16(down) || !aligned16(out) ||
        (norm ? !aligned16(norm->hidden) || (norm->w && !aligned16(norm->w)) : !aligned16(x)))
        return fail(HF_ERR_ARG, f + ": pointers must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) % kAlign)
        return fail(HF_ERR_ARG, f + ": workspace must be 256-byte aligned");
    const DenseWs L = layout(T, H, I);
    if (workspace_bytes < L.total)
        return fail(HF_ERR_ARG, f + ": workspace smaller than hf_dense_mlp_workspace_size");
    if (norm && norm->hidden != out) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(norm->hidden);
        const uintptr_t b = reinterpret_cast<uintptr_t>(out);
        const uintptr_t n = sizeof(float) * size_t(T) * H;
        if (a < b + n && b < a + n)
            return fail(HF_ERR_ARG, f + ": hidden_in and hidden_out overlap without being the "
                                        "same buffer");
    }
    int dev = 0;
    HF_CUDA(cudaGetDevice(&dev));
    const bool xf32 = x_dtype == HF_F32;
    const bool gemm = takes_gemm(T, H, I);
    if (!gemm && (gemv1_smem(H, xf32, 1) > 227 * 1024 || gemv2_smem(I, 1) > 227 * 1024))
        return fail(HF_ERR_ARG, f + ": H or I too large for the GEMV staging");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int32_t* plan = reinterpret_cast<int32_t*>(ws + L.plan);
    GroupW* groups = reinterpret_cast<GroupW*>(ws + L.groups);
    int32_t* perm = reinterpret_cast<int32_t*>(ws + L.perm);
    int* sched = reinterpret_cast<int*>(ws + L.sched);
    const PlanLayout pl = PlanLayout::make(1);
    const float* resid = norm ? norm->hidden : nullptr;

    RouteArgs ra{};
    ra.T = T;
    ra.H = H;
    ra.E = 0;
    ra.k = 0;
    ra.plan = plan;
    ra.pl = pl;
    ra.has_shared = 1;
    ra.shared_inter = I;
    ra.inter = I;
    ra.path = gemm ? HF_PATH_GEMM : HF_PATH_GEMV;
    ra.gemv_max = kDenseGemvMax;
    ra.gemm_ok = gemm;
    set_gemm_tiles(0, T, ra);
    // one group (the whole layer) makes few tiles at decode sizes: 128-row down
    // tiles of 32 tokens (48 x ceil(T/32) tiles at H = 6144) beat the MoE
    // decode shape of 256 x 16 here (measured 0.20 vs 0.26 ms at T = 64)
    if (T <= 64) {
        ra.gemm_bn2 = 32;
        ra.gemm_m2 = 128;
    }
    GroupW w{gate, upw, down, I, 0};
    HF_TRY(launch_dense_plan(ra, w, groups, perm, sched, st));

    if (!gemm) {
        if (norm) {
            x = ws + L.xn;
            HF_TRY(launch_rmsnorm(norm->hidden, norm->w, norm->eps, T, H,
                                  xf32 ? kNormF32 : kNormBf16, ws + L.xn, nullptr, st));
        }
        GemvArgs ga{};
        ga.groups = groups;
        ga.plan = plan;
        ga.pl = pl;
        ga.perm = perm;
        ga.x = x;
        ga.x_f32 = xf32;
        ga.T = T;
        ga.H = H;
        ga.k = 0;
        ga.inter_max = I;
        ga.mid = reinterpret_cast<float*>(ws + L.scratch);
        ga.y = out;
        ga.resid = resid;
        ga.te_cap = std::min(T, kGemvTE);
        ga.grid1 = gemv_grid(dev, true, xf32, H, I, 1, ga.te_cap);
        ga.grid2 = gemv_grid(dev, false, xf32, H, I, 1, ga.te_cap);
        HF_TRY(launch_gemv1(ga, st));
        return launch_gemv2(ga, st);
    }

    uint16_t* xp_hi = reinterpret_cast<uint16_t*>(ws + L.scratch);
    uint16_t* xp_lo = reinterpret_cast<uint16_t*>(ws + L.xp_lo);
    uint16_t* mid_hi = reinterpret_cast<uint16_t*>(ws + L.mid_hi);
    uint16_t* mid_lo = reinterpret_cast<uint16_t*>(ws + L.mid_lo);
    GemmMaps m1{}, m2{};
    if (norm) {  // the RMSNorm writes the GEMM's operand planes (token order) itself
        HF_TRY(launch_rmsnorm(norm->hidden, norm->w, norm->eps, T, H,
                              xf32 ? kNormHiLo : kNormBf16, xp_hi, xp_lo, st));
        HF_TRY(make_map_bf16(&m1.B0, xp_hi, H, T, H, 16));
        if (xf32) HF_TRY(make_map_bf16(&m1.B1, xp_lo, H, T, H, 16));
        else m1.B1 = m1.B0;
    } else if (xf32) {  // fp32 activations: split into bf16 hi + lo planes
        GatherArgs gx{};
        gx.plan = plan;
        gx.pl = pl;
        gx.perm = perm;
        gx.x = x;
        gx.T = T;
        gx.k = 0;
        gx.H = H;
        gx.device = dev;
        gx.xp_hi = xp_hi;
        gx.xp_lo = xp_lo;
        HF_TRY(launch_gather(gx, 1, st));
        HF_TRY(make_map_bf16(&m1.B0, xp_hi, H, T, H, 16));
        HF_TRY(make_map_bf16(&m1.B1, xp_lo, H, T, H, 16));
    } else {  // bf16 activations are already the GEMM's token-major operand
        HF_TRY(make_map_bf16(&m1.B0, x, H, T, H, 16));
        m1.B1 = m1.B0;
    }
    HF_TRY(make_map_bf16(&m1.A_sh, gate, H, I, H, 128));
    HF_TRY(make_map_bf16(&m1.A_sh2, upw, H, I, H, 128));
    m1.A = m1.A_sh;
    m1.B0_sh = m1.B0;
    m1.B1_sh = m1.B1;
    HF_TRY(make_map_bf16(&m2.A_sh, down, I, H, I, 128));
    m2.A = m2.A_sh2 = m2.A_sh;
    HF_TRY(make_map_bf16(&m2.B0, mid_hi, I, T, I, 16));
    HF_TRY(make_map_bf16(&m2.B1, mid_lo, I, T, I, 16));
    m2.B0_sh = m2.B0;
    m2.B1_sh = m2.B1;

    GemmArgs gm{};
    gm.plan = plan;
    gm.pl = pl;
    gm.which = 1;
    gm.H = H;
    gm.I = I;
    gm.Is = I;
    gm.Imax = I;
    gm.bn = ra.gemm_bn1;
    gm.mrows = ra.gemm_m1;
    gm.pair = ra.gemm_pair;
    gm.mid_hi = mid_hi;
    gm.mid_lo = mid_lo;
    gm.y = out;
    gm.resid = resid;
    gm.err = plan + pl.stats + 3;
    gm.timeout_ns = 2000ull * 1000 * 1000;
    gm.test_stall = 0;
    gm.sched = sched;
    const int nsm = num_sms(dev);
    HF_TRY(launch_gemm(m1, gm, xf32 ? 2 : 1, nsm, st));
    gm.which = 2;
    gm.bn = ra.gemm_bn2;
    gm.mrows = ra.gemm_m2;
    return launch_gemm(m2, gm, 2, nsm, st);
}

}  // namespace
}  // namespace hf

using namespace hf;

extern "C" {

size_t hf_dense_mlp_workspace_size(int T, int H, int I) {
    if (T <= 0 || H <= 0 || I <= 0) return 0;
    return layout(T, H, I).total;
}

hf_status hf_dense_mlp_forward(const uint16_t* gate, const uint16_t* upw, const uint16_t* down,
                               const void* x, hf_dtype x_dtype, int T, int H, int I, float* out,
                               void* workspace, size_t workspace_bytes, hf_stream stream) {
    return dense_run("hf_dense_mlp_forward", gate, upw, down, x, x_dtype, nullptr, T, H, I, out,
                     workspace, workspace_bytes, as_cuda(stream));
}

hf_status hf_dense_block_forward(const uint16_t* gate, const uint16_t* upw, const uint16_t* down,
                                 const uint16_t* norm_weight, float eps, hf_dtype act_dtype,
                                 const float* hidden_in, float* hidden_out, int T, int H, int I,
                                 void* workspace, size_t workspace_bytes, hf_stream stream) {
    const DenseNorm n{hidden_in, norm_weight, eps};
    return dense_run("hf_dense_block_forward", gate, upw, down, nullptr, act_dtype, &n, T, H, I,
                     hidden_out, workspace, workspace_bytes, as_cuda(stream));
}

hf_status hf_dense_mlp_status(const void* workspace, hf_stream stream) {
    if (!workspace) return fail(HF_ERR_ARG, "hf_dense_mlp_status: null workspace");
    HF_CUDA(cudaStreamSynchronize(as_cuda(stream)));
    const PlanLayout pl = PlanLayout::make(1);
    int word = 0;
    HF_CUDA(cudaMemcpy(&word, static_cast<const int32_t*>(workspace) + pl.stats + 3, sizeof(int),
                       cudaMemcpyDeviceToHost));
    if (word) return fail(HF_ERR_TIMEOUT, "hf_dense_mlp_forward: a GEMM wait ran out of time");
    return HF_OK;
}

}  // extern "C"
