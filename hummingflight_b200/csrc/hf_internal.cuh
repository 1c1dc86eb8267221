// hf_internal.cuh -- shared device helpers and host plumbing of libhf_moe.so.
#pragma once

#include <cuda.h>  // CUtensorMap (the encode entry point is fetched at run time)
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "hf_moe.h"

namespace hf {

// ------------------------------------------------------------------ errors
void set_error(const std::string& msg);
hf_status fail(hf_status s, const std::string& msg);
hf_status cuda_fail(cudaError_t e, const char* what);

#define HF_CUDA(call)                                                        \
    do {                                                                     \
        cudaError_t _e = (call);                                             \
        if (_e != cudaSuccess) return ::hf::cuda_fail(_e, #call);            \
    } while (0)

#define HF_TRY(call)                                                         \
    do {                                                                     \
        hf_status _s = (call);                                               \
        if (_s != HF_OK) return _s;                                          \
    } while (0)

inline cudaStream_t as_cuda(hf_stream s) { return reinterpret_cast<cudaStream_t>(s); }

// ------------------------------------------------------------------ limits
constexpr int kMaxTopK = 8;        // TopKResult holds 8 (compute/moe_router.h:12-16)
constexpr int kMaxExperts = 1024;  // top-k kernel keeps E/32 scores per lane
constexpr int kSmallRouteT = 128;  // single-CTA routing up to this many tokens
constexpr int kGemvTE = 4;         // tokens per grouped-GEMV chunk
constexpr int kGemv1Rows = 16;     // gate/up rows per GEMV1 unit (8 warps x 2)
constexpr int kGemv2Rows = 32;     // down rows per GEMV2 unit (8 warps x 4)
// AUTO with gemv_max_tokens = 0: a single token runs on the GEMV; every
// larger pass runs every segment on the tcgen05 GEMM, whose weight stream runs
// at the copy rate (the GEMV pair at 75-88 % of it). Measured on the GLM
// layer: 1 token GEMV 0.169 vs GEMM 0.197 ms; 2 / 4 / 8 / 16 tokens GEMM
// 0.29 / 0.48 / 0.70 / 1.04 ms vs single-token segments on the GEMV 0.37 /
// 0.55 / 0.78 / 1.09 ms.
constexpr int kGemvAutoBatch = 1;
constexpr int kGemvAutoMax = 1;

// Weights of one expert group (routed expert or the shared expert).
struct GroupW {
    const uint16_t* gate;  // [inter x H]
    const uint16_t* up;    // [inter x H]
    const uint16_t* down;  // [H x inter]: BF16, or FP16 holding w * 2^S when down_f16
    int inter;
    int down_f16;          // the down block is stored as FP16 (see down_scale)
    float down_scale;      // 2^-S: multiplies products with the FP16 down block
    int pad;
};

// Device plan of one forward, written by the routing kernels.
// Offsets are in int32 words from the start of the plan buffer.
struct PlanLayout {
    int G;            // groups = E + 1 (shared last, count 0 when absent)
    int counts;       // [G]
    int offsets;      // [G+1] positions
    int u1;           // [G+1] GEMV1 unit prefix
    int u2;           // [G+1] GEMV2 unit prefix
    int g1;           // [G+1] GEMM1 (gate/up) tile prefix
    int g2;           // [G+1] GEMM2 (down) tile prefix
    int stats;        // [4]: active experts, gemv segments, gemm segments, error word
    int words;        // total
    static PlanLayout make(int G) {
        PlanLayout p;
        p.G = G;
        p.counts = 0;
        p.offsets = p.counts + G;
        p.u1 = p.offsets + G + 1;
        p.u2 = p.u1 + G + 1;
        p.g1 = p.u2 + G + 1;
        p.g2 = p.g1 + G + 1;
        p.stats = p.g2 + G + 1;
        p.words = p.stats + 4;
        return p;
    }
};

// Everything the routing kernels need.
struct RouteArgs {
    const void* x;            // [T x H] bf16 or f32
    int x_f32;
    int T, H, E, k;           // k = min(top_k, E)
    const uint16_t* router;   // [E x H]
    const float* bias;        // [E] or null
    float scale;
    int norm;
    float* logits;            // [T x E]
    int32_t* ids;             // [T x k]
    float* w;                 // [T x k]
    float* margins;           // [T]
    int32_t* plan;            // PlanLayout
    PlanLayout pl;
    int has_shared;
    int shared_inter, inter;
    int32_t* perm;            // [T*k + T]
    int32_t* slot_pos;        // [T*k + T]
    uint32_t* masks;          // [nb x E x 4] (multi-block path)
    int32_t* blk_counts;      // [nb x E]
    int path;                 // hf_path
    int gemv_max;             // AUTO threshold
    int gemm_ok;              // shapes allow the tcgen05 GEMM (64-aligned)
    int gemm_bn1, gemm_bn2;   // token tile (columns per tile) of GEMM1 / GEMM2
    int gemm_m1, gemm_m2;     // weight rows per GEMM1 / GEMM2 tile (128 or 256)
    int gemm_pair;            // GEMM tiles run on CTA pairs
    int lsplit;               // logits are the sum of lsplit planes of [T x E] (split-K router)
    int* route_counter;       // zeroed device int: router + routing in one launch (null: two)
};

// ------------------------------------------------------------------ programmatic dependent launch
// A kernel launched with launch_pdl may start while the previous kernel of the
// stream still runs; it must call griddep_wait() before it reads anything that
// kernel writes (the wait returns once that grid has completed and its writes
// are visible). griddep_launch_dependents() lets the next PDL launch start
// early (without it, the next kernel starts when this one exits). Without a
// PDL predecessor griddep_wait() returns at once.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ------------------------------------------------------------------ device helpers
// Pulls [p, p + bytes) into L2, the grid's threads striding over 128-byte lines.
template <bool EVICT_LAST>
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
    const char* c = static_cast<const char*>(p);
    const size_t lines = bytes / 128, nthr = size_t(gridDim.x) * blockDim.x;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < lines; i += nthr) {
        if constexpr (EVICT_LAST)
            asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(c + i * 128));
        else
            asm volatile("prefetch.global.L2 [%0];" ::"l"(c + i * 128));
    }
}

// Read-only 16-byte loads (weights and activations never change during a
// kernel); not volatile, so the compiler may batch them for memory-level
// parallelism.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ld_nc_u4(const void* p) {
    uint4 r;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
    return __uint_as_float(uint32_t(h) << 16);
}

// BFloat16::fromF32 (compute/dtype_bf16.h:27-33): RNE without a NaN case.
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
    uint32_t u = __float_as_uint(f);
    return uint16_t((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// 8 consecutive elements of x as fp32 (bf16 widened exactly).
__device__ __forceinline__ void unpack8(const uint4 v, float (&o)[8]) {
    o[0] = bf16lo(v.x); o[1] = bf16hi(v.x);
    o[2] = bf16lo(v.y); o[3] = bf16hi(v.y);
    o[4] = bf16lo(v.z); o[5] = bf16hi(v.z);
    o[6] = bf16lo(v.w); o[7] = bf16hi(v.w);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// SiLU-gated product of the reference (glm_forward.cpp:444-446), IEEE ops.
__device__ __forceinline__ float swiglu(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}
// The same with the fast exponential and the fast division (a few ulp from
// swiglu, far below the rounding of mid to FP16 or to a BF16 hi + lo pair):
// the tensor-core epilogue evaluates it for every element of a tile. For
// g < -88 the exponential overflows and the quotient is -0, as in swiglu.
__device__ __forceinline__ float swiglu_fast(float g, float u) {
    return __fmul_rn(__fdividef(g, __fadd_rn(1.0f, __expf(-g))), u);
}

__device__ __forceinline__ int token_of_slot(int slot, int T, int k) {
    return slot < T * k ? slot / k : slot - T * k;
}

// Copies a unit/tile prefix [G+1], counts [G] and offsets [G] of the plan into
// shared memory (3G+1 words at sp), so per-unit lookups do not chain global
// loads. The caller synchronizes the block before use.
__device__ __forceinline__ void stage_plan(int32_t* sp, const int32_t* prefix, const int32_t* plan,
                                           const PlanLayout& pl) {
    const int G = pl.G;
    for (int i = threadIdx.x; i <= G; i += blockDim.x) sp[i] = prefix[i];
    for (int i = threadIdx.x; i < G; i += blockDim.x) {
        sp[G + 1 + i] = plan[pl.counts + i];
        sp[2 * G + 1 + i] = plan[pl.offsets + i];
    }
}

__host__ __device__ __forceinline__ size_t plan_smem_bytes(int G) {
    return (size_t(3 * G + 1) * 4 + 15) & ~size_t(15);
}

// Largest g with prefix[g] <= u (prefix non-decreasing, prefix[0] = 0).
__device__ __forceinline__ int find_group(const int32_t* prefix, int G, int u) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// ------------------------------------------------------------------ launchers
int num_sms(int device);
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device, size).
cudaError_t ensure_smem(const void* kernel, int bytes);

// Router logits; with `routed` non-null, small batches also run the whole
// routing in the same launch (then *routed = true and launch_route is skipped).
hf_status launch_router_logits(const RouteArgs& a, cudaStream_t st, bool* routed = nullptr);
// GEMM tiles (gemm_bn1, gemm_bn2, gemm_m2) for a pass over `rows` activation
// rows; bn_override (32, 64 or 128) forces both token tiles when non-zero.
void set_gemm_tiles(int bn_override, int rows, RouteArgs& ra);
// Work plan (counts, offsets, unit and tile prefixes) from per-group counts
// already in device memory (expert-parallel receivers, dense MLP).
hf_status launch_plan_from_counts(const RouteArgs& a, const int32_t* counts, cudaStream_t st);
// Expert-parallel receiver plan from device counts (fixed-capacity slabs of
// `cap` rows per source); see k_ep_plan. With `flags` it first waits (bounded)
// for every source's arrival flag to reach `seq` (peer-memory exchange).
// Output rows of an expert-parallel receiver's positions (yrow == nullptr:
// none written): peer_y[s] is rank s's output slab as mapped here.
struct EpRowOut {
    float** yrow;            // [positions] device
    float* const* peer_y;    // [W] device
    int rank, H;
    int esz;                 // bytes per output element: 4 (fp32) or 2 (FP16 plane)
};
// rmap (optional, [W x cap]): the slab row each received slot reads --
// sources send a token's row once per destination rank, however many of
// its experts live there (nullptr: row = arrival index).
hf_status launch_ep_plan(const RouteArgs& a, const int32_t* cnt, const int32_t* rmap, int W,
                         int El, int cap, int T_loc,
                         int32_t* perm, int32_t* row_pos, int32_t* recv_tot,
                         const unsigned long long* flags, unsigned long long seq,
                         unsigned long long timeout_ns, int* err, const EpRowOut& ro,
                         cudaStream_t st);
// Dense MLP pass: one group of all T tokens in order; writes groups[0] = w.
hf_status launch_dense_plan(const RouteArgs& a, const GroupW& w, GroupW* groups, int32_t* perm,
                            int* sched, cudaStream_t st);
// dst row i = src row (idx[i] / div), i < n; rows of row_bytes (multiple of 16).
hf_status launch_gather_rows(void* dst, const void* src, size_t row_bytes, int n,
                             const int32_t* idx, int div, cudaStream_t st);
// Top-k + permutation + plan; *launches receives the number of kernels.
hf_status launch_route(const RouteArgs& a, cudaStream_t st, int* launches);
hf_status launch_topk(const float* scores, int T, int E, const float* bias, int k, float scale,
                      int norm, int32_t* idx, float* w, int apply_sigmoid, float* margins,
                      cudaStream_t st);

struct GemvArgs {
    const GroupW* groups;   // [G] device
    const int32_t* plan;
    PlanLayout pl;
    const int32_t* perm;
    const void* x;          // [T x H]
    int x_f32;
    int T, H, k;
    int inter_max;          // mid row stride
    float* mid;             // [(T*k+T) x inter_max] fp32
    float* y;               // [(T*k+T) x H] fp32
    const float* resid;     // optional, one group whose positions are tokens (dense MLP):
                            // y = resid + down row; may alias y
    // the last group (the shared expert) is pulled into L2 by GEMV1 before it
    // waits for the routing kernel, its units run first (set when its three
    // matrices fit in L2 with room to spare)
    int prefetch_shared;
    int grid1, grid2;
    int te_cap;             // most tokens in one chunk: min(T, kGemvTE); sizes the staging
};
hf_status launch_gemv1(const GemvArgs& a, cudaStream_t st);
hf_status launch_gemv2(const GemvArgs& a, cudaStream_t st);
// Persistent grid (SM count x resident blocks) of GEMV1 (first) or GEMV2.
int gemv_grid(int device, bool first, bool xf32, int H, int inter_max, int G, int te = kGemvTE);
size_t gemv1_smem(int H, bool xf32, int G, int te = kGemvTE);
size_t gemv2_smem(int inter_max, int G, int te = kGemvTE);

// tcgen05 grouped GEMM (hf_gemm.cu).
struct GemmArgs {
    const int32_t* plan;
    PlanLayout pl;
    int which;              // 1: gate/up + SwiGLU -> mid hi/lo; 2: down -> y
    int H, I, Is, Imax, bn;
    int mrows;              // weight rows per tile: 128, or 256 (two row blocks, or a CTA pair)
    int pair;               // tiles run on CTA pairs (cta_group::2), 128 weight rows per CTA
    uint16_t* mid_hi;       // [slots x Imax] bf16
    uint16_t* mid_lo;
    float* y;               // [slots x H] fp32
    // optional (GEMM2, nsplit == 1, one group whose positions are tokens --
    // the dense MLP): y = resid + down row; may alias y
    const float* resid;
    int* err;               // error word (plan stats[3])
    unsigned long long timeout_ns;
    int test_stall;         // wait on a barrier nothing signals (test hook)
    int plan_smem;          // set by the launcher: plan arrays staged in shared memory
    // plan == nullptr: one group of dense_T rows in order (no device plan)
    int dense_T;
    // GEMM2 split-K: nsplit > 1 cuts the K blocks into runs of kbper; run s
    // writes its partial sums to y + s * split_stride (summed by the reader)
    int nsplit, kbper;
    long long split_stride;
    // tile scheduler: [0] next tile id, [1] CTAs done; zero before a launch,
    // left zero by it (device memory owned by the caller, one pair per stream)
    int* sched;
    // optional (GEMM2, nsplit == 1, no resid): output row of position p at
    // yrow[p] instead of y + p * H -- a row in another GPU's memory (a peer
    // mapping) when an expert-parallel receiver returns outputs from the
    // epilogue. With sig_flags set, every thread fences its stores system-wide
    // and the last CTA out stores sig_seq (release, system scope) to
    // sig_flags[d][sig_slot] for d < sig_n.
    float* const* yrow;
    unsigned long long* const* sig_flags;
    int sig_n, sig_slot;
    unsigned long long sig_seq;
    // FP16 down pass: GEMM1 writes mid as one FP16 plane holding mid * 2^-kMidF16Shift
    // (mid_hi), GEMM2 multiplies FP16 down rows (w * 2^S) by it and scales its
    // accumulator by 2^kMidF16Shift * groups[g].down_scale
    int down_f16;
    const GroupW* groups;
    // GEMM2 (no resid, nsplit == 1): outputs as one FP16 plane holding
    // y * 2^-kYF16Shift (y and yrow[] then address __half elements)
    int y16;
    // rows of one activation (B) box of the tensor maps passed: 16, or
    // kPairBoxB on CTA-pair passes given the wide maps (0 means 16)
    int box_b;
};
// activation box rows of the wide maps (a CTA of a 256-token pair tile loads
// its 128 token rows in 2 boxes instead of 8)
constexpr int kPairBoxB = 64;
// mid is stored as FP16 times 2^-6: finite up to 65504 * 64 ~ 4.2e6, full
// 11-bit precision from 2^-8 up; smaller values keep an absolute error
// below 2^-19
constexpr int kMidF16Shift = 6;
// Expert outputs of an all-GEMM forward are stored as FP16 times 2^-4:
// finite up to 65504 * 16 ~ 1.05e6 (beyond: HF_ERR_RANGE), full 11-bit
// precision from 2^-10 up; smaller values keep an absolute error below 2^-21
constexpr int kYF16Shift = 4;
struct GemmMaps {
    CUtensorMap A, A_sh;       // weights: routed view; shared expert gate (GEMM1) or down rows
    CUtensorMap A_sh2;         // shared expert up rows (GEMM1)
    CUtensorMap B0, B1;        // activations (hi, lo planes), routed K extent
    CUtensorMap B0_sh, B1_sh;  // the same with the shared expert's K extent
};
struct GatherArgs {
    const int32_t* plan;
    PlanLayout pl;
    const int32_t* perm;
    const void* x;
    int T, k, H, device;
    uint16_t* xp_hi;
    uint16_t* xp_lo;
    // optional (bf16 x, k > 1): slot -> position, so each token's row is read
    // once and written to all of its positions (token-major gather)
    const int32_t* slot_pos;
    int has_shared;
};
hf_status launch_gemm(const GemmMaps& m, const GemmArgs& a, int num_b, int grid, cudaStream_t st);
hf_status launch_gather(const GatherArgs& a, int x_f32, cudaStream_t st);
hf_status make_map_bf16(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                        uint64_t pitch, uint32_t box_rows);

// Device generator (hf_synth.cu).
hf_status synth_bf16(uint16_t* dst, uint64_t n, uint64_t key, float scale, cudaStream_t st);
hf_status synth_f32u(float* dst, uint64_t n, uint64_t key, float lo, float hi, cudaStream_t st);
uint64_t synth_key(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert);
float synth_normal_scale(double sigma);

struct CombineArgs {
    const float* y;        // [(T*k+T) x H]; FP16 elements (y * 2^-kYF16Shift) when y16
    int y16;
    const int32_t* slot_pos;
    const float* w;        // [T x k]
    int T, H, k, has_shared;
    float* out;            // [T x H]
    const float* resid;    // optional [T x H]: out = resid + (routed + shared); may alias out
    float* slot_out;       // optional [(T*k+T) x H] by slot id
};
hf_status launch_combine(const CombineArgs& a, cudaStream_t st);

// RMSNorm of fp32 rows with its output form (hf_norm.cu).
enum NormOut { kNormF32 = 0, kNormBf16 = 1, kNormHiLo = 2 };
hf_status launch_rmsnorm(const float* x, const uint16_t* w, float eps, int T, int H, int mode,
                         void* out, uint16_t* out_lo, cudaStream_t st);

hf_status launch_gemv_plain(const uint16_t* A, const float* x, float* y, int M, int K,
                            float alpha, float beta, cudaStream_t st);

}  // namespace hf
