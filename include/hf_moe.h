/*
 * hf_moe.h -- C ABI of the B200 (sm_100a) MoE layer for HummingFlight.
 *
 * One shared library (hummingflight_b200/libhf_moe.so) replaces the engine's
 * CPU MoE path and its sm_86 expert offload. Plain C types only: pointers,
 * sizes, an opaque context; CUDA streams are passed as hf_stream (the same
 * object as cudaStream_t, declared opaquely so callers need no CUDA headers).
 *
 * Every call returns an hf_status; nothing falls back to the CPU. A failed
 * call leaves a message for hf_last_error() (per thread). One context per
 * device; a context is used by one host thread at a time, as the reference's
 * single generation thread does (engine/scheduler.h:162-166).
 *
 * Reference interfaces replaced (paths in the HummingFlight source tree):
 *   GLMForward::moeLayer          model/glm_forward.h:93, glm_forward.cpp:509-661
 *   gemv_bf16_f32                 compute/cpu_kernels.h:16-17
 *   topKScores / TopKResult       compute/moe_router.h:12-16, :29-57
 *   gpuExpertCacheConfig / gpuExpertStage / gpuExpertFFN
 *                                 compute/cuda_backend.h:64-85
 *   Scheduler::getExpertPtr       engine/scheduler.h:80-84 ([gate|up|down] layout)
 *   Scheduler::getSharedProjectionPtr  engine/scheduler.h:93-96 (3 pointers)
 */
#ifndef HF_MOE_H
#define HF_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HF_MOE_ABI_VERSION 1

#if defined(__GNUC__)
#define HF_API __attribute__((visibility("default")))
#else
#define HF_API
#endif

typedef struct CUstream_st* hf_stream; /* == cudaStream_t; NULL = legacy default stream */

typedef enum hf_status {
    HF_OK = 0,
    HF_ERR_ARG = 1,         /* bad argument, shape or unsupported size          */
    HF_ERR_CUDA = 2,        /* a CUDA runtime/driver call or kernel failed      */
    HF_ERR_NCCL = 3,        /* expert-parallel exchange failed                  */
    HF_ERR_TIMEOUT = 4,     /* a bounded device wait gave up (error word set)   */
    HF_ERR_OOM = 5,         /* device allocation failed                         */
    HF_ERR_STATE = 6,       /* call out of order (e.g. weights not set)         */
    HF_ERR_UNSUPPORTED = 7, /* no device / wrong architecture                   */
    HF_ERR_RANGE = 8        /* a value beyond an FP16 plane of the tensor-core
                               path: a SwiGLU intermediate |silu(g) * u| > 4.2e6
                               or an expert output |y| > 1.05e6 (Inf included;
                               NaN propagates as in fp32): outputs invalid      */
} hf_status;

typedef enum hf_mem_kind { HF_MEM_HOST = 0, HF_MEM_DEVICE = 1 } hf_mem_kind;
typedef enum hf_dtype { HF_BF16 = 0, HF_F32 = 1 } hf_dtype;

/* Expert-path selection per expert segment (by its token count). */
typedef enum hf_path {
    HF_PATH_AUTO = 0,       /* grouped GEMV for short segments, tcgen05 GEMM else */
    HF_PATH_GEMV = 1,       /* always the CUDA-core grouped GEMV                   */
    HF_PATH_GEMM = 2        /* always the tcgen05 grouped GEMM                     */
} hf_path;

/* Layer shape and placement. Field names follow ModelConfig's MoE keys
 * (model/config.h; parsed at model/config.cpp:108-117). */
typedef struct hf_moe_config {
    int hidden_size;               /* hiddenSize (multiple of 8)                   */
    int num_experts;               /* numLocalExperts = n_routed_experts           */
    int num_experts_per_tok;       /* top-k, 1..8 (TopKResult holds 8)             */
    int moe_intermediate_size;     /* moeIntermediateSize (multiple of 8)          */
    int shared_intermediate_size;  /* nSharedExperts * moeIntermediateSize; 0=none */
    float routed_scaling_factor;   /* routedScalingFactor                          */
    int norm_topk_prob;            /* normTopkProb                                 */
    int num_layers;                /* layers this context holds weights for        */
    int max_tokens;                /* largest T of any forward (scratch sizing)    */
    int device;                    /* CUDA device ordinal                          */
    int path;                      /* hf_path                                      */
    int gemv_max_tokens;           /* AUTO: segments up to this use the GEMV; 0 = by pass
                                      size (the GEMV for single-token passes only) */
    /* expert parallelism (experts [r*E/W, (r+1)*E/W) on rank r); W=1: none */
    int ep_rank;
    int ep_world;
    const unsigned char* ep_unique_id; /* 128-byte NCCL unique id when ep_world > 1 */
} hf_moe_config;

/* Optional device outputs of a forward (any field may be NULL).
 * Routed slot (t, i) has slot id t*k + i; the shared expert's slot of token t
 * is T*k + t. Groups are the routed experts 0..E-1 then the shared expert E.
 * Positions order every slot by (group asc, token asc): the canonical
 * permutation into per-expert contiguous segments. */
typedef struct hf_moe_routing {
    int32_t* topk_ids;      /* [T*k]  TopKResult::indices per token, rank order */
    float* topk_weights;    /* [T*k]  TopKResult::weights                       */
    float* margins;         /* [T]    biased score of rank k-1 minus rank k     */
    int32_t* counts;        /* [E+1]  tokens per group (shared = T or 0)        */
    int32_t* offsets;       /* [E+2]  exclusive scan of counts                  */
    int32_t* perm;          /* [T*k+T] slot id at each position                 */
    float* slot_out;        /* [(T*k+T) x H] expert output of each slot, by slot id */
} hf_moe_routing;

typedef struct hf_moe_ctx hf_moe_ctx;

HF_API int hf_abi_version(void);
HF_API const char* hf_status_string(hf_status s);
/* Message of the last failed call on this thread ("" if none). */
HF_API const char* hf_last_error(void);

/* Replaces gpuExpertCacheConfig (compute/cuda_backend.h:64): allocates the
 * layer weights and the scratch for max_tokens on cfg->device. */
HF_API hf_status hf_moe_create(hf_moe_ctx** out, const hf_moe_config* cfg);
HF_API hf_status hf_moe_destroy(hf_moe_ctx* ctx);

/* Router weight mlp.gate.weight [E x H] BF16 and e_score_correction_bias [E]
 * fp32 (bias may be NULL: no correction), model/weight_index.cpp:20-27,222-236. */
HF_API hf_status hf_moe_set_router(hf_moe_ctx* ctx, int layer, const uint16_t* router_bf16,
                            const float* bias, hf_mem_kind kind);
/* One routed expert in Scheduler::getExpertPtr's layout [gate I*H | up I*H |
 * down H*I] BF16 (engine/scheduler.h:80-84); copied, so the caller may reuse
 * the buffer on return, as gpuExpertStage allows (cuda_backend.h:72-78).
 * Under expert parallelism only the owning rank accepts an eid. */
HF_API hf_status hf_moe_set_expert(hf_moe_ctx* ctx, int layer, int eid, const uint16_t* gate_up_down,
                            hf_mem_kind kind);
/* Shared expert from the three pointers of getSharedProjectionPtr
 * (engine/scheduler.h:93-96): gate [Is x H], up [Is x H], down [H x Is]. */
HF_API hf_status hf_moe_set_shared(hf_moe_ctx* ctx, int layer, const uint16_t* gate,
                            const uint16_t* up, const uint16_t* down, hf_mem_kind kind);
/* Device address of the resident [gate|up|down] block of expert eid
 * (eid == E: the shared expert), for loaders that write in place. */
HF_API hf_status hf_moe_expert_device_ptr(hf_moe_ctx* ctx, int layer, int eid, uint16_t** dev_ptr);
/* Device addresses of the router weight and bias. */
HF_API hf_status hf_moe_router_device_ptr(hf_moe_ctx* ctx, int layer, uint16_t** router, float** bias);
/* Marks a layer's weights complete (after in-place writes). set_* mark it too. */
HF_API hf_status hf_moe_mark_loaded(hf_moe_ctx* ctx, int layer);

/* The MoE layer over T tokens, asynchronous on `stream`: router GEMV ->
 * sigmoid -> + bias -> top-k -> permutation -> routed + shared SwiGLU experts
 * -> weighted combine (glm_forward.cpp:509-661). x: device [T x H], BF16 or
 * fp32 (x_dtype); out: device fp32 [T x H]. 0 <= T <= max_tokens. */
HF_API hf_status hf_moe_forward(hf_moe_ctx* ctx, int layer, const void* x, hf_dtype x_dtype, int T,
                         float* out, const hf_moe_routing* routing, hf_stream stream);
/* The same with HOST buffers: copies x in, runs the layer, copies out back and
 * waits. Pinned host memory makes the copies asynchronous DMA. */
HF_API hf_status hf_moe_forward_host(hf_moe_ctx* ctx, int layer, const void* x_host, hf_dtype x_dtype,
                              int T, float* out_host, hf_stream stream);
/* Drop-in for GLMForward::moeLayer(layer, input, output): one token, fp32 host
 * vectors of hidden_size, synchronous (model/glm_forward.h:93). */
HF_API hf_status hf_moe_layer(hf_moe_ctx* ctx, int layer, const float* input, float* output);

/* The MLP residual block of an MoE layer (glm_forward.cpp:785-796):
 * hidden_out = hidden_in + moeLayer(rmsNorm(post_attention_layernorm, hidden_in)),
 * asynchronous on `stream`. hidden_in / hidden_out: device fp32 [T x H], 16-byte
 * aligned, and may be the same buffer (the reference updates hiddenStates in
 * place). norm_weight: device BF16 [H] (postAttentionLayernorm), or NULL for
 * x * rms (rmsNorm without a weight pointer, :194-195); eps: config
 * rms_norm_eps. act_dtype: the form the normalised rows are handed to the
 * layer in -- HF_F32 (the reference's fp32 hand-off; the expert GEMMs read it
 * as a bf16 hi + lo pair) or HF_BF16 (rounded once, RNE: half the bytes and the
 * tensor-core router). The residual add is fused into the combine; the
 * normalised rows live in the context's input staging buffer. Expert
 * parallelism as for hf_moe_forward (every rank calls it, T may be 0). */
HF_API hf_status hf_moe_block_forward(hf_moe_ctx* ctx, int layer, const float* hidden_in,
                                      float* hidden_out, const uint16_t* norm_weight, float eps,
                                      hf_dtype act_dtype, int T, const hf_moe_routing* routing,
                                      hf_stream stream);

/* Routing only (router GEMV, sigmoid, bias, top-k, permutation) into `routing`. */
HF_API hf_status hf_moe_route(hf_moe_ctx* ctx, int layer, const void* x, hf_dtype x_dtype, int T,
                       const hf_moe_routing* routing, hf_stream stream);

/* Waits for the context's last stream and reports device-side failures of
 * the forwards since the previous check: HF_ERR_TIMEOUT when a bounded wait
 * inside a kernel gave up (the kernel drained, freed its tensor memory and
 * returned; the outputs of that forward are invalid, the context stays
 * usable). hf_moe_forward_host and hf_moe_layer check this themselves. */
HF_API hf_status hf_moe_synchronize(hf_moe_ctx* ctx);
/* Limit of every bounded device wait, in nanoseconds (default 2 s, 0 restores
 * it). Tests shorten it to make a wait run out on purpose. */
HF_API hf_status hf_moe_set_wait_timeout(hf_moe_ctx* ctx, uint64_t ns);
/* Test hook (failure detection without a GPU fault): while enabled, the
 * tensor-core kernels first wait on a barrier that nothing signals, so their
 * bounded wait runs out after the wait timeout and hf_moe_synchronize reports
 * HF_ERR_TIMEOUT. No counterpart in the reference, which has no device waits. */
HF_API hf_status hf_moe_debug_stall(hf_moe_ctx* ctx, int enable);

/* Expert parallelism (no reference counterpart: the reference is a single
 * process on one host). With ep_world = W > 1 each rank's context holds E/W
 * experts (by default [rank*E/W, (rank+1)*E/W); see hf_moe_set_placement)
 * plus the shared expert, and hf_moe_forward routes the rank's own T tokens,
 * exchanges token rows and expert outputs with the other ranks and combines
 * at the source in the reference's rank order, so outputs equal the
 * single-GPU outputs. The exchange is peer memory over NVLink when every rank
 * can map every other (stores into the other ranks' buffers, arrival flags
 * with bounded waits, no host synchronization; the down GEMM returns its
 * outputs from its epilogue), else NCCL (hf_moe_ep_transport). Every rank
 * must call the same forwards in the same order (T may differ, even 0).
 * NCCL is loaded at run time (libnccl.so.2). */
/* A fresh NCCL unique id (128 bytes) for hf_moe_config.ep_unique_id; rank 0
 * makes it and the caller broadcasts it to the other ranks. An id serves one
 * set of contexts (one communicator): make a new one for every hf_moe_create
 * round. */
HF_API hf_status hf_ep_unique_id(unsigned char* out128);

/* Expert placement of one layer (expert parallelism). order [E] lists global
 * expert ids; rank r owns the experts order[r*E/W .. (r+1)*E/W - 1] (the
 * default is order[j] = j, contiguous ranges). All ranks pass the same order.
 * Call before the layer's weights: the rank keeps only its own experts, so a
 * new placement marks the layer unloaded until its router (hf_moe_set_router,
 * hf_moe_synth_layer or hf_moe_load_safetensors) and experts are set again.
 * Ids everywhere in the API stay global (set_expert, routing outputs); with
 * a placement, write the router through hf_moe_set_router, not through the
 * pointer of hf_moe_router_device_ptr. No reference counterpart: the
 * reference keeps every expert on one host (its LRU/placement tiers decide
 * only which tier holds a weight, engine/scheduler.cpp). */
HF_API hf_status hf_moe_set_placement(hf_moe_ctx* ctx, int layer, const int32_t* order);

/* A placement that balances expected work: experts sorted by load (e.g.
 * routed token counts from a calibration batch, plus a constant for the
 * weight stream of an active expert), heaviest first, each to the least
 * loaded rank that still has room for E/world experts; each rank's experts
 * in ascending id. Writes order [E] for hf_moe_set_placement. */
HF_API hf_status hf_ep_balanced_placement(int E, int world, const long long* load, int32_t* order);

/* The exchange an expert-parallel context uses, agreed by all its ranks at
 * hf_moe_create: 0 none (one GPU), 1 peer memory over NVLink (CUDA IPC
 * mappings of the other ranks' slabs), 2 fixed slabs over NCCL, 3 NCCL with
 * counts read on the host. No reference counterpart (the reference runs on
 * one host process with no collective backend). */
HF_API hf_status hf_moe_ep_transport(hf_moe_ctx* ctx, int* transport);

/* Recovery after a forward that did not run on every rank (a rank skipped it,
 * so the others' bounded waits ran out and reported HF_ERR_TIMEOUT). Every
 * rank calls it, between forwards: it waits for the rank's own work, clears
 * the error, and agrees on the forward sequence numbers (one all-reduce), so
 * the next forward on all ranks is valid again. The counterpart of the
 * reference's bounded waits that give up and continue
 * (engine/scheduler.cpp:696-722). */
HF_API hf_status hf_moe_ep_resync(hf_moe_ctx* ctx);
/* The host-side order of one exchange, as the forward builds it (for tests
 * and external transports): send_counts / recv_counts [W x E_local] are the
 * rows this rank sends to / receives from each rank per local expert;
 * writes send_off, recv_off [W+1] (rows, source-major), local_counts
 * [E_local+1] (last: T_local when has_shared), local_rows [R + T_local] (for
 * each local position, expert-major then source rank, the row in [received
 * rows | local tokens]) and row_pos [R] (received row -> local position). */
HF_API hf_status hf_ep_plan(int world, int E_local, int T_local, int has_shared,
                            const int32_t* send_counts, const int32_t* recv_counts,
                            int32_t* send_off, int32_t* recv_off, int32_t* local_counts,
                            int32_t* local_rows, int32_t* row_pos);

/* Routing (router GEMV, sigmoid, bias, top-k, permutation) that allocates no
 * device memory, for callers that cannot call cudaMalloc: an engine whose
 * resident expert weights already hold the whole device, or a decode loop
 * that must not take the device-wide synchronization an allocation can
 * imply. No counterpart in the reference. Same kernels and outputs as
 * hf_moe_route, with no context: router [E x H] BF16, bias [E] or NULL, x
 * [T x H]; writes topk_ids/topk_weights [T*min(k,E)], counts [E+1], offsets
 * [E+2], perm [T*min(k,E) + T] (shared slots included when has_shared).
 * Scratch is a fixed array inside the library, one per device, kept until
 * the process exits: T <= 128, E <= 256, k <= 8, else HF_ERR_ARG. The first
 * call on a device looks the array up, so make it before any stream capture.
 * Calls that can overlap on the GPU share the array and race; calls ordered
 * on one stream do not. */
HF_API hf_status hf_moe_route_noalloc(const uint16_t* router_bf16, const float* bias,
                                      const void* x, hf_dtype x_dtype, int T, int H, int E,
                                      int top_k, float routed_scaling_factor, int norm_topk_prob,
                                      int has_shared, int32_t* topk_ids, float* topk_weights,
                                      int32_t* counts, int32_t* offsets, int32_t* perm,
                                      hf_stream stream);

/* Statistics of the most recent forward/route on this context (waits for it):
 * experts with at least one token, and segments on each expert path. */
HF_API hf_status hf_moe_last_stats(hf_moe_ctx* ctx, int* active_experts, int* gemv_segments,
                            int* gemm_segments);

/* Per-phase device time of forwards, from CUDA events recorded on the
 * forward's stream between its kernels (off by default; no counterpart in the
 * reference, whose GPU timing is one event pair per expert,
 * cuda_backend.cpp:464-477). Phases: 0 router logits, 1 top-k + permutation
 * + plan, 2 GEMV gate/up, 3 GEMV down, 4 GEMM gate/up, 5 GEMM down,
 * 6 combine, 7 expert-parallel dispatch (counts + rows to their ranks), 8
 * expert-parallel return (outputs back to their sources), 9 RMSNorm of the
 * residual block (hf_moe_block_forward). Kernel launches
 * (of this library) are counted whether or not timing is on. */
#define HF_MOE_PHASES 10
HF_API hf_status hf_moe_profile(hf_moe_ctx* ctx, int enable);
/* Waits for the recorded work, writes each phase's milliseconds and kernel
 * launches since the previous read (either pointer may be NULL), then resets. */
HF_API hf_status hf_moe_profile_read(hf_moe_ctx* ctx, double* phase_ms, long long* launches);

/* Device twin of gemv_bf16_f32 (compute/cpu_kernels.h:16-17):
 * y = alpha * A x + beta * y, A BF16 [M x K] row-major, x/y fp32, all device
 * pointers. Like the reference, y is read even when beta == 0. Any M, K >= 0. */
HF_API hf_status hf_gemv_bf16_f32(const uint16_t* A, const float* x, float* y, int M, int K, float alpha,
                           float beta, hf_stream stream);

/* Device twin of topKScores over T score rows (compute/moe_router.h:29-57):
 * scores [T x E] fp32 (post-sigmoid), bias [E] or NULL, writes idx/weights
 * [T x min(k,E)]. Ties go to the lower expert id. */
HF_API hf_status hf_topk_scores(const float* scores, int T, int E, const float* bias, int k, float scale,
                         int norm, int32_t* idx, float* weights, hf_stream stream);

/* Dense SwiGLU MLP (GLMForward::denseMlp, glm_forward.cpp:411-432; the
 * reference's per-token gemv_bf16_f32 x3 + fp32 SwiGLU) over T tokens.
 * gate, up: device BF16 [I x H]; down: device BF16 [H x I], three separate
 * pointers (16-byte aligned); x: device [T x H] bf16 or f32; out: device fp32
 * [T x H]. H and I multiples of 8 (of 64 for the tensor-core path, taken
 * from T = 2 tokens). workspace: device scratch, 256-byte aligned, of at least
 * hf_dense_mlp_workspace_size(T, H, I) bytes; not touched by the host, so one
 * workspace serves any number of layers called in stream order. Asynchronous
 * on `stream`; the reference's denseMlp is void, here argument errors return
 * HF_ERR_ARG before anything is enqueued. */
HF_API size_t hf_dense_mlp_workspace_size(int T, int H, int I);
HF_API hf_status hf_dense_mlp_forward(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                               const void* x, hf_dtype x_dtype, int T, int H, int I, float* out,
                               void* workspace, size_t workspace_bytes, hf_stream stream);
/* Waits for `stream` and reports whether the last hf_dense_mlp_forward on this
 * workspace hit a bounded-wait timeout (HF_ERR_TIMEOUT) -- no counterpart in
 * the reference, whose CPU GEMVs cannot time out. */
HF_API hf_status hf_dense_mlp_status(const void* workspace, hf_stream stream);

/* The MLP residual block of a dense layer (glm_forward.cpp:785-796 with
 * denseMlp): hidden_out = hidden_in + denseMlp(rmsNorm(norm_weight, hidden_in)).
 * Arguments as hf_dense_mlp_forward and hf_moe_block_forward (hidden_in and
 * hidden_out may alias; norm_weight NULL = no weight; act_dtype HF_F32 or
 * HF_BF16); the same workspace size. The RMSNorm writes the GEMM's operand
 * planes directly and the down projection's epilogue adds the residual. */
HF_API hf_status hf_dense_block_forward(const uint16_t* gate, const uint16_t* up,
                                        const uint16_t* down, const uint16_t* norm_weight,
                                        float eps, hf_dtype act_dtype, const float* hidden_in,
                                        float* hidden_out, int T, int H, int I, void* workspace,
                                        size_t workspace_bytes, hf_stream stream);

/* Device twin of GLMForward::rmsNorm (glm_forward.cpp:185-197) over T rows:
 * out = x * (1 / sqrt(mean(x^2) + eps)) * weight. x: device fp32 [T x H];
 * weight: device BF16 [H] or NULL (no weight); out: device [T x H] of
 * out_dtype (HF_F32, or HF_BF16 rounded to nearest even). H a multiple of 4,
 * pointers 16-byte aligned; out must not overlap x. */
HF_API hf_status hf_rmsnorm(const float* x, const uint16_t* weight, float eps, int T, int H,
                            void* out, hf_dtype out_dtype, hf_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* HF_MOE_H */
