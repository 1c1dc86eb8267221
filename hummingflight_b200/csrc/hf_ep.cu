// hf_ep.cu -- expert parallelism: experts sharded across the GPUs of one node,
// token rows exchanged over NVLink.
//
// The reference runs on one host with no collective backend (single-process
// CPU engine); this exchange is new. Rank r owns E/W experts -- by default
// [r*E/W, (r+1)*E/W), or those a placement gives it (hf_moe_set_placement;
// the router rows are stored in placed order, so the experts of one rank are
// one contiguous range of placed ids) -- plus a replica of the shared expert.
// One forward on the default transport, peer memory (CUDA IPC mappings of
// every rank's slabs, NVLink stores, no host round trip):
//
//  1. route the rank's own tokens over ALL experts; the canonical
//     permutation orders slots by expert, so the slots bound for rank d are
//     one contiguous range;
//  2. the pack kernel stores each token's activation row straight into its
//     destination's receive slab, once per destination rank however many of
//     its experts live there (with a slot -> row map beside the counts),
//     walking the destinations interleaved; then the per-expert counts, then
//     this forward's sequence number into every rank's arrival flag
//     (fence.sc.sys + st.release.sys);
//  3. the receiver's plan kernel waits (bounded) for every source's flag and
//     builds the plan from the counts and row maps on the device;
//  4. the same GEMV / tcgen05 GEMM kernels run on the local experts (received
//     rows, expert-major then source) and on the shared expert (local
//     tokens). On the GEMM path the down GEMM's epilogue stores every output
//     row (the FP16 plane, half the bytes of fp32) straight into its source's
//     output slab, and its last CTA raises the return flags, so the return
//     overlaps the GEMM tile by tile;
//  5. the source waits (bounded) for every rank's return flag and combines in
//     the reference's top-k rank order, reading the rows from its slab.
// Each slot's expert product and the combine order do not depend on W, so
// the output equals the single-GPU output bit for bit (given the same router
// logits). Without peer mappings (all ranks agree on the transport at
// create) the same slabs travel through NCCL for small batches, and large
// batches use an exchange sized on the host (counts read back, grouped
// ncclSend/ncclRecv).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, which returns the copy
// the process already uses, e.g. PyTorch's), so the library does not pin an
// NCCL build at link time.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <numeric>

#include "hf_ctx.cuh"
#include "hf_sm100.cuh"

namespace hf {

// ------------------------------------------------------------------ NCCL loader
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    std::string error;
    bool ok = false;
};

static NcclApi load_nccl() {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        a.error = std::string("cannot load libnccl.so.2: ") + dlerror();
        return a;
    }
    auto sym = [&](const char* n) { return dlsym(h, n); };
    a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(sym("ncclGetUniqueId"));
    a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(sym("ncclCommInitRank"));
    a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
    a.GroupStart = reinterpret_cast<decltype(a.GroupStart)>(sym("ncclGroupStart"));
    a.GroupEnd = reinterpret_cast<decltype(a.GroupEnd)>(sym("ncclGroupEnd"));
    a.Send = reinterpret_cast<decltype(a.Send)>(sym("ncclSend"));
    a.Recv = reinterpret_cast<decltype(a.Recv)>(sym("ncclRecv"));
    a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(sym("ncclAllReduce"));
    a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(sym("ncclGetErrorString"));
    a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.GroupStart && a.GroupEnd &&
           a.Send && a.Recv && a.AllReduce && a.GetErrorString;
    if (!a.ok) a.error = "libnccl.so.2 lacks a required symbol";
    return a;
}

static NcclApi& nccl() {
    static std::once_flag once;
    static NcclApi api;
    std::call_once(once, [] { api = load_nccl(); });
    return api;
}

static hf_status nccl_fail(ncclResult_t r, const char* what) {
    const char* s = nccl().GetErrorString ? nccl().GetErrorString(r) : "unknown";
    return fail(HF_ERR_NCCL, std::string(what) + ": " + s);
}

#define HF_NCCL(call)                                                  \
    do {                                                               \
        ncclResult_t _r = (call);                                      \
        if (_r != ncclSuccess) return ::hf::nccl_fail(_r, #call);      \
    } while (0)

// ------------------------------------------------------------------ exchange plan (host)
// Orders the received rows of one forward (see hf_ep_plan in include/hf_moe.h).
struct ExchangePlan {
    std::vector<int32_t> send_off, recv_off;  // [W+1] rows
    std::vector<int32_t> local_counts;        // [El + 1]
    int R = 0;
};

static void build_plan(int W, int El, int T, bool has_shared, const int32_t* send_counts,
                       const int32_t* recv_counts, ExchangePlan& p, int32_t* local_rows,
                       int32_t* row_pos) {
    p.send_off.assign(W + 1, 0);
    p.recv_off.assign(W + 1, 0);
    p.local_counts.assign(El + 1, 0);
    for (int d = 0; d < W; ++d) {
        int s = 0, r = 0;
        for (int j = 0; j < El; ++j) {
            s += send_counts[d * El + j];
            r += recv_counts[d * El + j];
            p.local_counts[j] += recv_counts[d * El + j];
        }
        p.send_off[d + 1] = p.send_off[d] + s;
        p.recv_off[d + 1] = p.recv_off[d] + r;
    }
    p.R = p.recv_off[W];
    p.local_counts[El] = has_shared ? T : 0;
    // local positions: expert-major, then source rank, then arrival order
    std::vector<int32_t> base(El + 1, 0);
    for (int j = 1; j <= El; ++j) base[j] = base[j - 1] + p.local_counts[j - 1];
    std::vector<int32_t> cursor(base.begin(), base.begin() + El);
    for (int s = 0; s < W; ++s) {
        int row = p.recv_off[s];
        for (int j = 0; j < El; ++j)
            for (int i = 0; i < recv_counts[s * El + j]; ++i, ++row) {
                const int pos = cursor[j]++;
                if (local_rows) local_rows[pos] = row;
                if (row_pos) row_pos[row] = pos;
            }
    }
    if (local_rows && has_shared)
        for (int t = 0; t < T; ++t) local_rows[base[El] + t] = p.R + t;
}

// ------------------------------------------------------------------ decode exchange kernels
// Small batches (decode) exchange fixed-capacity slabs so that no size has to
// reach the host: source s sends every destination `cap` rows (its rows for
// that rank's experts first, the rest unused) plus the per-expert counts, in
// one NCCL group; the receiver builds its plan from the counts on the device.

// This rank's routed rows into per-destination slabs: the slot at canonical
// position p (expert-major) goes to rank d = expert / El, slab row
// p - offsets[d * El].
__global__ void __launch_bounds__(256) k_ep_pack(const int32_t* perm, const int32_t* ids,
                                                 const int32_t* offsets, const uint4* x,
                                                 int row_vec, int n, int k, int El, int cap,
                                                 uint4* slab) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int p = warp; p < n; p += nw) {
        const int slot = perm[p];
        const int d = ids[slot] / El;
        const int r = p - offsets[d * El];
        const uint4* src = x + size_t(slot / k) * row_vec;
        uint4* dst = slab + (size_t(d) * cap + r) * row_vec;
        for (int c = lane; c < row_vec; c += 32) dst[c] = ld_nc_u4(src + c);
    }
}

// Receiver: expert outputs (local positions) back into per-source slabs in
// the order the rows arrived.
__global__ void __launch_bounds__(256) k_ep_unpack(const float4* y, const int32_t* row_pos,
                                                   const int32_t* recv_tot, int W, int cap,
                                                   int row_vec, float4* slab) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int idx = warp; idx < W * cap; idx += nw) {
        const int s = idx / cap;
        if (idx - s * cap >= recv_tot[s]) continue;
        const float4* src = y + size_t(row_pos[idx]) * row_vec;
        float4* dst = slab + size_t(idx) * row_vec;
        for (int c = lane; c < row_vec; c += 32) dst[c] = src[c];
    }
}

// Source: returned outputs to canonical positions; then the shared expert's
// outputs from the last group of the local plan.
__global__ void __launch_bounds__(256) k_ep_return(const int32_t* perm, const int32_t* ids,
                                                   const int32_t* offsets, int n, int k, int El,
                                                   int cap, const float4* slab, const float4* y_loc,
                                                   const int32_t* loc_shared_off, int n_shared,
                                                   int row_vec, float4* yrecv,
                                                   const unsigned long long* flags, int W,
                                                   unsigned long long seq,
                                                   unsigned long long timeout_ns, int* err) {
    if (flags) {  // peer-memory exchange: every rank's outputs are in the slabs
        if (threadIdx.x == 0) sm100::wait_flags_sys(flags, W, seq, timeout_ns, err);
        __syncthreads();
    }
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int p = warp; p < n + n_shared; p += nw) {
        const float4* src;
        if (p < n) {
            const int slot = perm[p];
            const int d = ids[slot] / El;
            src = slab + (size_t(d) * cap + (p - offsets[d * El])) * row_vec;
        } else {
            src = y_loc + size_t(*loc_shared_off + (p - n)) * row_vec;
        }
        float4* dst = yrecv + size_t(p) * row_vec;
        for (int c = lane; c < row_vec; c += 32) dst[c] = src[c];
    }
}

static int copy_grid(int nsm, int rows) { return std::max(1, std::min(nsm * 8, (rows + 7) / 8)); }

constexpr size_t kEpSlabBytes = size_t(64) << 20;     // largest slab set sent whole over NCCL
constexpr size_t kEpP2PSlabBytes = size_t(8) << 30;   // largest slab set reserved for peer stores

// ---- decode exchange over peer memory (NVLink): the same slabs, written by
// the producing kernels straight into the other GPUs' buffers (CUDA IPC
// mappings), with a per-forward sequence number as the arrival flag.
constexpr int kEpMaxRanks = 16;
struct PeerPtrs {                              // rank d's buffers, as mapped here
    char* x[kEpMaxRanks];                      // xslab_recv
    float* y[kEpMaxRanks];                     // yslab_recv
    int32_t* cnt[kEpMaxRanks];                 // cnt_recv (counts, then the slot -> row maps)
    unsigned long long* flags[kEpMaxRanks];    // [2W]: rows from s arrived / outputs from s
};

// The block that finishes last (device counter, reset by it) runs `tail`;
// every block fences its stores system-wide before counting itself in.
template <typename F>
__device__ __forceinline__ void ep_last_block(int* done, F tail) {
    __shared__ int s_last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(done, 1) == int(gridDim.x) - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();
    tail();
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) *done = 0;
}

// Rows into the destinations' slabs (at this rank's slab) in peer memory;
// then counts, then flags[d][rank] = seq on every rank.
// A token routed to several experts of one destination rank crosses NVLink
// once: only its slot with the smallest expert id there stores the row (at
// that slot's arrival row); every slot writes the row it reads into the
// destination's slot -> row map (after the counts: cnt[d][W * El + rank *
// cap + r]). Top-8 over 32-expert ranks sends ~5.3 rows a token at W = 8.
// With rowmap set, also records where each slot's output will be read back:
// routed slot -> row d * cap + r of this rank's output slab, the shared slot
// of local token t (slot n + t) -> row W * cap + t.
// Task order of a peer-memory dispatch. Canonical positions are
// destination-major, so walking them in order makes every source store into
// rank 0's slab first, then rank 1's, ...: all sources on one destination's
// links at a time. Task i instead goes to rank (rank + 1 + i) % W, its
// (i / W)-th slot: every source spreads its stores over every destination.
struct DispatchOrder {
    const int32_t* offsets;
    int W, El, rank, rounds;
    __device__ DispatchOrder(const int32_t* off, int W_, int El_, int rank_)
        : offsets(off), W(W_), El(El_), rank(rank_), rounds(0) {
        for (int d = 0; d < W; ++d) rounds = max(rounds, off[(d + 1) * El] - off[d * El]);
    }
    __device__ int tasks() const { return W * rounds; }
    // canonical position of task i, or -1 (past that destination's slots)
    __device__ int position(int i) const {
        const int d = (rank + 1 + i % W) % W, j = i / W;
        const int o = offsets[d * El];
        return j < offsets[(d + 1) * El] - o ? o + j : -1;
    }
};

// The token's first slot on rank d: smallest expert id there (ids of one
// token are distinct); all lanes of the warp call it, lane = top-k rank.
__device__ __forceinline__ int first_slot_on(const int32_t* ids, int t, int k, int El, int d,
                                             int lane) {
    unsigned key = 0xffffffffu;
    if (lane < k) {
        const int e = ids[t * k + lane];
        if (e / El == d) key = (unsigned(e) << 5) | unsigned(lane);
    }
    key = __reduce_min_sync(0xffffffffu, key);
    return t * k + int(key & 31u);
}

__global__ void __launch_bounds__(256) k_ep_pack_p2p(const int32_t* perm, const int32_t* ids,
                                                     const int32_t* slot_pos,
                                                     const int32_t* offsets, const uint4* x,
                                                     int row_vec, int n, int k, int El, int cap,
                                                     int rank, int W, const int32_t* cnt_src,
                                                     PeerPtrs pp, int* done,
                                                     unsigned long long seq, int32_t* rowmap,
                                                     int n_shared) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const DispatchOrder order(offsets, W, El, rank);
    for (int i = warp; i < order.tasks(); i += nw) {
        const int p = order.position(i);  // the same for every lane
        if (p < 0) continue;
        const int slot = perm[p];
        const int d = ids[slot] / El;
        const int off = offsets[d * El];
        const int r = p - off;
        const int t = slot / k;
        const int first = first_slot_on(ids, t, k, El, d, lane);
        if (first == slot) {
            const uint4* src = x + size_t(t) * row_vec;
            uint4* dst = reinterpret_cast<uint4*>(pp.x[d]) + (size_t(rank) * cap + r) * row_vec;
            // eight 16-byte loads in flight per lane before their stores cross NVLink
            for (int c0 = lane; c0 < row_vec; c0 += 32 * 8) {
                uint4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (c0 + 32 * u < row_vec) v[u] = ld_nc_u4(src + c0 + 32 * u);
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (c0 + 32 * u < row_vec) dst[c0 + 32 * u] = v[u];
            }
        }
        if (lane == 0) {
            pp.cnt[d][W * El + rank * cap + r] = first == slot ? r : slot_pos[first] - off;
            if (rowmap) rowmap[slot] = d * cap + r;
        }
    }
    if (rowmap)
        for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n_shared; t += gridDim.x * blockDim.x)
            rowmap[n + t] = W * cap + t;
    ep_last_block(done, [&] {
        for (int i = threadIdx.x; i < W * El; i += blockDim.x)
            pp.cnt[i / El][rank * El + i % El] = cnt_src[i];
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x < W) sm100::st_release_sys(pp.flags[threadIdx.x] + rank, seq);
    });
}

// Receiver: outputs back into each source's slab (at this rank's slab) in
// peer memory; then flags[s][W + rank] = seq.
__global__ void __launch_bounds__(256) k_ep_unpack_p2p(const float4* y, const int32_t* row_pos,
                                                       const int32_t* recv_tot, int W, int cap,
                                                       int row_vec, int rank, PeerPtrs pp,
                                                       int* done, unsigned long long seq) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int idx = warp; idx < W * cap; idx += nw) {
        const int s = idx / cap, i = idx - s * cap;
        if (i >= recv_tot[s]) continue;
        const float4* src = y + size_t(row_pos[idx]) * row_vec;
        float4* dst = reinterpret_cast<float4*>(pp.y[s]) + (size_t(rank) * cap + i) * row_vec;
        for (int c = lane; c < row_vec; c += 32) dst[c] = src[c];
    }
    ep_last_block(done, [&] {
        if (threadIdx.x < W) sm100::st_release_sys(pp.flags[threadIdx.x] + W + rank, seq);
    });
}

__global__ void k_ep_wait(const unsigned long long* flags, int n, unsigned long long seq,
                          unsigned long long timeout_ns, int* err) {
    if (threadIdx.x == 0) sm100::wait_flags_sys(flags, n, seq, timeout_ns, err);
}

// ------------------------------------------------------------------ state
struct EpState {
    ncclComm_t comm = nullptr;
    size_t R_cap = 0;
    int cap = 0;               // decode exchange: rows per source slab (0: not used)
    char* xslab_send = nullptr;   // [W x cap] rows
    char* xslab_recv = nullptr;   // [W x cap] received rows, then T_max local tokens
    float* yslab_send = nullptr;  // [W x cap x H]
    float* yslab_recv = nullptr;  // [W x cap x H]
    int32_t* recv_tot = nullptr;  // [W]
    // peer-memory exchange (decode): this rank's flags and the peers' mappings
    bool p2p = false;
    unsigned long long* flags = nullptr;  // [2W], this rank's arrival flags
    unsigned long long seq = 0;           // forwards exchanged so far
    PeerPtrs peers{};
    std::vector<void*> opened;            // IPC mappings to close
    // outputs returned from the down GEMM's epilogue (peer memory, GEMM path):
    // per-position output rows, the ranks' output slabs and flag arrays as
    // device tables, and slot -> row of this rank's output slab
    float** yrow = nullptr;                       // [R_cap + T_max]
    float** d_peer_y = nullptr;                   // [W]
    unsigned long long** d_peer_flags = nullptr;  // [W]
    int32_t* rowmap = nullptr;                    // [T_max * k + T_max]
    // the shared expert on the local tokens while the dispatch is in flight:
    // the dispatch runs on `side`, ordered by the two events
    cudaStream_t side = nullptr;
    cudaEvent_t ev_routed = nullptr, ev_packed = nullptr;
    GroupW* shared_group = nullptr;               // [1] the plan kernel's group slot
    void* xsend = nullptr;     // [T_max*k x H] activation rows in canonical order
    void* xall = nullptr;      // [(R_cap + T_max) x H] received rows, then local tokens
    float* ysend = nullptr;    // [R_cap x H] expert outputs in arrival order
    float* yrecv = nullptr;    // [(T_max*k + T_max) x H] outputs at canonical positions
    int32_t* cnt_recv = nullptr;   // [W x El] counts, then [W x cap] slot -> row maps
    int32_t* loc_counts = nullptr; // [El + 1]
    int32_t* row_pos = nullptr;    // [R_cap]
    int32_t* h_src = nullptr;      // pinned [E + 1]
    int32_t* h_recv = nullptr;     // pinned [W x El]
    int32_t* h_perm = nullptr;     // pinned [R_cap + T_max]
    int32_t* h_rowpos = nullptr;   // pinned [R_cap]
    int32_t* h_loc = nullptr;      // pinned [El + 1]
};

size_t ep_recv_cap(const hf_moe_ctx* c) {
    const size_t T = size_t(std::max(1, c->cfg.max_tokens));
    return size_t(c->world) * T * size_t(std::min(c->k, c->E_local));
}

// One value agreed by every rank: the minimum (or maximum) over the ranks of
// `v`, through the communicator on a private stream.
static hf_status allreduce_u64(EpState& e, unsigned long long* v, bool take_max) {
    NcclApi& n = nccl();
    unsigned long long* dv = nullptr;
    HF_TRY(dalloc(&dv, 1));
    cudaStream_t st = nullptr;
    hf_status s = HF_OK;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMemcpy(dv, v, sizeof(*v), cudaMemcpyHostToDevice) != cudaSuccess) {
        s = fail(HF_ERR_CUDA, "expert-parallel agreement: staging failed");
    } else {
        const ncclResult_t r =
            n.AllReduce(dv, dv, 1, ncclUint64, take_max ? ncclMax : ncclMin, e.comm, st);
        if (r != ncclSuccess) s = nccl_fail(r, "ncclAllReduce");
        else if (cudaStreamSynchronize(st) != cudaSuccess ||
                 cudaMemcpy(v, dv, sizeof(*v), cudaMemcpyDeviceToHost) != cudaSuccess)
            s = fail(HF_ERR_CUDA, "expert-parallel agreement: read-back failed");
    }
    if (st) cudaStreamDestroy(st);
    cudaFree(dv);
    return s;
}

// Maps every rank's slab receive buffers, counts and flags into this process
// (CUDA IPC handles gathered over the communicator). The ranks agree on the
// outcome: peer memory is used only when every rank mapped every peer, else
// every rank closes its mappings and all fall back to the NCCL exchanges
// together (a rank alone on NCCL would wait forever for sends its peers never
// make). Every rank therefore takes part in both exchanges below whatever
// fails locally. Test hook: HF_EP_FAIL_P2P_ON_RANK=r makes rank r report a
// failed mapping after it has opened its peers' handles.
struct HandleBlob {
    cudaIpcMemHandle_t h[4];
    int ok;
    int pad[3];
};

static hf_status setup_p2p(hf_moe_ctx* c) {
    EpState& e = *c->ep;
    NcclApi& n = nccl();
    const int W = c->world, me = c->rank;
    if (W > kEpMaxRanks) return fail(HF_ERR_ARG, "peer-memory exchange: too many ranks");
    constexpr int kBufs = 4;
    HandleBlob mine{};
    mine.ok = 1;
    if (dalloc(&e.flags, size_t(2) * W) != HF_OK ||
        cudaMemset(e.flags, 0, sizeof(unsigned long long) * 2 * W) != cudaSuccess)
        mine.ok = 0;
    void* mine_ptr[kBufs] = {e.xslab_recv, e.yslab_recv, e.cnt_recv, e.flags};
    for (int i = 0; i < kBufs && mine.ok; ++i)
        if (cudaIpcGetMemHandle(&mine.h[i], mine_ptr[i]) != cudaSuccess) mine.ok = 0;
    if (!mine.ok) {
        cudaGetLastError();
        std::memset(mine.h, 0, sizeof(mine.h));
    }
    const size_t hb = sizeof(HandleBlob);
    char* dev = nullptr;
    HF_TRY(dalloc(&dev, size_t(W) * hb));
    cudaStream_t st = nullptr;
    hf_status s = HF_OK;
    std::vector<HandleBlob> all(static_cast<size_t>(W));
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMemcpy(dev + size_t(me) * hb, &mine, hb, cudaMemcpyHostToDevice) != cudaSuccess) {
        s = fail(HF_ERR_CUDA, "peer-memory exchange: handle staging failed");
    } else {
        n.GroupStart();
        for (int d = 0; d < W; ++d) {
            if (d == me) continue;
            n.Send(dev + size_t(me) * hb, hb, ncclChar, d, e.comm, st);
            n.Recv(dev + size_t(d) * hb, hb, ncclChar, d, e.comm, st);
        }
        if (n.GroupEnd() != ncclSuccess || cudaStreamSynchronize(st) != cudaSuccess ||
            cudaMemcpy(all.data(), dev, size_t(W) * hb, cudaMemcpyDeviceToHost) != cudaSuccess)
            s = fail(HF_ERR_NCCL, "peer-memory exchange: handle exchange failed");
    }
    if (st) cudaStreamDestroy(st);
    cudaFree(dev);
    HF_TRY(s);
    bool every_handle = true;
    for (int d = 0; d < W; ++d) every_handle = every_handle && all[size_t(d)].ok;
    unsigned long long mapped = every_handle ? 1 : 0;
    if (every_handle) {
        for (int d = 0; d < W && mapped; ++d) {
            void* p[kBufs] = {mine_ptr[0], mine_ptr[1], mine_ptr[2], mine_ptr[3]};
            if (d != me)
                for (int i = 0; i < kBufs; ++i) {
                    if (cudaIpcOpenMemHandle(&p[i], all[size_t(d)].h[i],
                                             cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                        cudaGetLastError();
                        mapped = 0;
                        break;
                    }
                    e.opened.push_back(p[i]);
                }
            e.peers.x[d] = static_cast<char*>(p[0]);
            e.peers.y[d] = static_cast<float*>(p[1]);
            e.peers.cnt[d] = static_cast<int32_t*>(p[2]);
            e.peers.flags[d] = static_cast<unsigned long long*>(p[3]);
        }
        const char* hook = std::getenv("HF_EP_FAIL_P2P_ON_RANK");
        if (hook && std::atoi(hook) == me) mapped = 0;
    }
    HF_TRY(allreduce_u64(e, &mapped, false));  // every rank, every time
    if (!mapped) {
        for (void* p : e.opened) cudaIpcCloseMemHandle(p);
        e.opened.clear();
        e.peers = PeerPtrs{};
        return fail(HF_ERR_CUDA, "peer-memory exchange unavailable on some rank");
    }
    e.p2p = true;
    return HF_OK;
}

hf_status ep_create(hf_moe_ctx* c, const unsigned char* unique_id) {
    NcclApi& n = nccl();
    if (!n.ok) return fail(HF_ERR_NCCL, n.error);
    auto* e = new EpState();
    c->ep = e;
    const size_t T = size_t(std::max(1, c->T_max));
    e->R_cap = ep_recv_cap(c);
    const int W = c->world, El = c->E_local;
    HF_TRY(dalloc(&e->yrecv, (T * c->k + T) * c->H));
    // counts [W x El], then (peer memory) the slot -> row maps [W x cap]
    HF_TRY(dalloc(&e->cnt_recv, size_t(W) * El + size_t(W) * T * std::min(c->k, El)));
    HF_TRY(dalloc(&e->row_pos, e->R_cap));
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    HF_NCCL(n.CommInitRank(&e->comm, W, id, c->rank));

    // Slabs: every rank reserves, per source, room for every row that source
    // could send it (T_max tokens x min(k, El) slots). Over peer memory only
    // the rows that exist cross NVLink, so the slabs are used whenever they
    // fit kEpP2PSlabBytes; over NCCL the whole slab travels, so only while
    // small (kEpSlabBytes). Otherwise the exchange is sized on the host.
    const size_t cap = T * size_t(std::min(c->k, El));
    const size_t row4 = size_t(c->H) * 4;  // fp32 activations are the widest rows
    const size_t slab_bytes = size_t(W) * cap * row4;
    const bool try_p2p = !std::getenv("HF_EP_NCCL_ONLY") && W <= kEpMaxRanks &&
                         slab_bytes <= kEpP2PSlabBytes;
    if (try_p2p || slab_bytes <= kEpSlabBytes) {
        HF_TRY(dalloc(&e->xslab_recv, (size_t(W) * cap + T) * row4));
        // output slab: rows from every rank, then this rank's own shared-expert rows
        HF_TRY(dalloc(&e->yslab_recv, (size_t(W) * cap + T) * c->H));
        HF_TRY(dalloc(&e->recv_tot, size_t(W)));
    }
    if (try_p2p && setup_p2p(c) != HF_OK) {
        cudaGetLastError();  // no peer mappings: the NCCL exchanges below
        for (void* p : e->opened) cudaIpcCloseMemHandle(p);
        e->opened.clear();
        e->p2p = false;
    }
    if (e->p2p) {
        e->cap = int(cap);
        HF_TRY(dalloc(&e->yrow, e->R_cap + T));
        HF_TRY(dalloc(&e->d_peer_y, size_t(W)));
        HF_TRY(dalloc(&e->d_peer_flags, size_t(W)));
        HF_TRY(dalloc(&e->rowmap, T * c->k + T));
        HF_CUDA(cudaMemcpy(e->d_peer_y, e->peers.y, sizeof(float*) * W, cudaMemcpyHostToDevice));
        HF_CUDA(cudaMemcpy(e->d_peer_flags, e->peers.flags, sizeof(unsigned long long*) * W,
                           cudaMemcpyHostToDevice));
        HF_CUDA(cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking));
        HF_CUDA(cudaEventCreateWithFlags(&e->ev_routed, cudaEventDisableTiming));
        HF_CUDA(cudaEventCreateWithFlags(&e->ev_packed, cudaEventDisableTiming));
        HF_TRY(dalloc(&e->shared_group, size_t(1)));
    } else if (slab_bytes <= kEpSlabBytes) {
        e->cap = int(cap);
        HF_TRY(dalloc(&e->xslab_send, size_t(W) * cap * row4));
        HF_TRY(dalloc(&e->yslab_send, size_t(W) * cap * c->H));
    } else {
        cudaFree(e->xslab_recv);
        cudaFree(e->yslab_recv);
        e->xslab_recv = nullptr;
        e->yslab_recv = nullptr;
    }
    if (e->cap == 0) {  // host-sized exchange
        HF_TRY(dalloc(reinterpret_cast<float**>(&e->xsend), T * c->k * c->H));
        HF_TRY(dalloc(reinterpret_cast<float**>(&e->xall), (e->R_cap + T) * c->H));
        HF_TRY(dalloc(&e->ysend, e->R_cap * c->H));
        HF_TRY(dalloc(&e->loc_counts, size_t(El) + 1));
        HF_CUDA(cudaMallocHost(reinterpret_cast<void**>(&e->h_src), sizeof(int32_t) * (c->E + 1)));
        HF_CUDA(cudaMallocHost(reinterpret_cast<void**>(&e->h_recv), sizeof(int32_t) * W * El));
        HF_CUDA(cudaMallocHost(reinterpret_cast<void**>(&e->h_perm), sizeof(int32_t) * (e->R_cap + T)));
        HF_CUDA(cudaMallocHost(reinterpret_cast<void**>(&e->h_rowpos), sizeof(int32_t) * e->R_cap));
        HF_CUDA(cudaMallocHost(reinterpret_cast<void**>(&e->h_loc), sizeof(int32_t) * (El + 1)));
    }
    return HF_OK;
}

void ep_destroy(hf_moe_ctx* c) {
    EpState* e = c->ep;
    if (!e) return;
    if (e->side) cudaStreamSynchronize(e->side);
    for (void* p : e->opened) cudaIpcCloseMemHandle(p);
    if (e->comm) nccl().CommDestroy(e->comm);
    if (e->side) cudaStreamDestroy(e->side);
    if (e->ev_routed) cudaEventDestroy(e->ev_routed);
    if (e->ev_packed) cudaEventDestroy(e->ev_packed);
    cudaFree(e->shared_group);
    void* d[] = {e->xsend,      e->xall,       e->ysend,      e->yrecv,     e->cnt_recv,
                 e->loc_counts, e->row_pos,    e->xslab_send, e->xslab_recv, e->yslab_send,
                 e->yslab_recv, e->recv_tot,   e->flags,      e->yrow,      e->d_peer_y,
                 e->d_peer_flags, e->rowmap};
    for (void* p : d) cudaFree(p);
    void* h[] = {e->h_src, e->h_recv, e->h_perm, e->h_rowpos, e->h_loc};
    for (void* p : h)
        if (p) cudaFreeHost(p);
    delete e;
    c->ep = nullptr;
}

// ------------------------------------------------------------------ forward
// The shared expert over this rank's own T tokens as a pass of its own (a
// one-group plan, the tensor-core GEMMs), its outputs into rows W*cap + t of
// this rank's output slab, where the combine reads them. It needs nothing
// from the other ranks, so it runs while the dispatch is in flight.
static hf_status ep_shared_pass(hf_moe_ctx* c, LayerBuf& L, const void* x, hf_dtype xd, int T,
                                bool y16, cudaStream_t st) {
    EpState& e = *c->ep;
    RouteArgs ra{};
    ra.T = T;
    ra.H = c->H;
    ra.plan = c->plan;  // rebuilt by the receiver plan right after this pass (same stream)
    ra.pl = PlanLayout::make(1);
    ra.has_shared = 1;
    ra.shared_inter = c->Is;
    ra.inter = c->Is;
    ra.path = HF_PATH_GEMM;
    ra.gemm_ok = 1;
    set_gemm_tiles(c->gemm_bn, T, ra);
    const size_t n = size_t(c->Is) * c->H;
    GroupW w{L.shared, L.shared + n, L.shared + 2 * n, c->Is, 0, 1.0f, 0};  // GEMV fields: unused
    {
        PhaseTimer pp(c, st, 1);
        HF_TRY(launch_dense_plan(ra, w, e.shared_group, c->perm, c->sched, st));
        pp.done(1);
    }
    ExpertWork ws{};
    ws.down_f16 = L.down_f16;
    ws.plan = c->plan;
    ws.pl = ra.pl;
    ws.perm = c->perm;  // identity: slot t = token t (k = 0)
    ws.x = x;
    ws.x_f32 = xd == HF_F32;
    ws.T = T;
    ws.k = 0;
    // rows W * cap.. of the output slab, in the slab's element type
    const size_t yoff = size_t(c->world) * e.cap * c->H;
    ws.y = y16 ? reinterpret_cast<float*>(reinterpret_cast<__half*>(e.yslab_recv) + yoff)
               : e.yslab_recv + yoff;
    ws.y16 = y16;
    ws.bn1 = ra.gemm_bn1;
    ws.bn2 = ra.gemm_bn2;
    ws.m1 = ra.gemm_m1;
    ws.m2 = ra.gemm_m2;
    ws.pair = ra.gemm_pair;
    ws.maybe_gemm = true;
    ws.maybe_gemv = false;
    ws.groups_base = c->G - 1;  // the GEMM's group 0 is the layer's shared expert
    return run_experts(c, L, ws, st);
}

// The shared expert beside the dispatch pays at two ranks (config 3: the
// dispatch moves 403 MB a layer and the shared pass hides under it) and costs
// at eight (its three smaller launches lose more than the overlap gains:
// 18.3 -> 19.0 ms a step), so by default it runs early at W = 2 only.
static bool ep_shared_early(int world) {
    static const int knob = [] {
        const char* v = std::getenv("HF_EP_SHARED_EARLY");  // tuning knob: 0 never, 1 always
        return v ? std::atoi(v) : -1;
    }();
    return knob < 0 ? world == 2 : knob != 0;
}

// Slab exchange (peer memory at any size, NCCL for small batches): fixed
// per-source regions, counts and plan stay on the device.
static hf_status ep_forward_slabs(hf_moe_ctx* c, LayerBuf& L, const void* x, hf_dtype xd, int T,
                                  float* out, const float* resid, const hf_moe_routing* r,
                                  cudaStream_t st) {
    EpState& e = *c->ep;
    NcclApi& n = nccl();
    const int W = c->world, El = c->E_local, k = c->k, H = c->H, cap = e.cap;
    const size_t rowb = size_t(H) * (xd == HF_F32 ? 4 : 2);
    const bool has_shared = c->Is > 0;
    const int rows = W * cap;

    // every forward on every rank takes the next sequence number (peer memory)
    const unsigned long long seq = e.p2p ? ++e.seq : 0;
    int* err = c->plan + c->pl.stats + 3;

    // 1. route the local tokens over all experts; rows into per-destination slabs
    const RouteArgs ra = route_args(c, L, x, xd, T);
    // Expert paths of the receiver. Tiles and the GEMV threshold follow the
    // whole job's batch (T x W tokens): each local expert sees about as many
    // rows as it would on one GPU. On peer memory with every segment on the
    // tensor-core GEMM, the down GEMM's epilogue stores each output row
    // straight into its source's output slab and its last CTA raises the
    // return flags, so the return overlaps the GEMM and no copy kernel runs.
    RouteArgs rl = ra;
    rl.plan = c->plan;
    rl.pl = c->pl;
    set_gemm_tiles(c->gemm_bn, T * W, rl);
    rl.gemv_max = gemv_threshold(c, T * W);
    const bool maybe_gemm = rl.gemm_ok && (c->cfg.path == HF_PATH_GEMM || rows + T > rl.gemv_max);
    const bool maybe_gemv = !rl.gemm_ok || c->cfg.path == HF_PATH_GEMV ||
                            (c->cfg.path == HF_PATH_AUTO && rl.gemv_max > 0);
    const bool fused = e.p2p && e.yrow && maybe_gemm && !maybe_gemv;
    // expert outputs as the FP16 plane (every rank decides the same: the
    // GEMV possibility depends on the configuration only at W > 1)
    const bool y16 = y16_wanted(c, maybe_gemv);
    const size_t esz = y16 ? 2 : 4;
    const int yvec = int(size_t(H) * esz / 16);  // 16-byte vectors per output row
    // the shared expert runs as its own pass beside the dispatch (fused path)
    const bool early = fused && has_shared && T > 0 && e.side && ep_shared_early(W);
    if (T > 0) {
        HF_TRY(run_route(c, L, ra, st));
    } else {
        HF_CUDA(cudaMemsetAsync(c->plan_src + c->pl_src.counts, 0, sizeof(int32_t) * c->G_src, st));
    }
    const int32_t* cnt_src = c->plan_src + c->pl_src.counts;
    if (e.p2p) {
        // 2. rows straight into the destinations' slabs over NVLink, then the
        // counts and this rank's arrival flag on every rank (even with T = 0);
        // with `early`, on the side stream while the shared expert computes
        cudaStream_t sp = st;
        if (early) {
            HF_CUDA(cudaEventRecord(e.ev_routed, st));
            HF_CUDA(cudaStreamWaitEvent(e.side, e.ev_routed, 0));
            sp = e.side;
        }
        PhaseTimer px(c, sp, 7);
        // beside the shared expert's kernels the pack takes one block per SM,
        // which fits next to a GEMM CTA (a full grid would hold every SM until
        // it drained and the two would run one after the other)
        const int pack_grid = early ? std::min(c->nsm, copy_grid(c->nsm, std::max(1, T * k)))
                                    : copy_grid(c->nsm, std::max(1, T * k));
        k_ep_pack_p2p<<<pack_grid, 256, 0, sp>>>(
            c->perm_src, c->ids, c->slot_pos, c->plan_src + c->pl_src.offsets,
            static_cast<const uint4*>(x), int(rowb / 16), T * k, k, El, cap, c->rank, W, cnt_src,
            e.peers, c->sched + 6, seq, fused ? e.rowmap : nullptr, has_shared ? T : 0);
        HF_CUDA(cudaGetLastError());
        px.done(1);
        if (early) {
            HF_CUDA(cudaEventRecord(e.ev_packed, e.side));
            HF_TRY(ep_shared_pass(c, L, x, xd, T, y16, st));
            HF_CUDA(cudaStreamWaitEvent(st, e.ev_packed, 0));
        }
    } else {
        if (T > 0) {
            PhaseTimer p1(c, st, 1);
            k_ep_pack<<<copy_grid(c->nsm, T * k), 256, 0, st>>>(
                c->perm_src, c->ids, c->plan_src + c->pl_src.offsets, static_cast<const uint4*>(x),
                int(rowb / 16), T * k, k, El, cap, reinterpret_cast<uint4*>(e.xslab_send));
            HF_CUDA(cudaGetLastError());
            p1.done(1);
        }
        // 2. counts and slabs to every rank in one NCCL group
        PhaseTimer px(c, st, 7);
        HF_NCCL(n.GroupStart());
        for (int d = 0; d < W; ++d) {
            HF_NCCL(n.Send(cnt_src + d * El, El, ncclInt32, d, e.comm, st));
            HF_NCCL(n.Recv(e.cnt_recv + d * El, El, ncclInt32, d, e.comm, st));
            HF_NCCL(n.Send(e.xslab_send + size_t(d) * cap * rowb, size_t(cap) * rowb, ncclChar, d,
                           e.comm, st));
            HF_NCCL(n.Recv(e.xslab_recv + size_t(d) * cap * rowb, size_t(cap) * rowb, ncclChar, d,
                           e.comm, st));
        }
        HF_NCCL(n.GroupEnd());
        px.done(0);
    }
    // local tokens after the slabs (the shared expert's rows of the grouped pass)
    if (T > 0 && !early)
        HF_CUDA(cudaMemcpyAsync(e.xslab_recv + size_t(rows) * rowb, x, size_t(T) * rowb,
                                cudaMemcpyDeviceToDevice, st));

    // 3. receiver plan on the device (without the shared expert when it ran
    // early), then the local experts
    if (early) rl.has_shared = 0;
    {
        PhaseTimer pp(c, st, 1);
        const EpRowOut ro{fused ? e.yrow : nullptr, e.d_peer_y, c->rank, H, int(esz)};
        HF_TRY(launch_ep_plan(rl, e.cnt_recv, e.p2p ? e.cnt_recv + W * El : nullptr, W, El, cap,
                              T, c->perm, e.row_pos, e.recv_tot,
                              e.p2p ? e.flags : nullptr, seq, c->timeout_ns, err, ro, st));
        pp.done(1);
    }
    ExpertWork w{};
    w.down_f16 = L.down_f16;
    w.plan = c->plan;
    w.pl = c->pl;
    w.perm = c->perm;
    w.x = e.xslab_recv;
    w.x_f32 = xd == HF_F32;
    w.T = rows + T;
    w.k = 1;
    w.y = c->y;
    w.y16 = y16;
    w.bn1 = rl.gemm_bn1;
    w.bn2 = rl.gemm_bn2;
    w.m1 = rl.gemm_m1;
    w.m2 = rl.gemm_m2;
    w.pair = rl.gemm_pair;
    w.maybe_gemm = maybe_gemm;
    w.maybe_gemv = maybe_gemv;
    if (fused) {
        w.yrow = e.yrow;
        w.sig_flags = e.d_peer_flags;
        w.sig_n = W;
        w.sig_slot = W + c->rank;
        w.sig_seq = seq;
    }
    HF_TRY(run_experts(c, L, w, st));

    if (fused) {
        // 4. every rank's outputs for this rank's tokens are in its output slab
        // once every return flag shows this forward; 5. combine from there
        PhaseTimer py(c, st, 8);
        k_ep_wait<<<1, 32, 0, st>>>(e.flags + W, W, seq, c->timeout_ns, err);
        HF_CUDA(cudaGetLastError());
        py.done(1);
        if (T > 0)
            HF_TRY(run_combine(c, e.yslab_recv, y16, T, out, resid, r ? r->slot_out : nullptr, st,
                               e.rowmap));
        return HF_OK;
    }

    // 4. outputs back to their sources in arrival order, then to canonical positions
    const int n_shared = has_shared ? T : 0;
    const size_t yslab = size_t(cap) * H * esz;  // bytes of one source's output slab
    PhaseTimer py(c, st, 8);
    if (e.p2p) {
        k_ep_unpack_p2p<<<copy_grid(c->nsm, rows), 256, 0, st>>>(
            reinterpret_cast<const float4*>(c->y), e.row_pos, e.recv_tot, W, cap, yvec, c->rank,
            e.peers, c->sched + 7, seq);
        HF_CUDA(cudaGetLastError());
        if (T == 0) {  // no outputs to collect, but every rank waits for every rank
            k_ep_wait<<<1, 32, 0, st>>>(e.flags + W, W, seq, c->timeout_ns, err);
            HF_CUDA(cudaGetLastError());
        }
    } else {
        k_ep_unpack<<<copy_grid(c->nsm, rows), 256, 0, st>>>(
            reinterpret_cast<const float4*>(c->y), e.row_pos, e.recv_tot, W, cap, yvec,
            reinterpret_cast<float4*>(e.yslab_send));
        HF_CUDA(cudaGetLastError());
        char* ys = reinterpret_cast<char*>(e.yslab_send);
        char* yr = reinterpret_cast<char*>(e.yslab_recv);
        HF_NCCL(n.GroupStart());
        for (int d = 0; d < W; ++d) {
            HF_NCCL(n.Send(ys + size_t(d) * yslab, yslab, ncclChar, d, e.comm, st));
            HF_NCCL(n.Recv(yr + size_t(d) * yslab, yslab, ncclChar, d, e.comm, st));
        }
        HF_NCCL(n.GroupEnd());
    }
    if (T > 0) {
        k_ep_return<<<copy_grid(c->nsm, T * k + n_shared), 256, 0, st>>>(
            c->perm_src, c->ids, c->plan_src + c->pl_src.offsets, T * k, k, El, cap,
            reinterpret_cast<const float4*>(e.yslab_recv), reinterpret_cast<const float4*>(c->y),
            c->plan + c->pl.offsets + El, n_shared, yvec, reinterpret_cast<float4*>(e.yrecv),
            e.p2p ? e.flags + W : nullptr, W, seq, c->timeout_ns, err);
        HF_CUDA(cudaGetLastError());
    }
    py.done(T > 0 ? 2 : 1);
    // 5. combine in the reference order at the source
    if (T > 0) HF_TRY(run_combine(c, e.yrecv, y16, T, out, resid, r ? r->slot_out : nullptr, st));
    return HF_OK;
}

// Large batches: per-forward counts sized on the host, exact-size exchange.
static hf_status ep_forward_sized(hf_moe_ctx* c, LayerBuf& L, const void* x, hf_dtype xd, int T,
                                  float* out, const float* resid, const hf_moe_routing* r,
                                  cudaStream_t st) {
    EpState& e = *c->ep;
    NcclApi& n = nccl();
    const int W = c->world, El = c->E_local, k = c->k, H = c->H;
    const size_t elt = xd == HF_F32 ? 4 : 2;
    const size_t rowb = size_t(H) * elt;
    const bool has_shared = c->Is > 0;

    // 1. route the local tokens over all experts; gather their rows in slot order
    const RouteArgs ra = route_args(c, L, x, xd, T);
    if (T > 0) {
        HF_TRY(run_route(c, L, ra, st));
        PhaseTimer p1(c, st, 1);
        HF_TRY(launch_gather_rows(e.xsend, x, rowb, T * k, c->perm_src, k, st));
        p1.done(1);
    } else {
        HF_CUDA(cudaMemsetAsync(c->plan_src + c->pl_src.counts, 0, sizeof(int32_t) * c->G_src, st));
    }
    // 2. per-expert counts to every rank; read them back to size the exchange
    const int32_t* cnt_src = c->plan_src + c->pl_src.counts;
    PhaseTimer px(c, st, 7);
    HF_NCCL(n.GroupStart());
    for (int d = 0; d < W; ++d) {
        HF_NCCL(n.Send(cnt_src + d * El, El, ncclInt32, d, e.comm, st));
        HF_NCCL(n.Recv(e.cnt_recv + d * El, El, ncclInt32, d, e.comm, st));
    }
    HF_NCCL(n.GroupEnd());
    HF_CUDA(cudaMemcpyAsync(e.h_src, cnt_src, sizeof(int32_t) * c->E, cudaMemcpyDeviceToHost, st));
    HF_CUDA(cudaMemcpyAsync(e.h_recv, e.cnt_recv, sizeof(int32_t) * W * El, cudaMemcpyDeviceToHost, st));
    HF_CUDA(cudaStreamSynchronize(st));
    ExchangePlan p;
    build_plan(W, El, T, has_shared, e.h_src, e.h_recv, p, e.h_perm, e.h_rowpos);
    const int R = p.R;
    if (size_t(R) > e.R_cap) return fail(HF_ERR_STATE, "expert-parallel receive exceeds capacity");
    // slot ids of the receiver plan: received row r -> r; shared token t -> (R+T) + (R+t)
    for (int i = 0; i < R + (has_shared ? T : 0); ++i) {
        const int row = e.h_perm[i];
        e.h_perm[i] = row < R ? row : (R + T) + row;
    }
    int maxseg = 0;
    for (int j = 0; j <= El; ++j) {
        e.h_loc[j] = p.local_counts[j];
        maxseg = std::max(maxseg, p.local_counts[j]);
    }
    const int npos = R + (has_shared ? T : 0);
    if (npos > 0)
        HF_CUDA(cudaMemcpyAsync(c->perm, e.h_perm, sizeof(int32_t) * npos, cudaMemcpyHostToDevice, st));
    if (R > 0)
        HF_CUDA(cudaMemcpyAsync(e.row_pos, e.h_rowpos, sizeof(int32_t) * R, cudaMemcpyHostToDevice, st));
    HF_CUDA(cudaMemcpyAsync(e.loc_counts, e.h_loc, sizeof(int32_t) * (El + 1), cudaMemcpyHostToDevice, st));

    // 3. dispatch: rows for rank d's experts to rank d; then append local tokens
    char* xs = static_cast<char*>(e.xsend);
    char* xa = static_cast<char*>(e.xall);
    HF_NCCL(n.GroupStart());
    for (int d = 0; d < W; ++d) {
        const size_t ns = size_t(p.send_off[d + 1] - p.send_off[d]) * rowb;
        const size_t nr = size_t(p.recv_off[d + 1] - p.recv_off[d]) * rowb;
        if (ns) HF_NCCL(n.Send(xs + size_t(p.send_off[d]) * rowb, ns, ncclChar, d, e.comm, st));
        if (nr) HF_NCCL(n.Recv(xa + size_t(p.recv_off[d]) * rowb, nr, ncclChar, d, e.comm, st));
    }
    HF_NCCL(n.GroupEnd());
    if (T > 0) HF_CUDA(cudaMemcpyAsync(xa + size_t(R) * rowb, x, size_t(T) * rowb, cudaMemcpyDeviceToDevice, st));
    px.done(0);

    // 4. local experts over received rows, shared expert over local tokens
    RouteArgs rl = ra;
    rl.plan = c->plan;
    rl.pl = c->pl;
    rl.T = R + T;
    set_gemm_tiles(c->gemm_bn, T * W, rl);
    rl.gemv_max = gemv_threshold(c, T * W);
    {
        PhaseTimer pp(c, st, 1);
        HF_TRY(launch_plan_from_counts(rl, e.loc_counts, st));
        pp.done(1);
    }
    ExpertWork w{};
    w.down_f16 = L.down_f16;
    w.plan = c->plan;
    w.pl = c->pl;
    w.perm = c->perm;
    w.x = e.xall;
    w.x_f32 = xd == HF_F32;
    w.T = R + T;
    w.k = 1;
    w.y = c->y;
    w.bn1 = rl.gemm_bn1;
    w.bn2 = rl.gemm_bn2;
    w.m1 = rl.gemm_m1;
    w.m2 = rl.gemm_m2;
    w.pair = rl.gemm_pair;
    w.maybe_gemm = rl.gemm_ok && (c->cfg.path == HF_PATH_GEMM || maxseg > rl.gemv_max);
    w.maybe_gemv = !rl.gemm_ok || c->cfg.path == HF_PATH_GEMV ||
                   (c->cfg.path == HF_PATH_AUTO && rl.gemv_max > 0);
    // the same on every rank: maybe_gemv depends on the configuration only
    const bool y16 = y16_wanted(c, w.maybe_gemv);
    w.y16 = y16;
    if (npos > 0) HF_TRY(run_experts(c, L, w, st));

    // 5. outputs back to their sources, at canonical slot positions
    PhaseTimer py(c, st, 8);
    const size_t yrow = size_t(H) * (y16 ? 2 : 4);  // bytes of one output row
    if (R > 0) HF_TRY(launch_gather_rows(e.ysend, c->y, yrow, R, e.row_pos, 1, st));
    char* ys = reinterpret_cast<char*>(e.ysend);
    char* yr = reinterpret_cast<char*>(e.yrecv);
    HF_NCCL(n.GroupStart());
    for (int d = 0; d < W; ++d) {
        const size_t ns = size_t(p.recv_off[d + 1] - p.recv_off[d]) * yrow;
        const size_t nr = size_t(p.send_off[d + 1] - p.send_off[d]) * yrow;
        if (ns) HF_NCCL(n.Send(ys + size_t(p.recv_off[d]) * yrow, ns, ncclChar, d, e.comm, st));
        if (nr) HF_NCCL(n.Recv(yr + size_t(p.send_off[d]) * yrow, nr, ncclChar, d, e.comm, st));
    }
    HF_NCCL(n.GroupEnd());
    if (T > 0 && has_shared)
        HF_CUDA(cudaMemcpyAsync(yr + size_t(T) * k * yrow,
                                reinterpret_cast<const char*>(c->y) + size_t(R) * yrow,
                                size_t(T) * yrow, cudaMemcpyDeviceToDevice, st));
    py.done(R > 0 ? 1 : 0);
    // 6. combine in the reference order at the source
    if (T > 0) HF_TRY(run_combine(c, e.yrecv, y16, T, out, resid, r ? r->slot_out : nullptr, st));
    return HF_OK;
}

hf_status ep_forward(hf_moe_ctx* c, LayerBuf& L, const void* x, hf_dtype xd, int T, float* out,
                     const float* resid, const hf_moe_routing* r, cudaStream_t st) {
    if (c->ep->cap > 0) return ep_forward_slabs(c, L, x, xd, T, out, resid, r, st);
    return ep_forward_sized(c, L, x, xd, T, out, resid, r, st);
}

// ------------------------------------------------------------------ expert placement
// Router rows and bias of a placed layer: written in global expert order by
// the weight setters, then gathered into placed order (row j <- order[j]).
hf_status place_router(hf_moe_ctx* c, LayerBuf& L, cudaStream_t st) {
    if (L.order.empty()) return HF_OK;
    const size_t rows = size_t(c->E), rb = size_t(c->H) * 2;
    uint16_t* tmp = nullptr;
    HF_TRY(dalloc(&tmp, rows * c->H));
    hf_status s = launch_gather_rows(tmp, L.router, rb, int(rows), L.d_order, 1, st);
    if (s == HF_OK &&
        cudaMemcpyAsync(L.router, tmp, rows * rb, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        s = fail(HF_ERR_CUDA, "router placement copy failed");
    std::vector<float> b(rows), pb(rows);
    if (s == HF_OK &&
        (cudaMemcpyAsync(b.data(), L.bias, sizeof(float) * rows, cudaMemcpyDeviceToHost, st) !=
             cudaSuccess ||
         cudaStreamSynchronize(st) != cudaSuccess))
        s = fail(HF_ERR_CUDA, "bias placement read failed");
    if (s == HF_OK) {
        for (size_t j = 0; j < rows; ++j) pb[j] = b[size_t(L.order[j])];
        if (cudaMemcpy(L.bias, pb.data(), sizeof(float) * rows, cudaMemcpyHostToDevice) !=
            cudaSuccess)
            s = fail(HF_ERR_CUDA, "bias placement write failed");
    }
    cudaStreamSynchronize(st);
    cudaFree(tmp);
    return s;
}

// Routing outputs in global expert ids from the placed ones: ids through
// order[], counts to their experts, offsets rescanned, and each expert's
// segment of the permutation moved to its global offset (the order inside a
// segment, token then slot, does not depend on the labels). One block.
__global__ void __launch_bounds__(1024) k_unplace(const int32_t* order, int E, int T, int k,
                                                  const int32_t* ids_p, const int32_t* cnt_p,
                                                  const int32_t* off_p, const int32_t* perm_p,
                                                  int32_t* ids_o, int32_t* cnt_o, int32_t* off_o,
                                                  int32_t* perm_o) {
    extern __shared__ int32_t sm_u[];
    const int G = E + 1;
    int32_t* s_cnt = sm_u;          // [G] global order
    int32_t* s_off = s_cnt + G;     // [G + 1] global order
    int32_t* s_offp = s_off + G + 1;  // [G + 1] placed order
    for (int j = threadIdx.x; j < G; j += blockDim.x) {
        const int e = j < E ? order[j] : E;
        s_cnt[e] = cnt_p[j];
    }
    for (int j = threadIdx.x; j <= G; j += blockDim.x) s_offp[j] = off_p[j];
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int e = 0; e < G; ++e) {
            s_off[e] = acc;
            acc += s_cnt[e];
        }
        s_off[G] = acc;
    }
    __syncthreads();
    if (cnt_o)
        for (int e = threadIdx.x; e < G; e += blockDim.x) cnt_o[e] = s_cnt[e];
    if (off_o)
        for (int e = threadIdx.x; e <= G; e += blockDim.x) off_o[e] = s_off[e];
    if (ids_o)
        for (int i = threadIdx.x; i < T * k; i += blockDim.x) ids_o[i] = order[ids_p[i]];
    if (perm_o) {
        const int n = s_offp[G];
        for (int p = threadIdx.x; p < n; p += blockDim.x) {
            int lo = 0, hi = G - 1;  // group j of placed position p: s_offp[j] <= p < s_offp[j+1]
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (s_offp[mid] <= p) lo = mid;
                else hi = mid - 1;
            }
            const int e = lo < E ? order[lo] : E;
            perm_o[s_off[e] + (p - s_offp[lo])] = perm_p[p];
        }
    }
}

hf_status unplace_routing(hf_moe_ctx* c, const LayerBuf& L, const hf_moe_routing* r, int T,
                          cudaStream_t st) {
    const int G = c->E + 1;
    const size_t smem = sizeof(int32_t) * size_t(3 * G + 2);
    HF_CUDA(ensure_smem(reinterpret_cast<const void*>(k_unplace), int(smem)));
    k_unplace<<<1, 1024, smem, st>>>(L.d_order, c->E, T, c->k, c->ids, c->plan_src + c->pl_src.counts,
                                     c->plan_src + c->pl_src.offsets, c->perm_src, r->topk_ids,
                                     r->counts, r->offsets, r->perm);
    HF_CUDA(cudaGetLastError());
    return HF_OK;
}

int ep_transport(const hf_moe_ctx* c) {
    if (!c->ep) return 0;
    if (c->ep->p2p) return 1;
    return c->ep->cap > 0 ? 2 : 3;
}

// Every rank: wait for this rank's work, clear the error word, and adopt the
// largest forward sequence number of any rank, so that the next forward waits
// for flags that only that forward's stores can raise (flags left by a
// forward that ran on fewer than all ranks are below it).
hf_status ep_resync(hf_moe_ctx* c) {
    EpState& e = *c->ep;
    HF_CUDA(cudaDeviceSynchronize());
    HF_CUDA(cudaMemset(c->plan + c->pl.stats + 3, 0, sizeof(int)));
    unsigned long long s = e.seq;
    HF_TRY(allreduce_u64(e, &s, true));
    e.seq = s;
    return HF_OK;
}

}  // namespace hf

using namespace hf;

extern "C" hf_status hf_moe_set_placement(hf_moe_ctx* ctx, int layer, const int32_t* order) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_set_placement: null context");
    if (layer < 0 || layer >= int(ctx->layers.size()))
        return fail(HF_ERR_ARG, "hf_moe_set_placement: layer out of range");
    const int E = ctx->E;
    std::vector<int32_t> ord(static_cast<size_t>(E)), inv(static_cast<size_t>(E), -1);
    bool identity = true;
    for (int j = 0; j < E; ++j) {
        const int e = order ? order[j] : j;
        if (e < 0 || e >= E || inv[size_t(e)] >= 0)
            return fail(HF_ERR_ARG, "hf_moe_set_placement: order is not a permutation of 0..E-1");
        ord[size_t(j)] = e;
        inv[size_t(e)] = j;
        identity = identity && e == j;
    }
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(ctx_layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    const bool same = identity ? L.order.empty() : L.order == ord;
    if (same) return HF_OK;
    if (identity) {
        L.order.clear();
        L.inv.clear();
    } else {
        if (!L.d_order) HF_TRY(dalloc(&L.d_order, size_t(E)));
        HF_CUDA(cudaMemcpy(L.d_order, ord.data(), sizeof(int32_t) * E, cudaMemcpyHostToDevice));
        L.order = std::move(ord);
        L.inv = std::move(inv);
    }
    L.loaded = false;  // the rank's experts changed: the weights are set again
    return HF_OK;
}

extern "C" hf_status hf_ep_balanced_placement(int E, int world, const long long* load,
                                              int32_t* order) {
    if (E <= 0 || world <= 0 || E % world || !load || !order)
        return fail(HF_ERR_ARG, "hf_ep_balanced_placement: bad arguments (E must divide by world)");
    const int El = E / world;
    std::vector<int> idx(static_cast<size_t>(E));
    std::iota(idx.begin(), idx.end(), 0);
    // heaviest first (ties: lower id), each to the least-loaded rank with room
    std::stable_sort(idx.begin(), idx.end(),
                     [&](int a, int b) { return load[a] > load[b]; });
    std::vector<long long> sum(static_cast<size_t>(world), 0);
    std::vector<std::vector<int>> own(static_cast<size_t>(world));
    for (int e : idx) {
        int best = -1;
        for (int r = 0; r < world; ++r)
            if (int(own[size_t(r)].size()) < El && (best < 0 || sum[size_t(r)] < sum[size_t(best)]))
                best = r;
        own[size_t(best)].push_back(e);
        sum[size_t(best)] += load[e];
    }
    for (int r = 0; r < world; ++r) {
        std::sort(own[size_t(r)].begin(), own[size_t(r)].end());
        for (int l = 0; l < El; ++l) order[size_t(r) * El + l] = own[size_t(r)][size_t(l)];
    }
    return HF_OK;
}

extern "C" hf_status hf_moe_ep_transport(hf_moe_ctx* ctx, int* transport) {
    if (!ctx || !transport) return fail(HF_ERR_ARG, "hf_moe_ep_transport: null argument");
    *transport = ep_transport(ctx);
    return HF_OK;
}

extern "C" hf_status hf_moe_ep_resync(hf_moe_ctx* ctx) {
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_ep_resync: null context");
    if (!ctx->ep) return HF_OK;
    DeviceGuard dg(ctx->cfg.device);
    return ep_resync(ctx);
}

extern "C" hf_status hf_ep_unique_id(unsigned char* out) {
    if (!out) return fail(HF_ERR_ARG, "hf_ep_unique_id: null output");
    NcclApi& n = nccl();
    if (!n.ok) return fail(HF_ERR_NCCL, n.error);
    ncclUniqueId id;
    HF_NCCL(n.GetUniqueId(&id));
    static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
    std::memcpy(out, &id, sizeof(id));
    return HF_OK;
}

extern "C" hf_status hf_ep_plan(int world, int E_local, int T_local, int has_shared,
                                const int32_t* send_counts, const int32_t* recv_counts,
                                int32_t* send_off, int32_t* recv_off, int32_t* local_counts,
                                int32_t* local_rows, int32_t* row_pos) {
    if (world <= 0 || E_local <= 0 || T_local < 0 || !send_counts || !recv_counts)
        return fail(HF_ERR_ARG, "hf_ep_plan: bad arguments");
    ExchangePlan p;
    build_plan(world, E_local, T_local, has_shared != 0, send_counts, recv_counts, p, local_rows,
               row_pos);
    if (send_off) std::copy(p.send_off.begin(), p.send_off.end(), send_off);
    if (recv_off) std::copy(p.recv_off.begin(), p.recv_off.end(), recv_off);
    if (local_counts) std::copy(p.local_counts.begin(), p.local_counts.end(), local_counts);
    return HF_OK;
}
