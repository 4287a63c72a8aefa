// Host-side internals shared by the library's translation units.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <atomic>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/moe_b200.h"

namespace moe {

// Layout of the context's 256-byte status block (zeroed at creation; moe_sync clears the kernel
// words after an error):
//   [0, 4)      int status word (first device error code)
//   [64, 72)    decode kernel: 64-bit launch counter (its epochs)
//   [160, 164)  LM-head kernel: CTA completion ticket
//   [168, 232)  LM-head kernel: 8 64-bit argmax keys
constexpr size_t kStatusBlockBytes = 256;
constexpr size_t kStatusDecodeOff = 64;
constexpr size_t kStatusVocabTicketOff = 160;
constexpr size_t kStatusVocabKeysOff = 168;
constexpr size_t kStatusKernelEnd = 232;

// Tokens per chunk of the CUDA-core grouped GEMV kernels.
constexpr int kGemvTok = 8;

// Device copies of one layer's per-expert weight pointers; index E is the shared expert.
struct ExpertTables {
    const uint8_t* const* w1;  // [E+1]
    const uint8_t* const* w3;  // [E+1]
    const uint8_t* const* w2;  // [E+1]
};

struct Layer {
    moe_layer_spec spec;
    const uint8_t** tab = nullptr;  // device [3][E+1]
    std::vector<const uint8_t*> host_tab;  // the same pointers on the host (kernel parameters)
    bool tab_aligned16 = false;     // every expert weight pointer is 16-byte aligned
    const uint8_t* router_w_ptr = nullptr;
    const uint8_t* bias_ptr = nullptr;  // may be null
    const uint8_t* gate_ptr = nullptr;  // may be null
    // the layer that runs after this one (moe_layer_set_next): its router and shared expert are
    // prefetched into L2 by the single-token kernel
    const uint8_t* next_router = nullptr;
    size_t next_router_bytes = 0;
    const uint8_t* next_shared[3] = {nullptr, nullptr, nullptr};
    size_t next_shared_bytes[3] = {0, 0, 0};
    CUtensorMap* wmaps = nullptr;       // device [3][E+1] raw IQ4_XS maps (W1, W3, W2), or null
                                        // when the shapes do not suit the tensor-core path
    float* wsplit = nullptr;            // device [2][E][H]: router weight split (TF32 hi, rest)
    CUtensorMap rmaps[2];               // maps over wsplit (valid when wsplit != null)
    ExpertTables tables() const {
        const uint32_t n = spec.n_experts + 1;
        return ExpertTables{tab, tab + n, tab + 2 * n};
    }
    bool has_shared() const { return (spec.flags & MOE_F_SHARED) != 0; }
    bool subset() const { return (spec.flags & MOE_F_EXPERT_SUBSET) != 0; }
    bool ref36() const { return (spec.flags & MOE_F_REF36) != 0; }
    int slots() const { return static_cast<int>(spec.top_k) + (has_shared() ? 1 : 0); }
};

// Chunk of one bucket handled by the grouped kernels: tokens [start, start+n) of the sorted
// order, all routed to expert `bucket` (bucket == E: shared expert).
struct Chunk {
    int bucket;
    int start;
    int n;
    int pad;
};

// Per-call activation pointers, read by the kernels from device memory so that one captured
// CUDA graph serves every call with the same (layer, M, path): only the tiny kernel that writes
// this block changes between replays.
struct IoArgs {
    const float* x;      // [M][H] MoE input (router and experts)
    const float* resid;  // [M][H] residual added to the output, or null
    float* out;          // [M][H]
};

// fp16 activation tensor maps with 16-, 32-, 64- and 128-row boxes (64 columns, 128B swizzle):
// the tensor-core kernels load a token tile's B stage with one box of the smallest height that
// covers it (one large box streams ~2.4x faster per SM than the same bytes in 16-row boxes).
struct BMaps {
    CUtensorMap m[4];
};

// Token tile of one bucket for the tensor-core kernels: slots [p0, p0+n) of the sorted order.
struct TcTile {
    int bucket;
    int p0;
    int n;
    int pad;
};

// Expert-path selection (moe_set_path).
enum Path : int { kPathAuto = 0, kPathGemv = 1, kPathTcSmemA = 2, kPathTcTmemA = 3 };

// Workspace carve-up for one forward of up to `cap_tokens` tokens.
struct Workspace {
    uint8_t* base = nullptr;
    size_t bytes = 0;
    uint32_t cap_tokens = 0;
    uint32_t cap_experts = 0;
    uint32_t cap_slots = 0;
    uint32_t cap_hidden = 0;
    uint32_t cap_inter = 0;
    // regions
    float* logits = nullptr;      // [M][E+1]
    uint2* topk = nullptr;        // [M][k+1] {id, f32 bits}
    int* tilecnt = nullptr;       // [tiles][E+1]
    int* ranges = nullptr;        // [E+2]
    int* sorted_tok = nullptr;    // [S]
    float* sorted_w = nullptr;    // [S]
    int* slot_pos = nullptr;      // [M][k+1]
    Chunk* chunks = nullptr;      // [max_chunks]
    int* counters = nullptr;      // [8] device counters (n_chunks, ...)
    int* status = nullptr;        // device error status
    float* h = nullptr;           // [S][2I]: GEMV path h [S][I]; tensor-core path [g | u]
    float* ypart = nullptr;       // [S][H]
    TcTile* tiles13 = nullptr;    // tensor-core token tiles of <= 64 tokens
    TcTile* tiles2 = nullptr;     // tensor-core token tiles of <= 128 tokens
    uint32_t max_tiles13 = 0, max_tiles2 = 0;
    __half* x16 = nullptr;        // [S][H] gathered, scaled, K-permuted activations
    __half* h16 = nullptr;        // [S][I]
    int* xexp = nullptr;          // [S] power-of-two exponent of x16's scale
    float* xh = nullptr;          // [M][H] TF32 part of x (tensor-core router)
    float* xl = nullptr;          // [M][H] remainder x - xh
    float* xn = nullptr;          // [M][H] normalised layer input (moe_forward_norm)
    CUtensorMap xhmap, xlmap;
    const void* xh_base = nullptr;
    uint64_t xh_rows = 0, xh_cols = 0;
    int* hexp = nullptr;          // [S]
    // tensor maps (re-encoded when the buffers or the slot count change)
    BMaps xmap, hmap;
    const void* xmap_base = nullptr;
    const void* hmap_base = nullptr;
    uint64_t xmap_rows = 0, hmap_rows = 0, xmap_cols = 0, hmap_cols = 0;
    IoArgs* io = nullptr;         // device IoArgs of the current call
    unsigned long long* dx = nullptr;  // single-token kernel's epoch-tagged exchange entries
                                       // (decode_exchange_words), zeroed at allocation
    size_t dx_bytes = 0;
    uint32_t max_chunks = 0;
};

struct StageStat {
    std::string name;
    uint32_t calls = 0;
    double total_ms = 0.0;
};

// One captured forward (set_io + routing + experts + combine) for a (layer, M, path, stream).
struct GraphEntry {
    uint32_t layer = 0;
    uint32_t M = 0;
    int path = 0;
    cudaStream_t stream = nullptr;
    uint64_t ws_gen = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaGraphNode_t io_node = nullptr;
    uint64_t n_kernels = 0;
    uint64_t last_use = 0;
};

// NCCL entry points used by the expert-parallel layer (resolved at run time, nccl_dl.cu).
struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};
// Null (with *err set) when NCCL cannot be loaded.
const NcclApi* nccl_api(std::string* err);

// Expert-parallel state of a context (moe_ep_init / moe_forward_ep): the communicator and the
// exchange buffers, sized for n_ranks x capacity rows.
struct EpState {
    ncclComm_t comm = nullptr;
    uint32_t n_ranks = 0, rank = 0;
    uint32_t capacity = 0, hidden = 0, top_k = 0;  // buffer sizes
    uint8_t* buf = nullptr;
    uint8_t* plan = nullptr;
    float* send_x = nullptr;
    float* recv_x = nullptr;
    float* y_send = nullptr;
    float* y_recv = nullptr;
    uint2* send_rec = nullptr;
    uint2* recv_rec = nullptr;
    unsigned long long* flags = nullptr;  // [2][8]: per slot, the step each rank has published
    unsigned long long* epoch = nullptr;  // steps started by this rank
    // peer transport: the other ranks' exchange buffers mapped through CUDA IPC
    int transport = 1;                    // MOE_EP_TRANSPORT_PEER / _NCCL as requested
    bool peer = false;                    // the peer transport is active for the current buffers
    uint8_t* peer_base[8] = {};
    uint64_t off_recv_x = 0, off_recv_rec = 0, off_y_send = 0, off_flags = 0;
    // earlier buffer generations (replaced when a larger capacity was asked for): kept with their
    // mappings until the context is destroyed, so CUDA graphs captured against them stay valid
    struct Retired {
        uint8_t* buf;
        uint8_t* peer_base[8];
    };
    std::vector<Retired> retired;
    // set by moe_ep_abort (possibly from another thread): the communicator was aborted and freed
    std::atomic<bool> aborted{false};
    // back to the state of a context without a group (keeps nothing)
    void reset() {
        comm = nullptr;
        n_ranks = rank = capacity = hidden = top_k = 0;
        buf = plan = nullptr;
        send_x = recv_x = y_send = y_recv = nullptr;
        send_rec = recv_rec = nullptr;
        flags = epoch = nullptr;
        transport = 1;
        peer = false;
        for (auto& p : peer_base) p = nullptr;
        off_recv_x = off_recv_rec = off_y_send = off_flags = 0;
        retired.clear();
        aborted.store(false);
    }
};

struct Ctx {
    // CUDA graphs of moe_forward, keyed by (layer, M, path, stream)
    bool use_graphs = true;
    std::vector<GraphEntry> graphs;
    uint64_t ws_gen = 0, graph_clock = 0;
    // tracing: events of the current call and accumulated per-stage statistics
    bool prof = false;
    std::vector<cudaEvent_t> ev;
    std::vector<std::string> ev_names;
    std::vector<StageStat> stats;
    uint64_t launches = 0;
    int device = 0;
    uint8_t* base = nullptr;
    uint64_t bytes = 0;
    bool owns = false;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int sm_count = 148;
    int path = kPathAuto;
    std::string err;
    std::vector<Layer> layers;
    Workspace ws;
    // the shared expert's pass of a large-batch forward, on a second stream concurrently with
    // the routing (its own workspace; created on first use)
    Workspace ws_sh;
    cudaStream_t side_stream = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // moe_forward_host: kHostSlots device staging slots (x rows then out rows), copy streams and
    // the events that order them with the layer on `stream` (created on first use)
    static constexpr int kHostSlots = 3;
    float* host_stage[kHostSlots] = {};
    size_t host_stage_bytes = 0;  // per slot (x + out)
    int host_next = 0;
    cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;
    cudaEvent_t ev_in[kHostSlots] = {}, ev_done[kHostSlots] = {}, ev_out[kHostSlots] = {};
    float* ref36_scratch = nullptr;  // K-split partial sums of MOE_F_REF36 layers
    size_t ref36_scratch_bytes = 0;
    EpState ep;
};

// Kernel launchers (stream-ordered, no synchronisation).
int router_split_for(int M, int H);
void launch_set_io(IoArgs* dst, const float* x, const float* resid, float* out, cudaStream_t s);
const void* set_io_func();
void launch_router_logits(const Layer& L, const IoArgs* io, int M, float* logits, cudaStream_t s);
void launch_topk(const Layer& L, const float* logits, int n_split, bool gate_in_logits,
                 const IoArgs* io, int M, uint2* topk, int* status, cudaStream_t s);
void launch_bucket(int E, int k, bool routed, bool has_shared, const uint2* topk, int M, Workspace& ws,
                   int* ranges, int* sorted_tok, float* sorted_w, int* slot_pos, int* status,
                   cudaStream_t s);
void launch_gemv13(const Layer& L, const IoArgs* io, const Workspace& ws, int M, int max_chunks,
                   int sm_count, cudaStream_t s);
void launch_gemv2(const Layer& L, const Workspace& ws, int M, int max_chunks, int sm_count,
                  cudaStream_t s);
int tc_max_n(int mode);
bool tc_supported(int hidden, int inter);
void launch_convert_x(const IoArgs* io, const int* slot_pos, int M, int ns, int len, __half* dst,
                      int* sexp, cudaStream_t s);
void launch_convert_h(const float* gu, int n_rows, const int* n_used, int inter, __half* dst, int* sexp,
                      cudaStream_t s);
bool make_iq4_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes);
bool make_f32_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
void launch_split_tf32(const float* src, size_t n, float* hi, float* lo, cudaStream_t s);
// x -> TF32 parts; with gate_w, also the shared gate logit into column E of the logit planes.
void launch_split_x(const IoArgs* io, int M, int H, float* hi, float* lo, const float* gate_w, float* logits,
                    int n_split, int E, cudaStream_t s);
int router_tc_split(int M, int E, int H);
void launch_router_tc(const Layer& L, const CUtensorMap& xh, const CUtensorMap& xl, int M,
                      float* partial, int* status, cudaStream_t s);
void launch_tc13(const Layer& L, const BMaps& xmap, const Workspace& ws, int max_items,
                 int sm_count, bool a_tmem, cudaStream_t s);
void launch_tc2(const Layer& L, const BMaps& hmap, const Workspace& ws, int max_items,
                int sm_count, bool a_tmem, cudaStream_t s);
bool make_fp16_tmaps(BMaps* m, const void* base, uint64_t rows, uint64_t cols);
bool decode_supported(const Layer& L, int sm_count);
// 64-bit entries of the single-token kernel's exchange area: half-row logits and h.
size_t decode_exchange_words(int E, int k, int I);
// x == nullptr: activation pointers from ws.io; otherwise direct pointers, and norm_eps >= 0
// normalises x (RMSNorm) for the layer while x stays the residual when resid == x.  Returns 0,
// or -1 when the launch was refused.
int launch_decode(const Layer& L, const Workspace& ws, int* sync, int sm_count, cudaStream_t s,
                   const float* x = nullptr, const float* resid = nullptr, float* out = nullptr,
                   float norm_eps = -1.0f);
// ysh: unweighted shared-expert rows [M][H] of a separate shared pass (weighted by the gate in
// entry 0 of each routing record, added after the ns slots of ws), or null.
void launch_combine(const Layer& L, const Workspace& ws, const IoArgs* io, int M, int ns,
                    float scale, cudaStream_t s, const float* ysh = nullptr);
// Bucketing of a shared-expert-only pass: bucket E = every token in order, tiles of it.
void launch_shared_plan(int E, int M, Workspace& ws, cudaStream_t s);
// Expert-parallel dispatch plan (arena or workspace memory): mask[M], pos[M][n_ranks],
// offsets[2 * n_ranks] (block starts, rows used per block).
constexpr int kMaxEpRanks = 8;
struct EpPlan {
    uint32_t* mask;
    int* pos;
    int* offsets;
};
// Peer-transport addresses of one rank (device pointers valid on this rank's GPU: local or CUDA
// IPC mappings of the other ranks' exchange buffers).
struct EpPeers {
    float* x[kMaxEpRanks];      // block my_rank of rank d's receive rows
    uint2* rec[kMaxEpRanks];    // block my_rank of rank d's receive records
    const float* y[kMaxEpRanks];  // block my_rank of rank d's partial-row output
    unsigned long long* flag[2][kMaxEpRanks];  // this rank's slot in rank d's flags (dispatch, outputs)
};
void launch_ep_push(const float* x, const uint2* topk, EpPlan plan, int M, int H, int k, int epr, int n_ranks,
                    int my_rank, int capacity, const EpPeers& P, cudaStream_t s);
void launch_ep_signal(unsigned long long* epoch, bool bump, int n_ranks, const EpPeers& P, int slot,
                      cudaStream_t s);
void launch_ep_wait(const unsigned long long* flags, const unsigned long long* epoch, int n_ranks, int* status,
                    cudaStream_t s);
void launch_ep_pull_combine(EpPlan plan, int M, int n_ranks, int H, const EpPeers& P, const float* resid,
                            float scale, float* out, cudaStream_t s);
void launch_ep_plan(const uint2* topk, int M, int k, int epr, int n_ranks, int my_rank, int capacity,
                    EpPlan plan, int* status, cudaStream_t s);
void launch_ep_gather(const float* x, const uint2* topk, EpPlan plan, int M, int H, int k, int epr,
                      int n_ranks, int my_rank, float* send_x, uint2* send_rec, cudaStream_t s);
void launch_ep_combine(EpPlan plan, int M, int n_ranks, int H, const float* y_back, const float* resid,
                       float scale, float* out, cudaStream_t s);
void launch_rms_norm(const float* x, float* y, int M, int H, float eps, cudaStream_t s);
void launch_silu_mul(const float* g, const float* u, float* y, uint64_t n, int sm_count, cudaStream_t s);
void launch_dequant(const uint8_t* src, uint64_t n_blocks, float* dst, cudaStream_t s);
void launch_dequant_ref36(const uint8_t* src, uint64_t n_blocks, float* dst, cudaStream_t s);
// Expert products on the reference's 36-byte block format (MOE_F_REF36 layers): writes ws.h
// and ws.ypart like the GEMV path; scratch holds ref36_scratch_bytes(S, H, I).
bool ref36_supported(int H, int I);
size_t ref36_scratch_bytes(int S, int H, int I);
void launch_ref36_experts(const Layer& L, const Workspace& ws, int M, int slots, int max_chunks, float* scratch,
                          cudaStream_t s);
bool vocab_supported(int H, int M);
// Returns -1 when the shape does not fit the kernel's shared memory (nothing launched).
int launch_vocab(const uint8_t* w, int V, int H, const float* x, int M, float* logits, uint32_t* ids,
                 unsigned long long* keys, unsigned int* ticket, int* status, int sm_count,
                 cudaStream_t s);
void launch_synth(uint8_t* dst, uint64_t key, uint64_t block_start, uint64_t n_blocks,
                  cudaStream_t s);

// Upper bound on the chunk count: every non-empty bucket adds at most one partial chunk, and
// every chunk holds at least one slot.
inline int max_tiles_for(int M, int slots, int E, int nmax) {
    const int S = M * slots;
    const int nonempty = S < E + 1 ? S : E + 1;
    const int bound = (S + nmax - 1) / nmax + nonempty;
    return bound < S ? bound : S;
}

inline int max_chunks_for(int M, int slots, int E) {
    const int S = M * slots;
    const int nonempty = S < E + 1 ? S : E + 1;
    const int bound = (S + kGemvTok - 1) / kGemvTok + nonempty;
    return bound < S ? bound : S;
}

}  // namespace moe
