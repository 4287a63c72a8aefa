// C ABI entry points (include/moe_b200.h): context, arena, layers, routing, bucketing and the
// MoE layer forward.  Host-side validation happens here, before any launch: offsets must be
// non-zero (offset 0 is the reference's "missing tensor" sentinel, src/memory.rs:33,234),
// aligned and inside the arena; shapes must be ones the kernels support.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "moe_common.cuh"
#include "moe_internal.h"

using moe::Ctx;
using moe::Layer;
using moe::Workspace;

struct moe_ctx : public Ctx {};

namespace {

thread_local std::string g_create_error;

int fail(Ctx* c, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (c) c->err = buf; else g_create_error = buf;
    return code;
}

int cuda_fail(Ctx* c, cudaError_t e, const char* what) {
    return fail(c, MOE_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define MOE_CUDA(c, call)                                   \
    do {                                                    \
        cudaError_t e_ = (call);                            \
        if (e_ != cudaSuccess) return cuda_fail(c, e_, #call); \
    } while (0)

bool off_ok(const Ctx* c, uint64_t off, uint64_t bytes, uint64_t align) {
    if (off == 0 || off % align != 0) return false;
    if (off > c->bytes || bytes > c->bytes - off) return false;
    return true;
}

template <typename T>
T* at(const Ctx* c, uint64_t off) {
    return reinterpret_cast<T*>(c->base + off);
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

void free_ws(Workspace& ws) {
    if (ws.base) cudaFree(ws.base);
    ws = Workspace{};
}

// Grow the workspace to hold a forward of M tokens for (E, k, slots, H, I).
int ensure_ws_of(Ctx* c, Workspace& ws, uint32_t M, uint32_t E, uint32_t k, uint32_t slots, uint32_t H,
                 uint32_t I) {
    if (ws.base && M <= ws.cap_tokens && E <= ws.cap_experts && slots <= ws.cap_slots &&
        H <= ws.cap_hidden && I <= ws.cap_inter)
        return MOE_OK;
    M = std::max(M, ws.cap_tokens);
    E = std::max(E, ws.cap_experts);
    slots = std::max(std::max(slots, k + 1), ws.cap_slots);
    H = std::max(H, ws.cap_hidden);
    I = std::max(I, ws.cap_inter);
    const size_t S = static_cast<size_t>(M) * slots;
    const int tiles = (M + 255) / 256;
    const int max_chunks = moe::max_chunks_for(M, slots, E);
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off = align_up(off + bytes, 256); return o; };
    const size_t o_logits = take(sizeof(float) * 16 * M * (E + 1));  // up to 16 K splits
    const size_t o_topk = take(sizeof(uint2) * M * (slots + 1));
    const size_t o_tile = take(sizeof(int) * tiles * (E + 1));
    const size_t o_ranges = take(sizeof(int) * (E + 2));
    const size_t o_stok = take(sizeof(int) * S);
    const size_t o_sw = take(sizeof(float) * S);
    const size_t o_pos = take(sizeof(int) * M * slots);
    const size_t o_chunks = take(sizeof(moe::Chunk) * max_chunks);
    const size_t o_cnt = take(sizeof(int) * 8);
    const size_t o_h = take(sizeof(float) * S * 2 * I);
    const size_t o_y = take(sizeof(float) * S * H);
    const int max13 = moe::max_tiles_for(M, slots, E, moe::tc_max_n(13));
    const int max2 = moe::max_tiles_for(M, slots, E, moe::tc_max_n(2));
    const size_t o_t13 = take(sizeof(moe::TcTile) * max13);
    const size_t o_t2 = take(sizeof(moe::TcTile) * max2);
    const size_t o_x16 = take(sizeof(__half) * S * H);
    const size_t o_h16 = take(sizeof(__half) * S * I);
    const size_t o_xe = take(sizeof(int) * S);
    const size_t o_he = take(sizeof(int) * S);
    const size_t o_io = take(sizeof(moe::IoArgs));
    const size_t o_xh = take(sizeof(float) * M * H);
    const size_t o_xl = take(sizeof(float) * M * H);
    const size_t o_xn = take(sizeof(float) * M * H);
    const size_t dx_bytes = sizeof(unsigned long long) * moe::decode_exchange_words(E, slots - 1, I);
    const size_t o_dx = take(dx_bytes);
    const size_t total = off;
    int* status = ws.status;
    ws.status = nullptr;
    cudaStreamSynchronize(c->stream);
    free_ws(ws);
    c->ws_gen += 1;  // captured graphs refer to the old buffers
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, total);
    if (e != cudaSuccess) {
        cudaGetLastError();
        ws.status = status;
        return fail(c, MOE_E_OOM, "workspace of %zu bytes for %u tokens: %s", total, M,
                    cudaGetErrorString(e));
    }
    uint8_t* b = static_cast<uint8_t*>(p);
    ws.base = b;
    ws.bytes = total;
    ws.cap_tokens = M; ws.cap_experts = E; ws.cap_slots = slots; ws.cap_hidden = H; ws.cap_inter = I;
    ws.logits = reinterpret_cast<float*>(b + o_logits);
    ws.topk = reinterpret_cast<uint2*>(b + o_topk);
    ws.tilecnt = reinterpret_cast<int*>(b + o_tile);
    ws.ranges = reinterpret_cast<int*>(b + o_ranges);
    ws.sorted_tok = reinterpret_cast<int*>(b + o_stok);
    ws.sorted_w = reinterpret_cast<float*>(b + o_sw);
    ws.slot_pos = reinterpret_cast<int*>(b + o_pos);
    ws.chunks = reinterpret_cast<moe::Chunk*>(b + o_chunks);
    ws.counters = reinterpret_cast<int*>(b + o_cnt);
    ws.h = reinterpret_cast<float*>(b + o_h);
    ws.ypart = reinterpret_cast<float*>(b + o_y);
    ws.tiles13 = reinterpret_cast<moe::TcTile*>(b + o_t13);
    ws.tiles2 = reinterpret_cast<moe::TcTile*>(b + o_t2);
    ws.max_tiles13 = static_cast<uint32_t>(max13);
    ws.max_tiles2 = static_cast<uint32_t>(max2);
    ws.x16 = reinterpret_cast<__half*>(b + o_x16);
    ws.h16 = reinterpret_cast<__half*>(b + o_h16);
    ws.xexp = reinterpret_cast<int*>(b + o_xe);
    ws.hexp = reinterpret_cast<int*>(b + o_he);
    ws.io = reinterpret_cast<moe::IoArgs*>(b + o_io);
    ws.xh = reinterpret_cast<float*>(b + o_xh);
    ws.xl = reinterpret_cast<float*>(b + o_xl);
    ws.xn = reinterpret_cast<float*>(b + o_xn);
    ws.dx = reinterpret_cast<unsigned long long*>(b + o_dx);
    ws.dx_bytes = dx_bytes;
    // no stale epoch may match a later launch: the exchange entries start at zero (epoch 0 is
    // never used)
    e = cudaMemset(b + o_dx, 0, dx_bytes);
    if (e != cudaSuccess) return cuda_fail(c, e, "workspace exchange clear");
    ws.max_chunks = static_cast<uint32_t>(max_chunks);
    ws.status = status;
    return MOE_OK;
}

int ensure_ws(Ctx* c, uint32_t M, uint32_t E, uint32_t k, uint32_t slots, uint32_t H, uint32_t I) {
    return ensure_ws_of(c, c->ws, M, E, k, slots, H, I);
}

bool use_shared_split(const Ctx* c, const Layer& L, uint32_t M);

int ensure_layer_ws(Ctx* c, const Layer& L, uint32_t M) {
    int rc = ensure_ws(c, M, L.spec.n_experts, L.spec.top_k, static_cast<uint32_t>(L.slots()),
                       L.spec.hidden, L.spec.inter);
    if (rc) return rc;
    if (use_shared_split(c, L, M)) {
        c->ws_sh.status = c->ws.status;
        if ((rc = ensure_ws_of(c, c->ws_sh, M, L.spec.n_experts, 0, 1, L.spec.hidden, L.spec.inter))) return rc;
        if (!c->side_stream) {
            MOE_CUDA(c, cudaStreamCreateWithFlags(&c->side_stream, cudaStreamNonBlocking));
            MOE_CUDA(c, cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming));
            MOE_CUDA(c, cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming));
        }
    }
    if (!L.ref36()) return MOE_OK;
    // the reference-format path's K-split partial sums, grown like the workspace
    const size_t need = moe::ref36_scratch_bytes(static_cast<int>(c->ws.cap_tokens * c->ws.cap_slots),
                                                 static_cast<int>(c->ws.cap_hidden), static_cast<int>(c->ws.cap_inter));
    if (need <= c->ref36_scratch_bytes) return MOE_OK;
    cudaStreamSynchronize(c->stream);
    if (c->ref36_scratch) cudaFree(c->ref36_scratch);
    c->ref36_scratch = nullptr;
    c->ref36_scratch_bytes = 0;
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, need);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(c, MOE_E_OOM, "reference-format scratch of %zu bytes: %s", need, cudaGetErrorString(e));
    }
    c->ref36_scratch = static_cast<float*>(p);
    c->ref36_scratch_bytes = need;
    c->ws_gen += 1;  // captured graphs refer to the old buffer
    return MOE_OK;
}

// The decode kernel's grid-synchronisation words in the status block.
int* decode_sync(Ctx* c) {
    return reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(c->ws.status) + moe::kStatusDecodeOff);
}

struct DeviceGuard {
    explicit DeviceGuard(int dev) { cudaSetDevice(dev); }
};

int check_launch(Ctx* c, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, what);
    return MOE_OK;
}

int get_layer(Ctx* c, uint32_t id, Layer** L) {
    if (id >= c->layers.size()) return fail(c, MOE_E_INVALID, "unknown layer id %u", id);
    *L = &c->layers[id];
    return MOE_OK;
}

int check_tokens(Ctx* c, const Layer& L, uint64_t off, uint32_t M, const char* name) {
    if (!off_ok(c, off, static_cast<uint64_t>(M) * L.spec.hidden * 4, 16))
        return fail(c, MOE_E_INVALID, "%s offset %llu invalid for %u tokens", name,
                    static_cast<unsigned long long>(off), M);
    return MOE_OK;
}

// ---- tracing: one event per stage boundary of the current call --------------------------
void prof_begin(Ctx* c) {
    if (!c->prof) return;
    c->ev_names.clear();
    if (c->ev.empty()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        c->ev.push_back(e);
    }
    cudaEventRecord(c->ev[0], c->stream);
}

// Marks the end of a stage of `n_launch` kernels.
void stage(Ctx* c, const char* name, int n_launch) {
    c->launches += static_cast<uint64_t>(n_launch);
    if (!c->prof) return;
    c->ev_names.push_back(name);
    const size_t i = c->ev_names.size();
    while (c->ev.size() <= i) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        c->ev.push_back(e);
    }
    cudaEventRecord(c->ev[i], c->stream);
}

void prof_end(Ctx* c) {
    if (!c->prof || c->ev_names.empty()) return;
    cudaEventSynchronize(c->ev[c->ev_names.size()]);
    for (size_t i = 0; i < c->ev_names.size(); ++i) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, c->ev[i], c->ev[i + 1]);
        moe::StageStat* st = nullptr;
        for (auto& s : c->stats)
            if (s.name == c->ev_names[i]) st = &s;
        if (!st) {
            c->stats.push_back(moe::StageStat{c->ev_names[i], 0, 0.0});
            st = &c->stats.back();
        }
        st->calls += 1;
        st->total_ms += ms;
    }
    c->ev_names.clear();
}

void run_set_io(Ctx* c, const float* x, const float* resid, float* out) {
    moe::launch_set_io(c->ws.io, x, resid, out, c->stream);
    stage(c, "set_io", 1);
}

int ensure_tmap(Ctx* c, moe::BMaps* m, const void** base, uint64_t* rows, uint64_t* cols,
                const void* p, uint64_t r, uint64_t cl);

// Routing of M tokens (activations from ws.io) into ws.topk: tensor-core router (3xTF32) for
// batches above 8 tokens when the layer supports it, CUDA-core f32 otherwise.
int run_route(Ctx* c, const Layer& L, uint32_t M) {
    Workspace& ws = c->ws;
    const int E = static_cast<int>(L.spec.n_experts), H = static_cast<int>(L.spec.hidden);
    if (M > 8 && L.wsplit) {
        if (ws.xh_base != ws.xh || ws.xh_rows != M || ws.xh_cols != static_cast<uint64_t>(H)) {
            if (!moe::make_f32_tmap(&ws.xhmap, ws.xh, M, H, 256) || !moe::make_f32_tmap(&ws.xlmap, ws.xl, M, H, 256))
                return fail(c, MOE_E_CUDA, "cuTensorMapEncodeTiled failed for the router operands");
            ws.xh_base = ws.xh; ws.xh_rows = M; ws.xh_cols = static_cast<uint64_t>(H);
        }
        // the split kernel also computes the shared gate logit (column E of the logit planes)
        const bool gate = (L.spec.flags & MOE_F_SHARED_GATE) != 0 && L.gate_ptr;
        const int n_split = moe::router_tc_split(static_cast<int>(M), E, H);
        moe::launch_split_x(ws.io, static_cast<int>(M), H, ws.xh, ws.xl,
                            gate ? reinterpret_cast<const float*>(L.gate_ptr) : nullptr, ws.logits, n_split, E,
                            c->stream);
        stage(c, "router_split", 1);
        moe::launch_router_tc(L, ws.xhmap, ws.xlmap, static_cast<int>(M), ws.logits, ws.status, c->stream);
        stage(c, "router", 1);
        moe::launch_topk(L, ws.logits, n_split, gate, ws.io, static_cast<int>(M), ws.topk, ws.status, c->stream);
    } else {
        moe::launch_router_logits(L, ws.io, static_cast<int>(M), ws.logits, c->stream);
        stage(c, "router", 1);
        moe::launch_topk(L, ws.logits, moe::router_split_for(static_cast<int>(M), H), true, ws.io,
                         static_cast<int>(M), ws.topk, ws.status, c->stream);
    }
    stage(c, "topk", 1);
    return check_launch(c, "router");
}

// Expert path for a batch of M tokens: CUDA-core grouped GEMV for decode-sized batches,
// tcgen05 grouped GEMM otherwise (or as forced by moe_set_path).
int choose_path(const Ctx* c, const Layer& L, uint32_t M) {
    if (c->path != moe::kPathAuto) return c->path;
    return (M <= 8 || !L.wmaps) ? moe::kPathGemv : moe::kPathTcTmemA;
}

// Batches of at least kSplitMinTokens on the tensor-core path run the shared expert as a separate
// pass on a second stream, concurrently with the router, top-k and bucketing (it needs no
// routing); the combine adds its rows after the routed slots, in the order of a single pass, so
// the result is bit-identical.  MOE_B200_SHARED_SPLIT=0 keeps the single pass.
constexpr uint32_t kSplitMinTokens = 64;

bool use_shared_split(const Ctx* c, const Layer& L, uint32_t M) {
    static const bool enabled = [] {
        const char* e = std::getenv("MOE_B200_SHARED_SPLIT");
        return !(e && e[0] == '0');
    }();
    return enabled && M >= kSplitMinTokens && L.has_shared() && L.wmaps && choose_path(c, L, M) != moe::kPathGemv;
}

int ensure_tmap(Ctx* c, moe::BMaps* m, const void** base, uint64_t* rows, uint64_t* cols,
                const void* p, uint64_t r, uint64_t cl) {
    if (*base == p && *rows == r && *cols == cl) return MOE_OK;
    if (!moe::make_fp16_tmaps(m, p, r, cl))
        return fail(c, MOE_E_CUDA, "cuTensorMapEncodeTiled failed (rows %llu, cols %llu)",
                    static_cast<unsigned long long>(r), static_cast<unsigned long long>(cl));
    *base = p; *rows = r; *cols = cl;
    return MOE_OK;
}

// The shared expert over all M tokens on the side stream with its own workspace: unweighted rows
// in ws_sh.ypart [M][H].  Forked from the context's stream after set_io; joined before the
// combine (run_experts with split).
int fork_shared_pass(Ctx* c, const Layer& L, uint32_t M) {
    Workspace& w = c->ws_sh;
    const int E = static_cast<int>(L.spec.n_experts), H = static_cast<int>(L.spec.hidden);
    const int I = static_cast<int>(L.spec.inter);
    cudaStream_t s = c->side_stream;
    int rc = ensure_tmap(c, &w.xmap, &w.xmap_base, &w.xmap_rows, &w.xmap_cols, w.x16, M, H);
    if (rc) return rc;
    rc = ensure_tmap(c, &w.hmap, &w.hmap_base, &w.hmap_rows, &w.hmap_cols, w.h16, M, I);
    if (rc) return rc;
    MOE_CUDA(c, cudaEventRecord(c->ev_fork, c->stream));
    MOE_CUDA(c, cudaStreamWaitEvent(s, c->ev_fork, 0));
    moe::launch_shared_plan(E, static_cast<int>(M), w, s);
    moe::launch_convert_x(c->ws.io, w.slot_pos, static_cast<int>(M), 1, H, w.x16, w.xexp, s);
    const int tiles13 = (static_cast<int>(M) + moe::tc_max_n(13) - 1) / moe::tc_max_n(13);
    const int tiles2 = (static_cast<int>(M) + moe::tc_max_n(2) - 1) / moe::tc_max_n(2);
    const bool a_tmem = choose_path(c, L, M) == moe::kPathTcTmemA;
    moe::launch_tc13(L, w.xmap, w, tiles13 * (2 * I / 128), c->sm_count, a_tmem, s);
    moe::launch_convert_h(w.h, static_cast<int>(M), w.ranges + E + 1, I, w.h16, w.hexp, s);
    moe::launch_tc2(L, w.hmap, w, tiles2 * (H / 128), c->sm_count, a_tmem, s);
    c->launches += 5;
    MOE_CUDA(c, cudaEventRecord(c->ev_join, s));
    return check_launch(c, "shared pass");
}

// routed: use the routed entries of the records; shared: add the shared expert's slot; scale:
// the combine scale (the layer's, or 1 for expert-parallel partial rows); split: the shared
// expert's rows come from fork_shared_pass instead of a slot.
int run_experts(Ctx* c, const Layer& L, uint32_t M, bool routed, bool shared, float scale, bool split = false) {
    Workspace& ws = c->ws;
    if (split) shared = false;
    const int slots = static_cast<int>(L.spec.top_k) + (shared ? 1 : 0);
    const int E = static_cast<int>(L.spec.n_experts);
    moe::launch_bucket(E, static_cast<int>(L.spec.top_k), routed, shared, ws.topk,
                       static_cast<int>(M), ws, ws.ranges, ws.sorted_tok, ws.sorted_w,
                       ws.slot_pos, ws.status, c->stream);
    stage(c, "bucket", 3);
    const int path = choose_path(c, L, M);
    if (path != moe::kPathGemv && !L.wmaps)
        return fail(c, MOE_E_UNSUPPORTED, "tensor-core path needs hidden and inter multiples of 512");
    if (path == moe::kPathGemv && L.ref36()) {
        const int max_chunks = moe::max_chunks_for(static_cast<int>(M), slots, E);
        moe::launch_ref36_experts(L, ws, static_cast<int>(M), slots, max_chunks, c->ref36_scratch, c->stream);
        stage(c, "ref36", 4);
    } else if (path == moe::kPathGemv) {
        const int max_chunks = moe::max_chunks_for(static_cast<int>(M), slots, E);
        moe::launch_gemv13(L, ws.io, ws, static_cast<int>(M), max_chunks, c->sm_count, c->stream);
        stage(c, "gemv13", 1);
        moe::launch_gemv2(L, ws, static_cast<int>(M), max_chunks, c->sm_count, c->stream);
        stage(c, "gemv2", 1);
    } else {
        const bool a_tmem = path == moe::kPathTcTmemA;
        const uint64_t S = static_cast<uint64_t>(M) * slots;
        const int H = static_cast<int>(L.spec.hidden), I = static_cast<int>(L.spec.inter);
        int rc = ensure_tmap(c, &ws.xmap, &ws.xmap_base, &ws.xmap_rows, &ws.xmap_cols, ws.x16, S, H);
        if (rc) return rc;
        rc = ensure_tmap(c, &ws.hmap, &ws.hmap_base, &ws.hmap_rows, &ws.hmap_cols, ws.h16, S, I);
        if (rc) return rc;
        moe::launch_convert_x(ws.io, ws.slot_pos, static_cast<int>(M), slots, H, ws.x16, ws.xexp, c->stream);
        stage(c, "convert_x", 1);
        const int items13 = moe::max_tiles_for(static_cast<int>(M), slots, E, moe::tc_max_n(13)) * (2 * I / 128);
        moe::launch_tc13(L, ws.xmap, ws, items13, c->sm_count, a_tmem, c->stream);
        stage(c, "tc13", 1);
        moe::launch_convert_h(ws.h, static_cast<int>(S), ws.ranges + E + 1, I, ws.h16, ws.hexp, c->stream);
        stage(c, "convert_h", 1);
        const int items2 = moe::max_tiles_for(static_cast<int>(M), slots, E, moe::tc_max_n(2)) * (H / 128);
        moe::launch_tc2(L, ws.hmap, ws, items2, c->sm_count, a_tmem, c->stream);
        stage(c, "tc2", 1);
    }
    if (split) MOE_CUDA(c, cudaStreamWaitEvent(c->stream, c->ev_join, 0));
    moe::launch_combine(L, ws, ws.io, static_cast<int>(M), slots, scale, c->stream,
                        split ? c->ws_sh.ypart : nullptr);
    stage(c, "combine", 1);
    return check_launch(c, "experts");
}

// ---- CUDA graphs of moe_forward ------------------------------------------------------------
constexpr size_t kMaxGraphs = 64;

void destroy_graph(moe::GraphEntry& g) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    if (g.graph) cudaGraphDestroy(g.graph);
    g.exec = nullptr;
    g.graph = nullptr;
}

bool use_decode(const Ctx* c, const Layer& L, uint32_t M) {
    return M == 1 && (c->path == moe::kPathAuto || c->path == moe::kPathGemv) && moe::decode_supported(L, c->sm_count);
}

int record_forward(Ctx* c, const Layer& L, uint32_t M, const float* x, const float* resid, float* out) {
    if (use_decode(c, L, M)) {
        // single token: the whole layer in one fused launch with direct pointers (no graph or
        // pointer block needed); its launch counter lives after the status word
        if (moe::launch_decode(L, c->ws, decode_sync(c), c->sm_count, c->stream, x, resid, out, -1.0f))
            return check_launch(c, "decode (cooperative launch refused)");
        stage(c, "decode", 1);
        return check_launch(c, "decode");
    }
    run_set_io(c, x, resid, out);
    const bool split = use_shared_split(c, L, M) && c->ws_sh.cap_tokens >= M && c->side_stream;
    int rc = split ? fork_shared_pass(c, L, M) : MOE_OK;
    if (rc) return rc;
    rc = run_route(c, L, M);
    if (rc) return rc;
    return run_experts(c, L, M, true, L.has_shared(), L.spec.scale, split);
}

// Replay (capturing on first use) the forward of (layer, M, path) with new activation pointers:
// only the set_io node's arguments change between replays.
int graph_forward(Ctx* c, uint32_t layer, const Layer& L, uint32_t M, const float* x,
                  const float* resid, float* out) {
    const int path = choose_path(c, L, M);
    moe::GraphEntry* e = nullptr;
    for (auto& g : c->graphs)
        if (g.layer == layer && g.M == M && g.path == path && g.stream == c->stream && g.ws_gen == c->ws_gen)
            e = &g;
    if (!e) {
        // drop stale entries, then the least recently used one if the cache is full
        for (size_t i = 0; i < c->graphs.size();) {
            if (c->graphs[i].ws_gen != c->ws_gen) {
                destroy_graph(c->graphs[i]);
                c->graphs.erase(c->graphs.begin() + static_cast<long>(i));
            } else {
                ++i;
            }
        }
        if (c->graphs.size() >= kMaxGraphs) {
            size_t lru = 0;
            for (size_t i = 1; i < c->graphs.size(); ++i)
                if (c->graphs[i].last_use < c->graphs[lru].last_use) lru = i;
            destroy_graph(c->graphs[lru]);
            c->graphs.erase(c->graphs.begin() + static_cast<long>(lru));
        }
        moe::GraphEntry g;
        g.layer = layer; g.M = M; g.path = path; g.stream = c->stream; g.ws_gen = c->ws_gen;
        const uint64_t l0 = c->launches;
        MOE_CUDA(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        int rc = record_forward(c, L, M, x, resid, out);
        cudaGraph_t graph = nullptr;
        cudaError_t ce = cudaStreamEndCapture(c->stream, &graph);
        g.n_kernels = c->launches - l0;
        c->launches = l0;
        if (rc != MOE_OK) { if (graph) cudaGraphDestroy(graph); return rc; }
        if (ce != cudaSuccess) return cuda_fail(c, ce, "cudaStreamEndCapture");
        g.graph = graph;
        size_t n_root = 0;
        cudaGraphGetRootNodes(graph, nullptr, &n_root);
        if (n_root != 1) { destroy_graph(g); return fail(c, MOE_E_CUDA, "captured forward has %zu roots", n_root); }
        cudaGraphGetRootNodes(graph, &g.io_node, &n_root);
        ce = cudaGraphInstantiate(&g.exec, graph, 0);
        if (ce != cudaSuccess) { destroy_graph(g); return cuda_fail(c, ce, "cudaGraphInstantiate"); }
        c->graphs.push_back(g);
        e = &c->graphs.back();
    }
    e->last_use = ++c->graph_clock;
    moe::IoArgs* io = c->ws.io;
    void* args[4] = {&io, const_cast<float**>(&x), const_cast<float**>(&resid), &out};
    cudaKernelNodeParams p{};
    p.func = const_cast<void*>(moe::set_io_func());
    p.gridDim = dim3(1);
    p.blockDim = dim3(1);
    p.kernelParams = args;
    MOE_CUDA(c, cudaGraphExecKernelNodeSetParams(e->exec, e->io_node, &p));
    MOE_CUDA(c, cudaGraphLaunch(e->exec, c->stream));
    c->launches += e->n_kernels;
    return MOE_OK;
}

bool stream_capturing(Ctx* c) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(c->stream, &st) != cudaSuccess) return true;
    return st != cudaStreamCaptureStatusNone;
}

}  // namespace

extern "C" {

int moe_abi_version(void) { return MOE_B200_ABI_VERSION; }

static int ctx_init(int device, moe_ctx* c) {
    c->device = device;
    cudaDeviceProp prop;
    MOE_CUDA(c, cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(c, MOE_E_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a",
                    device, prop.major, prop.minor);
    c->sm_count = prop.multiProcessorCount;
    MOE_CUDA(c, cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking));
    c->stream = c->own_stream;
    const char* ng = std::getenv("MOE_B200_NO_GRAPHS");
    c->use_graphs = !(ng && ng[0] == '1');
    void* st = nullptr;
    MOE_CUDA(c, cudaMalloc(&st, moe::kStatusBlockBytes));
    MOE_CUDA(c, cudaMemset(st, 0, moe::kStatusBlockBytes));
    c->ws.status = static_cast<int*>(st);
    return MOE_OK;
}

int moe_ctx_create(int device, uint64_t arena_bytes, moe_ctx** out) {
    if (!out) return fail(nullptr, MOE_E_INVALID, "out is NULL");
    *out = nullptr;
    if (arena_bytes < 256) return fail(nullptr, MOE_E_INVALID, "arena too small");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || device < 0 || device >= n)
        return fail(nullptr, MOE_E_CUDA, "no CUDA device %d (%s)", device,
                    e == cudaSuccess ? "out of range" : cudaGetErrorString(e));
    cudaSetDevice(device);
    moe_ctx* c = new moe_ctx();
    int rc = ctx_init(device, c);
    if (rc != MOE_OK) { g_create_error = c->err; moe_ctx_destroy(c); return rc; }
    void* p = nullptr;
    e = cudaMalloc(&p, arena_bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(nullptr, MOE_E_OOM, "arena of %llu bytes: %s",
             static_cast<unsigned long long>(arena_bytes), cudaGetErrorString(e));
        moe_ctx_destroy(c);
        return MOE_E_OOM;
    }
    c->base = static_cast<uint8_t*>(p);
    c->bytes = arena_bytes;
    c->owns = true;
    *out = c;
    return MOE_OK;
}

int moe_ctx_create_external(int device, void* base, uint64_t bytes, moe_ctx** out) {
    if (!out || !base) return fail(nullptr, MOE_E_INVALID, "out/base is NULL");
    *out = nullptr;
    if (reinterpret_cast<uintptr_t>(base) % 256 != 0)
        return fail(nullptr, MOE_E_INVALID, "external arena must be 256-byte aligned");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || device < 0 || device >= n)
        return fail(nullptr, MOE_E_CUDA, "no CUDA device %d", device);
    cudaSetDevice(device);
    moe_ctx* c = new moe_ctx();
    int rc = ctx_init(device, c);
    if (rc != MOE_OK) { g_create_error = c->err; moe_ctx_destroy(c); return rc; }
    c->base = static_cast<uint8_t*>(base);
    c->bytes = bytes;
    c->owns = false;
    *out = c;
    return MOE_OK;
}

static void ep_release(Ctx* c);

void moe_ctx_destroy(moe_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto& L : c->layers) {
        if (L.tab) cudaFree(const_cast<uint8_t**>(L.tab));
        if (L.wmaps) cudaFree(L.wmaps);
        if (L.wsplit) cudaFree(L.wsplit);
    }
    for (auto& g : c->graphs) destroy_graph(g);
    ep_release(c);
    int* status = c->ws.status;
    free_ws(c->ws);
    if (status) cudaFree(status);
    if (c->ref36_scratch) cudaFree(c->ref36_scratch);
    c->ws_sh.status = nullptr;
    free_ws(c->ws_sh);
    if (c->h2d_stream) cudaStreamSynchronize(c->h2d_stream);
    if (c->d2h_stream) cudaStreamSynchronize(c->d2h_stream);
    for (int b = 0; b < Ctx::kHostSlots; ++b) {
        if (c->host_stage[b]) cudaFree(c->host_stage[b]);
        for (cudaEvent_t e : {c->ev_in[b], c->ev_done[b], c->ev_out[b]})
            if (e) cudaEventDestroy(e);
    }
    if (c->h2d_stream) cudaStreamDestroy(c->h2d_stream);
    if (c->d2h_stream) cudaStreamDestroy(c->d2h_stream);
    if (c->ev_fork) cudaEventDestroy(c->ev_fork);
    if (c->ev_join) cudaEventDestroy(c->ev_join);
    if (c->side_stream) cudaStreamDestroy(c->side_stream);
    if (c->owns && c->base) cudaFree(c->base);
    for (cudaEvent_t e : c->ev) cudaEventDestroy(e);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
}

int moe_last_error(const moe_ctx* c, char* buf, size_t n) {
    if (!buf || n == 0) return MOE_E_INVALID;
    const std::string& s = c ? c->err : g_create_error;
    std::snprintf(buf, n, "%s", s.c_str());
    return MOE_OK;
}

int moe_arena_upload(moe_ctx* c, uint64_t off, const void* host, uint64_t n) {
    if (!c || !host) return fail(c, MOE_E_INVALID, "NULL argument");
    if (n == 0) return MOE_OK;
    if (!off_ok(c, off, n, 1)) return fail(c, MOE_E_INVALID, "upload [%llu, +%llu) outside arena",
                                          (unsigned long long)off, (unsigned long long)n);
    DeviceGuard g(c->device);
    MOE_CUDA(c, cudaMemcpyAsync(c->base + off, host, n, cudaMemcpyHostToDevice, c->stream));
    return MOE_OK;
}

int moe_arena_download(moe_ctx* c, uint64_t off, void* host, uint64_t n) {
    if (!c || !host) return fail(c, MOE_E_INVALID, "NULL argument");
    if (n == 0) return MOE_OK;
    if (!off_ok(c, off, n, 1)) return fail(c, MOE_E_INVALID, "download [%llu, +%llu) outside arena",
                                          (unsigned long long)off, (unsigned long long)n);
    DeviceGuard g(c->device);
    MOE_CUDA(c, cudaMemcpyAsync(host, c->base + off, n, cudaMemcpyDeviceToHost, c->stream));
    MOE_CUDA(c, cudaStreamSynchronize(c->stream));
    return MOE_OK;
}

int moe_arena_ptr(moe_ctx* c, uint64_t off, void** dptr) {
    if (!c || !dptr) return fail(c, MOE_E_INVALID, "NULL argument");
    if (off >= c->bytes) return fail(c, MOE_E_INVALID, "offset outside arena");
    *dptr = c->base + off;
    return MOE_OK;
}

int moe_set_stream(moe_ctx* c, void* stream) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
    return MOE_OK;
}

int moe_sync(moe_ctx* c) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    DeviceGuard g(c->device);
    MOE_CUDA(c, cudaStreamSynchronize(c->stream));
    if (c->h2d_stream) MOE_CUDA(c, cudaStreamSynchronize(c->h2d_stream));
    if (c->d2h_stream) MOE_CUDA(c, cudaStreamSynchronize(c->d2h_stream));
    int st = 0;
    MOE_CUDA(c, cudaMemcpy(&st, c->ws.status, sizeof(int), cudaMemcpyDeviceToHost));
    if (st != 0) {
        cudaMemset(c->ws.status, 0, sizeof(int));
        // the decode kernel's grid counter and h maxima, the vocabulary argmax ticket and keys
        cudaMemset(decode_sync(c), 0, moe::kStatusKernelEnd - moe::kStatusDecodeOff);
        if (c->ws.dx) cudaMemset(c->ws.dx, 0, c->ws.dx_bytes);  // stale epochs go with the counter
        const char* what = st == moe::kDevBadExpert ? "expert id out of range"
                         : st == moe::kDevBadToken ? "token index out of range"
                         : st == moe::kDevOverflow ? "chunk list overflow"
                         : st == moe::kDevTimeout ? "wait timed out" : "device error";
        return fail(c, MOE_E_DEVICE, "kernel reported status %d (%s)", st, what);
    }
    return MOE_OK;
}

int moe_layer_create(moe_ctx* c, const moe_layer_spec* spec, const uint64_t* w1,
                     const uint64_t* w3, const uint64_t* w2, uint32_t* layer_id) {
    if (!c || !spec || !w1 || !w3 || !w2 || !layer_id) return fail(c, MOE_E_INVALID, "NULL argument");
    const moe_layer_spec& s = *spec;
    if (s.hidden == 0 || s.hidden % 256 != 0 || s.hidden > 16384)
        return fail(c, MOE_E_UNSUPPORTED, "hidden %u: must be a multiple of 256, <= 16384", s.hidden);
    if (s.inter != 256 && s.inter != 512 && s.inter != 1024)
        return fail(c, MOE_E_UNSUPPORTED, "inter %u: supported 256, 512, 1024", s.inter);
    if (s.n_experts == 0 || s.n_experts > moe::kMaxExperts)
        return fail(c, MOE_E_UNSUPPORTED, "n_experts %u: supported 1..256", s.n_experts);
    if (s.top_k == 0 || s.top_k > moe::kMaxTopK || s.top_k > s.n_experts)
        return fail(c, MOE_E_UNSUPPORTED, "top_k %u: supported 1..min(8, n_experts)", s.top_k);
    if ((s.flags & MOE_F_SHARED_GATE) && !(s.flags & MOE_F_SHARED))
        return fail(c, MOE_E_INVALID, "MOE_F_SHARED_GATE needs MOE_F_SHARED");
    const uint64_t H = s.hidden, I = s.inter, E = s.n_experts;
    if (!off_ok(c, s.router_w, E * H * 4, 16)) return fail(c, MOE_E_INVALID, "router_w offset invalid");
    if (s.router_bias && !off_ok(c, s.router_bias, E * 4, 4))
        return fail(c, MOE_E_INVALID, "router_bias offset invalid");
    if (s.flags & MOE_F_SHARED_GATE) {
        if (!off_ok(c, s.shared_gate, H * 4, 16)) return fail(c, MOE_E_INVALID, "shared_gate offset invalid");
    }
    const bool ref36 = (s.flags & MOE_F_REF36) != 0;
    if (ref36 && !moe::ref36_supported(static_cast<int>(H), static_cast<int>(I)))
        return fail(c, MOE_E_UNSUPPORTED, "MOE_F_REF36 needs hidden and inter multiples of 512");
    // GGUF IQ4_XS rows of 136-byte blocks, or the reference's 36-byte blocks of 32 weights
    const uint64_t b13 = ref36 ? H * I / 32 * 36 : I * (H / 256) * 136;
    const uint64_t b2 = ref36 ? H * I / 32 * 36 : H * (I / 256) * 136;
    std::vector<const uint8_t*> tab(3 * (E + 1), nullptr);
    const bool subset = (s.flags & MOE_F_EXPERT_SUBSET) != 0;
    for (uint64_t e = 0; e < E; ++e) {
        if (subset && w1[e] == 0 && w3[e] == 0 && w2[e] == 0) continue;  // held by another rank
        if (!off_ok(c, w1[e], b13, 256) || !off_ok(c, w3[e], b13, 256) || !off_ok(c, w2[e], b2, 256))
            return fail(c, MOE_E_INVALID, "expert %llu: weight offset missing, misaligned or outside arena",
                        static_cast<unsigned long long>(e));
        tab[e] = c->base + w1[e];
        tab[(E + 1) + e] = c->base + w3[e];
        tab[2 * (E + 1) + e] = c->base + w2[e];
    }
    if (s.flags & MOE_F_SHARED) {
        if (!off_ok(c, s.shared_w1, b13, 256) || !off_ok(c, s.shared_w3, b13, 256) ||
            !off_ok(c, s.shared_w2, b2, 256))
            return fail(c, MOE_E_INVALID, "shared expert weight offset missing, misaligned or outside arena");
        tab[E] = c->base + s.shared_w1;
        tab[(E + 1) + E] = c->base + s.shared_w3;
        tab[2 * (E + 1) + E] = c->base + s.shared_w2;
    }
    DeviceGuard g(c->device);
    void* d = nullptr;
    MOE_CUDA(c, cudaMalloc(&d, tab.size() * sizeof(void*)));
    MOE_CUDA(c, cudaMemcpy(d, tab.data(), tab.size() * sizeof(void*), cudaMemcpyHostToDevice));
    Layer L;
    L.spec = s;
    L.tab = static_cast<const uint8_t**>(d);
    L.host_tab = tab;
    L.tab_aligned16 = true;
    for (const uint8_t* q : tab)
        if (q && reinterpret_cast<uintptr_t>(q) % 16 != 0) L.tab_aligned16 = false;
    if (H % 32 == 0) {
        // router weight split for the tensor-core router: [Wh | Wl], each [E][H] f32
        void* wsd = nullptr;
        MOE_CUDA(c, cudaMalloc(&wsd, 2 * E * H * sizeof(float)));
        float* whp = static_cast<float*>(wsd);
        moe::launch_split_tf32(reinterpret_cast<const float*>(c->base + s.router_w), E * H, whp,
                               whp + E * H, c->stream);
        MOE_CUDA(c, cudaStreamSynchronize(c->stream));
        if (moe::make_f32_tmap(&L.rmaps[0], whp, E, H, 128) && moe::make_f32_tmap(&L.rmaps[1], whp + E * H, E, H, 128))
            L.wsplit = whp;
        else
            cudaFree(wsd);
    }
    if (!ref36 && moe::tc_supported(static_cast<int>(H), static_cast<int>(I))) {
        // raw IQ4_XS tensor maps for the tensor-core path: [W1 | W3 | W2][E+1]
        std::vector<CUtensorMap> maps(3 * (E + 1));
        bool ok = true;
        const uint64_t nb = E + 1;
        // absent entries (no shared expert, experts held by other ranks) repeat the maps of a
        // present expert; they are never used
        uint64_t first = E + 1;
        for (uint64_t e = 0; e <= E && first > E; ++e)
            if (tab[e]) first = e;
        ok = first <= E;
        for (uint64_t e = 0; e <= E && ok; ++e) {
            if (!tab[e]) continue;
            ok = moe::make_iq4_tmap(&maps[e], tab[e], I, b13 / I) &&
                 moe::make_iq4_tmap(&maps[nb + e], tab[nb + e], I, b13 / I) &&
                 moe::make_iq4_tmap(&maps[2 * nb + e], tab[2 * nb + e], H, b2 / H);
        }
        for (uint64_t e = 0; e <= E && ok; ++e) {
            if (tab[e]) continue;
            maps[e] = maps[first]; maps[nb + e] = maps[nb + first]; maps[2 * nb + e] = maps[2 * nb + first];
        }
        if (ok) {
            void* dm = nullptr;
            MOE_CUDA(c, cudaMalloc(&dm, maps.size() * sizeof(CUtensorMap)));
            MOE_CUDA(c, cudaMemcpy(dm, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
            L.wmaps = static_cast<CUtensorMap*>(dm);
        }
    }
    L.router_w_ptr = c->base + s.router_w;
    L.bias_ptr = s.router_bias ? c->base + s.router_bias : nullptr;
    L.gate_ptr = (s.flags & MOE_F_SHARED_GATE) ? c->base + s.shared_gate : nullptr;
    c->layers.push_back(L);
    *layer_id = static_cast<uint32_t>(c->layers.size() - 1);
    return MOE_OK;
}

int moe_reserve(moe_ctx* c, uint32_t layer_id, uint32_t max_tokens) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    DeviceGuard g(c->device);
    return ensure_layer_ws(c, *L, std::max(max_tokens, 1u));
}

int moe_route(moe_ctx* c, uint32_t layer_id, uint64_t x_off, uint32_t M, uint64_t topk_off) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    if (M == 0) return MOE_OK;
    if ((rc = check_tokens(c, *L, x_off, M, "x"))) return rc;
    const uint64_t rec = static_cast<uint64_t>(M) * (L->spec.top_k + 1) * 8;
    if (!off_ok(c, topk_off, rec, 8)) return fail(c, MOE_E_INVALID, "topk offset invalid");
    DeviceGuard g(c->device);
    if ((rc = ensure_layer_ws(c, *L, M))) return rc;
    run_set_io(c, at<float>(c, x_off), nullptr, nullptr);
    if ((rc = run_route(c, *L, M))) return rc;
    MOE_CUDA(c, cudaMemcpyAsync(c->base + topk_off, c->ws.topk, rec, cudaMemcpyDeviceToDevice, c->stream));
    return MOE_OK;
}

int moe_do_route(moe_ctx* c, uint32_t layer_id, uint64_t x_off, uint32_t M, uint16_t* routed,
                 float* weights, float* shared_gate) {
    if (!c || !routed || !weights) return fail(c, MOE_E_INVALID, "NULL argument");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    if (M == 0) return MOE_OK;
    if ((rc = check_tokens(c, *L, x_off, M, "x"))) return rc;
    DeviceGuard g(c->device);
    if ((rc = ensure_layer_ws(c, *L, M))) return rc;
    run_set_io(c, at<float>(c, x_off), nullptr, nullptr);
    if ((rc = run_route(c, *L, M))) return rc;
    const int k = static_cast<int>(L->spec.top_k);
    std::vector<uint2> rec(static_cast<size_t>(M) * (k + 1));
    MOE_CUDA(c, cudaMemcpyAsync(rec.data(), c->ws.topk, rec.size() * sizeof(uint2),
                                cudaMemcpyDeviceToHost, c->stream));
    if ((rc = moe_sync(c))) return rc;
    for (uint32_t t = 0; t < M; ++t) {
        const uint2* r = &rec[static_cast<size_t>(t) * (k + 1)];
        for (int s = 0; s < k; ++s) {
            routed[static_cast<size_t>(t) * k + s] = static_cast<uint16_t>(r[1 + s].x);
            float w;
            std::memcpy(&w, &r[1 + s].y, 4);
            weights[static_cast<size_t>(t) * k + s] = w;
        }
        if (shared_gate) std::memcpy(&shared_gate[t], &r[0].y, 4);
    }
    return MOE_OK;
}

int moe_bucket(moe_ctx* c, uint32_t n_experts, uint32_t top_k, int has_shared, uint64_t topk_off,
               uint32_t M, uint64_t ranges_off, uint64_t tokens_off, uint64_t weights_off,
               uint64_t slot_pos_off) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (n_experts == 0 || n_experts > moe::kMaxExperts || top_k == 0 || top_k > moe::kMaxTopK ||
        top_k > n_experts)
        return fail(c, MOE_E_UNSUPPORTED, "n_experts %u / top_k %u unsupported", n_experts, top_k);
    if (M == 0) return MOE_OK;
    const uint64_t slots = top_k + (has_shared ? 1 : 0);
    const uint64_t S = static_cast<uint64_t>(M) * slots;
    if (!off_ok(c, topk_off, static_cast<uint64_t>(M) * (top_k + 1) * 8, 8) ||
        !off_ok(c, ranges_off, (n_experts + 2) * 4ull, 4) || !off_ok(c, tokens_off, S * 4, 4) ||
        !off_ok(c, weights_off, S * 4, 4) || !off_ok(c, slot_pos_off, S * 4, 4))
        return fail(c, MOE_E_INVALID, "bucket buffer offsets invalid");
    DeviceGuard g(c->device);
    int rc = ensure_ws(c, M, n_experts, top_k, static_cast<uint32_t>(slots), 0, 0);
    if (rc) return rc;
    moe::launch_bucket(static_cast<int>(n_experts), static_cast<int>(top_k), true, has_shared != 0,
                       at<uint2>(c, topk_off), static_cast<int>(M), c->ws, at<int>(c, ranges_off),
                       at<int>(c, tokens_off), at<float>(c, weights_off), at<int>(c, slot_pos_off),
                       c->ws.status, c->stream);
    stage(c, "bucket", 3);
    return check_launch(c, "bucket");
}

// Staging slots and streams of moe_forward_host, grown to hold M tokens of width H.
static int ensure_host_stage(Ctx* c, uint32_t M, uint32_t H) {
    if (!c->h2d_stream) {
        MOE_CUDA(c, cudaStreamCreateWithFlags(&c->h2d_stream, cudaStreamNonBlocking));
        MOE_CUDA(c, cudaStreamCreateWithFlags(&c->d2h_stream, cudaStreamNonBlocking));
        for (int b = 0; b < Ctx::kHostSlots; ++b) {
            MOE_CUDA(c, cudaEventCreateWithFlags(&c->ev_in[b], cudaEventDisableTiming));
            MOE_CUDA(c, cudaEventCreateWithFlags(&c->ev_done[b], cudaEventDisableTiming));
            MOE_CUDA(c, cudaEventCreateWithFlags(&c->ev_out[b], cudaEventDisableTiming));
        }
    }
    const size_t need = 2 * static_cast<size_t>(M) * H * sizeof(float);
    if (need <= c->host_stage_bytes) return MOE_OK;
    // earlier calls may still use the old slots
    MOE_CUDA(c, cudaStreamSynchronize(c->stream));
    MOE_CUDA(c, cudaStreamSynchronize(c->h2d_stream));
    MOE_CUDA(c, cudaStreamSynchronize(c->d2h_stream));
    for (int b = 0; b < Ctx::kHostSlots; ++b) {
        if (c->host_stage[b]) cudaFree(c->host_stage[b]);
        c->host_stage[b] = nullptr;
    }
    c->host_stage_bytes = 0;
    for (int b = 0; b < Ctx::kHostSlots; ++b) {
        void* p = nullptr;
        const cudaError_t e = cudaMalloc(&p, need);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(c, MOE_E_OOM, "host staging of %zu bytes: %s", need, cudaGetErrorString(e));
        }
        c->host_stage[b] = static_cast<float*>(p);
    }
    c->host_stage_bytes = need;
    return MOE_OK;
}

int moe_forward_host(moe_ctx* c, uint32_t layer_id, const float* x_host, float* out_host, uint32_t M,
                     int add_residual) {
    if (!c || !x_host || !out_host) return fail(c, MOE_E_INVALID, "NULL argument");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    if (L->subset())
        return fail(c, MOE_E_UNSUPPORTED, "expert-subset layer: route with moe_route and run moe_forward_topk");
    if (M == 0) return MOE_OK;
    if (stream_capturing(c)) return fail(c, MOE_E_INVALID, "moe_forward_host cannot be captured");
    DeviceGuard g(c->device);
    const uint32_t H = L->spec.hidden;
    if ((rc = ensure_layer_ws(c, *L, M))) return rc;
    if ((rc = ensure_host_stage(c, M, H))) return rc;
    const int b = c->host_next;
    c->host_next = (b + 1) % Ctx::kHostSlots;
    const size_t bytes = static_cast<size_t>(M) * H * sizeof(float);
    float* xs = c->host_stage[b];
    float* os = xs + static_cast<size_t>(M) * H;
    // host -> slot b once the layer call that last used it has finished reading it
    MOE_CUDA(c, cudaStreamWaitEvent(c->h2d_stream, c->ev_done[b], 0));
    MOE_CUDA(c, cudaMemcpyAsync(xs, x_host, bytes, cudaMemcpyHostToDevice, c->h2d_stream));
    MOE_CUDA(c, cudaEventRecord(c->ev_in[b], c->h2d_stream));
    // the layer, once its rows are in and slot b's previous result has been read out
    MOE_CUDA(c, cudaStreamWaitEvent(c->stream, c->ev_in[b], 0));
    MOE_CUDA(c, cudaStreamWaitEvent(c->stream, c->ev_out[b], 0));
    const float* resid = add_residual ? xs : nullptr;
    if (c->use_graphs && !c->prof && !use_decode(c, *L, M))
        rc = graph_forward(c, layer_id, *L, M, xs, resid, os);
    else {
        prof_begin(c);
        rc = record_forward(c, *L, M, xs, resid, os);
        prof_end(c);
    }
    if (rc) return rc;
    MOE_CUDA(c, cudaEventRecord(c->ev_done[b], c->stream));
    // result -> host
    MOE_CUDA(c, cudaStreamWaitEvent(c->d2h_stream, c->ev_done[b], 0));
    MOE_CUDA(c, cudaMemcpyAsync(out_host, os, bytes, cudaMemcpyDeviceToHost, c->d2h_stream));
    MOE_CUDA(c, cudaEventRecord(c->ev_out[b], c->d2h_stream));
    return MOE_OK;
}

int moe_forward(moe_ctx* c, uint32_t layer_id, uint64_t x_off, uint64_t resid_off,
                uint64_t out_off, uint32_t M) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    if (L->subset())
        return fail(c, MOE_E_UNSUPPORTED, "expert-subset layer: route with moe_route and run moe_forward_topk");
    if (M == 0) return MOE_OK;
    if ((rc = check_tokens(c, *L, x_off, M, "x"))) return rc;
    if (resid_off && (rc = check_tokens(c, *L, resid_off, M, "resid"))) return rc;
    if ((rc = check_tokens(c, *L, out_off, M, "out"))) return rc;
    DeviceGuard g(c->device);
    if ((rc = ensure_layer_ws(c, *L, M))) return rc;
    const float* x = at<float>(c, x_off);
    const float* resid = resid_off ? at<float>(c, resid_off) : nullptr;
    float* out = at<float>(c, out_off);
    if (c->use_graphs && !c->prof && !stream_capturing(c) && !use_decode(c, *L, M))
        return graph_forward(c, layer_id, *L, M, x, resid, out);
    prof_begin(c);
    rc = record_forward(c, *L, M, x, resid, out);
    prof_end(c);
    return rc;
}

int moe_layer_set_next(moe_ctx* c, uint32_t layer_id, int32_t next_id) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    L->next_router = nullptr;
    L->next_router_bytes = 0;
    for (int i = 0; i < 3; ++i) { L->next_shared[i] = nullptr; L->next_shared_bytes[i] = 0; }
    if (next_id < 0) return MOE_OK;
    Layer* N;
    if ((rc = get_layer(c, static_cast<uint32_t>(next_id), &N))) return rc;
    const uint64_t H = N->spec.hidden, I = N->spec.inter, E = N->spec.n_experts;
    L->next_router = N->router_w_ptr;
    L->next_router_bytes = E * H * 4;
    if (N->has_shared() && N->tab) {
        std::vector<const uint8_t*> t(3 * (E + 1));
        MOE_CUDA(c, cudaMemcpy(t.data(), N->tab, t.size() * sizeof(void*), cudaMemcpyDeviceToHost));
        const bool ref36 = N->ref36();
        const uint64_t b13 = ref36 ? H * I / 32 * 36 : I * (H / 256) * 136;
        const uint64_t b2 = ref36 ? H * I / 32 * 36 : H * (I / 256) * 136;
        for (int i = 0; i < 3; ++i) {
            L->next_shared[i] = t[i * (E + 1) + E];
            L->next_shared_bytes[i] = i == 2 ? b2 : b13;
        }
    }
    return MOE_OK;
}

int moe_forward_norm(moe_ctx* c, uint32_t layer_id, uint64_t x_off, uint64_t out_off, uint32_t M,
                     float eps) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    if (L->subset())
        return fail(c, MOE_E_UNSUPPORTED, "expert-subset layer: route with moe_route and run moe_forward_topk");
    if (!(eps >= 0.f)) return fail(c, MOE_E_INVALID, "eps must be >= 0");
    if (M == 0) return MOE_OK;
    if ((rc = check_tokens(c, *L, x_off, M, "x"))) return rc;
    if ((rc = check_tokens(c, *L, out_off, M, "out"))) return rc;
    DeviceGuard g(c->device);
    if ((rc = ensure_layer_ws(c, *L, M))) return rc;
    const float* x = at<float>(c, x_off);
    float* out = at<float>(c, out_off);
    if (M == 1 && (c->path == moe::kPathAuto || c->path == moe::kPathGemv) && moe::decode_supported(*L, c->sm_count) &&
        out != x) {
        // one launch: normalisation inside the fused decode kernel, direct pointers
        if (moe::launch_decode(*L, c->ws, decode_sync(c), c->sm_count, c->stream, x, x, out, eps))
            return check_launch(c, "decode (cooperative launch refused)");
        stage(c, "decode", 1);
        return check_launch(c, "decode");
    }
    moe::launch_rms_norm(x, c->ws.xn, static_cast<int>(M), static_cast<int>(L->spec.hidden), eps, c->stream);
    stage(c, "rms_norm", 1);
    if ((rc = check_launch(c, "rms_norm"))) return rc;
    if (c->use_graphs && !c->prof && !stream_capturing(c) && !use_decode(c, *L, M))
        return graph_forward(c, layer_id, *L, M, c->ws.xn, x, out);
    prof_begin(c);
    rc = record_forward(c, *L, M, c->ws.xn, x, out);
    prof_end(c);
    return rc;
}

int moe_forward_routed(moe_ctx* c, uint32_t layer_id, uint64_t x_off, uint64_t resid_off,
                       uint64_t out_off, uint32_t M, const uint16_t* routed, const float* weights,
                       const float* shared_gate) {
    if (!c || !routed || !weights) return fail(c, MOE_E_INVALID, "NULL argument");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    if (L->subset())
        return fail(c, MOE_E_UNSUPPORTED, "expert-subset layer: route with moe_route and run moe_forward_topk");
    if (M == 0) return MOE_OK;
    if ((rc = check_tokens(c, *L, x_off, M, "x"))) return rc;
    if (resid_off && (rc = check_tokens(c, *L, resid_off, M, "resid"))) return rc;
    if ((rc = check_tokens(c, *L, out_off, M, "out"))) return rc;
    const int k = static_cast<int>(L->spec.top_k);
    const uint32_t E = L->spec.n_experts;
    std::vector<uint2> rec(static_cast<size_t>(M) * (k + 1));
    for (uint32_t t = 0; t < M; ++t) {
        uint2* r = &rec[static_cast<size_t>(t) * (k + 1)];
        float g = shared_gate ? shared_gate[t] : 1.0f;
        uint32_t gb;
        std::memcpy(&gb, &g, 4);
        r[0] = make_uint2(E, gb);
        for (int s = 0; s < k; ++s) {
            const uint16_t e = routed[static_cast<size_t>(t) * k + s];
            if (e >= E) return fail(c, MOE_E_INVALID, "token %u slot %d: expert %u >= %u", t, s, e, E);
            for (int s2 = 0; s2 < s; ++s2)
                if (routed[static_cast<size_t>(t) * k + s2] == e)
                    return fail(c, MOE_E_INVALID, "token %u: expert %u routed twice", t, e);
            uint32_t wb;
            std::memcpy(&wb, &weights[static_cast<size_t>(t) * k + s], 4);
            r[1 + s] = make_uint2(e, wb);
        }
    }
    DeviceGuard g(c->device);
    if ((rc = ensure_layer_ws(c, *L, M))) return rc;
    // Pageable source: the copy has left `rec` when cudaMemcpyAsync returns.
    MOE_CUDA(c, cudaMemcpyAsync(c->ws.topk, rec.data(), rec.size() * sizeof(uint2),
                                cudaMemcpyHostToDevice, c->stream));
    prof_begin(c);
    run_set_io(c, at<float>(c, x_off), resid_off ? at<float>(c, resid_off) : nullptr, at<float>(c, out_off));
    rc = run_experts(c, *L, M, true, L->has_shared(), L->spec.scale);
    prof_end(c);
    return rc;
}

int moe_forward_topk(moe_ctx* c, uint32_t layer_id, uint64_t x_off, uint64_t resid_off,
                     uint64_t out_off, uint32_t M, uint64_t topk_off, uint32_t flags) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    if (flags & ~(MOE_FT_NO_SHARED | MOE_FT_SHARED_ONLY | MOE_FT_UNSCALED))
        return fail(c, MOE_E_INVALID, "unknown flags 0x%x", flags);
    if ((flags & MOE_FT_NO_SHARED) && (flags & MOE_FT_SHARED_ONLY))
        return fail(c, MOE_E_INVALID, "MOE_FT_NO_SHARED and MOE_FT_SHARED_ONLY exclude each other");
    if ((flags & MOE_FT_SHARED_ONLY) && !L->has_shared())
        return fail(c, MOE_E_INVALID, "MOE_FT_SHARED_ONLY on a layer without a shared expert");
    if (M == 0) return MOE_OK;
    if ((rc = check_tokens(c, *L, x_off, M, "x"))) return rc;
    if (resid_off && (rc = check_tokens(c, *L, resid_off, M, "resid"))) return rc;
    if ((rc = check_tokens(c, *L, out_off, M, "out"))) return rc;
    const uint64_t rec = static_cast<uint64_t>(M) * (L->spec.top_k + 1) * 8;
    if (!off_ok(c, topk_off, rec, 8)) return fail(c, MOE_E_INVALID, "topk offset invalid");
    DeviceGuard g(c->device);
    if ((rc = ensure_layer_ws(c, *L, M))) return rc;
    MOE_CUDA(c, cudaMemcpyAsync(c->ws.topk, c->base + topk_off, rec, cudaMemcpyDeviceToDevice, c->stream));
    prof_begin(c);
    run_set_io(c, at<float>(c, x_off), resid_off ? at<float>(c, resid_off) : nullptr, at<float>(c, out_off));
    rc = run_experts(c, *L, M, !(flags & MOE_FT_SHARED_ONLY), L->has_shared() && !(flags & MOE_FT_NO_SHARED),
                     (flags & MOE_FT_UNSCALED) ? 1.0f : L->spec.scale);
    prof_end(c);
    return rc;
}

uint64_t moe_ep_plan_bytes(uint32_t M, uint32_t n_ranks) {
    const uint64_t a = (4ull * M + 255) / 256 * 256;
    const uint64_t b = (4ull * M * n_ranks + 255) / 256 * 256;
    return a + b + 8ull * n_ranks;
}

static moe::EpPlan ep_plan_at(Ctx* c, uint64_t plan_off, uint32_t M, uint32_t n_ranks) {
    const uint64_t a = (4ull * M + 255) / 256 * 256;
    const uint64_t b = (4ull * M * n_ranks + 255) / 256 * 256;
    return moe::EpPlan{at<uint32_t>(c, plan_off), at<int>(c, plan_off + a), at<int>(c, plan_off + a + b)};
}

static int ep_check_ranks(Ctx* c, uint32_t n_ranks, uint32_t my_rank, uint32_t capacity, uint32_t M) {
    if (n_ranks == 0 || n_ranks > static_cast<uint32_t>(moe::kMaxEpRanks) || my_rank >= n_ranks)
        return fail(c, MOE_E_UNSUPPORTED, "n_ranks %u (1..%d) / rank %u", n_ranks, moe::kMaxEpRanks, my_rank);
    if (capacity < M) return fail(c, MOE_E_INVALID, "capacity %u below the %u local tokens", capacity, M);
    return MOE_OK;
}

int moe_ep_dispatch(moe_ctx* c, uint32_t n_experts, uint32_t top_k, uint32_t n_ranks, uint32_t my_rank,
                    uint32_t capacity, uint64_t topk_off, uint64_t x_off, uint32_t M, uint32_t H,
                    uint64_t plan_off, uint64_t send_x_off, uint64_t send_topk_off) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    int rc = ep_check_ranks(c, n_ranks, my_rank, capacity, M);
    if (rc) return rc;
    if (n_experts == 0 || n_experts > moe::kMaxExperts || n_experts % n_ranks != 0 || top_k == 0 ||
        top_k > moe::kMaxTopK)
        return fail(c, MOE_E_UNSUPPORTED, "n_experts %u (a multiple of n_ranks %u), top_k %u", n_experts,
                    n_ranks, top_k);
    if (H == 0 || H % 4 != 0) return fail(c, MOE_E_INVALID, "H must be a positive multiple of 4");
    const uint64_t rows = static_cast<uint64_t>(n_ranks) * capacity;
    const uint64_t rec_bytes = rows * (top_k + 1) * 8;
    if (!off_ok(c, send_x_off, rows * H * 4, 16) || !off_ok(c, send_topk_off, rec_bytes, 8) ||
        !off_ok(c, plan_off, moe_ep_plan_bytes(std::max(M, 1u), n_ranks), 256) ||
        (M && (!off_ok(c, topk_off, static_cast<uint64_t>(M) * (top_k + 1) * 8, 8) ||
               !off_ok(c, x_off, static_cast<uint64_t>(M) * H * 4, 16))))
        return fail(c, MOE_E_INVALID, "ep dispatch buffer offsets invalid (send buffers hold n_ranks*capacity rows)");
    DeviceGuard g(c->device);
    // every record starts empty (id 0xFFFFFFFF): rows no token uses are skipped by the experts
    MOE_CUDA(c, cudaMemsetAsync(c->base + send_topk_off, 0xFF, rec_bytes, c->stream));
    if (M == 0) return MOE_OK;
    const moe::EpPlan plan = ep_plan_at(c, plan_off, M, n_ranks);
    const int epr = static_cast<int>(n_experts / n_ranks);
    moe::launch_ep_plan(at<uint2>(c, topk_off), static_cast<int>(M), static_cast<int>(top_k), epr,
                        static_cast<int>(n_ranks), static_cast<int>(my_rank), static_cast<int>(capacity),
                        plan, c->ws.status, c->stream);
    moe::launch_ep_gather(at<float>(c, x_off), at<uint2>(c, topk_off), plan, static_cast<int>(M),
                          static_cast<int>(H), static_cast<int>(top_k), epr, static_cast<int>(n_ranks),
                          static_cast<int>(my_rank), at<float>(c, send_x_off), at<uint2>(c, send_topk_off),
                          c->stream);
    stage(c, "ep_dispatch", 3);
    return check_launch(c, "ep_dispatch");
}

int moe_ep_combine(moe_ctx* c, uint32_t n_ranks, uint32_t capacity, uint32_t H, uint32_t M,
                   uint64_t plan_off, uint64_t y_back_off, uint64_t resid_off, uint64_t out_off, float scale) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    int rc = ep_check_ranks(c, n_ranks, 0, capacity, M);
    if (rc) return rc;
    if (H == 0 || H % 4 != 0) return fail(c, MOE_E_INVALID, "H must be a positive multiple of 4");
    if (M == 0) return MOE_OK;
    const uint64_t row = static_cast<uint64_t>(H) * 4, rows = static_cast<uint64_t>(M) * row;
    if (!off_ok(c, plan_off, moe_ep_plan_bytes(M, n_ranks), 256) ||
        !off_ok(c, y_back_off, static_cast<uint64_t>(n_ranks) * capacity * row, 16) ||
        (resid_off && !off_ok(c, resid_off, rows, 16)) || !off_ok(c, out_off, rows, 16))
        return fail(c, MOE_E_INVALID, "ep combine buffer offsets invalid");
    DeviceGuard g(c->device);
    moe::launch_ep_combine(ep_plan_at(c, plan_off, M, n_ranks), static_cast<int>(M), static_cast<int>(n_ranks),
                           static_cast<int>(H), at<float>(c, y_back_off),
                           resid_off ? at<float>(c, resid_off) : nullptr, scale, at<float>(c, out_off), c->stream);
    stage(c, "ep_combine", 1);
    return check_launch(c, "ep_combine");
}

// ---- expert parallelism over NCCL ----------------------------------------------------------

static int nccl_fail(Ctx* c, const moe::NcclApi* api, ncclResult_t r, const char* what) {
    return fail(c, MOE_E_CUDA, "%s: %s", what, api->error_string ? api->error_string(r) : "NCCL error");
}

// Per-peer blocks of `count` elements: block d of `send` goes to rank d, block d of `recv` comes
// from rank d (equal splits: nothing about the sizes is exchanged).
static int ep_alltoall(Ctx* c, const moe::NcclApi* api, const void* send, void* recv, size_t count,
                       ncclDataType_t type, size_t elem, const char* what) {
    const moe::EpState& ep = c->ep;
    ncclResult_t r = api->group_start();
    if (r != ncclSuccess) return nccl_fail(c, api, r, what);
    for (uint32_t d = 0; d < ep.n_ranks && r == ncclSuccess; ++d) {
        r = api->send(static_cast<const uint8_t*>(send) + d * count * elem, count, type, static_cast<int>(d),
                      ep.comm, c->stream);
        if (r == ncclSuccess)
            r = api->recv(static_cast<uint8_t*>(recv) + d * count * elem, count, type, static_cast<int>(d),
                          ep.comm, c->stream);
    }
    const ncclResult_t r2 = api->group_end();
    if (r != ncclSuccess) return nccl_fail(c, api, r, what);
    if (r2 != ncclSuccess) return nccl_fail(c, api, r2, what);
    return MOE_OK;
}

static moe::EpPlan ep_plan_ptr(uint8_t* base, uint32_t M, uint32_t n_ranks) {
    const uint64_t a = (4ull * M + 255) / 256 * 256;
    const uint64_t b = (4ull * M * n_ranks + 255) / 256 * 256;
    return moe::EpPlan{reinterpret_cast<uint32_t*>(base), reinterpret_cast<int*>(base + a),
                       reinterpret_cast<int*>(base + a + b)};
}

static void ep_close_peers(moe::EpState& ep) {
    for (uint32_t d = 0; d < 8; ++d) {
        if (ep.peer_base[d]) cudaIpcCloseMemHandle(ep.peer_base[d]);
        ep.peer_base[d] = nullptr;
    }
    ep.peer = false;
}

// Maps every other rank's exchange buffer (CUDA IPC handles all-gathered over the group).  The
// outcome is agreed by all ranks (an all-reduce of the local result), so either every rank uses
// the peer transport or none does.
// Every rank's buffer layout (capacity, width, record length) must be the same, or rank blocks
// would land at different offsets (and, with the peer transport, past a smaller peer buffer):
// checked whenever the buffers are (re)created, by an all-gather of the layouts.
static int ep_check_layout(Ctx* c, const moe::NcclApi* api) {
    moe::EpState& ep = c->ep;
    const uint32_t n = ep.n_ranks;
    if (n == 1) return MOE_OK;
    const uint32_t mine[4] = {ep.capacity, ep.hidden, ep.top_k, n};
    uint32_t* d = nullptr;
    MOE_CUDA(c, cudaMalloc(&d, sizeof(mine) * (n + 1)));
    cudaMemcpy(d + 4 * n, mine, sizeof(mine), cudaMemcpyHostToDevice);
    const ncclResult_t r = api->all_gather(d + 4 * n, d, 4, ncclUint32, ep.comm, c->stream);
    std::vector<uint32_t> all(4 * n);
    if (r == ncclSuccess) {
        cudaStreamSynchronize(c->stream);
        cudaMemcpy(all.data(), d, sizeof(mine) * n, cudaMemcpyDeviceToHost);
    }
    cudaFree(d);
    if (r != ncclSuccess) return nccl_fail(c, api, r, "layout exchange");
    for (uint32_t q = 0; q < n; ++q)
        if (std::memcmp(&all[4 * q], mine, sizeof(mine)) != 0)
            return fail(c, MOE_E_INVALID,
                        "expert-parallel ranks disagree: rank %u has capacity %u, hidden %u, top_k %u; rank %u "
                        "capacity %u, hidden %u, top_k %u (every rank must pass the same capacity and layer shape)",
                        ep.rank, mine[0], mine[1], mine[2], q, all[4 * q], all[4 * q + 1], all[4 * q + 2]);
    return MOE_OK;
}

static int ep_map_peers(Ctx* c, const moe::NcclApi* api) {
    moe::EpState& ep = c->ep;
    const uint32_t n = ep.n_ranks;
    int ok = 1;
    cudaIpcMemHandle_t mine;
    if (n > 1 && cudaIpcGetMemHandle(&mine, ep.buf) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
        std::memset(&mine, 0, sizeof(mine));
    }
    std::vector<cudaIpcMemHandle_t> all(n);
    void* tmp = nullptr;
    MOE_CUDA(c, cudaMalloc(&tmp, sizeof(cudaIpcMemHandle_t) * (n + 1) + 16));
    uint8_t* t = static_cast<uint8_t*>(tmp);
    int* flag = reinterpret_cast<int*>(t + sizeof(cudaIpcMemHandle_t) * (n + 1));
    int rc = MOE_OK;
    ncclResult_t r = ncclSuccess;
    if (n > 1) {
        cudaMemcpy(t + sizeof(cudaIpcMemHandle_t) * n, &mine, sizeof(mine), cudaMemcpyHostToDevice);
        r = api->all_gather(t + sizeof(cudaIpcMemHandle_t) * n, t, sizeof(mine), ncclUint8, ep.comm, c->stream);
        if (r == ncclSuccess) {
            cudaStreamSynchronize(c->stream);
            cudaMemcpy(all.data(), t, sizeof(cudaIpcMemHandle_t) * n, cudaMemcpyDeviceToHost);
            for (uint32_t d = 0; d < n && ok; ++d) {
                if (d == ep.rank) continue;
                void* p = nullptr;
                if (cudaIpcOpenMemHandle(&p, all[d], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                    cudaGetLastError();
                    ok = 0;
                } else {
                    ep.peer_base[d] = static_cast<uint8_t*>(p);
                }
            }
        }
    }
    if (r == ncclSuccess) {
        cudaMemcpy(flag, &ok, sizeof(int), cudaMemcpyHostToDevice);
        r = api->all_reduce(flag, flag, 1, ncclInt32, ncclMin, ep.comm, c->stream);
        if (r == ncclSuccess) {
            cudaStreamSynchronize(c->stream);
            cudaMemcpy(&ok, flag, sizeof(int), cudaMemcpyDeviceToHost);
        }
    }
    cudaFree(tmp);
    if (r != ncclSuccess) rc = nccl_fail(c, api, r, "peer handle exchange");
    if (!ok || rc != MOE_OK) ep_close_peers(ep);
    else ep.peer = true;
    return rc;
}

// Exchange buffers for n_ranks x capacity rows of width H with (k+1)-entry records, the step
// flags and epoch, and (peer transport) the mappings of the other ranks' buffers.  Collective
// when it reallocates: every rank calls it with the same sizes.
static int ensure_ep_buffers(Ctx* c, const moe::NcclApi* api, uint32_t capacity, uint32_t H, uint32_t k) {
    moe::EpState& ep = c->ep;
    const bool want_peer = ep.transport == MOE_EP_TRANSPORT_PEER;
    // rows are laid out with the layer's own width and record length, so those must match
    const bool same_shape = H == ep.hidden && k == ep.top_k;
    if (ep.buf && same_shape && capacity <= ep.capacity && ep.peer == (want_peer && ep.peer)) return MOE_OK;
    if (same_shape) capacity = std::max(capacity, ep.capacity);
    const uint64_t rows = static_cast<uint64_t>(ep.n_ranks) * capacity;
    const uint64_t xb = (rows * H * 4 + 255) / 256 * 256, rb = (rows * (k + 1) * 8 + 255) / 256 * 256;
    const uint64_t pb = (moe_ep_plan_bytes(capacity, ep.n_ranks) + 255) / 256 * 256;
    MOE_CUDA(c, cudaStreamSynchronize(c->stream));
    if (ep.buf) {  // retired, not freed: graphs captured against it may still be replayed
        moe::EpState::Retired r{ep.buf, {}};
        for (int d = 0; d < 8; ++d) r.peer_base[d] = ep.peer_base[d];
        ep.retired.push_back(r);
        for (int d = 0; d < 8; ++d) ep.peer_base[d] = nullptr;
        ep.peer = false;
    }
    ep.buf = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, pb + 4 * xb + 2 * rb + 256);
    if (e != cudaSuccess) {
        cudaGetLastError();
        // the other ranks are entering the layout exchange: take part with an empty layout, so
        // every rank fails (on the disagreement) instead of waiting for this one
        ep.capacity = ep.hidden = ep.top_k = 0;
        ep_check_layout(c, api);
        ep.capacity = ep.hidden = ep.top_k = 0;
        return fail(c, MOE_E_OOM, "expert-parallel buffers for %u x %u rows: %s", ep.n_ranks, capacity,
                    cudaGetErrorString(e));
    }
    uint8_t* b = static_cast<uint8_t*>(p);
    ep.buf = b;
    ep.plan = b;
    ep.send_x = reinterpret_cast<float*>(b + pb);
    ep.off_recv_x = pb + xb;
    ep.recv_x = reinterpret_cast<float*>(b + ep.off_recv_x);
    ep.off_y_send = pb + 2 * xb;
    ep.y_send = reinterpret_cast<float*>(b + ep.off_y_send);
    ep.y_recv = reinterpret_cast<float*>(b + pb + 3 * xb);
    ep.send_rec = reinterpret_cast<uint2*>(b + pb + 4 * xb);
    ep.off_recv_rec = pb + 4 * xb + rb;
    ep.recv_rec = reinterpret_cast<uint2*>(b + ep.off_recv_rec);
    ep.off_flags = pb + 4 * xb + 2 * rb;
    ep.flags = reinterpret_cast<unsigned long long*>(b + ep.off_flags);
    ep.epoch = ep.flags + 16;
    MOE_CUDA(c, cudaMemsetAsync(b + ep.off_flags, 0, 256, c->stream));
    MOE_CUDA(c, cudaStreamSynchronize(c->stream));
    ep.capacity = capacity;
    ep.hidden = H;
    ep.top_k = k;
    int rc = ep_check_layout(c, api);
    if (rc != MOE_OK) {
        ep.capacity = ep.hidden = ep.top_k = 0;  // the next call re-creates (and re-checks) them
        return rc;
    }
    if (want_peer) return ep_map_peers(c, api);
    return MOE_OK;
}

static void ep_release(Ctx* c) {
    moe::EpState& ep = c->ep;
    ep_close_peers(ep);
    for (auto& r : ep.retired) {
        for (int d = 0; d < 8; ++d)
            if (r.peer_base[d]) cudaIpcCloseMemHandle(r.peer_base[d]);
        cudaFree(r.buf);
    }
    if (ep.comm && !ep.aborted.load()) {  // an aborted communicator is already freed
        const moe::NcclApi* api = moe::nccl_api(nullptr);
        if (api) api->comm_destroy(ep.comm);
    }
    if (ep.buf) cudaFree(ep.buf);
    const int transport = ep.transport;
    ep.reset();
    ep.transport = transport;
}

// Peer addresses of this rank's blocks at every rank (see EpPeers).
static moe::EpPeers ep_peers(const moe::EpState& ep) {
    moe::EpPeers P{};
    const uint64_t rb = static_cast<uint64_t>(ep.rank) * ep.capacity;
    for (uint32_t d = 0; d < ep.n_ranks; ++d) {
        uint8_t* base = d == ep.rank ? ep.buf : ep.peer_base[d];
        P.x[d] = reinterpret_cast<float*>(base + ep.off_recv_x) + rb * ep.hidden;
        P.rec[d] = reinterpret_cast<uint2*>(base + ep.off_recv_rec) + rb * (ep.top_k + 1);
        P.y[d] = reinterpret_cast<const float*>(base + ep.off_y_send) + rb * ep.hidden;
        for (int s = 0; s < 2; ++s)
            P.flag[s][d] = reinterpret_cast<unsigned long long*>(base + ep.off_flags) + s * 8 + ep.rank;
    }
    return P;
}

int moe_ep_set_transport(moe_ctx* c, int transport) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (transport != MOE_EP_TRANSPORT_NCCL && transport != MOE_EP_TRANSPORT_PEER)
        return fail(c, MOE_E_INVALID, "unknown transport %d", transport);
    if (c->ep.transport != transport) {
        DeviceGuard g(c->device);
        MOE_CUDA(c, cudaStreamSynchronize(c->stream));
        c->ep.transport = transport;
        c->ep.capacity = 0;  // the next moe_forward_ep re-creates the buffers (collectively)
    }
    return MOE_OK;
}

int moe_ep_transport(moe_ctx* c, int* transport) {
    if (!c || !transport) return fail(c, MOE_E_INVALID, "NULL argument");
    *transport = c->ep.buf ? (c->ep.peer ? MOE_EP_TRANSPORT_PEER : MOE_EP_TRANSPORT_NCCL) : -1;
    return MOE_OK;
}

int moe_ep_unique_id(void* out, size_t n) {
    if (!out || n < sizeof(ncclUniqueId)) return fail(nullptr, MOE_E_INVALID, "unique id buffer below %zu bytes",
                                                       sizeof(ncclUniqueId));
    std::string err;
    const moe::NcclApi* api = moe::nccl_api(&err);
    if (!api) return fail(nullptr, MOE_E_UNSUPPORTED, "%s", err.c_str());
    ncclUniqueId id;
    const ncclResult_t r = api->get_unique_id(&id);
    if (r != ncclSuccess) return fail(nullptr, MOE_E_CUDA, "ncclGetUniqueId: %s", api->error_string(r));
    std::memcpy(out, &id, sizeof(id));
    return MOE_OK;
}

int moe_ep_init(moe_ctx* c, const void* unique_id, uint32_t n_ranks, uint32_t rank) {
    if (!c || !unique_id) return fail(c, MOE_E_INVALID, "NULL argument");
    if (n_ranks == 0 || n_ranks > static_cast<uint32_t>(moe::kMaxEpRanks) || rank >= n_ranks)
        return fail(c, MOE_E_UNSUPPORTED, "n_ranks %u (1..%d) / rank %u", n_ranks, moe::kMaxEpRanks, rank);
    std::string err;
    const moe::NcclApi* api = moe::nccl_api(&err);
    if (!api) return fail(c, MOE_E_UNSUPPORTED, "%s", err.c_str());
    DeviceGuard g(c->device);
    MOE_CUDA(c, cudaStreamSynchronize(c->stream));
    ep_release(c);
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = api->comm_init_rank(&comm, static_cast<int>(n_ranks), id, static_cast<int>(rank));
    if (r != ncclSuccess) return nccl_fail(c, api, r, "ncclCommInitRank");
    c->ep.comm = comm;
    c->ep.n_ranks = n_ranks;
    c->ep.rank = rank;
    return MOE_OK;
}

int moe_ep_abort(moe_ctx* c) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    moe::EpState& ep = c->ep;
    if (!ep.comm) return MOE_OK;
    if (ep.aborted.exchange(true)) return MOE_OK;
    const moe::NcclApi* api = moe::nccl_api(nullptr);
    if (api && api->comm_abort) api->comm_abort(ep.comm);
    return MOE_OK;
}

int moe_forward_ep(moe_ctx* c, uint32_t layer_id, uint64_t x_off, uint64_t resid_off, uint64_t out_off,
                   uint32_t M, uint32_t capacity) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    moe::EpState& ep = c->ep;
    if (!ep.comm) return fail(c, MOE_E_INVALID, "moe_ep_init has not been called on this context");
    if (ep.aborted.load()) return fail(c, MOE_E_CUDA, "the expert-parallel group was aborted (moe_ep_abort)");
    Layer* L;
    int rc = get_layer(c, layer_id, &L);
    if (rc) return rc;
    const uint32_t n = ep.n_ranks, E = L->spec.n_experts, k = L->spec.top_k, H = L->spec.hidden;
    if (E % n != 0) return fail(c, MOE_E_UNSUPPORTED, "%u experts do not split over %u ranks", E, n);
    // A rank whose own per-call arguments are bad must still take part in the exchange: the
    // other ranks are already waiting for its blocks (NCCL waits without a time limit).  It
    // joins as a rank with no tokens, serves its experts to the others, and reports the error.
    int local_rc = MOE_OK;
    if (capacity == 0 || capacity < M)
        local_rc = fail(c, MOE_E_INVALID, "capacity %u must be >= 1 and >= the %u local tokens", capacity, M);
    if (M && local_rc == MOE_OK) {
        if ((rc = check_tokens(c, *L, x_off, M, "x")) ||
            (resid_off && (rc = check_tokens(c, *L, resid_off, M, "resid"))) ||
            (rc = check_tokens(c, *L, out_off, M, "out")))
            local_rc = rc;
    }
    if (local_rc != MOE_OK) {
        M = 0;
        capacity = std::max(capacity, 1u);
    }
    const moe::NcclApi* api = moe::nccl_api(nullptr);
    DeviceGuard g(c->device);
    if ((rc = ensure_ep_buffers(c, api, capacity, H, k))) return rc;  // collective, agreed outcome
    capacity = ep.capacity;  // rank blocks are laid out with the buffers' capacity
    const uint32_t rows = n * capacity;
    // Without a workspace this rank cannot run its experts; it still completes the exchange and
    // returns NaN partial rows, so the tokens it should have served come out NaN on their ranks
    // instead of the group hanging.
    bool serve = true;
    if ((rc = ensure_layer_ws(c, *L, std::max(rows, M)))) {
        if (local_rc == MOE_OK) local_rc = rc;
        serve = false;
        M = 0;
    }
    const size_t rec = static_cast<size_t>(k + 1) * 8;
    const moe::EpPlan plan = ep_plan_ptr(ep.plan, std::max(M, 1u), n);
    const int epr = static_cast<int>(E / n);
    prof_begin(c);
    if (M) {
        run_set_io(c, at<float>(c, x_off), nullptr, nullptr);
        if ((rc = run_route(c, *L, M))) {
            if (local_rc == MOE_OK) local_rc = rc;
            M = 0;
        } else {
            moe::launch_ep_plan(c->ws.topk, static_cast<int>(M), static_cast<int>(k), epr, static_cast<int>(n),
                                static_cast<int>(ep.rank), static_cast<int>(capacity), plan, c->ws.status,
                                c->stream);
            stage(c, "ep_plan", 2);
        }
    }
    // this rank's experts on the received rows (or NaN rows when it cannot run them)
    auto run_local = [&]() -> int {
        if (!serve) {
            MOE_CUDA(c, cudaMemsetAsync(ep.y_send, 0xFF, static_cast<size_t>(rows) * H * 4, c->stream));
            return MOE_OK;
        }
        MOE_CUDA(c, cudaMemcpyAsync(c->ws.topk, ep.recv_rec, rows * rec, cudaMemcpyDeviceToDevice, c->stream));
        run_set_io(c, ep.recv_x, nullptr, ep.y_send);
        return run_experts(c, *L, rows, true, L->has_shared(), 1.0f);
    };
    const float* resid = resid_off ? at<float>(c, resid_off) : nullptr;
    if (ep.peer) {
        // rows and records stored into every owner's receive block over NVLink, then the
        // rank's experts, then each owner reads its partial rows from the expert ranks
        const moe::EpPeers P = ep_peers(ep);
        moe::launch_ep_push(at<float>(c, x_off), c->ws.topk, plan, static_cast<int>(M), static_cast<int>(H),
                            static_cast<int>(k), epr, static_cast<int>(n), static_cast<int>(ep.rank),
                            static_cast<int>(capacity), P, c->stream);
        moe::launch_ep_signal(ep.epoch, true, static_cast<int>(n), P, 0, c->stream);
        moe::launch_ep_wait(ep.flags, ep.epoch, static_cast<int>(n), c->ws.status, c->stream);
        stage(c, "ep_push", M ? 4 : 3);
        if ((rc = run_local())) return rc;
        moe::launch_ep_signal(ep.epoch, false, static_cast<int>(n), P, 1, c->stream);
        moe::launch_ep_wait(ep.flags + 8, ep.epoch, static_cast<int>(n), c->ws.status, c->stream);
        stage(c, "ep_sync", 2);
        if (M) {
            moe::launch_ep_pull_combine(plan, static_cast<int>(M), static_cast<int>(n), static_cast<int>(H), P,
                                        resid, L->spec.scale, at<float>(c, out_off), c->stream);
            stage(c, "ep_combine", 1);
        }
    } else {
        // 1-2. the rank blocks (empty records pad every block)
        MOE_CUDA(c, cudaMemsetAsync(ep.send_rec, 0xFF, rows * rec, c->stream));
        if (M) {
            moe::launch_ep_gather(at<float>(c, x_off), c->ws.topk, plan, static_cast<int>(M), static_cast<int>(H),
                                  static_cast<int>(k), epr, static_cast<int>(n), static_cast<int>(ep.rank), ep.send_x,
                                  ep.send_rec, c->stream);
            stage(c, "ep_dispatch", 1);
        }
        // 3. rows and records to their expert ranks
        if ((rc = ep_alltoall(c, api, ep.send_x, ep.recv_x, static_cast<size_t>(capacity) * H, ncclFloat32, 4,
                              "dispatch all-to-all")))
            return rc;
        if ((rc = ep_alltoall(c, api, ep.send_rec, ep.recv_rec, capacity * rec, ncclUint8, 1,
                              "record all-to-all")))
            return rc;
        stage(c, "ep_alltoall", 0);
        // 4. this rank's experts (and the shared expert for its own tokens) on every received row
        if ((rc = run_local())) return rc;
        // 5. partial rows back to their owners
        if ((rc = ep_alltoall(c, api, ep.y_send, ep.y_recv, static_cast<size_t>(capacity) * H, ncclFloat32, 4,
                              "combine all-to-all")))
            return rc;
        stage(c, "ep_alltoall", 0);
        // 6. out = resid + scale * sum of the partials in rank order
        if (M) {
            moe::launch_ep_combine(plan, static_cast<int>(M), static_cast<int>(n), static_cast<int>(H), ep.y_recv,
                                   resid, L->spec.scale, at<float>(c, out_off), c->stream);
            stage(c, "ep_combine", 1);
        }
    }
    prof_end(c);
    rc = check_launch(c, "forward_ep");
    return local_rc != MOE_OK ? local_rc : rc;
}

int moe_set_path(moe_ctx* c, int path) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (path < moe::kPathAuto || path > moe::kPathTcTmemA)
        return fail(c, MOE_E_INVALID, "unknown path %d", path);
    c->path = path;
    return MOE_OK;
}

int moe_profile(moe_ctx* c, int enable) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    c->prof = enable != 0;
    c->stats.clear();
    c->ev_names.clear();
    return MOE_OK;
}

int moe_profile_read(moe_ctx* c, moe_stage_stat* out, int max, int* n) {
    if (!c || !n) return fail(c, MOE_E_INVALID, "NULL argument");
    *n = static_cast<int>(c->stats.size());
    for (int i = 0; i < *n && i < max && out; ++i) {
        std::memset(&out[i], 0, sizeof(out[i]));
        std::snprintf(out[i].name, sizeof(out[i].name), "%s", c->stats[i].name.c_str());
        out[i].calls = c->stats[i].calls;
        out[i].total_ms = static_cast<float>(c->stats[i].total_ms);
    }
    return MOE_OK;
}

int moe_launch_count(moe_ctx* c, uint64_t* n) {
    if (!c || !n) return fail(c, MOE_E_INVALID, "NULL argument");
    *n = c->launches;
    return MOE_OK;
}

int moe_rms_norm(moe_ctx* c, uint64_t x_off, uint64_t y_off, uint32_t M, uint32_t H, float eps) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (M == 0) return MOE_OK;
    if (H == 0 || H % 4 != 0) return fail(c, MOE_E_INVALID, "H must be a positive multiple of 4");
    const uint64_t n = static_cast<uint64_t>(M) * H * 4;
    if (!off_ok(c, x_off, n, 16) || !off_ok(c, y_off, n, 16)) return fail(c, MOE_E_INVALID, "rms_norm offsets invalid");
    DeviceGuard g(c->device);
    moe::launch_rms_norm(at<float>(c, x_off), at<float>(c, y_off), static_cast<int>(M),
                         static_cast<int>(H), eps, c->stream);
    stage(c, "rms_norm", 1);
    return check_launch(c, "rms_norm");
}

int moe_vocab_logits(moe_ctx* c, uint64_t w_off, uint32_t V, uint32_t H, uint64_t x_off, uint32_t M,
                     uint64_t logits_off, uint64_t ids_off) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (M == 0 || V == 0) return MOE_OK;
    if (!moe::vocab_supported(static_cast<int>(H), static_cast<int>(M)))
        return fail(c, MOE_E_UNSUPPORTED, "vocab_logits: M=%u H=%u (need 1<=M<=8, H%%512==0, 512<=H<=4096)", M, H);
    if (V > 0x7FFFFFF0u) return fail(c, MOE_E_UNSUPPORTED, "vocab_logits: V=%u too large", V);
    if (logits_off == 0 && ids_off == 0) return fail(c, MOE_E_INVALID, "vocab_logits: no output");
    const uint64_t wb = static_cast<uint64_t>(V) * (H / 256) * 136;
    if (!off_ok(c, w_off, wb, 16)) return fail(c, MOE_E_INVALID, "vocab_logits weight offset invalid");
    if (!off_ok(c, x_off, static_cast<uint64_t>(M) * H * 4, 4))
        return fail(c, MOE_E_INVALID, "vocab_logits x offset invalid");
    if (logits_off && !off_ok(c, logits_off, static_cast<uint64_t>(M) * V * 4, 4))
        return fail(c, MOE_E_INVALID, "vocab_logits logits offset invalid");
    if (ids_off && !off_ok(c, ids_off, static_cast<uint64_t>(M) * 4, 4))
        return fail(c, MOE_E_INVALID, "vocab_logits ids offset invalid");
    DeviceGuard g(c->device);
    // argmax keys and the CTA ticket live in the status block, after the decode kernel's words
    uint8_t* sb = reinterpret_cast<uint8_t*>(c->ws.status);
    const int r = moe::launch_vocab(c->base + w_off, static_cast<int>(V), static_cast<int>(H),
                                    at<float>(c, x_off), static_cast<int>(M),
                                    logits_off ? at<float>(c, logits_off) : nullptr,
                                    ids_off ? at<uint32_t>(c, ids_off) : nullptr,
                                    reinterpret_cast<unsigned long long*>(sb + moe::kStatusVocabKeysOff),
                                    reinterpret_cast<unsigned int*>(sb + moe::kStatusVocabTicketOff), c->ws.status, c->sm_count,
                                    c->stream);
    if (r != 0) return fail(c, MOE_E_UNSUPPORTED, "vocab_logits: H=%u does not fit shared memory", H);
    stage(c, "vocab", 1);
    return check_launch(c, "vocab_logits");
}

int moe_silu_mul(moe_ctx* c, uint64_t g_off, uint64_t u_off, uint64_t y_off, uint64_t n) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (n == 0) return MOE_OK;
    if (!off_ok(c, g_off, n * 4, 4) || (u_off && !off_ok(c, u_off, n * 4, 4)) || !off_ok(c, y_off, n * 4, 4))
        return fail(c, MOE_E_INVALID, "silu_mul offsets invalid");
    DeviceGuard g(c->device);
    moe::launch_silu_mul(at<float>(c, g_off), u_off ? at<float>(c, u_off) : nullptr, at<float>(c, y_off), n,
                         c->sm_count, c->stream);
    stage(c, "silu_mul", 1);
    return check_launch(c, "silu_mul");
}

int moe_dequant_iq4xs(moe_ctx* c, uint64_t src_off, uint64_t n_blocks, uint64_t dst_off) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (n_blocks == 0) return MOE_OK;
    if (!off_ok(c, src_off, n_blocks * 136, 4) || !off_ok(c, dst_off, n_blocks * 1024, 4))
        return fail(c, MOE_E_INVALID, "dequant offsets invalid");
    DeviceGuard g(c->device);
    moe::launch_dequant(c->base + src_off, n_blocks, at<float>(c, dst_off), c->stream);
    return check_launch(c, "dequant");
}

int moe_dequant_ref36(moe_ctx* c, uint64_t src_off, uint64_t n_blocks, uint64_t dst_off) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (n_blocks == 0) return MOE_OK;
    if (!off_ok(c, src_off, n_blocks * 36, 4) || !off_ok(c, dst_off, n_blocks * 128, 4))
        return fail(c, MOE_E_INVALID, "dequant_ref36 offsets invalid");
    DeviceGuard g(c->device);
    moe::launch_dequant_ref36(c->base + src_off, n_blocks, at<float>(c, dst_off), c->stream);
    return check_launch(c, "dequant_ref36");
}

int moe_synth_iq4xs(moe_ctx* c, uint64_t dst_off, uint64_t key, uint64_t block_start,
                    uint64_t n_blocks) {
    if (!c) return fail(c, MOE_E_INVALID, "NULL context");
    if (n_blocks == 0) return MOE_OK;
    if (!off_ok(c, dst_off, n_blocks * 136, 8)) return fail(c, MOE_E_INVALID, "synth offset invalid");
    DeviceGuard g(c->device);
    moe::launch_synth(c->base + dst_off, key, block_start, n_blocks, c->stream);
    return check_launch(c, "synth");
}

}  // extern "C"
