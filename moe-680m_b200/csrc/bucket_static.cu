// moe_bucket_static: the bucketing launch of moe_bucket for callers that cannot allocate device
// memory.  Some callers own no allocator at all (an engine that carves everything out of one
// arena it sized up front, code running where cudaMalloc is forbidden or would stall other
// streams, or a host that only hands over pre-allocated buffers); moe_bucket needs a context
// whose workspace it grows with cudaMalloc.  This variant keeps its scratch (per-tile expert
// counts, the chunk list and counters) in one file-scope device array of fixed size, so it
// never allocates.
//
// Limits and sharing: up to kStaticMaxTokens tokens, 256 experts, top-8.  The array lives on
// every GPU that loads this library until the process exits, and every call on that GPU uses
// the same array: calls whose work overlaps on the GPU (different streams, no ordering between
// them) race on it and must be serialised by the caller.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "moe_common.cuh"
#include "moe_internal.h"

namespace moe {
namespace {

constexpr uint32_t kStaticMaxTokens = 8192;  // the reference's largest prefill batch
constexpr uint32_t kStaticTiles = (kStaticMaxTokens + 255) / 256;
constexpr size_t kTileCntBytes = sizeof(int) * kStaticTiles * (kMaxExperts + 1);
constexpr uint32_t kStaticMaxChunks = (kStaticMaxTokens * (kMaxTopK + 1) + kGemvTok - 1) / kGemvTok +
                                      kMaxExperts + 1;
constexpr size_t kChunkOff = (kTileCntBytes + 255) / 256 * 256;
constexpr size_t kCounterOff = kChunkOff + (sizeof(Chunk) * kStaticMaxChunks + 255) / 256 * 256;
constexpr size_t kScratchBytes = kCounterOff + 256;  // about 190 KB

static __device__ __align__(256) uint8_t g_bucket_scratch[kScratchBytes];

// Device address of g_bucket_scratch in the current CUDA context.  The address is looked up
// with that context current and cached per context (a primary context recreated after
// cudaDeviceReset, or a second context on the same device, gets its own lookup), so a stale
// address of a destroyed context is never reused.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CUcontext current_context() {
    static std::atomic<CtxGetCurrentFn> fn{nullptr};
    CtxGetCurrentFn f = fn.load(std::memory_order_acquire);
    if (!f) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p)
            return nullptr;
        f = reinterpret_cast<CtxGetCurrentFn>(p);
        fn.store(f, std::memory_order_release);
    }
    CUcontext c = nullptr;
    return f(&c) == CUDA_SUCCESS ? c : nullptr;
}

constexpr int kCacheSlots = 64;
std::mutex g_cache_mu;
CUcontext g_cache_ctx[kCacheSlots];
uint8_t* g_cache_ptr[kCacheSlots];
int g_cache_n = 0;

uint8_t* scratch_for_current_context() {
    const CUcontext c = current_context();
    if (!c) return nullptr;
    std::lock_guard<std::mutex> lk(g_cache_mu);
    for (int i = 0; i < g_cache_n; ++i)
        if (g_cache_ctx[i] == c) return g_cache_ptr[i];
    void* q = nullptr;
    if (cudaGetSymbolAddress(&q, g_bucket_scratch) != cudaSuccess || !q) {
        cudaGetLastError();
        return nullptr;
    }
    // a full cache recycles the oldest slot (contexts that old are normally gone)
    const int slot = g_cache_n < kCacheSlots ? g_cache_n++ : 0;
    g_cache_ctx[slot] = c;
    g_cache_ptr[slot] = static_cast<uint8_t*>(q);
    return static_cast<uint8_t*>(q);
}

// The status code alone reports the failure (there is no context to hold a message).
int static_fail(int code, const char*) { return code; }

}  // namespace
}  // namespace moe

extern "C" {

int moe_bucket_static(uint32_t n_experts, uint32_t top_k, int has_shared, const void* topk,
                      uint32_t M, int32_t* ranges, int32_t* tokens, float* weights,
                      int32_t* slot_pos, void* stream) {
    using namespace moe;
    if (M == 0) return MOE_OK;
    if (!topk || !ranges || !tokens || !weights || !slot_pos)
        return static_fail(MOE_E_INVALID, "moe_bucket_static: NULL buffer");
    if (n_experts == 0 || n_experts > kMaxExperts || top_k == 0 || top_k > kMaxTopK || top_k > n_experts)
        return static_fail(MOE_E_UNSUPPORTED, "moe_bucket_static: n_experts must be 1..256 and top_k 1..min(8, n_experts)");
    if (M > kStaticMaxTokens)
        return static_fail(MOE_E_UNSUPPORTED,
                           "moe_bucket_static: M exceeds the fixed scratch limit of 8192 tokens");
    uint8_t* base = scratch_for_current_context();
    if (!base) return static_fail(MOE_E_CUDA, "moe_bucket_static: no current context or cudaGetSymbolAddress failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Nothing has to start at zero: the tile counts, the chunk list and the counters are fully
    // written by one launch before the next reads them.  There is no status word: nothing could
    // read it back without synchronising, so a routed id outside [0, E) is dropped (its slot_pos
    // is -1) and reported nowhere.
    Workspace ws;  // a view of the static array; nothing is allocated
    ws.tilecnt = reinterpret_cast<int*>(base);
    ws.chunks = reinterpret_cast<Chunk*>(base + kChunkOff);
    ws.max_chunks = kStaticMaxChunks;
    ws.counters = reinterpret_cast<int*>(base + kCounterOff);
    ws.tiles13 = nullptr;  // no tensor-core tile lists
    ws.tiles2 = nullptr;
    launch_bucket(static_cast<int>(n_experts), static_cast<int>(top_k), true, has_shared != 0,
                  static_cast<const uint2*>(topk), static_cast<int>(M), ws, ranges, tokens, weights,
                  slot_pos, nullptr, s);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return static_fail(MOE_E_CUDA, cudaGetErrorString(e));
    return MOE_OK;
}

}  // extern "C"
