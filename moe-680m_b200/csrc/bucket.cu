// Prefix-sum bucketing of (token, slot) pairs by expert (moe-680m src/router.rs:55-97,
// build_expert_batches), on the device and deterministic.
//
// Three launches:
//  1. count:   per 256-token tile, one warp per 32 tokens builds bitmasks mask[w][e] (bit =
//              lane whose token picked expert e); tile counts are popcounts.
//  2. scan:    per expert, exclusive scan over tiles; exclusive scan over experts -> ranges;
//              chunk list of the grouped expert kernels.
//  3. scatter: recomputes the masks; a slot's position is its tile offset plus the popcount of
//              the lower warps' masks and of the lower lanes of its own warp.  Positions are
//              therefore in token order inside each bucket (the reference's stable fill).
// A routed record whose expert id is kNoExpert (0xFFFFFFFF) is an empty slot: it gets no
// position (slot_pos -1); so does the shared slot of a token whose entry 0 has id kNoExpert.
// Expert-parallel ranks use them for experts another rank owns and for padding rows.
// Bucket E holds the shared expert: every token, in order (the reference instead counts the
// shared slot into bucket shared_id = 0, which it also uses for routed expert 0).
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"

#include <algorithm>

namespace moe {

namespace {

constexpr int kTile = 256;  // tokens per tile (8 warps x 32)
constexpr int kScanThreads = 288;  // >= kMaxExperts + 1, whole warps

__device__ __forceinline__ void build_masks(uint32_t* masks, int nb, const uint2* topk, int M,
                                            int E, int k, int routed, int has_shared, int* status) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 8 * nb; i += blockDim.x) masks[i] = 0u;
    __syncthreads();
    const int t = blockIdx.x * kTile + tid;
    if (t < M) {
        const uint2* rec = topk + static_cast<size_t>(t) * (k + 1);
        for (int s = 0; s < (routed ? k : 0); ++s) {
            if (rec[1 + s].x == kNoExpert) continue;  // empty slot
            const int e = static_cast<int>(rec[1 + s].x);
            if (e < 0 || e >= E) { set_dev_error(status, kDevBadExpert); continue; }
            atomicOr(&masks[warp * nb + e], 1u << lane);
        }
        if (has_shared && rec[0].x != kNoExpert) atomicOr(&masks[warp * nb + E], 1u << lane);
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kTile)
bucket_count_kernel(const uint2* __restrict__ topk, int M, int E, int k, int routed, int has_shared,
                    int* __restrict__ tilecnt, int* status) {
    extern __shared__ uint32_t masks[];  // [8][E+1]
    const int nb = E + 1;
    build_masks(masks, nb, topk, M, E, k, routed, has_shared, status);
    for (int e = threadIdx.x; e < nb; e += blockDim.x) {
        int c = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) c += __popc(masks[w * nb + e]);
        tilecnt[static_cast<size_t>(blockIdx.x) * nb + e] = c;
    }
}

// One CTA.  tilecnt[tile][e] -> absolute offset of tile's first slot in bucket e (in place);
// ranges[0..E+1]; chunks of at most kGemvTok tokens per bucket; tensor-core token tiles.
struct TileLists {
    TcTile* t13;
    int max13;
    TcTile* t2;
    int max2;
    int n13, n2;  // tokens per tile
};

// Block-wide exclusive scan of int4 values (one per thread), returns the block total.
__device__ __forceinline__ int4 block_exscan4(int4 v, int4* warp_tot, int4& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int4 inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ax = __shfl_up_sync(0xffffffffu, inc.x, o), ay = __shfl_up_sync(0xffffffffu, inc.y, o);
        const int az = __shfl_up_sync(0xffffffffu, inc.z, o), aw = __shfl_up_sync(0xffffffffu, inc.w, o);
        if (lane >= o) { inc.x += ax; inc.y += ay; inc.z += az; inc.w += aw; }
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int4 t = lane < nw ? warp_tot[lane] : make_int4(0, 0, 0, 0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ax = __shfl_up_sync(0xffffffffu, t.x, o), ay = __shfl_up_sync(0xffffffffu, t.y, o);
            const int az = __shfl_up_sync(0xffffffffu, t.z, o), aw = __shfl_up_sync(0xffffffffu, t.w, o);
            if (lane >= o) { t.x += ax; t.y += ay; t.z += az; t.w += aw; }
        }
        if (lane < nw) warp_tot[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    const int4 before = warp > 0 ? warp_tot[warp - 1] : make_int4(0, 0, 0, 0);
    total = warp_tot[nw - 1];
    return make_int4(before.x + inc.x - v.x, before.y + inc.y - v.y, before.z + inc.z - v.z,
                     before.w + inc.w - v.w);
}

// One CTA, one thread per bucket (blockDim >= E+1).  tilecnt[tile][e] -> absolute offset of
// the tile's first slot in bucket e (in place); ranges[0..E+1]; the chunk list of the CUDA-core
// kernels and the token-tile lists of the tensor-core kernels.
__global__ void __launch_bounds__(kScanThreads)
bucket_scan_kernel(int* __restrict__ tilecnt, int n_tiles, int E, int* __restrict__ ranges,
                   Chunk* __restrict__ chunks, int max_chunks, TileLists lists,
                   int* __restrict__ counters, int* status) {
    __shared__ int4 warp_tot[32];
    const int nb = E + 1;
    const int e = threadIdx.x;
    int cnt = 0;
    if (e < nb) {
        for (int tl = 0; tl < n_tiles; ++tl) {
            const int c = tilecnt[static_cast<size_t>(tl) * nb + e];
            tilecnt[static_cast<size_t>(tl) * nb + e] = cnt;
            cnt += c;
        }
    }
    const int4 v = make_int4(cnt, (cnt + kGemvTok - 1) / kGemvTok, (cnt + lists.n13 - 1) / lists.n13,
                             (cnt + lists.n2 - 1) / lists.n2);
    int4 total;
    const int4 first = block_exscan4(v, warp_tot, total);
    if (e < nb) {
        ranges[e] = first.x;
        for (int tl = 0; tl < n_tiles; ++tl) tilecnt[static_cast<size_t>(tl) * nb + e] += first.x;
        int ci = first.y;
        for (int s = 0; s < cnt && ci < max_chunks; s += kGemvTok, ++ci)
            chunks[ci] = Chunk{e, first.x + s, min(kGemvTok, cnt - s), 0};
        if (lists.t13) {
            int ti = first.z;
            for (int s = 0; s < cnt && ti < lists.max13; s += lists.n13, ++ti)
                lists.t13[ti] = TcTile{e, first.x + s, min(lists.n13, cnt - s), 0};
            ti = first.w;
            for (int s = 0; s < cnt && ti < lists.max2; s += lists.n2, ++ti)
                lists.t2[ti] = TcTile{e, first.x + s, min(lists.n2, cnt - s), 0};
        }
    }
    if (threadIdx.x == 0) {
        ranges[nb] = total.x;
        int c = total.y, a13 = total.z, a2 = total.w;
        if (c > max_chunks) { set_dev_error(status, kDevOverflow); c = max_chunks; }
        if (lists.t13) {  // without tile lists (moe_bucket_static) there is nothing to overflow
            if (a13 > lists.max13) { set_dev_error(status, kDevOverflow); a13 = lists.max13; }
            if (a2 > lists.max2) { set_dev_error(status, kDevOverflow); a2 = lists.max2; }
        } else {
            a13 = a2 = 0;
        }
        counters[0] = c;
        counters[1] = a13;
        counters[2] = a2;
    }
}

__global__ void __launch_bounds__(kTile)
bucket_scatter_kernel(const uint2* __restrict__ topk, int M, int E, int k, int routed, int has_shared,
                      const int* __restrict__ tileoff, int* __restrict__ sorted_tok,
                      float* __restrict__ sorted_w, int* __restrict__ slot_pos, int* status) {
    extern __shared__ uint32_t masks[];
    const int nb = E + 1;
    build_masks(masks, nb, topk, M, E, k, routed, has_shared, status);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = blockIdx.x * kTile + tid;
    if (t >= M) return;
    const int* off = tileoff + static_cast<size_t>(blockIdx.x) * nb;
    const uint32_t lt = (1u << lane) - 1u;
    const uint2* rec = topk + static_cast<size_t>(t) * (k + 1);
    const int ns = k + (has_shared ? 1 : 0);
    int* sp = slot_pos + static_cast<size_t>(t) * ns;
    for (int s = 0; s < ns; ++s) {
        const uint2 r = rec[s == k ? 0 : 1 + s];  // slot k: the shared expert, record entry 0
        int e;
        if (s == k) e = r.x == kNoExpert ? -1 : E;
        else e = (!routed || r.x >= static_cast<uint32_t>(E)) ? -1 : static_cast<int>(r.x);
        if (e < 0) { sp[s] = -1; continue; }
        int pos = off[e] + __popc(masks[warp * nb + e] & lt);
        for (int w = 0; w < warp; ++w) pos += __popc(masks[w * nb + e]);
        sorted_tok[pos] = t;
        sorted_w[pos] = __uint_as_float(r.y);
        sp[s] = pos;
    }
}

// ---- small batches: count, scan and scatter in one CTA ---------------------------------------
// For up to kSmallMaxTokens tokens one CTA of 1024 threads does all three steps (one launch
// instead of three), one token per thread: the token's routing record is read once into
// registers; per-warp bitmasks give each slot's rank among the earlier tokens exactly as in the
// three-launch path, so the results are identical.  The chunk and tile lists are written by all
// threads in parallel (entry -> bucket by binary search over the per-bucket list offsets).
constexpr int kSmallThreads = 1024;
constexpr int kSmallWarps = kSmallThreads / 32;
constexpr int kSmallMaxTokens = kSmallThreads;
constexpr int kSortMax = kSmallThreads;  // tile lists longer than this keep bucket order

// Stable sort of a tile list by token count, descending (one CTA; n <= kSortMax entries, else
// left as is): each entry's rank is the number of entries that precede it in the new order.
__device__ void sort_tiles(TcTile* list, int n, TcTile* buf, int* nbuf) {
    if (n > kSortMax) return;
    const int i = threadIdx.x;
    if (i < n) {
        buf[i] = list[i];
        nbuf[i] = list[i].n;
    }
    __syncthreads();
    if (i < n) {
        const int ni = nbuf[i];
        int r[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // independent partial counts
        int j = 0;
        for (; j + 8 <= n; j += 8) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int nj = nbuf[j + u];
                r[u] += (nj > ni || (nj == ni && j + u < i)) ? 1 : 0;
            }
        }
        for (; j < n; ++j) r[0] += (nbuf[j] > ni || (nbuf[j] == ni && j < i)) ? 1 : 0;
        const int rank = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        list[rank] = buf[i];
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kSmallThreads)
bucket_small_kernel(const uint2* __restrict__ topk, int M, int E, int k, int routed, int has_shared,
                    int* __restrict__ ranges, int* __restrict__ sorted_tok, float* __restrict__ sorted_w,
                    int* __restrict__ slot_pos, Chunk* __restrict__ chunks, int max_chunks, TileLists lists,
                    int* __restrict__ counters, int* status) {
    extern __shared__ uint32_t masks[];  // [32][E+1]
    // per bucket: first slot, first chunk, first gate/up tile, first down tile (+ totals at nb)
    __shared__ int4 first_s[kMaxExperts + 2];
    __shared__ int4 warp_tot[32];
    __shared__ TcTile tsort[kSortMax];
    __shared__ int tsort_n[kSortMax];
    const int nb = E + 1, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = tid;
    // the token's slots: bucket (or -1) and gate weight, read once
    int eb[kMaxTopK + 1];
    uint32_t wb[kMaxTopK + 1];
    {
        uint2 rec[kMaxTopK + 1];
#pragma unroll
        for (int i = 0; i <= kMaxTopK; ++i)
            rec[i] = (t < M && i <= k) ? topk[static_cast<size_t>(t) * (k + 1) + i] : make_uint2(kNoExpert, 0u);
#pragma unroll
        for (int s = 0; s <= kMaxTopK; ++s) {
            // slot s < k: routed entry 1 + s; slot k: the shared expert (record entry 0)
            const uint2 r = s < k ? rec[(1 + s) <= kMaxTopK ? 1 + s : kMaxTopK] : rec[0];
            int e = -1;
            if (s < k) {
                if (routed && r.x != kNoExpert) {
                    if (r.x >= static_cast<uint32_t>(E)) set_dev_error(status, kDevBadExpert);
                    else e = static_cast<int>(r.x);
                }
            } else if (s == k) {
                e = (has_shared && r.x != kNoExpert) ? E : -1;
            }
            eb[s] = t < M ? e : -1;
            wb[s] = r.y;
        }
    }
    for (int i = tid; i < kSmallWarps * nb; i += kSmallThreads) masks[i] = 0u;
    __syncthreads();
#pragma unroll
    for (int s = 0; s <= kMaxTopK; ++s)
        if (eb[s] >= 0) atomicOr(&masks[warp * nb + eb[s]], 1u << lane);
    __syncthreads();
    // 1. counts and 2. scan
    int c_e = 0;
    if (tid < nb) {
#pragma unroll 4
        for (int w = 0; w < kSmallWarps; ++w) c_e += __popc(masks[w * nb + tid]);
    }
    const int4 v = make_int4(c_e, (c_e + kGemvTok - 1) / kGemvTok, (c_e + lists.n13 - 1) / lists.n13,
                             (c_e + lists.n2 - 1) / lists.n2);
    int4 total;
    const int4 first = block_exscan4(v, warp_tot, total);
    if (tid < nb) {
        ranges[tid] = first.x;
        first_s[tid] = first;
    }
    if (tid == 0) {
        ranges[nb] = total.x;
        first_s[nb] = total;
        int c = total.y, a13 = total.z, a2 = total.w;
        if (c > max_chunks) { set_dev_error(status, kDevOverflow); c = max_chunks; }
        if (lists.t13) {
            if (a13 > lists.max13) { set_dev_error(status, kDevOverflow); a13 = lists.max13; }
            if (a2 > lists.max2) { set_dev_error(status, kDevOverflow); a2 = lists.max2; }
        } else {
            a13 = a2 = 0;
        }
        counters[0] = c;
        counters[1] = a13;
        counters[2] = a2;
    }
    __syncthreads();
    // chunk and tile lists, one entry per thread
    const int* fs = reinterpret_cast<const int*>(first_s);  // field f of bucket b at fs[4 * b + f]
    auto bucket_of = [&](int f, int i) {
        int lo = 0, hi = nb - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (fs[4 * mid + f] <= i) lo = mid;
            else hi = mid - 1;
        }
        return lo;
    };
    for (int ci = tid; ci < min(total.y, max_chunks); ci += kSmallThreads) {
        const int e = bucket_of(1, ci);
        const int q = (ci - fs[4 * e + 1]) * kGemvTok, cnt = fs[4 * (e + 1)] - fs[4 * e];
        chunks[ci] = Chunk{e, fs[4 * e] + q, min(kGemvTok, cnt - q), 0};
    }
    if (lists.t13) {
        for (int ti = tid; ti < min(total.z, lists.max13); ti += kSmallThreads) {
            const int e = bucket_of(2, ti);
            const int q = (ti - fs[4 * e + 2]) * lists.n13, cnt = fs[4 * (e + 1)] - fs[4 * e];
            lists.t13[ti] = TcTile{e, fs[4 * e] + q, min(lists.n13, cnt - q), 0};
        }
        for (int ti = tid; ti < min(total.w, lists.max2); ti += kSmallThreads) {
            const int e = bucket_of(3, ti);
            const int q = (ti - fs[4 * e + 3]) * lists.n2, cnt = fs[4 * (e + 1)] - fs[4 * e];
            lists.t2[ti] = TcTile{e, fs[4 * e] + q, min(lists.n2, cnt - q), 0};
        }
    }
    // the down-projection tile list largest first: that kernel deals items round robin and its
    // short items cost in proportion to their tile's token count (its epilogue), so the largest
    // tiles are spread over the first rounds (stable: equal sizes keep their order; the results
    // do not depend on it).  The gate/up list gained nothing from the same order (measured).
    if (lists.t2) {
        __syncthreads();  // the lists above are complete
        sort_tiles(lists.t2, min(total.w, lists.max2), tsort, tsort_n);
    }
    // 3. positions in token order
    if (t < M) {
        const uint32_t lt = (1u << lane) - 1u;
        const int ns = k + (has_shared ? 1 : 0);
        int* sp = slot_pos + static_cast<size_t>(t) * ns;
#pragma unroll
        for (int s = 0; s <= kMaxTopK; ++s) {
            if (s >= ns) break;
            const int e = eb[s];
            if (e < 0) { sp[s] = -1; continue; }
            int pos = fs[4 * e] + __popc(masks[warp * nb + e] & lt);
            for (int w = 0; w < warp; ++w) pos += __popc(masks[w * nb + e]);
            sorted_tok[pos] = t;
            sorted_w[pos] = __uint_as_float(wb[s]);
            sp[s] = pos;
        }
    }
}

// The bucketing of a shared-expert-only pass (no routing needed): bucket E holds every token
// in order, so slot position = token; tensor-core tiles of up to n13 / n2 tokens.
__global__ void shared_plan_kernel(int M, int E, int* __restrict__ ranges, int* __restrict__ sorted_tok,
                                   float* __restrict__ sorted_w, int* __restrict__ slot_pos, TileLists lists,
                                   int* __restrict__ counters) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < M) {
        sorted_tok[i] = i;
        sorted_w[i] = 1.0f;
        slot_pos[i] = i;
    }
    if (i <= E) ranges[i] = 0;
    if (i == 0) {
        ranges[E + 1] = M;
        int a13 = 0, a2 = 0;
        for (int q = 0; q < M && a13 < lists.max13; q += lists.n13, ++a13)
            lists.t13[a13] = TcTile{E, q, min(lists.n13, M - q), 0};
        for (int q = 0; q < M && a2 < lists.max2; q += lists.n2, ++a2)
            lists.t2[a2] = TcTile{E, q, min(lists.n2, M - q), 0};
        counters[0] = 0;
        counters[1] = a13;
        counters[2] = a2;
    }
}

}  // namespace

void launch_shared_plan(int E, int M, Workspace& ws, cudaStream_t s) {
    TileLists tl{ws.tiles13, static_cast<int>(ws.max_tiles13), ws.tiles2,
                 static_cast<int>(ws.max_tiles2), tc_max_n(13), tc_max_n(2)};
    const int n = std::max(M, E + 1);
    shared_plan_kernel<<<(n + 255) / 256, 256, 0, s>>>(M, E, ws.ranges, ws.sorted_tok, ws.sorted_w, ws.slot_pos,
                                                       tl, ws.counters);
}

void launch_bucket(int E, int k, bool routed, bool has_shared, const uint2* topk, int M, Workspace& ws,
                   int* ranges, int* sorted_tok, float* sorted_w, int* slot_pos, int* status,
                   cudaStream_t s) {
    TileLists tl{ws.tiles13, static_cast<int>(ws.max_tiles13), ws.tiles2,
                 static_cast<int>(ws.max_tiles2), tc_max_n(13), tc_max_n(2)};
    if (M <= kSmallMaxTokens) {  // one launch
        const size_t smem_s = static_cast<size_t>(kSmallWarps) * (E + 1) * sizeof(uint32_t);
        static bool attr_set[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64 || !attr_set[dev]) {
            cudaFuncSetAttribute(bucket_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmallWarps * (kMaxExperts + 1) * sizeof(uint32_t)));
            if (dev >= 0 && dev < 64) attr_set[dev] = true;
        }
        bucket_small_kernel<<<1, kSmallThreads, smem_s, s>>>(topk, M, E, k, routed ? 1 : 0, has_shared ? 1 : 0,
                                                             ranges, sorted_tok, sorted_w, slot_pos, ws.chunks,
                                                             static_cast<int>(ws.max_chunks), tl, ws.counters,
                                                             status);
        return;
    }
    const int n_tiles = (M + kTile - 1) / kTile;
    const size_t smem = 8 * (E + 1) * sizeof(uint32_t);
    bucket_count_kernel<<<n_tiles, kTile, smem, s>>>(topk, M, E, k, routed ? 1 : 0, has_shared ? 1 : 0,
                                                     ws.tilecnt, status);
    bucket_scan_kernel<<<1, kScanThreads, 0, s>>>(ws.tilecnt, n_tiles, E, ranges, ws.chunks,
                                          static_cast<int>(ws.max_chunks), tl, ws.counters, status);
    bucket_scatter_kernel<<<n_tiles, kTile, smem, s>>>(topk, M, E, k, routed ? 1 : 0, has_shared ? 1 : 0,
                                                       ws.tilecnt, sorted_tok, sorted_w, slot_pos,
                                                       status);
}

}  // namespace moe
