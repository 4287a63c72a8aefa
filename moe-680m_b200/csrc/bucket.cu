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
// Bucket E holds the shared expert: every token, in order (the reference instead counts the
// shared slot into bucket shared_id = 0, which it also uses for routed expert 0).
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

constexpr int kTile = 256;  // tokens per tile (8 warps x 32)

__device__ __forceinline__ void build_masks(uint32_t* masks, int nb, const uint2* topk, int M,
                                            int E, int k, int* status) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 8 * nb; i += blockDim.x) masks[i] = 0u;
    __syncthreads();
    const int t = blockIdx.x * kTile + tid;
    if (t < M) {
        const uint2* rec = topk + static_cast<size_t>(t) * (k + 1);
        for (int s = 0; s < k; ++s) {
            const int e = static_cast<int>(rec[1 + s].x);
            if (e < 0 || e >= E) { set_dev_error(status, kDevBadExpert); continue; }
            atomicOr(&masks[warp * nb + e], 1u << lane);
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kTile)
bucket_count_kernel(const uint2* __restrict__ topk, int M, int E, int k, int has_shared,
                    int* __restrict__ tilecnt, int* status) {
    extern __shared__ uint32_t masks[];  // [8][E+1]
    const int nb = E + 1;
    build_masks(masks, nb, topk, M, E, k, status);
    const int tile_tokens = min(kTile, M - static_cast<int>(blockIdx.x) * kTile);
    for (int e = threadIdx.x; e < nb; e += blockDim.x) {
        int c = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) c += __popc(masks[w * nb + e]);
        if (e == E && has_shared) c = tile_tokens;
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

__global__ void __launch_bounds__(1024)
bucket_scan_kernel(int* __restrict__ tilecnt, int n_tiles, int E, int* __restrict__ ranges,
                   Chunk* __restrict__ chunks, int max_chunks, TileLists lists,
                   int* __restrict__ counters, int* status) {
    __shared__ int tot[kMaxExperts + 2];
    __shared__ int nch[kMaxExperts + 2];
    __shared__ int f13[kMaxExperts + 2];
    __shared__ int f2[kMaxExperts + 2];
    const int nb = E + 1;
    for (int e = threadIdx.x; e < nb; e += blockDim.x) {
        int run = 0;
        for (int tl = 0; tl < n_tiles; ++tl) {
            const int c = tilecnt[static_cast<size_t>(tl) * nb + e];
            tilecnt[static_cast<size_t>(tl) * nb + e] = run;
            run += c;
        }
        tot[e] = run;
        nch[e] = (run + kGemvTok - 1) / kGemvTok;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int r = 0, c = 0, a13 = 0, a2 = 0;
        for (int e = 0; e < nb; ++e) {
            ranges[e] = r;
            const int cnt = tot[e];
            r += cnt;
            const int n = nch[e];
            nch[e] = c;  // first chunk index of bucket e
            c += n;
            f13[e] = a13;
            a13 += (cnt + lists.n13 - 1) / lists.n13;
            f2[e] = a2;
            a2 += (cnt + lists.n2 - 1) / lists.n2;
            tot[e] = ranges[e];
        }
        ranges[nb] = r;
        if (c > max_chunks) { set_dev_error(status, kDevOverflow); c = max_chunks; }
        if (a13 > lists.max13) { set_dev_error(status, kDevOverflow); a13 = lists.max13; }
        if (a2 > lists.max2) { set_dev_error(status, kDevOverflow); a2 = lists.max2; }
        counters[0] = c;
        counters[1] = a13;
        counters[2] = a2;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nb; e += blockDim.x) {
        const int base = tot[e];
        for (int tl = 0; tl < n_tiles; ++tl) tilecnt[static_cast<size_t>(tl) * nb + e] += base;
        const int cnt = ranges[e + 1] - ranges[e];
        int ci = nch[e];
        for (int s = 0; s < cnt; s += kGemvTok, ++ci) {
            if (ci >= max_chunks) break;
            chunks[ci] = Chunk{e, ranges[e] + s, min(kGemvTok, cnt - s), 0};
        }
        if (lists.t13) {
            int ti = f13[e];
            for (int s = 0; s < cnt && ti < lists.max13; s += lists.n13, ++ti)
                lists.t13[ti] = TcTile{e, ranges[e] + s, min(lists.n13, cnt - s), 0};
            ti = f2[e];
            for (int s = 0; s < cnt && ti < lists.max2; s += lists.n2, ++ti)
                lists.t2[ti] = TcTile{e, ranges[e] + s, min(lists.n2, cnt - s), 0};
        }
    }
}

__global__ void __launch_bounds__(kTile)
bucket_scatter_kernel(const uint2* __restrict__ topk, int M, int E, int k, int has_shared,
                      const int* __restrict__ tileoff, int* __restrict__ sorted_tok,
                      float* __restrict__ sorted_w, int* __restrict__ slot_pos, int* status) {
    extern __shared__ uint32_t masks[];
    const int nb = E + 1;
    build_masks(masks, nb, topk, M, E, k, status);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = blockIdx.x * kTile + tid;
    if (t >= M) return;
    const int* off = tileoff + static_cast<size_t>(blockIdx.x) * nb;
    const uint32_t lt = (1u << lane) - 1u;
    const uint2* rec = topk + static_cast<size_t>(t) * (k + 1);
    const int ns = k + (has_shared ? 1 : 0);
    int* sp = slot_pos + static_cast<size_t>(t) * ns;
    for (int s = 0; s < k; ++s) {
        const int e = static_cast<int>(rec[1 + s].x);
        if (e < 0 || e >= E) { sp[s] = -1; continue; }
        int pos = off[e] + __popc(masks[warp * nb + e] & lt);
        for (int w = 0; w < warp; ++w) pos += __popc(masks[w * nb + e]);
        sorted_tok[pos] = t;
        sorted_w[pos] = __uint_as_float(rec[1 + s].y);
        sp[s] = pos;
    }
    if (has_shared) {
        const int pos = off[E] + tid;
        sorted_tok[pos] = t;
        sorted_w[pos] = __uint_as_float(rec[0].y);
        sp[k] = pos;
    }
}

}  // namespace

void launch_bucket(int E, int k, bool has_shared, const uint2* topk, int M, Workspace& ws,
                   int* ranges, int* sorted_tok, float* sorted_w, int* slot_pos, int* status,
                   cudaStream_t s) {
    const int n_tiles = (M + kTile - 1) / kTile;
    const size_t smem = 8 * (E + 1) * sizeof(uint32_t);
    bucket_count_kernel<<<n_tiles, kTile, smem, s>>>(topk, M, E, k, has_shared ? 1 : 0,
                                                     ws.tilecnt, status);
    TileLists tl{ws.tiles13, static_cast<int>(ws.max_tiles13), ws.tiles2,
                 static_cast<int>(ws.max_tiles2), tc_max_n(13), tc_max_n(2)};
    bucket_scan_kernel<<<1, 1024, 0, s>>>(ws.tilecnt, n_tiles, E, ranges, ws.chunks,
                                          static_cast<int>(ws.max_chunks), tl, ws.counters, status);
    bucket_scatter_kernel<<<n_tiles, kTile, smem, s>>>(topk, M, E, k, has_shared ? 1 : 0,
                                                       ws.tilecnt, sorted_tok, sorted_w, slot_pos,
                                                       status);
}

}  // namespace moe
