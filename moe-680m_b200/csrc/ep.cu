// Expert-parallel prefill: the device side of the dispatch and combine around an all-to-all.
//
// Rank d of N owns experts [d*epr, (d+1)*epr), epr = E/N.  Every rank sends every peer a block
// of `capacity` rows (capacity >= the tokens of any rank), so the all-to-alls have fixed,
// equal splits: no count exchange and no host synchronisation, and a whole layer can be
// replayed from a CUDA graph.  For the M local tokens of rank r:
//   plan:    mask[t] = bit d set when one of token t's k routed experts lives on rank d, and
//            bit r always (the shared expert of r's own tokens runs on r); pos[t][d] = rank of
//            t among the tokens with bit d (token order);
//   gather:  send_x[d*capacity + pos[t][d]] = x[t] (f32 row, exact) and the token's routing
//            record keeping only rank d's experts (others kNoExpert), with the shared entry 0
//            kept for d == r and emptied otherwise; rows no token uses carry empty records;
//   combine: out[t] = resid[t] + scale * sum over d in mask, ascending, of the partial row
//            y_back[d*capacity + pos[t][d]] returned by rank d (sum_j w_j E_j(x) over d's
//            experts, plus gate * S(x) from rank r itself).
// The single-device reference has no counterpart; this follows the exchange steps of the
// expert-parallel layout (router -> per-rank histogram -> dispatch -> local grouped experts ->
// return of one partial row per (token, rank) -> ordered sum).
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

constexpr int kScanT = 1024;

__global__ void ep_mask_kernel(const uint2* __restrict__ topk, int M, int k, int epr, int n_ranks,
                               int my_rank, uint32_t* __restrict__ mask, int* status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= M) return;
    const uint2* rec = topk + static_cast<size_t>(t) * (k + 1);
    uint32_t m = 1u << my_rank;
    for (int s = 0; s < k; ++s) {
        const uint32_t e = rec[1 + s].x;
        if (e == kNoExpert) continue;
        const uint32_t d = e / static_cast<uint32_t>(epr);
        if (d >= static_cast<uint32_t>(n_ranks)) { set_dev_error(status, kDevBadExpert); continue; }
        m |= 1u << d;
    }
    mask[t] = m;
}

// One CTA: per rank d, exclusive scan of mask bit d over the tokens (each thread a contiguous
// run of tokens), pair counts and rank offsets.
__global__ void __launch_bounds__(kScanT) ep_scan_kernel(const uint32_t* __restrict__ mask, int M,
                                                         int n_ranks, int capacity, int* __restrict__ pos,
                                                         int* __restrict__ offsets) {
    __shared__ int wsum[kScanT / 32][kMaxEpRanks];
    __shared__ int tot[kMaxEpRanks];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (M + kScanT - 1) / kScanT;
    const int t0 = min(M, tid * per), t1 = min(M, t0 + per);
    int cnt[kMaxEpRanks];
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) cnt[d] = 0;
    for (int t = t0; t < t1; ++t) {
        const uint32_t m = mask[t];
#pragma unroll
        for (int d = 0; d < kMaxEpRanks; ++d) cnt[d] += (m >> d) & 1u;
    }
    // inclusive warp scan, then over warps
    int inc[kMaxEpRanks];
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) {
        int v = cnt[d];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += u;
        }
        inc[d] = v;
        if (lane == 31) wsum[warp][d] = v;
    }
    __syncthreads();
    if (tid < kMaxEpRanks) {
        int run = 0;
        for (int w = 0; w < kScanT / 32; ++w) {
            const int v = wsum[w][tid];
            wsum[w][tid] = run;
            run += v;
        }
        tot[tid] = run;
    }
    __syncthreads();
    int base[kMaxEpRanks];
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) base[d] = wsum[warp][d] + inc[d] - cnt[d];
    for (int t = t0; t < t1; ++t) {
        const uint32_t m = mask[t];
#pragma unroll
        for (int d = 0; d < kMaxEpRanks; ++d) {
            if (d < n_ranks) {
                pos[static_cast<size_t>(t) * n_ranks + d] = ((m >> d) & 1u) ? base[d] : -1;
                base[d] += (m >> d) & 1u;
            }
        }
    }
    if (tid == 0) {  // block d starts at d * capacity; offsets[n_ranks + d] = rows used in it
        for (int d = 0; d < n_ranks; ++d) {
            offsets[d] = d * capacity;
            offsets[n_ranks + d] = tot[d];
        }
    }
}

// Warp per token: its row and record to every rank it visits.
__global__ void ep_gather_kernel(const float* __restrict__ x, const uint2* __restrict__ topk,
                                 const uint32_t* __restrict__ mask, const int* __restrict__ pos,
                                 const int* __restrict__ offsets, int M, int H, int k, int epr,
                                 int n_ranks, int my_rank, float* __restrict__ send_x,
                                 uint2* __restrict__ send_rec) {
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= M) return;
    const uint32_t m = mask[t];
    if (!m) return;
    const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
    const uint2* rec = topk + static_cast<size_t>(t) * (k + 1);
    const uint2 r = lane <= k ? rec[lane] : make_uint2(0, 0);
    for (int d = 0; d < n_ranks; ++d) {
        if (!((m >> d) & 1u)) continue;
        const size_t p = static_cast<size_t>(offsets[d] + pos[static_cast<size_t>(t) * n_ranks + d]);
        float4* dst = reinterpret_cast<float4*>(send_x + p * H);
        for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
        if (lane <= k) {
            uint2 o = r;
            if (lane > 0) {
                const uint32_t e = r.x;
                o.x = (e != kNoExpert && e / static_cast<uint32_t>(epr) == static_cast<uint32_t>(d))
                          ? e : kNoExpert;
            } else if (d != my_rank) {
                o.x = kNoExpert;  // the shared expert runs on the token's own rank
            }
            send_rec[p * (k + 1) + lane] = o;
        }
    }
}

__global__ void ep_combine_kernel(const uint32_t* __restrict__ mask, const int* __restrict__ pos,
                                  const int* __restrict__ offsets, int n_ranks, int H,
                                  const float* __restrict__ y_back, const float* __restrict__ resid,
                                  float scale, float* __restrict__ out) {
    const int t = blockIdx.x;
    const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
    if (c >= H) return;
    const uint32_t m = mask[t];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < n_ranks; ++d) {
        if (!((m >> d) & 1u)) continue;
        const size_t p = static_cast<size_t>(offsets[d] + pos[static_cast<size_t>(t) * n_ranks + d]);
        const float4 y = *reinterpret_cast<const float4*>(y_back + p * H + c);
        acc.x += y.x; acc.y += y.y; acc.z += y.z; acc.w += y.w;
    }
    const size_t row = static_cast<size_t>(t) * H + c;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (resid) r = *reinterpret_cast<const float4*>(resid + row);
    r.x = fmaf(scale, acc.x, r.x); r.y = fmaf(scale, acc.y, r.y);
    r.z = fmaf(scale, acc.z, r.z); r.w = fmaf(scale, acc.w, r.w);
    *reinterpret_cast<float4*>(out + row) = r;
}

// ---- peer transport: rows and records stored straight into the owner ranks' receive blocks,
// partial rows read straight from the expert ranks' output blocks (NVLink loads/stores through
// CUDA IPC mappings; plain loads and stores only) --------------------------------------------

// CTA per (token, destination rank): the token's row and reduced record to block my_rank of
// rank d when the token visits d.  One CTA per pair (instead of one warp per token looping over
// its ranks) keeps thousands of NVLink stores in flight from every SM.
constexpr int kPushThreads = 128;

__global__ void __launch_bounds__(kPushThreads)
ep_push_kernel(const float* __restrict__ x, const uint2* __restrict__ topk, const uint32_t* __restrict__ mask,
               const int* __restrict__ pos, int M, int H, int k, int epr, int n_ranks, int my_rank, EpPeers P) {
    const int t = blockIdx.x, d = blockIdx.y, tid = threadIdx.x;
    if (t >= M || !((mask[t] >> d) & 1u)) return;
    const size_t p = static_cast<size_t>(pos[static_cast<size_t>(t) * n_ranks + d]);
    const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
    float4* dst = reinterpret_cast<float4*>(P.x[d] + p * H);
    for (int i = tid; i < H / 4; i += kPushThreads) dst[i] = __ldg(src + i);
    if (tid <= k) {
        uint2 o = topk[static_cast<size_t>(t) * (k + 1) + tid];
        if (tid > 0) {
            const uint32_t e = o.x;
            o.x = (e != kNoExpert && e / static_cast<uint32_t>(epr) == static_cast<uint32_t>(d)) ? e : kNoExpert;
        } else if (d != my_rank) {
            o.x = kNoExpert;  // the shared expert runs on the token's own rank
        }
        P.rec[d][p * (k + 1) + tid] = o;
    }
    __threadfence_system();
}

// Empty records for the rows [used_d, capacity) of block my_rank at every rank d (used_d from the
// scan's counts, or 0 when this rank has no tokens).
__global__ void ep_fill_kernel(const int* __restrict__ counts, int n_ranks, int capacity, int k, EpPeers P) {
    const int per = capacity * (k + 1);
    for (int d = 0; d < n_ranks; ++d) {
        const int used = counts ? counts[d] * (k + 1) : 0;
        for (int i = used + blockIdx.x * blockDim.x + threadIdx.x; i < per; i += gridDim.x * blockDim.x)
            P.rec[d][i] = make_uint2(kNoExpert, kNoExpert);
    }
    __threadfence_system();
}

// Publish step progress to every rank: flag[d] (this rank's slot at rank d) = epoch, after
// bumping the local epoch when `bump` (one bump per layer step).
__global__ void ep_signal_kernel(unsigned long long* epoch, int bump, int n_ranks, EpPeers P, int slot) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    const unsigned long long e = *epoch + static_cast<unsigned long long>(bump);
    if (bump) *epoch = e;
    for (int d = 0; d < n_ranks; ++d)
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(P.flag[slot][d]), "l"(e) : "memory");
}

// Wait until every rank has published this step to slot `slot` of this rank's flags (bounded:
// gives up after 1 s, records kDevTimeout and returns).
__global__ void ep_wait_kernel(const unsigned long long* flags, const unsigned long long* epoch, int n_ranks,
                               int* status) {
    const int d = threadIdx.x;
    if (d >= n_ranks) return;
    const unsigned long long e = *epoch;
    unsigned long long v, t0, now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (uint32_t i = 0;; ++i) {
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + d) : "memory");
        if (v >= e) break;
        if ((i & 255u) == 255u) {
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (now - t0 > 1000000000ull) { set_dev_error(status, kDevTimeout); break; }
        }
    }
}

// out[t] = resid[t] + scale * sum over the ranks d in mask (ascending) of the partial row that
// rank d computed for t, read from rank d's output block.
__global__ void ep_pull_combine_kernel(const uint32_t* __restrict__ mask, const int* __restrict__ pos,
                                       int n_ranks, int H, EpPeers P, const float* __restrict__ resid,
                                       float scale, float* __restrict__ out) {
    const int t = blockIdx.x;
    const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
    if (c >= H) return;
    const uint32_t m = mask[t];
    // every remote row is requested before any is added (the NVLink round trips overlap), then
    // the rows are summed in rank order
    float4 y[kMaxEpRanks];
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) {
        y[d] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (d < n_ranks && ((m >> d) & 1u)) {
            const size_t p = static_cast<size_t>(pos[static_cast<size_t>(t) * n_ranks + d]);
            y[d] = *reinterpret_cast<const float4*>(P.y[d] + p * H + c);
        }
    }
    const size_t row = static_cast<size_t>(t) * H + c;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (resid) r = *reinterpret_cast<const float4*>(resid + row);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) {
        if (d < n_ranks && ((m >> d) & 1u)) {
            acc.x += y[d].x; acc.y += y[d].y; acc.z += y[d].z; acc.w += y[d].w;
        }
    }
    r.x = fmaf(scale, acc.x, r.x); r.y = fmaf(scale, acc.y, r.y);
    r.z = fmaf(scale, acc.z, r.z); r.w = fmaf(scale, acc.w, r.w);
    *reinterpret_cast<float4*>(out + row) = r;
}

}  // namespace

void launch_ep_push(const float* x, const uint2* topk, EpPlan plan, int M, int H, int k, int epr, int n_ranks,
                    int my_rank, int capacity, const EpPeers& P, cudaStream_t s) {
    if (M > 0)
        ep_push_kernel<<<dim3(M, n_ranks), kPushThreads, 0, s>>>(x, topk, plan.mask, plan.pos, M, H, k, epr, n_ranks,
                                                                 my_rank, P);
    ep_fill_kernel<<<32, 256, 0, s>>>(M > 0 ? plan.offsets + n_ranks : nullptr, n_ranks, capacity, k, P);
}

void launch_ep_signal(unsigned long long* epoch, bool bump, int n_ranks, const EpPeers& P, int slot,
                      cudaStream_t s) {
    ep_signal_kernel<<<1, 32, 0, s>>>(epoch, bump ? 1 : 0, n_ranks, P, slot);
}

void launch_ep_wait(const unsigned long long* flags, const unsigned long long* epoch, int n_ranks, int* status,
                    cudaStream_t s) {
    ep_wait_kernel<<<1, 32, 0, s>>>(flags, epoch, n_ranks, status);
}

void launch_ep_pull_combine(EpPlan plan, int M, int n_ranks, int H, const EpPeers& P, const float* resid,
                            float scale, float* out, cudaStream_t s) {
    dim3 grid(M, (H / 4 + 255) / 256);
    ep_pull_combine_kernel<<<grid, 256, 0, s>>>(plan.mask, plan.pos, n_ranks, H, P, resid, scale, out);
}

void launch_ep_plan(const uint2* topk, int M, int k, int epr, int n_ranks, int my_rank, int capacity,
                    EpPlan plan, int* status, cudaStream_t s) {
    ep_mask_kernel<<<(M + 255) / 256, 256, 0, s>>>(topk, M, k, epr, n_ranks, my_rank, plan.mask, status);
    ep_scan_kernel<<<1, kScanT, 0, s>>>(plan.mask, M, n_ranks, capacity, plan.pos, plan.offsets);
}

void launch_ep_gather(const float* x, const uint2* topk, EpPlan plan, int M, int H, int k, int epr,
                      int n_ranks, int my_rank, float* send_x, uint2* send_rec, cudaStream_t s) {
    ep_gather_kernel<<<(M * 32 + 255) / 256, 256, 0, s>>>(x, topk, plan.mask, plan.pos, plan.offsets, M,
                                                         H, k, epr, n_ranks, my_rank, send_x, send_rec);
}

void launch_ep_combine(EpPlan plan, int M, int n_ranks, int H, const float* y_back, const float* resid,
                       float scale, float* out, cudaStream_t s) {
    dim3 grid(M, (H / 4 + 255) / 256);
    ep_combine_kernel<<<grid, 256, 0, s>>>(plan.mask, plan.pos, plan.offsets, n_ranks, H, y_back, resid,
                                           scale, out);
}

}  // namespace moe
