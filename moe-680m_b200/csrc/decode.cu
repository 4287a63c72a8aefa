// Fused single-token MoE layer (decode, M = 1): router, softmax + top-k, shared and routed
// SwiGLU experts and the weighted combine in one launch -- the whole per-token path of
// moe-680m's router.comp + router_topk.comp + do_route + the 18 w1_w3_fused / w2_scatter
// dispatches of record_and_submit_moe's decode branch (src/inference.rs:734-762).
//
// One CTA per SM, 16 warps.  Phases:
//   1. every warp computes router rows (x . Wr[e], f32; row E = the shared-expert gate g . x);
//      the last CTA to finish (ticket counter) does softmax + top-k and publishes the routing
//      by bumping a generation word;
//   2. gate/up work units (expert slot, row j): h[slot][j] = silu(W1[j].x) * (W3[j].x), slots
//      0..k-1 routed, slot k shared.  Warps start with the shared expert's units, which need no
//      routing, and wait for the routing generation before their first routed unit;
//   3. grid barrier, then out[n] = resid[n] + scale * sum_s w_s * (W2_s[n] . h_s).
// The ticket counter and the barrier reset themselves (generation scheme), so the kernel can be
// replayed from a CUDA graph.  Every spin wait gives up after 100 ms, records kDevTimeout in
// the status word and continues, so a broken launch cannot hang the GPU.
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

#ifdef MOE_TC_TRACE
__device__ unsigned long long g_dec_trace[4][8];  // CTAs 0..3: phase timestamps (debug builds)
#define DEC_TRACE(i) do { if (blockIdx.x < 4 && threadIdx.x == 0) g_dec_trace[blockIdx.x][i] = tc::globaltimer_ns(); } while (0)
extern "C" int moe_debug_dec_trace(unsigned long long* out) {
    return cudaMemcpyFromSymbol(out, g_dec_trace, sizeof(g_dec_trace)) == cudaSuccess ? 0 : -2;
}
#else
#define DEC_TRACE(i) do {} while (0)
#endif

namespace {

constexpr int kDWarps = 16;
constexpr uint64_t kSpinLimitNs = 100000000ull;  // 100 ms

struct DecodeArgs {
    const IoArgs* io;
    const float* wr;      // [E][H]
    const float* bias;    // [E] or null
    const float* gate_w;  // [H] or null (gate 1.0)
    ExpertTables tabs;
    int H, I, E, k;
    int has_shared;
    float scale;
    float* logits;        // [E+1]
    uint2* topk;          // [k+1] records
    float* h;             // [k+1][I]
    int* sync;            // [0] ticket, [1] routing generation, [2] barrier count, [3] barrier gen
    int* status;
};

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Wait until *gen differs from `seen` (bounded).
__device__ __forceinline__ void wait_gen(const int* gen, int seen, int* status) {
    if (ld_volatile(gen) != seen) return;
    const uint64_t t0 = tc::globaltimer_ns();
    while (ld_volatile(gen) == seen) {
        __nanosleep(64);
        if (tc::globaltimer_ns() - t0 > kSpinLimitNs) { set_dev_error(status, kDevTimeout); return; }
    }
}

// Grid barrier (every CTA calls it once per launch); thread 0 of each CTA takes part.
__device__ void grid_barrier(int* count, int* gen, int* status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const int seen = ld_volatile(gen);
        __threadfence();
        if (atomicAdd(count, 1) == static_cast<int>(gridDim.x) - 1) {
            *reinterpret_cast<volatile int*>(count) = 0;
            __threadfence();
            atomicAdd(gen, 1);
        } else {
            wait_gen(gen, seen, status);
        }
        __threadfence();
    }
    __syncthreads();
}

// Dot of one IQ4_XS row (K = nsb sub-blocks of 32) with padded activations in shared memory.
__device__ __forceinline__ float row_dot(const uint8_t* row, const float* xs, int nsb, int lane) {
    float acc = 0.f;
    for (int sb = lane; sb < nsb; sb += 32) {
        const SubBlk s = load_subblk(row, sb);
        acc = fmaf(iq4_subscale(s.hdr.x, s.hdr.y, sb & 7), dot_subblk(s, xs + sb * 36), acc);
    }
    return warp_sum(acc);
}

__global__ void __launch_bounds__(32 * kDWarps, 1) decode_kernel(const DecodeArgs a) {
    extern __shared__ __align__(16) float sm[];
    float* xs = sm;                          // padded x [H]
    float* hs = sm + padded_len(a.H);        // padded h [k+1][I] (phase 3)
    __shared__ int route_seen;
    __shared__ int eid[kMaxTopK + 1];
    __shared__ float wgt[kMaxTopK + 1];
    __shared__ const uint8_t* p1[kMaxTopK + 1];
    __shared__ const uint8_t* p3[kMaxTopK + 1];
    __shared__ const uint8_t* p2[kMaxTopK + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gwarp = blockIdx.x * kDWarps + warp, nwarps = gridDim.x * kDWarps;
    const float* x = a.io->x;
    const int H = a.H, I = a.I, E = a.E, k = a.k;
    const int ns = k + (a.has_shared ? 1 : 0);

    DEC_TRACE(0);
    if (threadIdx.x == 0) route_seen = ld_volatile(&a.sync[1]);
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(xs + padded_idx(i)) = *reinterpret_cast<const float4*>(x + i);
    __syncthreads();

    // ---- phase 1: router rows, each split in 4 column quarters ------------------------------
    const int n_rows = E + (a.gate_w ? 1 : 0);
    const int qlen = H / 4;
    for (int w = gwarp; w < n_rows * 4; w += nwarps) {
        const int r = w >> 2, part = w & 3;
        const float* wrow = (r < E ? a.wr + static_cast<size_t>(r) * H : a.gate_w) + part * qlen;
        float acc = 0.f;
        for (int i = lane * 4; i < qlen; i += 128) {
            const float4 wv = __ldg(reinterpret_cast<const float4*>(wrow + i));
            const float4 xv = *reinterpret_cast<const float4*>(xs + padded_idx(part * qlen + i));
            acc = fmaf(wv.x, xv.x, acc); acc = fmaf(wv.y, xv.y, acc);
            acc = fmaf(wv.z, xv.z, acc); acc = fmaf(wv.w, xv.w, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) a.logits[part * (E + 1) + r] = acc;
    }
    __syncthreads();
    DEC_TRACE(1);
    if (threadIdx.x == 0) {
        __threadfence();
        const bool last = atomicAdd(&a.sync[0], 1) == static_cast<int>(gridDim.x) - 1;
        route_seen = last ? -1 - route_seen : route_seen;  // negative: this CTA routes
    }
    __syncthreads();
    if (route_seen < 0 && warp == 0) {
        // softmax + top-k over the E logits (router_topk.comp:36-92), ties to the lower index;
        // the four quarter sums of a logit are added in a fixed order
        __threadfence();
        float p[8];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            float l = -INFINITY;
            if (e < E) {
                l = ((__ldcg(a.logits + e) + __ldcg(a.logits + (E + 1) + e)) + __ldcg(a.logits + 2 * (E + 1) + e)) +
                    __ldcg(a.logits + 3 * (E + 1) + e);
                if (a.bias) l += a.bias[e];
            }
            p[i] = l;
            mx = fmaxf(mx, l);
        }
        mx = warp_max(mx);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) { p[i] = lane + 32 * i < E ? expf(p[i] - mx) : 0.f; sum += p[i]; }
        sum = warp_sum(sum);
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = lane + 32 * i < E ? (sum > 0.f ? p[i] / sum : 0.f) : -1.f;
        for (int r = 0; r < k; ++r) {
            float bv = -2.f;
            int bi = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < 8; ++i) if (p[i] > bv) { bv = p[i]; bi = lane + 32 * i; }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (bi >= E) { set_dev_error(a.status, kDevBadExpert); bi = 0; }
            if ((bi & 31) == lane) {
#pragma unroll
                for (int i = 0; i < 8; ++i) if (lane + 32 * i == bi) p[i] = -3.f;
            }
            if (lane == 0) a.topk[1 + r] = make_uint2(static_cast<uint32_t>(bi), __float_as_uint(bv));
        }
        if (lane == 0) {
            float g = 1.0f;
            if (a.gate_w) {
                const int e = E;
                const float z = ((__ldcg(a.logits + e) + __ldcg(a.logits + (E + 1) + e)) +
                                 __ldcg(a.logits + 2 * (E + 1) + e)) + __ldcg(a.logits + 3 * (E + 1) + e);
                g = 1.0f / (1.0f + expf(-z));
            }
            a.topk[0] = make_uint2(static_cast<uint32_t>(E), __float_as_uint(g));
            a.sync[0] = 0;
            __threadfence();
            atomicAdd(&a.sync[1], 1);  // publish the routing
        }
    }
    const int seen = route_seen < 0 ? -1 - route_seen : route_seen;

    // ---- phase 2: gate/up units ------------------------------------------------------------
    // Per-slot weight pointers and combine weights are cached in shared memory; each warp
    // issues the loads of its next unit before computing the current one.
    const size_t rb13 = static_cast<size_t>(H / kQK) * kBlockBytes;
    const int nsb_h = H / 32;  // <= 64: two sub-blocks per lane at most
    if (threadIdx.x == 0 && a.has_shared) {
        p1[k] = a.tabs.w1[E]; p3[k] = a.tabs.w3[E]; p2[k] = a.tabs.w2[E];
    }
    __syncthreads();
    auto load_unit = [&](const uint8_t* r1, const uint8_t* r3, SubBlk (&b1)[2], SubBlk (&b3)[2]) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int sb = lane + 32 * i;
            if (sb < nsb_h) { b1[i] = load_subblk(r1, sb); b3[i] = load_subblk(r3, sb); }
        }
    };
    auto finish_unit = [&](int slot, int j, const SubBlk (&b1)[2], const SubBlk (&b3)[2]) {
        float g = 0.f, up = 0.f;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int sb = lane + 32 * i;
            if (sb < nsb_h) {
                g = fmaf(iq4_subscale(b1[i].hdr.x, b1[i].hdr.y, sb & 7), dot_subblk(b1[i], xs + sb * 36), g);
                up = fmaf(iq4_subscale(b3[i].hdr.x, b3[i].hdr.y, sb & 7), dot_subblk(b3[i], xs + sb * 36), up);
            }
        }
        g = warp_sum(g);
        up = warp_sum(up);
        if (lane == 0) a.h[static_cast<size_t>(slot) * I + j] = silu_f(g) * up;
    };
    // runs units u = first, first+nwarps, ... < n of slot(u) = slot0 + u / I, row u % I
    auto run_units = [&](int n, int slot0) {
        SubBlk c1[2], c3[2], n1[2], n3[2];
        int u = gwarp;
        if (u < n) { const int sl = slot0 + u / I, j = u % I; load_unit(p1[sl] + j * rb13, p3[sl] + j * rb13, c1, c3); }
        for (; u < n; u += nwarps) {
            const int un = u + nwarps;
            if (un < n) { const int sl = slot0 + un / I, j = un % I; load_unit(p1[sl] + j * rb13, p3[sl] + j * rb13, n1, n3); }
            finish_unit(slot0 + u / I, u % I, c1, c3);
#pragma unroll
            for (int i = 0; i < 2; ++i) { c1[i] = n1[i]; c3[i] = n3[i]; }
        }
    };
    if (a.has_shared) run_units(I, k);  // the shared expert needs no routing
    if (threadIdx.x == 0) {
        wait_gen(&a.sync[1], seen, a.status);
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x < ns) {
        const int s2 = threadIdx.x;  // slots 0..k-1 routed, k shared (record 0)
        const uint2 r = __ldcg(reinterpret_cast<const uint2*>(a.topk) + (s2 < k ? 1 + s2 : 0));
        int e = s2 < k ? static_cast<int>(r.x) : E;
        if (e < 0 || e > E) { set_dev_error(a.status, kDevBadExpert); e = 0; }
        eid[s2] = e;
        wgt[s2] = __uint_as_float(r.y);
        if (s2 < k) { p1[s2] = a.tabs.w1[e]; p3[s2] = a.tabs.w3[e]; p2[s2] = a.tabs.w2[e]; }
    }
    __syncthreads();
    run_units(k * I, 0);
    DEC_TRACE(2);
    grid_barrier(&a.sync[2], &a.sync[3], a.status);
    DEC_TRACE(3);

    // ---- phase 3: down projection + weighted combine + residual ----------------------------
    for (int i = threadIdx.x * 4; i < ns * I; i += blockDim.x * 4) {
        const int s = i / I, c = i - s * I;
        *reinterpret_cast<float4*>(hs + s * padded_len(I) + padded_idx(c)) =
            __ldcg(reinterpret_cast<const float4*>(a.h + static_cast<size_t>(s) * I + c));
    }
    __syncthreads();
    const int spr = I / 32, rpi = 32 / spr;  // sub-blocks per W2 row; rows per warp pass
    const int r_in = lane / spr, sb = lane - r_in * spr;
    const size_t rb2 = static_cast<size_t>(I / kQK) * kBlockBytes;
    const float* resid = a.io->resid;
    float* out = a.io->out;
    for (int n0 = gwarp * rpi; n0 < H; n0 += nwarps * rpi) {
        const int n = n0 + r_in;
        // the 9 experts' sub-blocks of row n are loaded together, then reduced in slot order
        SubBlk b[kMaxTopK + 1];
#pragma unroll
        for (int s = 0; s < kMaxTopK + 1; ++s)
            if (s < ns) b[s] = load_subblk(p2[s] + n * rb2, sb);
        float y = 0.f;
#pragma unroll
        for (int s = 0; s < kMaxTopK + 1; ++s) {
            if (s < ns) {
                const float d = iq4_subscale(b[s].hdr.x, b[s].hdr.y, sb & 7) *
                                dot_subblk(b[s], hs + s * padded_len(I) + sb * 36);
                y = fmaf(wgt[s], d, y);
            }
        }
        for (int o = spr >> 1; o > 0; o >>= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (sb == 0 && n < H) out[n] = (resid ? resid[n] : 0.f) + a.scale * y;
    }
    __syncthreads();
    DEC_TRACE(4);
}

}  // namespace

bool decode_supported(const Layer& L) {
    return L.spec.hidden <= 2048 && L.spec.inter >= 256 && L.spec.inter <= 1024 &&
           L.spec.n_experts <= kMaxExperts;
}

void launch_decode(const Layer& L, const Workspace& ws, int* sync, int sm_count, cudaStream_t s) {
    DecodeArgs a;
    a.io = ws.io;
    a.wr = reinterpret_cast<const float*>(L.router_w_ptr);
    a.bias = reinterpret_cast<const float*>(L.bias_ptr);
    a.gate_w = reinterpret_cast<const float*>(L.gate_ptr);
    a.tabs = L.tables();
    a.H = static_cast<int>(L.spec.hidden);
    a.I = static_cast<int>(L.spec.inter);
    a.E = static_cast<int>(L.spec.n_experts);
    a.k = static_cast<int>(L.spec.top_k);
    a.has_shared = L.has_shared() ? 1 : 0;
    a.scale = L.spec.scale;
    a.logits = ws.logits;
    a.topk = ws.topk;
    a.h = ws.h;
    a.sync = sync;
    a.status = ws.status;
    const size_t smem = sizeof(float) * (padded_len(a.H) + (kMaxTopK + 1) * padded_len(a.I));
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    decode_kernel<<<sm_count, 32 * kDWarps, smem, s>>>(a);
}

}  // namespace moe
