// Router projection, softmax and top-k (moe-680m shaders/router.comp, shaders/router_topk.comp,
// src/router.rs:23-51).
//
// logits[t][e] = x[t] . Wr[e] (+ bias[e]) for e < E, and logits[t][E] = x[t] . g (the shared
// expert gate) when the layer has one.  Both are f32 with f32 accumulation.  Every output is
// produced by the same fixed-order reduction whatever its row or column, so identical router
// rows give bit-identical logits (ties are then real ties, broken toward the lower index).
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

// ---- small M: one warp per (router row, block of up to 8 tokens) ---------------------------
constexpr int kRowsPerCta = 4;  // warps per CTA

template <int TOK>
__global__ void __launch_bounds__(32 * kRowsPerCta)
router_gemv_kernel(const IoArgs* __restrict__ io, int M, int H, const float* __restrict__ wr,
                   const float* __restrict__ gate_w, int E, int n_rows,
                   float* __restrict__ logits) {
    const float* __restrict__ x = io->x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kRowsPerCta + warp;
    const int t0 = blockIdx.y * TOK;
    if (row >= n_rows) return;
    const float* w = row < E ? wr + static_cast<size_t>(row) * H : gate_w;
    float acc[TOK];
#pragma unroll
    for (int t = 0; t < TOK; ++t) acc[t] = 0.f;
    const int nt = min(TOK, M - t0);
    const int n4 = H / 4;
    for (int i = lane; i < n4; i += 32) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + i);
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
            if (t < nt) {
                const float4 xv =
                    __ldg(reinterpret_cast<const float4*>(x + static_cast<size_t>(t0 + t) * H) + i);
                acc[t] = fmaf(wv.x, xv.x, acc[t]);
                acc[t] = fmaf(wv.y, xv.y, acc[t]);
                acc[t] = fmaf(wv.z, xv.z, acc[t]);
                acc[t] = fmaf(wv.w, xv.w, acc[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < TOK; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0 && t < nt) logits[static_cast<size_t>(t0 + t) * (E + 1) + row] = v;
    }
}

// ---- larger M: 64x64 register-tiled SGEMM with a K split ------------------------------------
// partial[ks][t][e] over K range ks; the top-k kernel sums the splits in order.
constexpr int kTM = 64, kTE = 64, kTK = 16;

__global__ void __launch_bounds__(256)
router_gemm_kernel(const IoArgs* __restrict__ io, int M, int H, const float* __restrict__ wr,
                   const float* __restrict__ gate_w, int E, int n_rows, int k_len,
                   float* __restrict__ partial) {
    const float* __restrict__ x = io->x;
    __shared__ __align__(16) float xs[kTK][kTM + 4];
    __shared__ __align__(16) float ws[kTK][kTE + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;  // tx: experts, ty: tokens
    const int t0 = blockIdx.x * kTM, e0 = blockIdx.y * kTE;
    const int kbeg = blockIdx.z * k_len;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    // loader mapping: 64 rows x 16 k = 256 float4 -> one float4 per thread
    const int lr = tid >> 2, lk = (tid & 3) * 4;
    const int xt = t0 + lr, we = e0 + lr;
    const float* xrow = xt < M ? x + static_cast<size_t>(xt) * H : nullptr;
    const float* wrow = we < E ? wr + static_cast<size_t>(we) * H : (we < n_rows ? gate_w : nullptr);

    for (int k0 = kbeg; k0 < kbeg + k_len; k0 += kTK) {
        float4 xv = make_float4(0.f, 0.f, 0.f, 0.f), wv = xv;
        if (xrow) xv = __ldg(reinterpret_cast<const float4*>(xrow + k0 + lk));
        if (wrow) wv = __ldg(reinterpret_cast<const float4*>(wrow + k0 + lk));
        __syncthreads();
        xs[lk + 0][lr] = xv.x; xs[lk + 1][lr] = xv.y; xs[lk + 2][lr] = xv.z; xs[lk + 3][lr] = xv.w;
        ws[lk + 0][lr] = wv.x; ws[lk + 1][lr] = wv.y; ws[lk + 2][lr] = wv.z; ws[lk + 3][lr] = wv.w;
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kTK; ++kk) {
            const float4 a = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
    }
    float* out = partial + static_cast<size_t>(blockIdx.z) * M * (E + 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + tx * 4 + j;
            if (e < n_rows) out[static_cast<size_t>(t) * (E + 1) + e] = acc[i][j];
        }
    }
}

// ---- softmax + top-k: one warp per token ----------------------------------------------------
// Probabilities p = exp(l - max) / sum (router_topk.comp:36-60).  Top-k keeps the k largest p,
// descending, ties toward the lower expert index (strict '>' insertion, router_topk.comp:67-85).
template <int NS>
__global__ void __launch_bounds__(128)
topk_kernel(const float* __restrict__ partial, int M, int E, int k,
            const float* __restrict__ bias, int shared_mode, int gate_in_logits,
            const IoArgs* __restrict__ io, const float* __restrict__ gate_w, int H,
            uint2* __restrict__ topk, int* status) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const int t = warp;
    // all NS x 8 partial loads are independent; the splits are then added in a fixed order
    float part[NS][8];
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            part[s][i] = e < E ? partial[(static_cast<size_t>(s) * M + t) * (E + 1) + e] : 0.f;
        }
    float p[8];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        float l = -INFINITY;
        if (e < E) {
            l = 0.f;
#pragma unroll
            for (int s = 0; s < NS; ++s) l += part[s][i];
            if (bias) l += bias[e];
        }
        p[i] = l;
        mx = fmaxf(mx, l);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        p[i] = e < E ? expf(p[i] - mx) : 0.f;
        sum += p[i];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        p[i] = e < E ? (sum > 0.f ? p[i] / sum : 0.f) : -1.f;
    }
    uint2* rec = topk + static_cast<size_t>(t) * (k + 1);
    for (int r = 0; r < k; ++r) {
        float bv = -2.f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (p[i] > bv) { bv = p[i]; bi = lane + 32 * i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (bi >= E) { set_dev_error(status, kDevBadExpert); bi = 0; }
        if ((bi & 31) == lane) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (lane + 32 * i == bi) p[i] = -3.f;  // taken
        }
        if (lane == 0) rec[1 + r] = make_uint2(static_cast<uint32_t>(bi), __float_as_uint(bv));
    }
    float g = 1.0f;
    if (shared_mode == 2) {
        float z = 0.f;
        if (gate_in_logits) {
#pragma unroll
            for (int s = 0; s < NS; ++s) z += partial[(static_cast<size_t>(s) * M + t) * (E + 1) + E];
        } else {  // gate logit g . x[t], fixed-order warp reduction
            const float* xr = io->x + static_cast<size_t>(t) * H;
            for (int i = lane * 4; i < H; i += 128) {
                const float4 a = *reinterpret_cast<const float4*>(xr + i);
                const float4 b = *reinterpret_cast<const float4*>(gate_w + i);
                z = fmaf(a.x, b.x, z); z = fmaf(a.y, b.y, z); z = fmaf(a.z, b.z, z); z = fmaf(a.w, b.w, z);
            }
            z = warp_sum(z);
        }
        g = 1.0f / (1.0f + expf(-z));
    }
    if (lane == 0) rec[0] = make_uint2(static_cast<uint32_t>(E), __float_as_uint(g));
}

}  // namespace

constexpr int kGemmSplit = 4;

int router_split_for(int M, int H) {
    if (M <= 8) return 1;
    return (H % (kGemmSplit * kTK) == 0) ? kGemmSplit : 1;
}

void launch_router_logits(const Layer& L, const IoArgs* x, int M, float* logits, cudaStream_t s) {
    const int E = L.spec.n_experts, H = L.spec.hidden;
    const bool gate = (L.spec.flags & MOE_F_SHARED_GATE) != 0;
    const int n_rows = E + (gate ? 1 : 0);
    const float* wr = reinterpret_cast<const float*>(L.router_w_ptr);
    const float* gw = reinterpret_cast<const float*>(L.gate_ptr);
    if (M <= 8) {
        dim3 grid((n_rows + kRowsPerCta - 1) / kRowsPerCta, 1);
        if (M == 1)
            router_gemv_kernel<1><<<grid, 32 * kRowsPerCta, 0, s>>>(x, M, H, wr, gw, E, n_rows, logits);
        else
            router_gemv_kernel<8><<<grid, 32 * kRowsPerCta, 0, s>>>(x, M, H, wr, gw, E, n_rows, logits);
    } else {
        const int split = router_split_for(M, H);
        dim3 grid((M + kTM - 1) / kTM, (n_rows + kTE - 1) / kTE, split);
        router_gemm_kernel<<<grid, 256, 0, s>>>(x, M, H, wr, gw, E, n_rows, H / split, logits);
    }
}

void launch_topk(const Layer& L, const float* logits, int n_split, bool gate_in_logits,
                 const IoArgs* io, int M, uint2* topk, int* status, cudaStream_t s) {
    const int E = L.spec.n_experts;
    const int shared_mode = (L.spec.flags & MOE_F_SHARED_GATE) ? 2 : 1;
    const float* bias = reinterpret_cast<const float*>(L.bias_ptr);
    const int grid = (M + 3) / 4;
    const float* gw = reinterpret_cast<const float*>(L.gate_ptr);
    const int k = static_cast<int>(L.spec.top_k), H = static_cast<int>(L.spec.hidden);
    const int gl = gate_in_logits ? 1 : 0;
#define MOE_TOPK(NS) topk_kernel<NS><<<grid, 128, 0, s>>>(logits, M, E, k, bias, shared_mode, gl, io, gw, H, topk, status)
    switch (n_split) {
        case 1: MOE_TOPK(1); break;
        case 2: MOE_TOPK(2); break;
        case 4: MOE_TOPK(4); break;
        case 8: MOE_TOPK(8); break;
        default: MOE_TOPK(16); break;
    }
#undef MOE_TOPK
}

}  // namespace moe
