// Grouped IQ4_XS expert products on CUDA cores, for small buckets (decode, batched decode):
// the roles of moe-680m's w1_w3_fused(_m1).comp + silu_mult.comp (gate/up and SiLU) and
// w2(_scatter)(_m1).comp (down projection), regrouped by expert bucket.
//
// Work item = (chunk of <= TOK tokens of one bucket, block of output rows).  A CTA stages the
// chunk's activation rows in shared memory (gathered through the sorted token list), then
// each warp streams whole weight rows with 8-byte streaming loads, decodes every nibble once
// in registers (kvalues_iq4nl lookup via byte permutes, exact f32) and applies it to all the
// chunk's tokens.  Accumulation is f32; every (row, token) result is reduced in a fixed order.
//
//   gemv13: h[p][j] = silu(W1[j] . x_t) * (W3[j] . x_t)          (p = sorted slot position)
//   gemv2:  ypart[p][n] = W2[n] . h[p]                            (unweighted; combine weights)
#include <cuda_runtime.h>

#include <algorithm>

#include "moe_common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

constexpr int kWarps = 8;
constexpr int kRows13 = 16;  // gate/up row pairs per work item
constexpr int kRows2 = 64;   // down-projection rows per work item
constexpr int kMaxSbLane = 2;  // sub-blocks per lane per pass along a W1/W3 row

// Decode one qs word into 8 exact floats in x order (j0..j0+3 low nibbles, then +16).
__device__ __forceinline__ void decode_word(uint32_t q, float (&w)[8]) {
    uint32_t r0, r1;
    kv_lookup8(q, r0, r1);
    w[0] = kv_float<0>(r0);  // j0
    w[4] = kv_float<1>(r0);  // j0+16
    w[1] = kv_float<2>(r0);  // j0+1
    w[5] = kv_float<3>(r0);  // j0+17
    w[2] = kv_float<0>(r1);
    w[6] = kv_float<1>(r1);
    w[3] = kv_float<2>(r1);
    w[7] = kv_float<3>(r1);
}

// acc[t] += dl * sum_j kv_j * xs_t[j] over one sub-block, for the chunk's n tokens.
template <int TOK>
__device__ __forceinline__ void subblk_fma(const SubBlk& s, float dl, const float* xs, int stride,
                                           int n, float (&acc)[TOK]) {
    float part[TOK];
#pragma unroll
    for (int t = 0; t < TOK; ++t) part[t] = 0.f;
    const uint32_t words[4] = {s.q01.x, s.q01.y, s.q23.x, s.q23.y};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        float w[8];
        decode_word(words[wi], w);
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
            if (t < n) {
                const float4* x4 = reinterpret_cast<const float4*>(xs + t * stride);
                const float4 a = x4[wi], b = x4[4 + wi];
                float v = part[t];
                v = fmaf(w[0], a.x, v); v = fmaf(w[1], a.y, v);
                v = fmaf(w[2], a.z, v); v = fmaf(w[3], a.w, v);
                v = fmaf(w[4], b.x, v); v = fmaf(w[5], b.y, v);
                v = fmaf(w[6], b.z, v); v = fmaf(w[7], b.w, v);
                part[t] = v;
            }
        }
    }
#pragma unroll
    for (int t = 0; t < TOK; ++t) acc[t] = fmaf(dl, part[t], acc[t]);
}

// Stage rows src[idx[t]] (len floats) into padded shared memory dst[t].
__device__ __forceinline__ void stage_rows(float* dst, int stride, const float* src, int len,
                                           const int* idx, int n, bool gather) {
    const int n4 = len / 4;
    for (int i = threadIdx.x; i < n * n4; i += blockDim.x) {
        const int t = i / n4, c = i - t * n4;
        const int row = gather ? idx[t] : t;
        const float4 v = __ldg(reinterpret_cast<const float4*>(src + static_cast<size_t>(row) * len) + c);
        const int k = c * 4;
        *reinterpret_cast<float4*>(dst + t * stride + padded_idx(k)) = v;
    }
}

template <int TOK>
__global__ void __launch_bounds__(32 * kWarps)
gemv13_kernel(const IoArgs* __restrict__ io, int H, int I, ExpertTables tabs,
              const int* __restrict__ sorted_tok, const Chunk* __restrict__ chunks,
              const int* __restrict__ counters, float* __restrict__ h) {
    const float* __restrict__ x = io->x;
    extern __shared__ __align__(16) float xs[];
    const int stride = padded_len(H);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rb_per_chunk = I / kRows13;
    const int n_items = counters[0] * rb_per_chunk;
    const int nsb = H / 32;
    const size_t row_bytes = static_cast<size_t>(H / kQK) * kBlockBytes;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int c = item / rb_per_chunk, rb = item - c * rb_per_chunk;
        const Chunk ch = chunks[c];
        const int n = min(ch.n, TOK);
        __syncthreads();
        stage_rows(xs, stride, x, H, sorted_tok + ch.start, n, true);
        __syncthreads();
        const uint8_t* w1 = tabs.w1[ch.bucket];
        const uint8_t* w3 = tabs.w3[ch.bucket];
        for (int j = rb * kRows13 + warp; j < (rb + 1) * kRows13; j += kWarps) {
            const uint8_t* r1 = w1 + j * row_bytes;
            const uint8_t* r3 = w3 + j * row_bytes;
            float g[TOK], u[TOK];
#pragma unroll
            for (int t = 0; t < TOK; ++t) { g[t] = 0.f; u[t] = 0.f; }
            for (int base = 0; base < nsb; base += 32 * kMaxSbLane) {
                SubBlk a[kMaxSbLane], b[kMaxSbLane];
#pragma unroll
                for (int i = 0; i < kMaxSbLane; ++i) {
                    const int sb = base + lane + 32 * i;
                    if (sb < nsb) { a[i] = load_subblk(r1, sb); b[i] = load_subblk(r3, sb); }
                }
#pragma unroll
                for (int i = 0; i < kMaxSbLane; ++i) {
                    const int sb = base + lane + 32 * i;
                    if (sb < nsb) {
                        const float* xp = xs + sb * 36;
                        subblk_fma<TOK>(a[i], iq4_subscale(a[i].hdr.x, a[i].hdr.y, sb & 7), xp, stride, n, g);
                        subblk_fma<TOK>(b[i], iq4_subscale(b[i].hdr.x, b[i].hdr.y, sb & 7), xp, stride, n, u);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < TOK; ++t) {
                const float gs = warp_sum(g[t]);
                const float us = warp_sum(u[t]);
                if (lane == t && t < n) h[static_cast<size_t>(ch.start + t) * I + j] = silu_f(gs) * us;
            }
        }
    }
}

template <int TOK>
__global__ void __launch_bounds__(32 * kWarps)
gemv2_kernel(int H, int I, ExpertTables tabs, const Chunk* __restrict__ chunks,
             const int* __restrict__ counters, const float* __restrict__ h,
             float* __restrict__ ypart) {
    extern __shared__ __align__(16) float hs[];
    const int stride = padded_len(I);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int spr = I / 32;          // sub-blocks per row: 8, 16 or 32
    const int rpi = 32 / spr;        // rows per warp pass
    const int r_in = lane / spr, sb = lane - r_in * spr;
    const int rb_per_chunk = H / kRows2;
    const int n_items = counters[0] * rb_per_chunk;
    const size_t row_bytes = static_cast<size_t>(I / kQK) * kBlockBytes;
    constexpr int kPass = 4;  // passes issued together per warp
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int c = item / rb_per_chunk, rb = item - c * rb_per_chunk;
        const Chunk ch = chunks[c];
        const int n = min(ch.n, TOK);
        __syncthreads();
        stage_rows(hs, stride, h + static_cast<size_t>(ch.start) * I, I, nullptr, n, false);
        __syncthreads();
        const uint8_t* w2 = tabs.w2[ch.bucket];
        const int row_end = (rb + 1) * kRows2;
        for (int n0 = rb * kRows2 + warp * rpi * kPass; n0 < row_end; n0 += kWarps * rpi * kPass) {
            SubBlk a[kPass];
#pragma unroll
            for (int p = 0; p < kPass; ++p) {
                const int row = n0 + p * rpi + r_in;
                if (row < row_end) a[p] = load_subblk(w2 + row * row_bytes, sb);
            }
#pragma unroll
            for (int p = 0; p < kPass; ++p) {
                const int row = n0 + p * rpi + r_in;
                float y[TOK];
#pragma unroll
                for (int t = 0; t < TOK; ++t) y[t] = 0.f;
                if (row < row_end)
                    subblk_fma<TOK>(a[p], iq4_subscale(a[p].hdr.x, a[p].hdr.y, sb & 7),
                                    hs + sb * 36, stride, n, y);
#pragma unroll
                for (int t = 0; t < TOK; ++t) {
                    float v = y[t];
                    for (int o = spr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (sb == 0 && t < n && row < row_end)
                        ypart[static_cast<size_t>(ch.start + t) * H + row] = v;
                }
            }
        }
    }
}

// out[t] = resid[t] + scale * sum_s w_s * ypart[pos[t][s]]  (slots in order: routed by
// descending weight, then shared), float4 per thread.
__global__ void __launch_bounds__(256)
combine_kernel(const float* __restrict__ ypart, const int* __restrict__ slot_pos,
               const float* __restrict__ sorted_w, int ns, int H, float scale,
               const IoArgs* __restrict__ io, const float* __restrict__ ysh, const uint2* __restrict__ topk,
               int k) {
    const float* __restrict__ resid = io->resid;
    float* __restrict__ out = io->out;
    const int t = blockIdx.x;
    const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
    if (c >= H) return;
    const int* pos = slot_pos + static_cast<size_t>(t) * ns;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < ns; ++s) {
        const int p = pos[s];
        if (p < 0) continue;
        const float w = sorted_w[p];
        const float4 y = *reinterpret_cast<const float4*>(ypart + static_cast<size_t>(p) * H + c);
        acc.x = fmaf(w, y.x, acc.x); acc.y = fmaf(w, y.y, acc.y);
        acc.z = fmaf(w, y.z, acc.z); acc.w = fmaf(w, y.w, acc.w);
    }
    if (ysh) {  // the shared expert's row of a separate shared pass, weighted by its gate, last
        const uint2 r0 = topk[static_cast<size_t>(t) * (k + 1)];
        if (r0.x != kNoExpert) {
            const float w = __uint_as_float(r0.y);
            const float4 y = *reinterpret_cast<const float4*>(ysh + static_cast<size_t>(t) * H + c);
            acc.x = fmaf(w, y.x, acc.x); acc.y = fmaf(w, y.y, acc.y);
            acc.z = fmaf(w, y.z, acc.z); acc.w = fmaf(w, y.w, acc.w);
        }
    }
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (resid) r = *reinterpret_cast<const float4*>(resid + static_cast<size_t>(t) * H + c);
    r.x = fmaf(scale, acc.x, r.x); r.y = fmaf(scale, acc.y, r.y);
    r.z = fmaf(scale, acc.z, r.z); r.w = fmaf(scale, acc.w, r.w);
    *reinterpret_cast<float4*>(out + static_cast<size_t>(t) * H + c) = r;
}

template <typename K>
void set_smem(K kern, size_t bytes) {
    if (bytes > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(bytes));
}

__global__ void set_io_kernel(IoArgs* dst, const float* x, const float* resid, float* out) {
    dst->x = x;
    dst->resid = resid;
    dst->out = out;
}

}  // namespace

void launch_set_io(IoArgs* dst, const float* x, const float* resid, float* out, cudaStream_t s) {
    set_io_kernel<<<1, 1, 0, s>>>(dst, x, resid, out);
}

const void* set_io_func() { return reinterpret_cast<const void*>(&set_io_kernel); }

void launch_gemv13(const Layer& L, const IoArgs* x, const Workspace& ws, int M, int max_chunks,
                   int sm_count, cudaStream_t s) {
    const int H = L.spec.hidden, I = L.spec.inter;
    const int items = max_chunks * (I / kRows13);
    if (M == 1) {  // one token per bucket (decode)
        const size_t smem = padded_len(H) * sizeof(float);
        set_smem(gemv13_kernel<1>, smem);
        const int grid = std::min(items, sm_count * 8);
        gemv13_kernel<1><<<grid, 32 * kWarps, smem, s>>>(x, H, I, L.tables(), ws.sorted_tok,
                                                         ws.chunks, ws.counters, ws.h);
    } else {
        const size_t smem = static_cast<size_t>(kGemvTok) * padded_len(H) * sizeof(float);
        set_smem(gemv13_kernel<kGemvTok>, smem);
        const int grid = std::min(items, sm_count * 3);
        gemv13_kernel<kGemvTok><<<grid, 32 * kWarps, smem, s>>>(x, H, I, L.tables(), ws.sorted_tok,
                                                                ws.chunks, ws.counters, ws.h);
    }
}

void launch_gemv2(const Layer& L, const Workspace& ws, int M, int max_chunks, int sm_count,
                  cudaStream_t s) {
    const int H = L.spec.hidden, I = L.spec.inter;
    const int items = max_chunks * (H / kRows2);
    if (M == 1) {
        const size_t smem = padded_len(I) * sizeof(float);
        const int grid = std::min(items, sm_count * 8);
        gemv2_kernel<1><<<grid, 32 * kWarps, smem, s>>>(H, I, L.tables(), ws.chunks, ws.counters,
                                                        ws.h, ws.ypart);
    } else {
        const size_t smem = static_cast<size_t>(kGemvTok) * padded_len(I) * sizeof(float);
        set_smem(gemv2_kernel<kGemvTok>, smem);
        const int grid = std::min(items, sm_count * 6);
        gemv2_kernel<kGemvTok><<<grid, 32 * kWarps, smem, s>>>(H, I, L.tables(), ws.chunks,
                                                               ws.counters, ws.h, ws.ypart);
    }
}

void launch_combine(const Layer& L, const Workspace& ws, const IoArgs* io, int M, int ns, float scale,
                    cudaStream_t s, const float* ysh) {
    const int H = L.spec.hidden;
    dim3 grid(M, (H / 4 + 255) / 256);
    combine_kernel<<<grid, 256, 0, s>>>(ws.ypart, ws.slot_pos, ws.sorted_w, ns, H, scale, io, ysh, ws.topk,
                                        static_cast<int>(L.spec.top_k));
}

}  // namespace moe
