// Expert products on the reference's own weight format (layers created with MOE_F_REF36): the
// 36-byte, 32-weight blocks of moe-680m's shaders/common.glsl:59-86, stored the way its shaders
// address them, W[K][N] with weight (k, n) at flat index k * N + n (w1_w3_fused_m1.comp:46-47,
// w2_scatter_m1.comp:41).  A block covers 32 consecutive outputs n of one input k: f16 scales d0
// (positions 0-15) and d2 (16-31) at bytes 0 and 2, the low 4 bits of position p in byte
// 4 + p/2 (low nibble for even p), bit 4 in byte 20 + p/8 (bit p % 8); w = (q - 8) * d, the f16
// scales converted with the shaders' flush of subnormals.
//
// This is the compatibility path (weights 2.1x the bytes of GGUF IQ4_XS; CUDA cores, f32): the
// grouped GEMV of the library on the same chunks of one bucket (up to 8 tokens each).  Gate/up:
// CTA (chunk, K split) computes partial sums of the 2I outputs [W1 | W3] for its K range, one
// thread per output (a warp's 32 outputs share one block per k, read as a broadcast); a second
// kernel adds the splits in a fixed order and writes h = silu(g) * u per slot row, the layout the
// library's down-projection and combine read.  Down: the same over W2 into the unweighted
// per-slot rows; the library's combine then applies weights, scale and residual.
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

constexpr int kRefThreads = 512;
constexpr int kRefSplit = 16;  // K splits (gate/up: H / 16 inputs each; down: I / 16)

__device__ __forceinline__ float ref_f16(uint32_t b) {
    const uint32_t sgn = (b & 0x8000u) << 16, e = (b & 0x7C00u) >> 10, m = b & 0x03FFu;
    if (e == 0u) return __uint_as_float(sgn);
    const uint32_t e32 = e == 31u ? 255u : e + 112u;
    return __uint_as_float(sgn | (e32 << 23) | (m << 13));
}

// Weight (k, n) of a [K][N] reference-format matrix.
__device__ __forceinline__ float ref36_weight(const uint8_t* w, int N, int k, int n) {
    const uint64_t idx = static_cast<uint64_t>(k) * N + n;
    const uint32_t* b = reinterpret_cast<const uint32_t*>(w + (idx >> 5) * 36);
    const uint32_t p = static_cast<uint32_t>(idx & 31);
    const uint32_t w0 = __ldg(b);
    const uint32_t dbits = p < 16 ? (w0 & 0xFFFFu) : (w0 >> 16);
    const uint32_t qw = __ldg(b + 1 + (p >> 3));         // bytes 4 + 4 (p/8) .. : nibbles of p
    const uint32_t hw = __ldg(b + 5);                    // bytes 20..23: bit 4 of every p
    uint32_t q = (qw >> (((p >> 1) & 3) * 8 + (p & 1) * 4)) & 0xFu;
    q |= ((hw >> p) & 1u) << 4;
    return (static_cast<float>(q) - 8.0f) * ref_f16(dbits);
}

// partial[split][p][o] for the chunk's slot rows p: o < N0 from matrix A ([K][N0]), o >= N0 from
// matrix B ([K][N0]) (gate/up: A = W1, B = W3); down: B == null, N0 = N.
__global__ void __launch_bounds__(kRefThreads)
ref36_partial_kernel(const IoArgs* __restrict__ io, const float* __restrict__ src_rows, int src_ld,
                     const int* __restrict__ sorted_tok, bool by_token, const Chunk* __restrict__ chunks, const int* __restrict__ n_chunks,
                     const uint8_t* const* __restrict__ tab_a, const uint8_t* const* __restrict__ tab_b,
                     int K, int N0, int n_out, float* __restrict__ partial, size_t split_stride) {
    extern __shared__ float xs[];  // [kGemvTok][K / kRefSplit]
    const int ci = blockIdx.x;
    if (ci >= *n_chunks) return;
    const Chunk ch = chunks[ci];
    const int kl = K / kRefSplit, k0 = blockIdx.y * kl;
    const float* src = src_rows ? src_rows : io->x;
    for (int i = threadIdx.x; i < ch.n * kl; i += blockDim.x) {
        const int t = i / kl, kk = i - t * kl;
        const int p = ch.start + t;
        const size_t row = by_token ? static_cast<size_t>(sorted_tok[p]) : static_cast<size_t>(p);
        xs[t * kl + kk] = src[row * src_ld + k0 + kk];
    }
    __syncthreads();
    const uint8_t* wa = tab_a[ch.bucket];
    const uint8_t* wb = tab_b ? tab_b[ch.bucket] : nullptr;
    for (int o = threadIdx.x; o < n_out; o += blockDim.x) {
        const uint8_t* w = o < N0 ? wa : wb;
        const int n = o < N0 ? o : o - N0;
        float acc[kGemvTok];
#pragma unroll
        for (int t = 0; t < kGemvTok; ++t) acc[t] = 0.f;
        for (int kk = 0; kk < kl; ++kk) {
            const float wv = ref36_weight(w, N0, k0 + kk, n);
#pragma unroll
            for (int t = 0; t < kGemvTok; ++t)
                if (t < ch.n) acc[t] = fmaf(xs[t * kl + kk], wv, acc[t]);
        }
        float* out = partial + blockIdx.y * split_stride;
#pragma unroll
        for (int t = 0; t < kGemvTok; ++t)
            if (t < ch.n) out[static_cast<size_t>(ch.start + t) * n_out + o] = acc[t];
    }
}

// Sum of the K splits in split order for the used slot rows: gate/up -> h = silu(g) * u
// ([S][I]); down -> y ([S][H]).
__global__ void ref36_finish_kernel(const float* __restrict__ partial, size_t split_stride,
                                    const int* __restrict__ n_used, int n_rows, int n_out, int swiglu,
                                    float* __restrict__ dst) {
    const int n_dst = swiglu ? n_out / 2 : n_out;
    const int used = min(n_rows, *n_used);
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
         i < static_cast<size_t>(used) * n_dst; i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t p = i / n_dst, j = i - p * n_dst;
        float a = 0.f, b = 0.f;
        for (int s = 0; s < kRefSplit; ++s) {
            a += partial[s * split_stride + p * n_out + j];
            if (swiglu) b += partial[s * split_stride + p * n_out + n_dst + j];
        }
        dst[i] = swiglu ? silu_f(a) * b : a;
    }
}

}  // namespace

size_t ref36_scratch_bytes(int S, int H, int I) {
    const int widest = H > 2 * I ? H : 2 * I;
    return static_cast<size_t>(kRefSplit) * S * widest * sizeof(float);
}

bool ref36_supported(int H, int I) { return H % (32 * kRefSplit) == 0 && I % (32 * kRefSplit) == 0; }

void launch_ref36_experts(const Layer& L, const Workspace& ws, int M, int slots, int max_chunks, float* scratch,
                          cudaStream_t s) {
    const int H = static_cast<int>(L.spec.hidden), I = static_cast<int>(L.spec.inter);
    const int S = M * slots;
    const ExpertTables t = L.tables();
    // gate/up: x rows by token, [W1 | W3], K = H
    {
        const size_t stride = static_cast<size_t>(S) * 2 * I;
        const size_t smem = static_cast<size_t>(kGemvTok) * (H / kRefSplit) * sizeof(float);
        ref36_partial_kernel<<<dim3(max_chunks, kRefSplit), kRefThreads, smem, s>>>(
            ws.io, nullptr, H, ws.sorted_tok, true, ws.chunks, ws.counters, t.w1, t.w3, H, I, 2 * I, scratch, stride);
        ref36_finish_kernel<<<1184, 256, 0, s>>>(scratch, stride, ws.ranges + L.spec.n_experts + 1, S, 2 * I, 1,
                                                 ws.h);
    }
    // down: h rows by slot position, W2, K = I
    {
        const size_t stride = static_cast<size_t>(S) * H;
        const size_t smem = static_cast<size_t>(kGemvTok) * (I / kRefSplit) * sizeof(float);
        ref36_partial_kernel<<<dim3(max_chunks, kRefSplit), kRefThreads, smem, s>>>(
            ws.io, ws.h, I, ws.sorted_tok, false, ws.chunks, ws.counters, t.w2, nullptr, I, H, H, scratch, stride);
        ref36_finish_kernel<<<1184, 256, 0, s>>>(scratch, stride, ws.ranges + L.spec.n_experts + 1, S, H, 0,
                                                 ws.ypart);
    }
}

}  // namespace moe
