// Utility kernels: f32 IQ4_XS decode (dequant check), synthetic IQ4_XS weights, RMSNorm glue.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "moe_common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

// One warp per block: lane l decodes weights 8l..8l+7 of the 256 (sub-block l/4).
__global__ void dequant_kernel(const uint8_t* __restrict__ src, uint64_t n_blocks,
                               float* __restrict__ dst) {
    const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= n_blocks) return;
    const uint8_t* blk = src + warp * kBlockBytes;
    const uint32_t h0 = *reinterpret_cast<const uint32_t*>(blk);
    const uint32_t h1 = *reinterpret_cast<const uint32_t*>(blk + 4);
    const int ib = lane >> 2, w = lane & 3;  // sub-block, word inside its 16 qs bytes
    const uint32_t q = *reinterpret_cast<const uint32_t*>(blk + 8 + ib * 16 + w * 4);
    const float dl = iq4_subscale(h0, h1, ib);
    uint32_t r0, r1;
    kv_lookup8(q, r0, r1);
    float* o = dst + warp * kQK + ib * 32;
    const int j0 = w * 4;
    o[j0 + 0] = dl * kv_float<0>(r0);
    o[j0 + 16] = dl * kv_float<1>(r0);
    o[j0 + 1] = dl * kv_float<2>(r0);
    o[j0 + 17] = dl * kv_float<3>(r0);
    o[j0 + 2] = dl * kv_float<0>(r1);
    o[j0 + 18] = dl * kv_float<1>(r1);
    o[j0 + 3] = dl * kv_float<2>(r1);
    o[j0 + 19] = dl * kv_float<3>(r1);
}

// splitmix64 (Steele, Lea & Flood 2014): the published finaliser constants.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Thread per 8-byte word of the output; word i of block b = splitmix64(key + 17*b + i).
__global__ void synth_kernel(uint8_t* __restrict__ dst, uint64_t key, uint64_t block_start,
                             uint64_t n_blocks) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t n_words = n_blocks * 17;
    if (i >= n_words) return;
    const uint64_t b = i / 17, w = i - b * 17;
    uint64_t v = splitmix64(key + (block_start + b) * 17 + w);
    if (w == 0) {
        const float u = static_cast<float>(static_cast<uint32_t>(v >> 40)) * (1.0f / 16777216.0f);
        const float d = __fadd_rn(0.005f, __fmul_rn(0.015f, u));
        const uint64_t hb = __half_as_ushort(__float2half_rn(d));
        v = (v & ~0xFFFFull) | hb;
    }
    // 136-byte blocks are 8-byte aligned: store as two 4-byte halves (alignment 8 holds too).
    reinterpret_cast<uint64_t*>(dst)[i] = v;
}

// One CTA per token: y = x * rsqrt(mean(x^2) + eps) (shaders/rms_norm.comp:36-58, no gain).
__global__ void __launch_bounds__(256)
rms_norm_kernel(const float* __restrict__ x, float* __restrict__ y, int H, float eps) {
    __shared__ float red[8];
    const float* xr = x + static_cast<size_t>(blockIdx.x) * H;
    float* yr = y + static_cast<size_t>(blockIdx.x) * H;
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) tot += red[w];
    const float r = 1.0f / sqrtf(tot / static_cast<float>(H) + eps);
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
        float4 v = *reinterpret_cast<const float4*>(xr + i);
        v.x *= r; v.y *= r; v.z *= r; v.w *= r;
        *reinterpret_cast<float4*>(yr + i) = v;
    }
}

// y[i] = silu(g[i]) * (u ? u[i] : 1), silu(v) = v / (1 + e^-v) (shaders/silu_mult.comp:21-38,
// shaders/common.glsl:106-108).
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ y,
                                uint64_t n) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float v = silu_f(g[i]);
        y[i] = u ? v * u[i] : v;
    }
}

}  // namespace

// The reference's own 36-byte weight block (shaders/common.glsl:59-86, "IQ4_XS" there): 32
// weights, f16 scales d0 (weights 0-15) and d2 (16-31) at bytes 0 and 2, low 4 bits of weight p
// in byte 4 + p/2 (low nibble for even p), bit 4 in byte 20 + p/8, bit p%8; w = (q - 8) * d in
// f32.  The shader's f16 -> f32 conversion flushes subnormals to signed zero and keeps inf/NaN;
// this decoder does the same, so it reproduces the shipped shaders' weights bit for bit.
__device__ __forceinline__ float ref_f16_to_f32(uint32_t b) {
    const uint32_t sgn = (b & 0x8000u) << 16, e = (b & 0x7C00u) >> 10, m = b & 0x03FFu;
    if (e == 0u) return __uint_as_float(sgn);
    const uint32_t e32 = e == 31u ? 255u : e + 112u;
    return __uint_as_float(sgn | (e32 << 23) | (m << 13));
}

__global__ void dequant_ref36_kernel(const uint8_t* __restrict__ src, uint64_t n_blocks,
                                     float* __restrict__ dst) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // weight
    if (i >= n_blocks * 32) return;
    const uint8_t* b = src + (i >> 5) * 36;
    const uint32_t p = static_cast<uint32_t>(i & 31);
    const uint32_t dbits = p < 16 ? (b[0] | (b[1] << 8)) : (b[2] | (b[3] << 8));
    uint32_t q = (b[4 + (p >> 1)] >> ((p & 1) * 4)) & 0xFu;
    q |= ((b[20 + (p >> 3)] >> (p & 7)) & 1u) << 4;
    dst[i] = (static_cast<float>(q) - 8.0f) * ref_f16_to_f32(dbits);
}

void launch_dequant_ref36(const uint8_t* src, uint64_t n_blocks, float* dst, cudaStream_t s) {
    const uint64_t n = n_blocks * 32;
    dequant_ref36_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(src, n_blocks, dst);
}

void launch_dequant(const uint8_t* src, uint64_t n_blocks, float* dst, cudaStream_t s) {
    const uint64_t threads = n_blocks * 32;
    dequant_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(src, n_blocks, dst);
}

void launch_synth(uint8_t* dst, uint64_t key, uint64_t block_start, uint64_t n_blocks,
                  cudaStream_t s) {
    const uint64_t words = n_blocks * 17;
    synth_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, s>>>(dst, key, block_start,
                                                                           n_blocks);
}

void launch_rms_norm(const float* x, float* y, int M, int H, float eps, cudaStream_t s) {
    rms_norm_kernel<<<M, 256, 0, s>>>(x, y, H, eps);
}

void launch_silu_mul(const float* g, const float* u, float* y, uint64_t n, int sm_count, cudaStream_t s) {
    const uint64_t blocks = std::min<uint64_t>((n + 255) / 256, static_cast<uint64_t>(sm_count) * 8);
    silu_mul_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(g, u, y, n);
}

}  // namespace moe
