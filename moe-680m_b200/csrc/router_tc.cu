// Router projection for batches (M > 8) on the tensor cores, with f32-level accuracy from three
// TF32 products: logits = Wh.xh + Wh.xl + Wl.xh, where v = vh + vl splits every f32 value into
// its round-to-nearest TF32 part and the remainder (the dropped xl.Wl term is ~2^-22 relative).
// The role of moe-680m's shaders/router.comp (x . ffn_gate), with an f32 router weight.
//
// One CTA per (128-expert tile, <=256-token tile, K split): warp 0 lane 0 streams the four
// operand tiles (Wh, Wl: 128 x 32; xh, xl: 256 x 32 f32, 128-byte swizzle) with TMA into a
// 2-stage ring, warp 1 (one elected lane) issues tcgen05.mma kind::tf32 (M=128, N=tokens, K=8) into one
// TMEM accumulator, warps 2-5 write the f32 partial logits partial[split][token][expert]; the
// top-k kernel sums the splits in a fixed order.  Identical router rows go through identical
// operations, so they still produce identical logits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

namespace {

using namespace tc;

constexpr int kRThreads = 6 * 32;
constexpr int kRStages = 2;
constexpr int kRTokMax = 256;
constexpr int kWTile = 128 * 128;          // bytes: 128 rows x 32 f32
constexpr int kXTile = kRTokMax * 128;     // bytes: 256 rows x 32 f32
constexpr int kRStage = 2 * kWTile + 2 * kXTile;
constexpr size_t kRSmem = static_cast<size_t>(kRStages) * kRStage + 256 + 1024;

// Instruction descriptor, kind::tf32: TF32 A and B (K-major), f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

__global__ void __launch_bounds__(kRThreads, 1)
router_tc_kernel(const __grid_constant__ CUtensorMap wh_map, const __grid_constant__ CUtensorMap wl_map,
                 const __grid_constant__ CUtensorMap xh_map, const __grid_constant__ CUtensorMap xl_map,
                 int M, int E, int k_len, float* __restrict__ partial, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRStages * kRStage);
    uint64_t* empty = full + kRStages;
    uint64_t* accf = empty + kRStages;
    uint32_t* tmem_p = reinterpret_cast<uint32_t*>(accf + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_p + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * 128, t0 = blockIdx.y * kRTokMax, split = blockIdx.z;
    const int ntok = min(kRTokMax, M - t0);
    const int N = (ntok + 15) & ~15;
    const int kbeg = split * k_len, nst = k_len / 32;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(accf, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_p, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_p;

    if (warp == 0) {
        if (lane == 0) {
            for (int s = 0; s < nst && !*abort; ++s) {
                const int slot = s % kRStages;
                if (!mbar_wait(&empty[slot], ((s / kRStages) & 1) ^ 1, abort)) break;
                uint8_t* st = smem + slot * kRStage;
                mbar_arrive_expect_tx(&full[slot], 2 * kWTile + 2 * kXTile);
                const int k = kbeg + s * 32;
                tma_load_2d(st, &wh_map, k, e0, &full[slot]);
                tma_load_2d(st + kWTile, &wl_map, k, e0, &full[slot]);
                tma_load_2d(st + 2 * kWTile, &xh_map, k, t0, &full[slot]);
                tma_load_2d(st + 2 * kWTile + kXTile, &xl_map, k, t0, &full[slot]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // whole warp loops; one elected lane issues (keeps the MMA operands warp-uniform)
        const uint32_t idesc = idesc_tf32(128, N);
        bool ok = true;
        for (int s = 0; s < nst; ++s) {
            const int slot = s % kRStages;
            if (!mbar_wait_warp(&full[slot], (s / kRStages) & 1, abort)) { ok = false; break; }
            tc_fence_after();
            const uint32_t base = smem_u32(smem + slot * kRStage);
            if (elect_one()) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint64_t wh = sw128_desc(base + 32 * j);
                    const uint64_t wl = sw128_desc(base + kWTile + 32 * j);
                    const uint64_t xh = sw128_desc(base + 2 * kWTile + 32 * j);
                    const uint64_t xl = sw128_desc(base + 2 * kWTile + kXTile + 32 * j);
                    mma_tf32(tmem, wh, xh, idesc, (s | j) != 0);
                    mma_tf32(tmem, wh, xl, idesc, 1);
                    mma_tf32(tmem, wl, xh, idesc, 1);
                }
                mma_commit(&empty[slot]);
            }
            __syncwarp();
        }
        if (ok && elect_one()) mma_commit(accf);
        __syncwarp();
    } else {
        const int q = warp & 3;
        const int e = e0 + q * 32 + lane;
        if (mbar_wait(accf, 0, abort)) {
            tc_fence_after();
            float* out = partial + static_cast<size_t>(split) * M * (E + 1);
            for (int c0 = 0; c0 < ntok; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < 16; ++t)
                    if (c0 + t < ntok && e < E)
                        out[static_cast<size_t>(t0 + c0 + t) * (E + 1) + e] = __uint_as_float(v[t]);
            }
        }
    }
    __syncthreads();
    if (*abort) {
        if (threadIdx.x == 0) set_dev_error(status, kDevTimeout);
        for (int i = 0; i < 200; ++i) __nanosleep(1000);
    }
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 256);
}

// v -> (round-to-nearest TF32 part, remainder), elementwise.
__global__ void split_tf32_kernel(const float* __restrict__ src, size_t n, float* __restrict__ hi,
                                  float* __restrict__ lo) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float v = src[i];
        uint32_t h;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
        const float hf = __uint_as_float(h);
        hi[i] = hf;
        lo[i] = v - hf;
    }
}

// One CTA (128 threads) per token: x[t] -> (TF32 part, remainder) for the router operands and,
// when the layer has a shared-expert gate, the gate logit g . x[t] (f32, fixed-order reduction)
// into column E of the first logit plane, with zeros in column E of the other n_split - 1
// planes, so that the top-k kernel's in-order sum of the planes returns it unchanged.
__global__ void __launch_bounds__(128)
split_x_kernel(const IoArgs* __restrict__ io, int M, int H, float* __restrict__ hi, float* __restrict__ lo,
               const float* __restrict__ gate_w, float* __restrict__ logits, int n_split, int E) {
    __shared__ float red[4];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float4* src = reinterpret_cast<const float4*>(io->x + static_cast<size_t>(t) * H);
    float4* h4 = reinterpret_cast<float4*>(hi + static_cast<size_t>(t) * H);
    float4* l4 = reinterpret_cast<float4*>(lo + static_cast<size_t>(t) * H);
    float z = 0.f;
    for (int i = tid; i < H / 4; i += 128) {
        const float4 v = src[i];
        float vv[4] = {v.x, v.y, v.z, v.w}, hh[4], ll[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t h;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(vv[j]));
            hh[j] = __uint_as_float(h);
            ll[j] = vv[j] - hh[j];
        }
        h4[i] = make_float4(hh[0], hh[1], hh[2], hh[3]);
        l4[i] = make_float4(ll[0], ll[1], ll[2], ll[3]);
        if (gate_w) {
            const float4 g = reinterpret_cast<const float4*>(gate_w)[i];
            z = fmaf(v.x, g.x, z); z = fmaf(v.y, g.y, z); z = fmaf(v.z, g.z, z); z = fmaf(v.w, g.w, z);
        }
    }
    if (!gate_w) return;
    z = warp_sum(z);
    if ((tid & 31) == 0) red[tid >> 5] = z;
    __syncthreads();
    if (tid < n_split) {
        const float zz = tid == 0 ? ((red[0] + red[1]) + (red[2] + red[3])) : 0.f;
        logits[(static_cast<size_t>(tid) * M + t) * (E + 1) + E] = zz;
    }
}

}  // namespace

// 2D tensor map over an f32 [rows][cols] row-major matrix, box box_rows x 32 cols, 128B swizzle.
bool make_f32_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);

void launch_split_tf32(const float* src, size_t n, float* hi, float* lo, cudaStream_t s) {
    split_tf32_kernel<<<1184, 256, 0, s>>>(src, n, hi, lo);
}

void launch_split_x(const IoArgs* io, int M, int H, float* hi, float* lo, const float* gate_w, float* logits,
                    int n_split, int E, cudaStream_t s) {
    split_x_kernel<<<M, 128, 0, s>>>(io, M, H, hi, lo, gate_w, logits, n_split, E);
}

int router_tc_split(int M, int E, int H) {
    const int tiles = ((E + 127) / 128) * ((M + kRTokMax - 1) / kRTokMax);
    int split = 1;
    while (split < 16 && tiles * split * 2 <= 160 && (H / 32) % (split * 2) == 0) split *= 2;
    return split;
}

void launch_router_tc(const Layer& L, const CUtensorMap& xh, const CUtensorMap& xl, int M,
                      float* partial, int* status, cudaStream_t s) {
    const int E = static_cast<int>(L.spec.n_experts), H = static_cast<int>(L.spec.hidden);
    const int split = router_tc_split(M, E, H);
    cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kRSmem));
    dim3 grid((E + 127) / 128, (M + kRTokMax - 1) / kRTokMax, split);
    router_tc_kernel<<<grid, kRThreads, kRSmem, s>>>(L.rmaps[0], L.rmaps[1], xh, xl, M, E, H / split,
                                                     partial, status);
}

}  // namespace moe
