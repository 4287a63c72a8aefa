// Fused single-token MoE layer (decode, M = 1): router, softmax + top-k, shared and routed
// SwiGLU experts and the weighted combine in one launch -- the whole per-token path of
// moe-680m's router.comp + router_topk.comp + do_route + the 18 w1_w3_fused / w2_scatter
// dispatches of record_and_submit_moe's decode branch (src/inference.rs:734-762).
//
// One CTA per SM, 16 warps.  Phases:
//   1. every warp computes router-row quarters (x . Wr[e], f32; row E = the shared-expert gate
//      g . x) and each CTA arrives on a grid counter;
//   2. gate/up work units (expert slot, row j): h[slot][j] = silu(W1[j].x) * (W3[j].x), slots
//      0..k-1 routed, slot k shared.  Warps first run the shared expert's units, which need no
//      routing; then every CTA waits for all router rows, computes softmax + top-k itself from
//      the logits (identically in every CTA) and runs its routed units;
//   3. after a second arrival on the counter: out[n] = resid[n] + scale * sum_s w_s (W2_s[n].h_s),
//      one warp per output row.
// Expert rows are copied to shared memory with coalesced 16-byte cp.async (a 32-lane load then
// covers 4 whole 128-byte lines) and decoded from there; loading the sub-block layout directly
// from global memory touches each line with several partial requests and is limited by the
// SM's outstanding-request capacity.
//
// Expert dot products are integer: the IQ4_XS codes are exact bytes (kvalue + 128), the
// activation row (x, or one slot of h) is rounded to 16-bit fixed point with a power-of-two
// scale chosen from its largest magnitude, and dp2a accumulates code x activation products of a
// 32-weight sub-block exactly in int32.  Each sub-block sum is then converted to f32, multiplied
// by its scale d*(ls-32) and accumulated in f32 in a fixed order.  The only rounding besides
// f32 accumulation is the 16-bit activation grid (relative step 2^-15 of the row maximum).  The
// max |h| of a slot is gathered during phase 2 (per CTA, then one 64-bit atomicMax per slot
// whose high word is the launch's epoch, so stale values of earlier launches always lose).
//
// Grid synchronisation uses one 64-bit counter that only grows: every CTA adds 1 at each of the
// two arrival points, so a launch of G CTAs adds 2G and a launch finds its base by rounding the
// value it reads at entry down to a multiple of 2G.  Nothing has to be reset between launches
// (CUDA-graph replay is safe).  Every spin wait gives up after 100 ms, records kDevTimeout and
// continues; moe_sync then clears the counter along with the status word.
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

#ifdef MOE_TC_TRACE
__device__ unsigned long long g_dec_trace[160][16];
__device__ volatile int g_route_done[160];  // per CTA: phase timestamps (debug builds)
#define DEC_TRACE(i) do { if (blockIdx.x < 160 && threadIdx.x == 0) g_dec_trace[blockIdx.x][i] = tc::globaltimer_ns(); } while (0)
#define DEC_TRACE_R(i) do { if (blockIdx.x < 160 && threadIdx.x == 32 * kRouteWarp) g_dec_trace[blockIdx.x][i] = tc::globaltimer_ns(); } while (0)
extern "C" int moe_debug_dec_trace(unsigned long long* out) {
    return cudaMemcpyFromSymbol(out, g_dec_trace, sizeof(g_dec_trace)) == cudaSuccess ? 0 : -2;
}
#else
#define DEC_TRACE(i) do {} while (0)
#define DEC_TRACE_R(i) do {} while (0)
#endif

namespace {

constexpr int kDWarps = 16;
constexpr int kDThreads = 32 * kDWarps;
constexpr int kRouteWarp = kDWarps - 1;  // its units come last in the unit order
constexpr uint64_t kSpinLimitNs = 100000000ull;  // 100 ms
constexpr int kMaxH = 2048;                      // decode_supported limits
constexpr int kMaxI = 512;
// 16-bit activation pairs in shared memory: sub-block sb (32 values) occupies words
// [sb*kQW, sb*kQW+16); word 4w+i holds values 4w+i (low half) and 16+4w+i (high half), the
// pairing of one IQ4_XS qs word's low and high nibbles.  Word 16 holds 128 * (sum of the 32
// values), the correction for codes stored as kvalue + 128.  The stride of 20 words keeps the
// 16-byte loads of 8 consecutive lanes on distinct banks.
constexpr int kQW = 20;
constexpr int kMaxRow13 = kMaxH / kQK * kBlockBytes;  // bytes of one W1/W3 row
constexpr int kMaxRow2 = kMaxI / kQK * kBlockBytes;   // bytes of one W2 row
constexpr size_t kDecodeSmem = sizeof(float) * padded_len(kMaxH) + sizeof(uint32_t) * (kMaxH / 32) * kQW +
                               sizeof(uint32_t) * (kMaxTopK + 1) * (kMaxI / 32) * kQW +
                               size_t(kDWarps) * 4 * kMaxRow13 + size_t(kDWarps) * (kMaxTopK + 1) * kMaxRow2;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Sub-block `sb` of a row staged in shared memory (the layout of load_subblk).
__device__ __forceinline__ SubBlk lds_subblk(const uint8_t* row, int sb) {
    const uint8_t* blk = row + (sb >> 3) * kBlockBytes;
    SubBlk s;
    s.hdr = *reinterpret_cast<const uint2*>(blk);
    const uint2* q = reinterpret_cast<const uint2*>(blk + 8 + (sb & 7) * 16);
    s.q01 = q[0];
    s.q23 = q[1];
    return s;
}

struct DecodeArgs {
    const IoArgs* io;     // activation pointers in device memory (graph replay), or null:
    const float* x_direct;       // ... then these (a direct launch)
    const float* resid_direct;
    float* out_direct;
    float norm_eps;       // >= 0: the layer input is RMSNorm(x) (no gain), the residual x
    const uint8_t* pf[4];  // next layer's router and shared W1, W3, W2 (L2 prefetch), or null
    uint32_t pf_bytes[4];
    const float* wr;      // [E][H]
    const float* bias;    // [E] or null
    const float* gate_w;  // [H] or null (gate 1.0)
    ExpertTables tabs;
    int H, I, E, k;
    int has_shared;
    float scale;
    float* logits;        // [4][E+1] column-quarter partial logits
    uint2* topk;          // [k+1] records (written by CTA 0 for inspection)
    float* h;             // [k+1][I]
    unsigned long long* counter;
    unsigned long long* hmax;  // [k+1]: (launch epoch << 32) | bits of max |h| per slot
    int* status;
};

__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Exact integer dot of one IQ4_XS sub-block with 32 packed 16-bit activations (kQW layout):
// sum over j of kv(code_j) * a_j.
__device__ __noinline__ int dot_subblk_i16(const SubBlk& s, const uint32_t* aq) {
    const uint4* a4 = reinterpret_cast<const uint4*>(aq);
    const uint32_t w[4] = {s.q01.x, s.q01.y, s.q23.x, s.q23.y};
    int acc = -static_cast<int>(aq[16]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t r0, r1;
        kv_lookup8(w[i], r0, r1);  // r0 bytes: codes 4i, 16+4i, 4i+1, 17+4i (+128)
        const uint4 av = a4[i];
        acc = dp2a_lo(av.x, r0, acc);
        acc = dp2a_hi(av.y, r0, acc);
        acc = dp2a_lo(av.z, r1, acc);
        acc = dp2a_hi(av.w, r1, acc);
    }
    return acc;
}

// 16-bit fixed-point value of v at scale sc (a power of two), clamped to +-32767.
__device__ __forceinline__ int q16(float v, float sc) {
    return max(-32767, min(32767, __float2int_rn(v * sc)));
}

// Scale 2^e with max_abs * 2^e in [16384, 32768), or 1 for an all-zero row.
__device__ __forceinline__ float q16_scale(float max_abs) {
    if (!(max_abs > 0.f) || !isfinite(max_abs)) return 1.f;
    int e;
    frexpf(max_abs, &e);  // max_abs = m * 2^e, m in [0.5, 1)
    return ldexpf(1.f, 15 - e);
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0, after a __syncthreads of its CTA: arrive on the counter (no return value needed).
__device__ __forceinline__ void grid_arrive(unsigned long long* counter) {
    __threadfence();
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" :: "l"(counter) : "memory");
}

// Thread 0: wait until the counter reaches `target` (bounded).
__device__ __forceinline__ void grid_wait(const unsigned long long* counter, unsigned long long target,
                                          int* status) {
    if (ld_acquire_u64(counter) >= target) return;
    const uint64_t t0 = tc::globaltimer_ns();
    while (ld_acquire_u64(counter) < target) {
        if (tc::globaltimer_ns() - t0 > kSpinLimitNs) { set_dev_error(status, kDevTimeout); return; }
    }
}

__global__ void __launch_bounds__(kDThreads, 1) decode_kernel(const DecodeArgs a) {
    extern __shared__ __align__(16) float sm[];
    float* xs = sm;                                                      // padded f32 x (router)
    uint32_t* xq = reinterpret_cast<uint32_t*>(sm + padded_len(kMaxH));  // [H/32][kQW]
    uint32_t* hq = xq + kMaxH / 32 * kQW;                                // [k+1][I/32][kQW]
    uint8_t* st13 = reinterpret_cast<uint8_t*>(hq + (kMaxTopK + 1) * (kMaxI / 32) * kQW);  // W1/W3 rows
    uint8_t* st2 = st13 + kDWarps * 4 * kMaxRow13;                       // W2 rows
    __shared__ const uint8_t* tw[3][kMaxExperts + 1];  // expert weight pointers W1, W3, W2
    __shared__ unsigned long long base;
    __shared__ float red[kDWarps];
    __shared__ float wgt[kMaxTopK + 1];
    __shared__ int slot_e[kMaxTopK + 1];
    __shared__ uint32_t s_hmax[kMaxTopK + 1];  // bits of max |h| per slot over this CTA's units
    __shared__ float hscale[kMaxTopK + 1], hw[kMaxTopK + 1];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gwarp = blockIdx.x * kDWarps + warp, nwarps = gridDim.x * kDWarps;
    const float* x = a.io ? a.io->x : a.x_direct;
    const int H = a.H, I = a.I, E = a.E, k = a.k;
    const int ns = k + (a.has_shared ? 1 : 0);
    const unsigned long long G = gridDim.x;

    DEC_TRACE(0);
    // Warps are numbered with the CTAs interleaved (pw), so that the shared expert's units,
    // which come first, spread over every SM instead of filling the first few.
    const int pw = warp * static_cast<int>(G) + static_cast<int>(blockIdx.x);
    const int g_sh = a.has_shared ? I : 0;
    const int total = g_sh + k * I;
    const int n_my = pw < total ? (total - pw + nwarps - 1) / nwarps : 0;  // this warp's units
    const int n_sh = pw < g_sh ? (g_sh - pw + nwarps - 1) / nwarps : 0;    // ... of them shared
    const int rb13 = H / kQK * kBlockBytes, nch13 = rb13 / 16;
    uint8_t* st_w = st13 + warp * 4 * kMaxRow13;  // this warp's [2 units][W1, W3] row staging
    // unit t of this warp: rows j of W1 and W3 of expert e into staging slot t & 1
    auto issue_unit = [&](int t, const uint8_t* w1e, const uint8_t* w3e) {
        const int g = pw + t * nwarps;
        const size_t off = static_cast<size_t>(g < g_sh ? g : (g - g_sh) % I) * rb13;
        uint8_t* dst = st_w + (t & 1) * 2 * kMaxRow13;
        for (int c = lane; c < 2 * nch13; c += 32) {
            const int m = c >= nch13 ? 1 : 0, o = (c - m * nch13) * 16;
            cp_async16(dst + m * kMaxRow13 + o, (m ? w3e : w1e) + off + o);
        }
    };
    const uint8_t* sh1 = nullptr;
    const uint8_t* sh3 = nullptr;
    if (n_sh > 0) {
        sh1 = a.tabs.w1[E];
        sh3 = a.tabs.w3[E];
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {  // the first two shared units start loading at once
        if (t < n_sh) issue_unit(t, sh1, sh3);
        cp_commit();
    }
    // x, then the expert pointer tables into registers; the tables are stored to shared
    // memory after the router rows, hiding their latency
    float4 xv4[kMaxH / (4 * kDThreads)];
#pragma unroll
    for (int t = 0; t < kMaxH / (4 * kDThreads); ++t) {
        const int i = (tid + t * kDThreads) * 4;
        if (i < H) xv4[t] = *reinterpret_cast<const float4*>(x + i);
    }
    constexpr int kTabPerThread = (3 * (kMaxExperts + 1) + kDThreads - 1) / kDThreads;
    const uint8_t* tv[kTabPerThread];
#pragma unroll
    for (int t = 0; t < kTabPerThread; ++t) {
        const int i = tid + t * kDThreads;
        const int m = i / (E + 1), e = i - m * (E + 1);
        tv[t] = i < 3 * (E + 1) ? (m == 0 ? a.tabs.w1 : m == 1 ? a.tabs.w3 : a.tabs.w2)[e] : nullptr;
    }
    if (tid == 0) {
        const unsigned long long v = ld_acquire_u64(a.counter);
        base = v - v % (2 * G);
        if (a.has_shared) slot_e[k] = E;
    }
    if (tid <= kMaxTopK) s_hmax[tid] = 0u;
    if (a.norm_eps >= 0.f) {
        // RMSNorm of the layer input (rms_norm.comp: x / sqrt(mean(x^2) + eps), no gain), the
        // sum of squares reduced in a fixed order in every CTA
        float ss = 0.f;
#pragma unroll
        for (int t = 0; t < kMaxH / (4 * kDThreads); ++t) {
            const int i = (tid + t * kDThreads) * 4;
            if (i < H) {
                const float4 v = xv4[t];
                ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kDWarps; ++w) tot += red[w];
        const float r = 1.0f / sqrtf(tot / static_cast<float>(H) + a.norm_eps);
        __syncthreads();  // red[] reused below
#pragma unroll
        for (int t = 0; t < kMaxH / (4 * kDThreads); ++t) {
            xv4[t].x *= r; xv4[t].y *= r; xv4[t].z *= r; xv4[t].w *= r;
        }
    }
    float mx = 0.f;
#pragma unroll
    for (int t = 0; t < kMaxH / (4 * kDThreads); ++t) {
        const int i = (tid + t * kDThreads) * 4;
        if (i < H) {
            const float4 v = xv4[t];
            *reinterpret_cast<float4*>(xs + padded_idx(i)) = v;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            if ((v.x * 0.f + v.y * 0.f) + (v.z * 0.f + v.w * 0.f) != 0.f) mx = INFINITY;  // NaN or inf
        }
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();  // xs complete

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
    __syncthreads();  // this CTA's logits are written
    DEC_TRACE(1);
    if (tid == 0) grid_arrive(a.counter);
    // x as 16-bit pairs for the experts (scale from the block maximum of |x|)
    mx = red[0];
#pragma unroll
    for (int w = 1; w < kDWarps; ++w) mx = fmaxf(mx, red[w]);
    const bool x_finite = isfinite(mx);
    const float sx = q16_scale(mx), inv_sx = 1.f / sx;
    for (int p = tid; p < H / 2; p += kDThreads) {  // 16 consecutive lanes per sub-block
        const int sb = p >> 4, wi = p & 15;
        const int j = sb * 32 + (wi >> 2) * 4 + (wi & 3);
        const int lo = q16(xs[padded_idx(j)], sx), hi = q16(xs[padded_idx(j + 16)], sx);
        xq[sb * kQW + wi] = (static_cast<uint32_t>(lo) & 0xFFFFu) | (static_cast<uint32_t>(hi) << 16);
        int sum = lo + hi;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (wi == 0) xq[sb * kQW + 16] = static_cast<uint32_t>(128 * sum);
    }
#pragma unroll
    for (int t = 0; t < kTabPerThread; ++t) {
        const int i = tid + t * kDThreads;
        if (i < 3 * (E + 1)) tw[i / (E + 1)][i % (E + 1)] = tv[t];
    }
    __syncthreads();  // xq, tw, slot_e[k]

    // ---- phase 2: gate/up units ------------------------------------------------------------
    // Units g = 0 .. total-1 in one global sequence (the shared expert's I rows first), unit g
    // on the warp with pw = g mod (warps in the grid).  A unit's two rows are copied into this
    // warp's staging slot with 16-byte cp.async (coalesced: 4 full lines per instruction), two
    // units in flight, and decoded from shared memory.
    const int nsb_h = H / 32;  // <= 64: two sub-blocks per lane at most
    auto compute_unit = [&](int t) {
        const uint8_t* s1 = st_w + (t & 1) * 2 * kMaxRow13;
        const uint8_t* s3 = s1 + kMaxRow13;
        float gt = 0.f, up = 0.f;
#pragma unroll 1
        for (int i = 0; i < 2; ++i) {  // not unrolled: code size (instruction-cache misses) matters
            const int sb = lane + 32 * i;
            if (sb < nsb_h) {
                const uint32_t* aq = xq + sb * kQW;
                const SubBlk b1 = lds_subblk(s1, sb), b3 = lds_subblk(s3, sb);
                gt = fmaf(iq4_subscale(b1.hdr.x, b1.hdr.y, sb & 7), static_cast<float>(dot_subblk_i16(b1, aq)), gt);
                up = fmaf(iq4_subscale(b3.hdr.x, b3.hdr.y, sb & 7), static_cast<float>(dot_subblk_i16(b3, aq)), up);
            }
        }
        gt = warp_sum(gt) * inv_sx;
        up = warp_sum(up) * inv_sx;
        if (!x_finite) gt = up = __int_as_float(0x7fc00000);
        const int g = pw + t * nwarps;
        const int slot = g < g_sh ? k : (g - g_sh) / I, j = g < g_sh ? g : (g - g_sh) % I;
        if (lane == 0) {
            const float hv = silu_f(gt) * up;
            a.h[static_cast<size_t>(slot) * I + j] = hv;
            atomicMax(&s_hmax[slot], __float_as_uint(fabsf(hv)));  // NaN bits exceed inf's
        }
    };
    // runs units [t0, t1) of this warp; units t0 and t0+1 were issued (or committed empty)
    auto run_units = [&](int t0, int t1, auto&& issue) {
        for (int t = t0; t < t1; ++t) {
            cp_wait<1>();
            __syncwarp();
            compute_unit(t);
            __syncwarp();  // the slot is free again
            if (t + 2 < t1) issue(t + 2);
            cp_commit();
        }
    };
    run_units(0, n_sh, [&](int t) { issue_unit(t, sh1, sh3); });
    DEC_TRACE(2);

    // ---- routing, computed redundantly by every CTA by one warp from the published logits ---
    // softmax over E (router_topk.comp:36-92) with max and sum reduced in a fixed order, so
    // every CTA derives identical probabilities; then k rounds of selection: the largest
    // probability (as its bit pattern, probabilities being non-negative) among the experts not
    // taken yet, ties to the lower expert index.
    if (warp == kRouteWarp) {
        if (lane == 0) grid_wait(a.counter, base + G, a.status);
        __syncwarp();
        DEC_TRACE_R(3);
        const float* lg = a.logits;
        float pv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // unconditional (clamped) loads, so all issue at once
            const int e = min(lane + 32 * i, E - 1);
            const float b = a.bias ? a.bias[e] : 0.f;
            pv[i] = (((__ldcg(lg + e) + __ldcg(lg + (E + 1) + e)) + __ldcg(lg + 2 * (E + 1) + e)) +
                     __ldcg(lg + 3 * (E + 1) + e)) + b;
        }
        float lmax = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) if (lane + 32 * i < E) lmax = fmaxf(lmax, pv[i]);
        lmax = warp_max(lmax);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            pv[i] = lane + 32 * i < E ? expf(pv[i] - lmax) : 0.f;
            sum += pv[i];
        }
        sum = warp_sum(sum);
        uint32_t key[8];
        uint32_t avail = 0;  // bit i: expert lane + 32 i exists and is not taken
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float p = sum > 0.f ? pv[i] / sum : 0.f;
            key[i] = __float_as_uint(p);
            if (p != p) { set_dev_error(a.status, kDevBadExpert); key[i] = 0; }  // NaN logits
            if (lane + 32 * i < E) avail |= 1u << i;
        }
        DEC_TRACE_R(9);
        for (int r = 0; r < k; ++r) {
            uint32_t best = 0;
            int bi = -1;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (((avail >> i) & 1u) && (bi < 0 || key[i] > best)) { best = key[i]; bi = i; }
            const uint32_t m = __reduce_max_sync(0xffffffffu, bi >= 0 ? best : 0u);
            const uint32_t cand = (bi >= 0 && best == m) ? static_cast<uint32_t>(lane + 32 * bi) : 0xFFFFu;
            const uint32_t e = __reduce_min_sync(0xffffffffu, cand);
            if (e == cand) avail &= ~(1u << bi);  // the winner lane drops it
            if (lane == 0) {
                slot_e[r] = static_cast<int>(e);
                wgt[r] = __uint_as_float(m);
                if (blockIdx.x == 0) a.topk[1 + r] = make_uint2(e, m);
            }
        }
        if (lane == 0) {  // the shared-expert gate sigmoid(g . x), or 1 without a gate weight
            float gt = 1.0f;
            if (a.gate_w) {
                const float z = ((__ldcg(lg + E) + __ldcg(lg + (E + 1) + E)) + __ldcg(lg + 2 * (E + 1) + E)) +
                                __ldcg(lg + 3 * (E + 1) + E);
                gt = 1.0f / (1.0f + expf(-z));
            }
            if (a.has_shared) wgt[k] = gt;
            if (blockIdx.x == 0) a.topk[0] = make_uint2(static_cast<uint32_t>(E), __float_as_uint(gt));
        }
    }
    __syncthreads();
    DEC_TRACE(4);

    cp_wait<0>();  // only empty groups can be pending here
    auto issue_routed = [&](int t) {
        const int g = pw + t * nwarps;
        const int e = slot_e[(g - g_sh) / I];
        issue_unit(t, tw[0][e], tw[1][e]);
    };
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        if (n_sh + u < n_my) issue_routed(n_sh + u);
        cp_commit();
    }
    run_units(n_sh, n_my, issue_routed);

    // ---- phase 3: down projection + weighted combine + residual ----------------------------
    // warp per output row n (n = pw, pw + warps in the grid, ...); the row's W2 sub-blocks of
    // every slot are staged in shared memory by cp.async, the first row's before the grid
    // barrier.  Lane group gi (spr lanes, one per sub-block of the row) takes the slots
    // s = gi, gi + G2, ...; partial sums are reduced across the warp in a fixed order.
    const int rb2 = I / kQK * kBlockBytes, nch2 = rb2 / 16;
    uint8_t* st_d = st2 + warp * (kMaxTopK + 1) * kMaxRow2;
    auto issue_row = [&](int n) {
        for (int c = lane; c < ns * nch2; c += 32) {
            const int s = c / nch2, o = (c - s * nch2) * 16;
            cp_async16(st_d + s * kMaxRow2 + o, tw[2][slot_e[s]] + static_cast<size_t>(n) * rb2 + o);
        }
        cp_commit();
    };
    if (pw < H) issue_row(pw);
    __syncthreads();  // this CTA's h rows are written
    DEC_TRACE(5);
    // per-slot maxima of |h| from every CTA, tagged with this launch's epoch so that values
    // left by earlier launches lose (no reset needed); released by the barrier arrival
    const unsigned long long epoch = (base / (2 * G) + 1) << 32;
    if (tid < ns) atomicMax(a.hmax + tid, epoch | s_hmax[tid]);
    __syncthreads();
    if (tid == 0) {
        grid_arrive(a.counter);
        grid_wait(a.counter, base + 2 * G, a.status);
    }
    __syncthreads();
    DEC_TRACE(6);
    if (pw >= H) {  // warps without an output row: pull the next layer's fixed weights into L2
        const int idle = nwarps - H, me = pw - H;
#pragma unroll 1
        for (int r = 0; r < 4; ++r) {
            if (!a.pf[r]) continue;
            for (uint32_t o = (static_cast<uint32_t>(me) * 32 + lane) * 128; o < a.pf_bytes[r];
                 o += static_cast<uint32_t>(idle) * 32 * 128)
                asm volatile("prefetch.global.L2 [%0];" :: "l"(a.pf[r] + o));
        }
    }
    constexpr int kPairIt = ((kMaxTopK + 1) * kMaxI / 2 + kDThreads - 1) / kDThreads;
    float hlo[kPairIt], hhi[kPairIt];
#pragma unroll
    for (int it = 0; it < kPairIt; ++it) {  // every load issued before any is used
        const int q = tid + it * kDThreads;
        if (q < ns * I / 2) {
            const int j = (q >> 4) * 32 + ((q & 15) >> 2) * 4 + (q & 3);
            hlo[it] = __ldcg(a.h + j);
            hhi[it] = __ldcg(a.h + j + 16);
        }
    }
    // h as 16-bit pairs per slot (kQW layout), scale from the slot's max |h|
    if (tid < ns) {
        const unsigned long long v = __ldcg(a.hmax + tid);
        const float m = (v & ~0xFFFFFFFFull) == epoch ? __uint_as_float(static_cast<uint32_t>(v)) : __int_as_float(0x7fc00000);
        const float sc = q16_scale(m);
        hscale[tid] = sc;
        hw[tid] = isfinite(m) ? wgt[tid] / sc : __int_as_float(0x7fc00000);
    }
    __syncthreads();
#pragma unroll
    for (int it = 0; it < kPairIt; ++it) {  // 16 consecutive lanes per sub-block
        const int q = tid + it * kDThreads;
        if (q >= ns * I / 2) break;
        const int gsb = q >> 4, wi = q & 15;           // gsb = slot * (I/32) + sub-block
        const float sc = hscale[gsb / (I / 32)];
        const int lo = q16(hlo[it], sc), hi = q16(hhi[it], sc);
        hq[gsb * kQW + wi] = (static_cast<uint32_t>(lo) & 0xFFFFu) | (static_cast<uint32_t>(hi) << 16);
        int s16 = lo + hi;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
        if (wi == 0) hq[gsb * kQW + 16] = static_cast<uint32_t>(128 * s16);
    }
    __syncthreads();
    DEC_TRACE(7);
    const int spr = I / 32, G2 = 32 / spr;
    const int gi = lane / spr, sb = lane - gi * spr;
    const int nslot = (ns + G2 - 1) / G2;
    const float* resid = a.io ? a.io->resid : a.resid_direct;
    float* out = a.io ? a.io->out : a.out_direct;
    for (int n = pw; n < H; n += nwarps) {
        cp_wait<0>();
        __syncwarp();
        float y = 0.f;
#pragma unroll 1
        for (int t = 0; t < nslot; ++t) {
            const int s = gi + t * G2;
            if (s < ns) {
                const SubBlk b = lds_subblk(st_d + s * kMaxRow2, sb);
                const float d = iq4_subscale(b.hdr.x, b.hdr.y, sb & 7) *
                                static_cast<float>(dot_subblk_i16(b, hq + (s * spr + sb) * kQW));
                y = fmaf(hw[s], d, y);
            }
        }
        __syncwarp();  // staging free
        if (n + nwarps < H) issue_row(n + nwarps);
        y = warp_sum(y);
        if (!x_finite) y = __int_as_float(0x7fc00000);
        if (lane == 0) out[n] = (resid ? resid[n] : 0.f) + a.scale * y;
    }
    cp_wait<0>();
    DEC_TRACE(8);
}

}  // namespace

bool decode_supported(const Layer& L) {
    // rows of whole 16-byte chunks (H and I multiples of 512) from 16-byte aligned experts
    return L.tab_aligned16 && L.spec.hidden <= kMaxH && L.spec.hidden % 512 == 0 &&
           L.spec.inter <= kMaxI && L.spec.inter % 512 == 0 && L.spec.n_experts <= kMaxExperts;
}

void launch_decode(const Layer& L, const Workspace& ws, int* sync, int sm_count, cudaStream_t s,
                   const float* x, const float* resid, float* out, float norm_eps) {
    DecodeArgs a;
    a.io = x ? nullptr : ws.io;
    a.x_direct = x;
    a.resid_direct = resid;
    a.out_direct = out;
    a.norm_eps = norm_eps;
    a.pf[0] = L.next_router;
    a.pf_bytes[0] = static_cast<uint32_t>(L.next_router_bytes);
    for (int i = 0; i < 3; ++i) {
        a.pf[1 + i] = L.next_shared[i];
        a.pf_bytes[1 + i] = static_cast<uint32_t>(L.next_shared_bytes[i]);
    }
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
    a.counter = reinterpret_cast<unsigned long long*>(sync);
    a.hmax = a.counter + 1;
    a.status = ws.status;
    // once per device (not during a stream capture that may follow the first call)
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kDecodeSmem));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    decode_kernel<<<sm_count, kDThreads, kDecodeSmem, s>>>(a);
}

}  // namespace moe
