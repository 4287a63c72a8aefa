// Fused single-token MoE layer (decode, M = 1): router, softmax + top-k, shared and routed
// SwiGLU experts and the weighted combine in one launch -- the whole per-token path of
// moe-680m's router.comp + router_topk.comp + do_route + the 18 w1_w3_fused / w2_scatter
// dispatches of record_and_submit_moe's decode branch (src/inference.rs:734-762).
//
// One CTA per SM (cooperative launch, so every CTA is resident; programmatic dependent launch
// lets a layer's prologue overlap the previous launch's tail), 16 warps.  Each CTA owns:
//   * router half-rows t = c, c + G, ... of the 2 (E + 1) halves (row E: the shared-expert gate
//     g . x), f32 dot products of the f32 router weight with x, on warps 4..15;
//   * one 32-value sub-block of h: CTA c < (k + 1) I / 32 computes units j0..j0+31 of one slot
//     (unit j: rows j of W1 and W3, h[j] = silu(W1[j] . x) * (W3[j] . x)); the shared expert's
//     sub-blocks come first, so those CTAs start without waiting for the routing;
//   * a set of output rows n, over which it computes
//     out[n] = resid[n] + scale * sum_s w_s (W2_s[n] . h_s) for all k + 1 slots.
// Work of other CTAs is consumed through two exchanges in global memory:
//   * the half-row logits carry the launch's epoch in their high 32 bits (64-bit stores and
//     loads are single-copy atomic); the routing warp of each CTA polls them until every entry
//     shows the current epoch, so the data itself is the barrier (one L2 round trip after the
//     last producer), then computes softmax + top-k itself, identically in every CTA (fixed
//     reduction order, ties to the lower index);
//   * h: each active CTA publishes its sub-block already packed (16-bit fixed point with its
//     power-of-two scale) and arrives once on a 64-bit counter with a release reduction; thread 0
//     of each CTA polls the counter (acquire) and the CTA then reads all of packed h.
//
// Weights move by bulk copies (cp.async.bulk, completion counted on mbarriers): a shared-expert
// CTA requests its W1/W3 rows at entry, a routed CTA right after the routing step (chunks of 4
// units; the rows are contiguous); W2 rows of this CTA's output rows follow and are in shared
// memory long before h is complete.  Warps waiting for the routing park on a named barrier, so
// they take no issue slots from the routing warp.
//
// Dot products are integer: IQ4_XS codes are exact bytes (kvalue + 128); activations (x, and
// each slot of h) are rounded to 16-bit fixed point with a power-of-two scale per 32-value
// sub-block, chosen from that sub-block's largest magnitude (relative step 2^-15 of it); dp2a
// accumulates a sub-block's code x activation products exactly in int32, which is then scaled
// by d * (ls - 32) / activation scale and accumulated in f32 in a fixed order.
//
// Epochs: thread 0 of every CTA reads the counter at entry (v); each of the launch's G CTAs
// adds 1 after publishing its h sub-block (CTAs without one add 1 as well), so a launch adds G.
// No CTA can arrive before every CTA of its launch has read the counter (an arrival follows a
// CTA-wide barrier that the routing warp reaches only after the logits exchange of its launch,
// which needs every CTA's logits, each published after that CTA's read), so all CTAs read the same v, use
// epoch v / G + 1 for the logits and wait for v + G.  Nothing is reset between launches
// (CUDA-graph replay is safe).  Every wait gives up after 100 ms, records kDevTimeout and lets
// the CTA finish (in-flight bulk copies are drained first); moe_sync then clears the counter
// and the exchange entries.
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

#ifdef MOE_TC_TRACE
__device__ unsigned long long g_dec_trace[160][16];
#define DEC_TRACE(i) do { if (blockIdx.x < 160 && threadIdx.x == 0) g_dec_trace[blockIdx.x][i] = tc::globaltimer_ns(); } while (0)
#define DEC_TRACE_W(i, w) do { if (blockIdx.x < 160 && threadIdx.x == 32 * (w)) g_dec_trace[blockIdx.x][i] = tc::globaltimer_ns(); } while (0)
#define DEC_CLOCK_W(i, w) do { if (blockIdx.x < 160 && threadIdx.x == 32 * (w)) g_dec_trace[blockIdx.x][i] = clock64(); } while (0)
__device__ unsigned long long g_dec_clk0[160][16];  // warp 0's own clock (sub-partition counter)
#define DEC_CLK0(i) do { if (blockIdx.x < 160 && threadIdx.x == 0) g_dec_clk0[blockIdx.x][i] = clock64(); } while (0)
extern "C" int moe_debug_dec_clk0(unsigned long long* out) {
    return cudaMemcpyFromSymbol(out, g_dec_clk0, sizeof(g_dec_clk0)) == cudaSuccess ? 0 : -2;
}
extern "C" int moe_debug_dec_trace(unsigned long long* out) {
    return cudaMemcpyFromSymbol(out, g_dec_trace, sizeof(g_dec_trace)) == cudaSuccess ? 0 : -2;
}
#else
#define DEC_TRACE(i) do {} while (0)
#define DEC_TRACE_W(i, w) do {} while (0)
#define DEC_CLOCK_W(i, w) do {} while (0)
#define DEC_CLK0(i) do {} while (0)
#endif

namespace {

constexpr int kDWarps = 16;
constexpr int kDThreads = 32 * kDWarps;
constexpr int kRouteWarp = kDWarps - 1;
constexpr uint64_t kSpinLimitNs = 100000000ull;  // 100 ms
constexpr int kMaxH = 2048;                      // decode_supported limits
constexpr int kMaxI = 512;
constexpr int kMinGrid = 144;                    // per-CTA slices below are sized for G >= 144
constexpr int kUnits = 32;                        // gate/up units per CTA: one sub-block of h
constexpr int kMaxRoutedUnits = kUnits;            // 2 per warp
constexpr int kMaxRows2 = (kMaxH + kMinGrid - 1) / kMinGrid;                  // 15
static_assert(kUnits == 2 * kDWarps, "two units per warp");
static_assert(kMaxRows2 <= kDWarps, "one output row per warp");
// The routed rows arrive in chunks of 4 units (one bulk copy of 4 W1 rows and one of 4 W3 rows;
// a chunk that straddles two slots takes two copies per matrix), each chunk on its own mbarrier:
// few large copies (the bulk-copy unit takes ~70 cycles per request) that still let the warps of
// early chunks start while later chunks land.
constexpr int kChunkUnits = 4;
constexpr int kMaxChunks = (kMaxRoutedUnits + kChunkUnits - 1) / kChunkUnits;  // 8
static_assert(kMaxChunks * 2 * kChunkUnits <= 4 * kDWarps, "chunk staging fits the routed staging");
// 16-bit activation pairs of one 32-value sub-block: word w (< 16) holds values w (low half) and
// w + 16 (high half), the pairing of one IQ4_XS qs word's low and high nibbles; word 16 holds
// 128 * (sum of the 32 values), the correction for codes stored as kvalue + 128; word 17 the f32
// bits of 1 / scale.  The stride of 20 words keeps the 16-byte loads of 8 consecutive lanes on
// distinct banks.
constexpr int kQW = 20;
constexpr int kRow13 = kMaxH / kQK * kBlockBytes;  // bytes of one W1/W3 row (1088)
constexpr int kRow2 = kMaxI / kQK * kBlockBytes;   // bytes of one W2 row (272)
constexpr size_t kStRouted = size_t(kDWarps) * 4 * kRow13;             // [warp][W1 a, W1 b, W3 a, W3 b]
constexpr size_t kStW2 = size_t(kMaxTopK + 1) * kMaxRows2 * kRow2;      // [slot][row]
constexpr size_t kDecodeSmem = kStRouted + kStW2 + sizeof(float) * kMaxH +
                               sizeof(uint32_t) * (kMaxH / 32) * kQW +
                               sizeof(uint32_t) * (kMaxTopK + 1) * (kMaxI / 32) * kQW;

struct DecodeArgs {
    const IoArgs* io;            // activation pointers in device memory (graph replay), or null:
    const float* x_direct;       // ... then these (a direct launch)
    const float* resid_direct;
    float* out_direct;
    float norm_eps;              // >= 0: the layer input is RMSNorm(x) (no gain), the residual x
    const uint8_t* pf[4];        // next layer's router and shared W1, W3, W2 (L2 prefetch), or null
    uint32_t pf_bytes[4];
    const float* wr;             // [E][H]
    const float* bias;           // [E] or null
    const float* gate_w;         // [H] or null (gate 1.0)
    const uint8_t* tw[3][kMaxExperts + 1];  // expert weight pointers W1, W3, W2 (index E: shared)
    int H, I, E, k;
    int has_shared;
    float scale;
    uint2* topk;                 // [k+1] records (written by CTA 0 for inspection)
    unsigned long long* xlog;    // [2 (E+1)] tagged half-row logits
    unsigned long long* xh;      // [k+1][I] tagged h
    unsigned long long* counter;
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

// Exact integer dot of one IQ4_XS sub-block (its four qs words) with 32 packed 16-bit
// activations (kQW layout): sum over j of kv(code_j) * a_j.  Four independent partial sums keep
// the dp2a dependency chains short (the pipe is quarter rate; with a handful of warps per
// sub-partition a single 16-long chain leaves it idle most of the time).
__device__ __forceinline__ int dot_subblk_i16(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                              const uint32_t* aq) {
    const uint4* a4 = reinterpret_cast<const uint4*>(aq);
    const uint32_t w[4] = {w0, w1, w2, w3};
    int acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t r0, r1;
        kv_lookup8(w[i], r0, r1);  // r0 bytes: codes 4i, 16+4i, 4i+1, 17+4i (+128)
        const uint4 av = a4[i];
        acc[i] = dp2a_lo(av.x, r0, 0);
        acc[i] = dp2a_hi(av.y, r0, acc[i]);
        acc[i] = dp2a_lo(av.z, r1, acc[i]);
        acc[i] = dp2a_hi(av.w, r1, acc[i]);
    }
    return ((acc[0] + acc[1]) + (acc[2] + acc[3])) - static_cast<int>(aq[16]);
}

// f32 contribution of one staged sub-block against packed activations: scale(d, ls) x
// (1 / activation scale) x exact integer dot.
__device__ __forceinline__ float subblk_dot(const uint8_t* row, int sb, const uint32_t* aq) {
    const SubBlk b = lds_subblk(row, sb);
    return iq4_subscale(b.hdr.x, b.hdr.y, sb & 7) * __uint_as_float(aq[17]) *
           static_cast<float>(dot_subblk_i16(b.q01.x, b.q01.y, b.q23.x, b.q23.y, aq));
}

// Biased exponent field f of the power-of-two scale 2^(f - 127) that brings a sub-block's largest
// magnitude m (bits mb, finite, > 0) into [16384, 32768): m = 1.x * 2^(E - 127) needs
// 2^(141 - E), i.e. f = 268 - E, clamped to the normal range (sub-blocks below 2^-113 keep
// fewer bits).  An all-zero sub-block gets scale 1 (f = 127).
__device__ __forceinline__ uint32_t q16_scale_field(uint32_t mb) {
    if (mb == 0u) return 127u;
    const int e = static_cast<int>(mb >> 23);
    return static_cast<uint32_t>(min(254, max(1, 268 - e)));
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long tag(uint32_t epoch, float v) {
    return (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
}

// Bounded wait on an mbarrier phase (a whole warp, or one thread); false on timeout.  Between
// tests the warp sleeps, so waiting warps leave the issue slots to the warps still computing.
__device__ __noinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = tc::globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(64);
        if (tc::mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 0u && tc::globaltimer_ns() - t0 > kSpinLimitNs) return false;
    }
}

// CTA named barrier 1 (barrier 0 is __syncthreads): warps park on it without issuing.
__device__ __forceinline__ void named_sync(int n) { asm volatile("bar.sync 1, %0;" :: "r"(n) : "memory"); }
__device__ __forceinline__ void named_arrive(int n) { asm volatile("bar.arrive 1, %0;" :: "r"(n) : "memory"); }

// One warp packs N sub-blocks at once (the collectives of the N sub-blocks are independent, so
// their latencies overlap): v[i] is lane's value of sub-block first + 16 i, written to
// base + (first + 16 i) * kQW when that index is below nsb.  Each sub-block gets 16-bit fixed
// point at its own power-of-two scale; a non-finite value makes its inverse scale NaN, so every
// product with the sub-block is NaN.
template <int N>
__device__ __forceinline__ void pack_subblocks(const float (&v)[N], uint32_t* base, int first, int nsb, int lane) {
    uint32_t mb[N];
#pragma unroll
    for (int i = 0; i < N; ++i) mb[i] = __reduce_max_sync(0xffffffffu, __float_as_uint(v[i]) & 0x7FFFFFFFu);
    int q[N];
    uint32_t f[N];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        f[i] = mb[i] < 0x7F800000u ? q16_scale_field(mb[i]) : 127u;
        q[i] = max(-32767, min(32767, __float2int_rn(v[i] * __uint_as_float(f[i] << 23))));
    }
    int hi[N], sum[N];
#pragma unroll
    for (int i = 0; i < N; ++i) hi[i] = __shfl_down_sync(0xffffffffu, q[i], 16);
#pragma unroll
    for (int i = 0; i < N; ++i) sum[i] = __reduce_add_sync(0xffffffffu, q[i]);
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int g = first + 16 * i;
        if (g >= nsb) continue;
        uint32_t* dst = base + g * kQW;
        if (lane < 16) dst[lane] = (static_cast<uint32_t>(q[i]) & 0xFFFFu) | (static_cast<uint32_t>(hi[i]) << 16);
        if (lane == 0) {
            dst[16] = static_cast<uint32_t>(128 * sum[i]);
            dst[17] = mb[i] < 0x7F800000u ? ((254u - f[i]) << 23) : 0x7fc00000u;  // 1 / scale, or NaN
        }
    }
}

// Order-preserving map of a float onto unsigned integers (NaN: 0, below every number).
__device__ __forceinline__ uint32_t f2ord(float f) {
    const uint32_t u = __float_as_uint(f);
    if (f != f) return 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t o) {
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

// Compare-exchange of (key desc, index asc) pairs.
__device__ __forceinline__ void cx(uint32_t& ka, uint32_t& ia, uint32_t& kb, uint32_t& ib) {
    const bool sw = kb > ka || (kb == ka && ib < ia);
    const uint32_t k0 = sw ? kb : ka, i0 = sw ? ib : ia;
    kb = sw ? ka : kb;
    ib = sw ? ia : ib;
    ka = k0;
    ia = i0;
}

// Routing of one token by one warp from the half-row logits (v0/v1: lane's experts lane + 32 i;
// g0/g1: the gate row's halves): softmax over E (router_topk.comp:36-92) with max and sum
// reduced in a fixed order, so that every CTA derives identical probabilities
// p_e = exp(l_e - max) * (1 / sum), then the k largest p in descending order, ties to the lower
// expert index.  Each lane sorts its 8 candidates once; a round then takes the warp maximum of
// the lanes' heads (a tie between heads goes to the lower index) and the winning lane pops its
// head, writing the slot's expert and probability.  Lane k writes the shared expert's slot
// (gate sigmoid(g . x), or 1 without a gate weight).  CTA 0 also writes the routing record.
__device__ __noinline__ void route_warp(const float* lg, float gz, int E, int k, bool has_gate, bool has_shared,
                                       int* status, int* slot_e, float* wgt, uint2* topk_rec) {
    const int lane = threadIdx.x & 31;
    float pv[8];
    uint32_t om = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        pv[i] = lg[min(lane + 32 * i, E - 1)];
        if (lane + 32 * i < E) om = max(om, f2ord(pv[i]));
    }
    const float lmax = ord2f(__reduce_max_sync(0xffffffffu, om));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        pv[i] = lane + 32 * i < E ? expf(pv[i] - lmax) : 0.f;
        sum += pv[i];
    }
    sum = warp_sum(sum);
    const float inv = sum > 0.f ? 1.0f / sum : 0.f;
    uint32_t key[8], idx[8];
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float p = pv[i] * inv;
        bad = bad || (p != p);
        key[i] = (p == p) ? __float_as_uint(p) : 0u;  // NaN logits: reported, ranked as 0
        idx[i] = lane + 32 * i < E ? static_cast<uint32_t>(lane + 32 * i) : 0xFFFFu;
    }
    if (bad) set_dev_error(status, kDevBadExpert);
    // sorting network of 8 (19 compare-exchanges), descending by key, ascending index on ties
    cx(key[0], idx[0], key[1], idx[1]); cx(key[2], idx[2], key[3], idx[3]);
    cx(key[4], idx[4], key[5], idx[5]); cx(key[6], idx[6], key[7], idx[7]);
    cx(key[0], idx[0], key[2], idx[2]); cx(key[1], idx[1], key[3], idx[3]);
    cx(key[4], idx[4], key[6], idx[6]); cx(key[5], idx[5], key[7], idx[7]);
    cx(key[1], idx[1], key[2], idx[2]); cx(key[5], idx[5], key[6], idx[6]);
    cx(key[0], idx[0], key[4], idx[4]); cx(key[3], idx[3], key[7], idx[7]);
    cx(key[1], idx[1], key[5], idx[5]); cx(key[2], idx[2], key[6], idx[6]);
    cx(key[1], idx[1], key[4], idx[4]); cx(key[3], idx[3], key[6], idx[6]);
    cx(key[2], idx[2], key[4], idx[4]); cx(key[3], idx[3], key[5], idx[5]);
    cx(key[3], idx[3], key[4], idx[4]);
    uint32_t my_e = 0, my_m = 0;  // lane r: slot r's expert and probability bits
    // rounds without divergence: the winning lane pops its head by selects; the slot's expert
    // comes from the winner by a shuffle that is off the rounds' dependency chain
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
        if (r >= k) break;
        const uint32_t m = __reduce_max_sync(0xffffffffu, key[0]);
        const unsigned tie = __ballot_sync(0xffffffffu, key[0] == m);
        // equal probabilities in several heads (rare): the lower expert index; computed
        // alongside, selected without a branch
        const uint32_t wmin = __reduce_min_sync(0xffffffffu, key[0] == m ? idx[0] : 0xFFFFu) & 31u;
        const uint32_t win = __popc(tie) == 1 ? static_cast<uint32_t>(__ffs(tie) - 1) : wmin;
        const uint32_t e = __shfl_sync(0xffffffffu, idx[0], static_cast<int>(win));
        const bool won = static_cast<uint32_t>(lane) == win;
#pragma unroll
        for (int i = 0; i < 7; ++i) {
            key[i] = won ? key[i + 1] : key[i];
            idx[i] = won ? idx[i + 1] : idx[i];
        }
        key[7] = won ? 0u : key[7];
        idx[7] = won ? 0xFFFFu : idx[7];
        my_e = lane == r ? e : my_e;
        my_m = lane == r ? m : my_m;
    }
    if (lane < k) {
        slot_e[lane] = static_cast<int>(my_e);
        wgt[lane] = __uint_as_float(my_m);
        if (topk_rec) topk_rec[1 + lane] = make_uint2(my_e, my_m);
    }
    if (lane == 0) {
        float gt = 1.0f;
        if (has_gate) gt = 1.0f / (1.0f + expf(-gz));
        if (has_shared) {
            slot_e[k] = E;
            wgt[k] = gt;
        }
        if (topk_rec) topk_rec[0] = make_uint2(static_cast<uint32_t>(E), __float_as_uint(gt));
    }
}

__global__ void __launch_bounds__(kDThreads, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* st_r = smem;                         // W1/W3 rows of this CTA's 32 units, by chunks
    uint8_t* st_2 = st_r + kStRouted;             // raw W2 rows [slot][row]
    float* xs = reinterpret_cast<float*>(st_2 + kStW2);                 // f32 x (router)
    uint32_t* xq = reinterpret_cast<uint32_t*>(xs + kMaxH);             // [H/32][kQW]
    uint32_t* hq = xq + (kMaxH / 32) * kQW;                             // [k+1][I/32][kQW]
    __shared__ __align__(8) uint64_t bar_w2, bar_c[kMaxChunks];
    __shared__ float hloc[kUnits];               // this CTA's h values
    __shared__ unsigned long long s_base;
    __shared__ float red[kDWarps];
    __shared__ float wgt[kMaxTopK + 1];
    __shared__ int slot_e[kMaxTopK + 1];
    __shared__ float s_bias[kMaxExperts];
    __shared__ float s_lg[kMaxExperts];          // routing logits (bias added)
    __shared__ int s_failed;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
    const float* x = a.io ? a.io->x : a.x_direct;
    const int H = a.H, I = a.I, E = a.E, k = a.k;
    const int ns = k + (a.has_shared ? 1 : 0);
    const int rb13 = H / kQK * kBlockBytes, rb2 = I / kQK * kBlockBytes;
    const int spr = I / 32;  // sub-blocks per h slot
    // this CTA's slices: one 32-value sub-block of h (slot my_slot, values j0 .. j0 + 31; the
    // shared expert's sub-blocks first), or none; output rows [n0, n1)
    const int sbid = c;
    const bool active = sbid < ns * spr;
    const bool sh_cta = active && a.has_shared && sbid < spr;
    const int my_slot = !active ? -1 : (a.has_shared ? (sh_cta ? k : sbid / spr - 1) : sbid / spr);
    const int j0 = (sbid % spr) * kUnits;
    const int n0 = c * H / G, n1 = (c + 1) * H / G;
    const int nrows = n1 - n0;
    const int T = 2 * (E + (a.gate_w ? 1 : 0)), half = H / 2;
    // router half-row task of this warp (warps 4..15; decode_supported bounds the count)
    const int task = warp >= 4 ? c + G * (warp - 4) : T;

    DEC_TRACE(0);
    DEC_CLK0(0);
    // with programmatic dependent launch, wait here for the previous kernel on the stream (its
    // memory included) before reading anything it may have written
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // ---- every independent load first: x, this warp's router half-row, pointer tables, bias --
    if (tid == 0) {
        s_failed = 0;
        s_base = ld_relaxed_u64(a.counter);
        tc::mbar_init(&bar_w2, 1);
        for (int i = 0; i < kMaxChunks; ++i) tc::mbar_init(&bar_c[i], 1);
        tc::fence_mbar_init();
        // W2 rows [n0, n1) of every slot land on bar_w2: all bytes expected now, the shared
        // slot's copy issued now, the routed slots' after the routing step
        tc::mbar_arrive_expect_tx(&bar_w2, static_cast<uint32_t>(ns * nrows * rb2));
        if (a.has_shared)
            tc::bulk_load(st_2 + static_cast<size_t>(k) * kMaxRows2 * kRow2,
                          a.tw[2][E] + static_cast<size_t>(n0) * rb2, static_cast<uint32_t>(nrows * rb2), &bar_w2);
    }
    float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);  // H <= 2048 = 4 x 512 threads
    if (tid * 4 < H) xv = *reinterpret_cast<const float4*>(x + tid * 4);
    float4 wv[kMaxH / 2 / 128];
    const int hf = task & 1;
    if (task < T) {
        const int r = task >> 1;
        const float* wrow = (r < E ? a.wr + static_cast<size_t>(r) * H : a.gate_w) + hf * half;
#pragma unroll
        for (int i = 0; i < kMaxH / 2 / 128; ++i)
            if (lane * 4 + 128 * i < half) wv[i] = __ldg(reinterpret_cast<const float4*>(wrow + lane * 4 + 128 * i));
    }
    // the router bias is needed only at the routing step: loaded now, stored after the first
    // barrier
    const float bias_v = (a.bias && tid < E) ? a.bias[tid] : 0.f;
    if (a.norm_eps >= 0.f) {
        // RMSNorm of the layer input (rms_norm.comp: x / sqrt(mean(x^2) + eps), no gain), the
        // sum of squares reduced in a fixed order in every CTA
        float ss = fmaf(xv.x, xv.x, 0.f);
        ss = fmaf(xv.y, xv.y, ss); ss = fmaf(xv.z, xv.z, ss); ss = fmaf(xv.w, xv.w, ss);
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll 1
        for (int w = 0; w < kDWarps; ++w) tot += red[w];
        const float r = 1.0f / sqrtf(tot / static_cast<float>(H) + a.norm_eps);
        xv.x *= r; xv.y *= r; xv.z *= r; xv.w *= r;
    }
    bool fin = true;
    if (tid * 4 < H) {
        *reinterpret_cast<float4*>(xs + tid * 4) = xv;
        fin = isfinite(xv.x) && isfinite(xv.y) && isfinite(xv.z) && isfinite(xv.w);
    }
    const bool x_finite = __syncthreads_and(fin) != 0;  // also: xs, barriers, s_base, tables
    const unsigned long long base = s_base;
    const uint32_t epoch = static_cast<uint32_t>(base / static_cast<unsigned long long>(G)) + 1u;
    if (tid < E) s_bias[tid] = bias_v;
    DEC_TRACE(1);
    // W1/W3 rows of the CTA's 32 units (rows j0 .. j0 + 31 of one expert) in 8 chunks of 4 units,
    // each chunk one bulk copy per matrix on its own mbarrier; lanes 0-15 of one warp issue them
    auto issue_units = [&](const uint8_t* w1e, const uint8_t* w3e) {
        const int ch = lane >> 1, m = lane & 1;
        if (lane < 2 * kMaxChunks && m == 0)  // expected bytes posted before any copy is issued
            tc::mbar_arrive_expect_tx(&bar_c[ch], static_cast<uint32_t>(2 * kChunkUnits * rb13));
        __syncwarp();
        if (lane < 2 * kMaxChunks)
            tc::bulk_load(st_r + static_cast<size_t>(ch) * 2 * kChunkUnits * kRow13 + m * kChunkUnits * rb13,
                          (m ? w3e : w1e) + static_cast<size_t>(j0 + ch * kChunkUnits) * rb13,
                          static_cast<uint32_t>(kChunkUnits * rb13), &bar_c[ch]);
        __syncwarp();
    };
    if (sh_cta && warp == 1) issue_units(a.tw[0][E], a.tw[1][E]);  // needs no routing

    // ---- router half-row of this warp (f32), published with the launch's epoch --------------
    if (task < T) {
        const float* xrow = xs + hf * half;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxH / 2 / 128; ++i) {
            if (lane * 4 + 128 * i < half) {
                const float4 xv4 = *reinterpret_cast<const float4*>(xrow + lane * 4 + 128 * i);
                acc = fmaf(wv[i].x, xv4.x, acc); acc = fmaf(wv[i].y, xv4.y, acc);
                acc = fmaf(wv[i].z, xv4.z, acc); acc = fmaf(wv[i].w, xv4.w, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) st_relaxed_u64(a.xlog + task, tag(epoch, acc));
    }
    // x as 16-bit pairs per sub-block, for the experts
    {
        constexpr int kPerX = kMaxH / 32 / kDWarps;  // 4
        float v[kPerX];
#pragma unroll
        for (int i = 0; i < kPerX; ++i) {
            const int g = warp + kDWarps * i;
            v[i] = g < H / 32 ? xs[g * 32 + lane] : 0.f;
        }
        pack_subblocks<kPerX>(v, xq, warp, H / 32, lane);
    }
    __syncthreads();  // xq complete
    DEC_TRACE(2);

    // ---- routing (one warp per CTA), then the routed copies ----------------------------------
    if (warp == kRouteWarp) {
        unsigned long long v0[8], v1[8], g0 = 0, g1 = 0;
        const uint64_t t0 = tc::globaltimer_ns();
        for (;;) {
            bool ok = true;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int e = min(lane + 32 * i, E - 1);
                v0[i] = ld_relaxed_u64(a.xlog + 2 * e);
                v1[i] = ld_relaxed_u64(a.xlog + 2 * e + 1);
            }
            if (a.gate_w) {
                g0 = ld_relaxed_u64(a.xlog + 2 * E);
                g1 = ld_relaxed_u64(a.xlog + 2 * E + 1);
                ok = (g0 >> 32) == epoch && (g1 >> 32) == epoch;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) ok = ok && (v0[i] >> 32) == epoch && (v1[i] >> 32) == epoch;
            if (__all_sync(0xffffffffu, ok)) break;
            if (tc::globaltimer_ns() - t0 > kSpinLimitNs) {
                set_dev_error(a.status, kDevTimeout);
                if (lane == 0) s_failed = 1;
                break;
            }
            __nanosleep(64);
        }
        DEC_TRACE_W(3, kRouteWarp);
        DEC_CLOCK_W(12, kRouteWarp);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (lane + 32 * i < E)
                s_lg[lane + 32 * i] = (__uint_as_float(static_cast<uint32_t>(v0[i])) +
                                       __uint_as_float(static_cast<uint32_t>(v1[i]))) + s_bias[lane + 32 * i];
        __syncwarp();
        route_warp(s_lg, __uint_as_float(static_cast<uint32_t>(g0)) + __uint_as_float(static_cast<uint32_t>(g1)), E, k,
                   a.gate_w != nullptr, a.has_shared != 0, a.status, slot_e, wgt, c == 0 ? a.topk : nullptr);
        __syncwarp();
        DEC_CLOCK_W(13, kRouteWarp);
        DEC_TRACE_W(9, kRouteWarp);
        DEC_CLOCK_W(15, kRouteWarp);
        if (active && !sh_cta) issue_units(a.tw[0][slot_e[my_slot]], a.tw[1][slot_e[my_slot]]);
        __syncwarp();
        if (!sh_cta) named_arrive(kDThreads);  // the parked warps may read the routing now
        if (lane < k)  // routed W2 rows [n0, n1) of slot `lane`
            tc::bulk_load(st_2 + static_cast<size_t>(lane) * kMaxRows2 * kRow2,
                          a.tw[2][slot_e[lane]] + static_cast<size_t>(n0) * rb2, static_cast<uint32_t>(nrows * rb2),
                          &bar_w2);
        DEC_CLOCK_W(14, kRouteWarp);
        DEC_TRACE_W(4, kRouteWarp);
    }

    // ---- gate/up units: warp w computes units 2w, 2w + 1 (rows j0 + 2w, j0 + 2w + 1) ----------
    {
        // in a routed CTA every warp but the routing warp parks on barrier 1 during the routing
        // step (parked warps issue nothing); a shared-expert CTA's data needs no routing
        if (!sh_cta && warp != kRouteWarp) named_sync(kDThreads);
        DEC_CLK0(11);
        if (active) {
            const int ch = (2 * warp) / kChunkUnits;
            if (!bar_wait(&bar_c[ch], 0)) { set_dev_error(a.status, kDevTimeout); if (lane == 0) s_failed = 1; }
            DEC_CLK0(12);
#pragma unroll 1
            for (int q = 0; q < 2; ++q) {
                const int lu = 2 * warp + q, iu = lu - ch * kChunkUnits;
                const uint8_t* s1 = st_r + static_cast<size_t>(ch) * 2 * kChunkUnits * kRow13 + iu * rb13;
                const uint8_t* s3 = s1 + kChunkUnits * rb13;
                float gt = 0.f, up = 0.f;
#pragma unroll 2
                for (int sb = lane; sb < H / 32; sb += 32) {
                    const uint32_t* aq = xq + sb * kQW;
                    gt += subblk_dot(s1, sb, aq);
                    up += subblk_dot(s3, sb, aq);
                }
                gt = warp_sum(gt);
                up = warp_sum(up);
                float hv = silu_f(gt) * up;
                if (!x_finite) hv = __int_as_float(0x7fc00000);
                if (lane == 0) hloc[lu] = hv;
                DEC_CLK0(13 + q);
            }
        }
    }
    __syncthreads();  // hloc complete
    DEC_TRACE(5);
    uint32_t* hx = reinterpret_cast<uint32_t*>(a.xh);  // packed h exchange: [slots x I/32][kQW]
    if (warp == 0) {
        // publish this CTA's sub-block packed (16-bit pairs, its own power-of-two scale), then
        // arrive: one arrival per CTA, after the stores (release orders the warp's stores, which
        // __syncwarp has made visible to lane 0)
        if (active) {
            float v[1] = {hloc[lane]};
            pack_subblocks<1>(v, hx + static_cast<size_t>(sbid) * kQW, 0, 1, lane);
        }
        __syncwarp();
        if (lane == 0) asm volatile("red.release.gpu.global.add.u64 [%0], 1;" :: "l"(a.counter) : "memory");
    }
    DEC_CLK0(1);
    if (tid == 0) {  // wait for every CTA's arrival
        const unsigned long long target = base + static_cast<unsigned long long>(G);
        const uint64_t t0 = tc::globaltimer_ns();
        while (ld_acquire_u64(a.counter) < target) {
            if (tc::globaltimer_ns() - t0 > kSpinLimitNs) {
                set_dev_error(a.status, kDevTimeout);
                s_failed = 1;
                break;
            }
            __nanosleep(20);
        }
    }
    DEC_CLK0(5);
    __syncthreads();
    DEC_TRACE(6);
    DEC_CLK0(6);
    // every CTA's packed sub-block of h into shared memory (the slots' sub-blocks in order: the
    // shared expert's first when there is one)
    {
        const int P = ns * spr;
        for (int i = tid; i < P * kQW / 4; i += kDThreads)
            reinterpret_cast<uint4*>(hq)[i] = __ldcg(reinterpret_cast<const uint4*>(hx) + i);
    }
    DEC_CLK0(8);
    __syncthreads();  // hq, slot_e, wgt
    DEC_TRACE(7);
    DEC_CLK0(9);

    // the next kernel on the stream may start launching (it waits for this grid's completion
    // in its own griddepcontrol.wait before reading anything)
    asm volatile("griddepcontrol.launch_dependents;");
    // ---- down projection + weighted combine + residual --------------------------------------
    // Thread t takes the (slot, sub-block) pair p = t mod P (P = slots x I/32) for the output
    // rows r = t / P, t / P + 3, ... : its packed activations stay in registers across the rows,
    // and the pair partials (each weighted by its slot's routing weight) go to shared memory;
    // then warp r sums row r's P partials in a fixed order.
    const float* resid = a.io ? a.io->resid : a.resid_direct;
    float* out = a.io ? a.io->out : a.out_direct;
    float* part = reinterpret_cast<float*>(st_r);  // [kMaxRows2][P]; the W1/W3 staging is free
    {
        const int P = ns * spr;
        if (!bar_wait(&bar_w2, 0)) { set_dev_error(a.status, kDevTimeout); if (lane == 0) s_failed = 1; }
        if (tid < 3 * P) {
            // pair pp is exchange sub-block pp: the shared expert's sub-blocks come first
            const int pp = tid % P, r0 = tid / P, sb = pp % spr;
            const int s = a.has_shared ? (pp < spr ? k : pp / spr - 1) : pp / spr;
            const uint32_t* aq = hq + pp * kQW;
            const uint4 a0 = reinterpret_cast<const uint4*>(aq)[0], a1 = reinterpret_cast<const uint4*>(aq)[1];
            const uint4 a2 = reinterpret_cast<const uint4*>(aq)[2], a3 = reinterpret_cast<const uint4*>(aq)[3];
            const int corr = static_cast<int>(aq[16]);
            const float f = wgt[s] * __uint_as_float(aq[17]);
            const uint8_t* rows = st_2 + static_cast<size_t>(s) * kMaxRows2 * kRow2 + (sb >> 3) * kBlockBytes;
            // the thread's rows unrolled completely, so that their loads and lookups interleave
#pragma unroll
            for (int i = 0; i < (kMaxRows2 + 2) / 3; ++i) {
                const int r = r0 + 3 * i;
                if (r >= nrows) break;
                const uint8_t* blk = rows + static_cast<size_t>(r) * rb2;
                const uint2 hdr = *reinterpret_cast<const uint2*>(blk);
                // the qs bytes of a sub-block start 8 bytes into a 16-byte unit: two 8-byte loads
                const uint2 q01 = *reinterpret_cast<const uint2*>(blk + 8 + (sb & 7) * 16);
                const uint2 q23 = *reinterpret_cast<const uint2*>(blk + 16 + (sb & 7) * 16);
                const uint32_t w[4] = {q01.x, q01.y, q23.x, q23.y};
                const uint4 av[4] = {a0, a1, a2, a3};
                int acc[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint32_t k0, k1;
                    kv_lookup8(w[i], k0, k1);
                    acc[i] = dp2a_lo(av[i].x, k0, 0);
                    acc[i] = dp2a_hi(av[i].y, k0, acc[i]);
                    acc[i] = dp2a_lo(av[i].z, k1, acc[i]);
                    acc[i] = dp2a_hi(av[i].w, k1, acc[i]);
                }
                const int dot = ((acc[0] + acc[1]) + (acc[2] + acc[3])) - corr;
                part[r * P + pp] = f * iq4_subscale(hdr.x, hdr.y, sb & 7) * static_cast<float>(dot);
            }
        }
        __syncthreads();
        if (warp < nrows) {
            float y = 0.f;
#pragma unroll 1
            for (int i = lane; i < P; i += 32) y += part[warp * P + i];
            y = warp_sum(y);
            if (!x_finite) y = __int_as_float(0x7fc00000);
            if (lane == 0) out[n0 + warp] = (resid ? resid[n0 + warp] : 0.f) + a.scale * y;
        }
    }
    DEC_CLK0(10);
    DEC_TRACE(8);
    // pull this CTA's slice of the next layer's fixed weights into L2
#pragma unroll 1
    for (int r = 0; r < 4; ++r) {
        if (!a.pf[r]) continue;
        const uint32_t nl = (a.pf_bytes[r] + 127) / 128;
        for (uint32_t l = static_cast<uint32_t>(c) + static_cast<uint32_t>(G) * tid; l < nl;
             l += static_cast<uint32_t>(G) * kDThreads)
            asm volatile("prefetch.global.L2 [%0];" :: "l"(a.pf[r] + static_cast<size_t>(l) * 128));
    }
    __syncthreads();
    DEC_TRACE(10);
    if (s_failed && tid == 0) {  // drain bulk copies still landing in this CTA's shared memory
        bar_wait(&bar_w2, 0);
        if (active)
            for (int ch = 0; ch < kMaxChunks; ++ch) bar_wait(&bar_c[ch], 0);
    }
}

}  // namespace

size_t decode_exchange_words(int E, int k, int I) {
    return static_cast<size_t>(2) * (E + 1) + static_cast<size_t>(k + 1) * I;
}

bool decode_supported(const Layer& L, int sm_count) {
    // rows of whole 16-byte chunks (H and I multiples of 512) from 16-byte aligned experts, a
    // grid large enough for the per-CTA slices of the shared memory plan, and at most one router
    // half-row per warp 4..15
    const int T = 2 * (static_cast<int>(L.spec.n_experts) + 1);
    const int ns = static_cast<int>(L.spec.top_k) + (L.has_shared() ? 1 : 0);
    return !L.ref36() && L.tab_aligned16 && L.spec.hidden <= kMaxH && L.spec.hidden % 512 == 0 &&
           L.spec.inter <= kMaxI && L.spec.inter % 512 == 0 && L.spec.n_experts <= kMaxExperts &&
           sm_count >= kMinGrid && T <= (kDWarps - 4) * sm_count &&
           ns * static_cast<int>(L.spec.inter / 32) <= sm_count;  // one h sub-block per CTA
}

int launch_decode(const Layer& L, const Workspace& ws, int* sync, int sm_count, cudaStream_t s,
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
    a.H = static_cast<int>(L.spec.hidden);
    a.I = static_cast<int>(L.spec.inter);
    a.E = static_cast<int>(L.spec.n_experts);
    for (int m = 0; m < 3; ++m)
        for (int e = 0; e <= a.E; ++e) a.tw[m][e] = L.host_tab[static_cast<size_t>(m) * (a.E + 1) + e];
    a.k = static_cast<int>(L.spec.top_k);
    a.has_shared = L.has_shared() ? 1 : 0;
    a.scale = L.spec.scale;
    a.topk = ws.topk;
    a.xlog = ws.dx;
    a.xh = ws.dx + 2 * (a.E + 1);
    a.counter = reinterpret_cast<unsigned long long*>(sync);
    a.status = ws.status;
    // once per device (not during a stream capture that may follow the first call)
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kDecodeSmem));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    // cooperative: the CTAs wait on each other's exchange entries, so all must be resident
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count));
    cfg.blockDim = dim3(kDThreads);
    cfg.dynamicSmemBytes = kDecodeSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;  // cooperative, and the next kernel on the stream may launch early (PDL)
    return cudaLaunchKernelEx(&cfg, decode_kernel, a) == cudaSuccess ? 0 : -1;
}

}  // namespace moe
