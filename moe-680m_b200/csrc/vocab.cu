// Vocabulary projection with an IQ4_XS weight matrix: the LM head and the MTP output heads of
// moe-680m (src/inference.rs:319-330 and :355-360, dispatched on shaders/attn_output.comp),
// logits[m][n] = sum_h x[m][h] * W[n][h] for a matrix W of V rows (GGUF row layout, each row
// H/256 IQ4_XS blocks), at most 8 activation rows, with an optional fused greedy argmax (the
// reference's util::argmax, src/util.rs:66-76, run on the host over the downloaded logits).
//
// The pass is a single read of W (V * H/256 * 136 bytes; 270 MB for the 248,320 x 2048 head),
// so it is bound by HBM bandwidth.  Layout of the work:
//   * persistent grid, one CTA per SM; a chunk of 16*R consecutive rows (R = 4 for one
//     activation row with H <= 2048, else 2) is one contiguous byte range of W and is copied to shared memory
//     by a single bulk copy (cp.async.bulk, completion counted on an mbarrier) issued by a
//     producer warp into a ring of up to 8 stages;
//   * 16 consumer warps take R rows each per chunk: lane l decodes sub-blocks l, l+32, ... of
//     each row once and applies them to every activation row;
//   * the products are integer, as in the single-token layer kernel: activations are rounded to
//     16-bit fixed point with a power-of-two scale per row (from its largest magnitude), dp2a
//     sums code x activation over a 32-weight sub-block exactly, and the sub-block sums are
//     scaled by d*(ls-32) and accumulated in f32 in a fixed order (then a fixed warp tree).
//   * argmax: every lane t keeps the best (value, lowest index) key of activation row t over its
//     warp's rows; keys meet in shared memory, then in 64-bit global atomics, and the last CTA
//     to finish (a ticket counter) writes the token ids and resets the keys and the ticket, so
//     repeated launches and CUDA-graph replays need no host-side reset.
// Every mbarrier wait is bounded (100 ms); a timeout records kDevTimeout in the status word and
// the CTA drains its own copies in flight before it exits.
#include <cuda_runtime.h>

#include <algorithm>

#include "moe_common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

namespace {

constexpr int kVWarps = 16;                    // consumer warps
// rows per warp per chunk: independent rows give the decode/dot chains instruction-level
// parallelism (measured at M=1 on 248,320 x 2048: 1 row 110 us, 2 rows 94 us, 4 rows 90 us)
// (4 rows only with the register-held activations, H <= 2048, so that two or more stages fit)
template <int MT, int NL>
constexpr int vocab_rows() { return MT == 1 && NL > 0 ? 4 : 2; }
constexpr int kVThreads = 32 * (kVWarps + 1);  // + the producer warp
constexpr int kVMaxStages = 8;
constexpr int kVQW = 20;  // words per 32-value group of packed 16-bit activations (see below)
constexpr uint64_t kVSpinNs = 100000000ull;
constexpr int kVHeader = 256;  // barriers, block keys, scales, abort flag
constexpr int kVSmemMax = 232448;

// Packed 16-bit activations of one row: sub-block sb (values 32sb..32sb+31) occupies words
// [sb*kVQW, sb*kVQW+16); word 4w+i holds values 4w+i (low half) and 16+4w+i (high half), the
// pairing of the low and high nibbles of one qs byte; word 16 holds 128 * (sum of the 32
// values), the correction for codes stored as kvalue + 128.

struct VocabArgs {
    const uint8_t* w;
    const float* x;       // [M][H]
    float* logits;        // [M][V] or null
    uint32_t* ids;        // [M] or null
    unsigned long long* keys;  // [8] argmax keys (zero between launches)
    unsigned int* ticket;      // CTA completion counter (zero between launches)
    int* status;
    int V, H, M, n_chunks, stages;
    uint32_t row_bytes;
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

__device__ __forceinline__ int q16(float v, float sc) {
    return max(-32767, min(32767, __float2int_rn(v * sc)));
}

// 2^e with max_abs * 2^e in [16384, 32768), or 1 for an all-zero row.
__device__ __forceinline__ float q16_scale(float max_abs) {
    if (!(max_abs > 0.f)) return 1.f;
    int e;
    frexpf(max_abs, &e);
    return ldexpf(1.f, 15 - e);
}

// Sub-block sb of a row staged in shared memory: its 32 codes as kv+128 bytes in r (byte order
// of kv_lookup8 for the four qs words) and its scale d*(ls-32).
__device__ __forceinline__ float decode_subblk(const uint8_t* row, int sb, uint32_t (&r)[8]) {
    const uint8_t* blk = row + (sb >> 3) * kBlockBytes;
    const uint2 hdr = *reinterpret_cast<const uint2*>(blk);
    const uint2* qp = reinterpret_cast<const uint2*>(blk + 8 + (sb & 7) * 16);
    const uint2 q01 = qp[0], q23 = qp[1];
    kv_lookup8(q01.x, r[0], r[1]);
    kv_lookup8(q01.y, r[2], r[3]);
    kv_lookup8(q23.x, r[4], r[5]);
    kv_lookup8(q23.y, r[6], r[7]);
    return iq4_subscale(hdr.x, hdr.y, sb & 7);
}

// Exact sum over the sub-block of kv(code_j) * a_j, a in the packed 17-word layout.
__device__ __forceinline__ int dot_codes(const uint32_t (&aw)[17], const uint32_t (&r)[8]) {
    int d = -static_cast<int>(aw[16]);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        d = dp2a_lo(aw[4 * w], r[2 * w], d);
        d = dp2a_hi(aw[4 * w + 1], r[2 * w], d);
        d = dp2a_lo(aw[4 * w + 2], r[2 * w + 1], d);
        d = dp2a_hi(aw[4 * w + 3], r[2 * w + 1], d);
    }
    return d;
}

// Order-preserving argmax key: larger value first, then lower index; 0 = no candidate.  -0 is
// folded into +0 (the reference compares with >, so equal values keep the first index), and
// NaN and -inf never win (v > -inf fails for both).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    if (!(v > -INFINITY)) return 0ull;
    v += 0.f;
    const uint32_t b = __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(o) << 32) | (0xFFFFFFFFu - idx);
}

template <int MT, int NL>
__global__ void __launch_bounds__(kVThreads, 1) vocab_kernel(const VocabArgs a) {
    constexpr int kVRows = vocab_rows<MT, NL>();
    constexpr int kVChunkRows = kVWarps * kVRows;
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* empty = full + kVMaxStages;
    unsigned long long* bkey = reinterpret_cast<unsigned long long*>(empty + kVMaxStages);  // [8]
    float* xinv = reinterpret_cast<float*>(bkey + 8);                                        // [8]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(xinv + 8);
    uint32_t* xq = reinterpret_cast<uint32_t*>(sm + kVHeader);  // [MT][H/32][kVQW]
    const int nsb = a.H / 32;
    const size_t xq_bytes = static_cast<size_t>(MT) * nsb * kVQW * 4;
    uint8_t* stage0 = sm + ((kVHeader + xq_bytes + 127) / 128) * 128;
    const uint32_t chunk_bytes = a.row_bytes * kVChunkRows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = a.stages, M = a.M;

    if (tid < 8) bkey[tid] = 0ull;
    if (warp == kVWarps) {
        // producer: one lane initialises the ring, issues the first S chunks before the CTA-wide
        // barrier (overlapping the activation packing), then streams the rest
        int issued = 0;
        int c = blockIdx.x;
        auto issue = [&](int s) {
            const int rows = min(kVChunkRows, a.V - c * kVChunkRows);
            const uint32_t bytes = static_cast<uint32_t>(rows) * a.row_bytes;
            tc::mbar_arrive_expect_tx(&full[s], bytes);
            tc::bulk_load(stage0 + static_cast<size_t>(s) * chunk_bytes,
                          a.w + static_cast<size_t>(c) * chunk_bytes, bytes, &full[s]);
        };
        if (lane == 0) {
            for (int s = 0; s < S; ++s) {
                tc::mbar_init(&full[s], 1);
                tc::mbar_init(&empty[s], kVWarps);
            }
            tc::fence_mbar_init();
            *abort_flag = 0;
            for (; c < a.n_chunks && issued < S; c += gridDim.x, ++issued) issue(issued);
        }
        __syncwarp();
        __syncthreads();
        if (lane == 0) {
            for (; c < a.n_chunks; c += gridDim.x, ++issued) {
                const int s = issued % S;
                if (!tc::mbar_wait(&empty[s], ((issued / S) & 1) ^ 1, abort_flag, kVSpinNs)) break;
                issue(s);
            }
            // drain: the copies still in flight land before the CTA's shared memory goes away
            for (int i = max(0, issued - S); i < issued; ++i) {
                uint64_t t0 = 0;
                for (uint32_t n = 0; !tc::mbar_try_wait(&full[i % S], (i / S) & 1); ++n) {
                    if (n == 0) t0 = tc::globaltimer_ns();
                    else if ((n & 63u) == 0u && tc::globaltimer_ns() - t0 > kVSpinNs) break;
                }
            }
        }
        __syncwarp();
    } else {
        // activation row `warp` as packed 16-bit pairs
        if (warp < M) {
            const float* xr = a.x + static_cast<size_t>(warp) * a.H;
            float mx = 0.f;
            bool nonfinite = false;
            for (int j = lane; j < a.H; j += 32) {
                const float v = __ldg(xr + j);
                nonfinite |= !isfinite(v);
                mx = fmaxf(mx, fabsf(v));
            }
            mx = warp_max(mx);
            const bool finite = !__any_sync(0xffffffffu, nonfinite);  // else the row's logits are NaN
            const float sc = q16_scale(finite ? mx : 0.f);
            if (lane == 0) xinv[warp] = finite ? 1.f / sc : __int_as_float(0x7fc00000);
            uint32_t* q = xq + static_cast<size_t>(warp) * nsb * kVQW;
            for (int p = lane; p < a.H / 2; p += 32) {  // 16 consecutive lanes per sub-block
                const int sb = p >> 4, wi = p & 15;
                const int j = sb * 32 + (wi >> 2) * 4 + (wi & 3);
                const int lo = q16(__ldg(xr + j), sc), hi = q16(__ldg(xr + j + 16), sc);
                q[sb * kVQW + wi] = (static_cast<uint32_t>(lo) & 0xFFFFu) | (static_cast<uint32_t>(hi) << 16);
                int sum = lo + hi;
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                if (wi == 0) q[sb * kVQW + 16] = static_cast<uint32_t>(128 * sum);
            }
        }
        __syncthreads();
        float inv[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) inv[t] = t < M ? xinv[t] : 0.f;
        // NL > 0: lane l always takes sub-blocks l, l+32, ..., so its packed activations stay in
        // registers (NL*17 words per row); shared-memory reads of them bound the rate otherwise
        uint32_t xreg[NL > 0 ? MT : 1][NL > 0 ? NL : 1][17];
        if constexpr (NL > 0) {
#pragma unroll
            for (int t = 0; t < MT; ++t)
#pragma unroll
                for (int n = 0; n < NL; ++n)
#pragma unroll
                    for (int w = 0; w < 17; ++w)
                        xreg[t][n][w] = t < M ? xq[(static_cast<size_t>(t) * nsb + lane + 32 * n) * kVQW + w] : 0u;
        }
        unsigned long long best = 0ull;  // lane t: activation row t
        int i = 0;
        for (int c = blockIdx.x; c < a.n_chunks; c += gridDim.x, ++i) {
            const int s = i % S;
            if (!tc::mbar_wait_warp(&full[s], (i / S) & 1, abort_flag)) break;
            const int row0 = (c * kVWarps + warp) * kVRows;
            if (row0 < a.V) {
                // rows row0 .. row0+kVRows-1 (rows past V in the last chunk are computed from stale
                // shared memory and not stored)
                const uint8_t* rp = stage0 + static_cast<size_t>(s) * chunk_bytes +
                                    static_cast<size_t>(warp) * kVRows * a.row_bytes;
                float acc[kVRows][MT];
#pragma unroll
                for (int rr = 0; rr < kVRows; ++rr)
#pragma unroll
                    for (int t = 0; t < MT; ++t) acc[rr][t] = 0.f;
                if constexpr (NL > 0) {
#pragma unroll
                    for (int n = 0; n < NL; ++n) {
#pragma unroll
                        for (int rr = 0; rr < kVRows; ++rr) {
                            uint32_t r[8];
                            const float dl = decode_subblk(rp + rr * a.row_bytes, lane + 32 * n, r);
#pragma unroll
                            for (int t = 0; t < MT; ++t)
                                if (t < M)
                                    acc[rr][t] = fmaf(dl, static_cast<float>(dot_codes(xreg[t][n], r)), acc[rr][t]);
                        }
                    }
                } else {
                    for (int sb = lane; sb < nsb; sb += 32) {
#pragma unroll
                        for (int rr = 0; rr < kVRows; ++rr) {
                            uint32_t r[8];
                            const float dl = decode_subblk(rp + rr * a.row_bytes, sb, r);
#pragma unroll
                            for (int t = 0; t < MT; ++t) {
                                if (t < M) {
                                    const uint32_t* aq = xq + (static_cast<size_t>(t) * nsb + sb) * kVQW;
                                    const uint4* a4 = reinterpret_cast<const uint4*>(aq);
                                    uint32_t aw[17];
#pragma unroll
                                    for (int w = 0; w < 4; ++w) {
                                        const uint4 av = a4[w];
                                        aw[4 * w] = av.x; aw[4 * w + 1] = av.y; aw[4 * w + 2] = av.z; aw[4 * w + 3] = av.w;
                                    }
                                    aw[16] = aq[16];
                                    acc[rr][t] = fmaf(dl, static_cast<float>(dot_codes(aw, r)), acc[rr][t]);
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int rr = 0; rr < kVRows; ++rr) {
                    const int row = row0 + rr;
#pragma unroll
                    for (int t = 0; t < MT; ++t) {
                        if (t < M) {
                            const float v = warp_sum(acc[rr][t]) * inv[t];
                            if (lane == t && row < a.V) {
                                if (a.logits) a.logits[static_cast<size_t>(t) * a.V + row] = v;
                                const unsigned long long k = argmax_key(v, static_cast<uint32_t>(row));
                                best = k > best ? k : best;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[s]);
        }
        if (a.ids && lane < M && best) atomicMax(&bkey[lane], best);
    }
    __syncthreads();
    if (tid == 0) {
        if (*abort_flag) set_dev_error(a.status, kDevTimeout);
        if (a.ids) {
            for (int t = 0; t < M; ++t)
                if (bkey[t]) atomicMax(&a.keys[t], bkey[t]);
            __threadfence();
            const unsigned int done = atomicAdd(a.ticket, 1u);
            if (done == gridDim.x - 1) {  // last CTA: every other CTA's keys are visible
                __threadfence();
                for (int t = 0; t < M; ++t) {
                    const unsigned long long k = atomicExch(&a.keys[t], 0ull);
                    a.ids[t] = k ? 0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull) : 0u;
                }
                atomicExch(a.ticket, 0u);
            }
        }
    }
}

template <int MT, int NL>
size_t vocab_smem(int H, int stages, uint32_t row_bytes) {
    constexpr int kVChunkRows = kVWarps * vocab_rows<MT, NL>();
    const size_t xq = static_cast<size_t>(MT) * (H / 32) * kVQW * 4;
    return (kVHeader + xq + 127) / 128 * 128 + static_cast<size_t>(stages) * row_bytes * kVChunkRows;
}

template <int MT, int NL>
int launch_vocab_t(VocabArgs a, int sm_count, cudaStream_t s) {
    constexpr int kVChunkRows = kVWarps * vocab_rows<MT, NL>();
    a.n_chunks = (a.V + kVChunkRows - 1) / kVChunkRows;
    const size_t base = vocab_smem<MT, NL>(a.H, 0, a.row_bytes);
    const size_t chunk = static_cast<size_t>(a.row_bytes) * kVChunkRows;
    if (base + 2 * chunk > static_cast<size_t>(kVSmemMax)) return -1;
    a.stages = static_cast<int>(std::min<size_t>(kVMaxStages, (kVSmemMax - base) / chunk));
    const size_t smem = vocab_smem<MT, NL>(a.H, a.stages, a.row_bytes);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        cudaFuncSetAttribute(vocab_kernel<MT, NL>, cudaFuncAttributeMaxDynamicSharedMemorySize, kVSmemMax);
        attr_set[dev] = true;
    }
    const int grid = std::min(a.n_chunks, sm_count);
    vocab_kernel<MT, NL><<<grid, kVThreads, smem, s>>>(a);
    return 0;
}

}  // namespace

bool vocab_supported(int H, int M) {
    return M >= 1 && M <= 8 && H >= 512 && H <= 4096 && H % 512 == 0;
}

int launch_vocab(const uint8_t* w, int V, int H, const float* x, int M, float* logits, uint32_t* ids,
                 unsigned long long* keys, unsigned int* ticket, int* status, int sm_count,
                 cudaStream_t s) {
    VocabArgs a{};
    a.w = w; a.x = x; a.logits = logits; a.ids = ids; a.keys = keys; a.ticket = ticket;
    a.status = status; a.V = V; a.H = H; a.M = M;
    a.row_bytes = static_cast<uint32_t>(H / kQK * kBlockBytes);
    // activations in registers when each lane's share is small (H = 1024 or 2048, M <= 2)
    const int nl = (H == 1024 || H == 2048) ? H / 1024 : 0;
    if (M <= 1) return nl == 2 ? launch_vocab_t<1, 2>(a, sm_count, s)
                     : nl == 1 ? launch_vocab_t<1, 1>(a, sm_count, s) : launch_vocab_t<1, 0>(a, sm_count, s);
    if (M <= 2) return nl == 2 ? launch_vocab_t<2, 2>(a, sm_count, s)
                     : nl == 1 ? launch_vocab_t<2, 1>(a, sm_count, s) : launch_vocab_t<2, 0>(a, sm_count, s);
    if (M <= 4) return launch_vocab_t<4, 0>(a, sm_count, s);
    return launch_vocab_t<8, 0>(a, sm_count, s);
}

}  // namespace moe
