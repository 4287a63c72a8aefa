// Grouped IQ4_XS expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM), for buckets
// of several tokens (prefill, batched decode): the roles of moe-680m's w1_w3_fused.comp +
// silu_mult.comp and w2.comp / w2_scatter.comp, regrouped by expert bucket.
//
// Formulation: D[feature][token] = W[feature][:] . X[token][:], i.e. the expert's output
// features are the MMA M dimension (128 rows per tile) and the bucket's tokens the N dimension
// (16..NMAX), so a bucket of a few tokens still fills 128-row MMAs.
//
// One persistent CTA per SM (448 threads, warp-specialised), looping over work items
// (token tile of one bucket x 128-row feature tile):
//   warps 0-7   dequantise IQ4_XS rows (kvalues_iq4nl lookup by byte permutes, fp16 scale per
//               32-weight sub-block) and write the fp16 A operand into TMEM (tcgen05.st) or
//               into 128-byte-swizzled shared memory, 64 K values per stage;
//   warp 8      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=16..NMAX, K=16) and
//               tcgen05.commit;
//   warp 9      lane 0 loads the B operand (fp16 activations, pre-scaled per slot by a power of
//               two, K permuted to match the decode order) with 2D TMA tile loads;
//   warps 10-13 epilogue: TMEM -> registers, undo the activation scale, then
//                 gemm13: h = silu(g) * u  ->  h32[slot][feature]     (f32)
//                 gemm2:  y                ->  ypart[slot][feature]   (f32, unweighted)
// The accumulators are double-buffered in TMEM so the epilogue of one item overlaps the main
// loop of the next.  Every mbarrier wait is bounded: on timeout the CTA records an error
// status, stops issuing work, lets in-flight operations drain and frees its TMEM.
//
// K order inside each 64-wide stage is permuted (the same way for A and B): position
// q = 32*s + 8*w + 2*i + h holds k = 32*s + 4*w + i + 16*h, which is the order in which one
// 32-bit word of IQ4_XS nibbles decodes (low nibbles k..k+3, high nibbles k+16..k+19).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "moe_common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

namespace {

using namespace tc;

constexpr int kStages = 4;
constexpr int kProdWarps = 8;
constexpr int kThreads = 14 * 32;
constexpr int kMmaWarp = 8, kTmaWarp = 9;  // warps 10-13: epilogue
constexpr int kTmemCols = 512;
constexpr int kBoxRows = 16;  // TMA box: 16 rows x 64 fp16

template <int MODE>
struct Cfg;
template <>
struct Cfg<13> {                         // gate (W1) + up (W3), K = hidden
    static constexpr int kNMax = 64;
    static constexpr int kMats = 2;
    static constexpr int kAccStride = 128;  // TMEM columns per accumulator buffer
    static constexpr int kAColsPerStage = 64;
};
template <>
struct Cfg<2> {                          // down (W2), K = inter
    static constexpr int kNMax = 128;
    static constexpr int kMats = 1;
    static constexpr int kAccStride = 128;
    static constexpr int kAColsPerStage = 32;
};

struct TcArgs {
    ExpertTables tabs;
    const TcTile* tiles;
    const int* counters;  // counters[counter_idx] = number of tiles
    int counter_idx;
    int row_tiles;        // feature tiles of 128 rows
    int K;                // contraction length (multiple of 256)
    int row_bytes;        // IQ4_XS bytes per weight row
    const int* sexp;      // per-slot power-of-two exponent of the B operand scale
    float* out;           // gemm13: h32 [S][I]; gemm2: ypart [S][H]
    int out_ld;
    int* status;
};

// ---- dequantisation ---------------------------------------------------------------------------
// Two fp16 weights (lo/hi nibble of one qs byte) from kv+128 bytes: build 1024+u halves with a
// byte permute, subtract 1152 (exact), multiply by the sub-block scale.
__device__ __forceinline__ uint32_t pair_f16(uint32_t r, uint32_t sel, __half2 scale) {
    const uint32_t m = prmt(r, 0x64646464u, sel);
    __half2 v = *reinterpret_cast<const __half2*>(&m);
    v = __hmul2(__hsub2(v, __half2half2(__ushort_as_half(0x6480))), scale);  // 0x6480 = 1152
    return *reinterpret_cast<uint32_t*>(&v);
}

// One qs word -> 4 packed fp16x2 (8 weights in permuted K order).
__device__ __forceinline__ void word_f16(uint32_t q, __half2 scale, uint32_t* o) {
    uint32_t r0, r1;
    kv_lookup8(q, r0, r1);
    o[0] = pair_f16(r0, 0x4140u, scale);
    o[1] = pair_f16(r0, 0x4342u, scale);
    o[2] = pair_f16(r1, 0x4140u, scale);
    o[3] = pair_f16(r1, 0x4342u, scale);
}

__device__ __forceinline__ __half2 subscale_h2(uint32_t h0, uint32_t h1, int ib) {
    const __half d = __ushort_as_half(static_cast<unsigned short>(h0 & 0xFFFFu));
    const int ls = static_cast<int>(((h1 >> (4 * ib)) & 0xFu) | (((h0 >> (16 + 2 * ib)) & 3u) << 4));
    const __half s = __hmul(d, __int2half_rn(ls - 32));
    return __half2half2(s);
}

// Raw bytes of one producer thread for one stage.  gemm13: 2 sub-blocks (32 qs bytes) of one
// row; gemm2: 1 sub-block (16 qs bytes) of one row.
template <int MODE>
struct Raw {
    uint2 hdr;
    uint2 q[MODE == 13 ? 4 : 2];
};

template <int MODE>
__device__ __forceinline__ void load_raw(Raw<MODE>& r, const uint8_t* row, int s, int half) {
    const uint8_t* blk = row + (s >> 2) * kBlockBytes;
    r.hdr = ldg_stream_u2(blk);
    if constexpr (MODE == 13) {
        const uint8_t* q = blk + 8 + (s & 3) * 32;
#pragma unroll
        for (int i = 0; i < 4; ++i) r.q[i] = ldg_stream_u2(q + 8 * i);
    } else {
        const uint8_t* q = blk + 8 + ((s & 3) * 2 + half) * 16;
        r.q[0] = ldg_stream_u2(q);
        r.q[1] = ldg_stream_u2(q + 8);
    }
}

// Decode: gemm13 -> 32 words (64 weights), gemm2 -> 16 words (32 weights).
template <int MODE>
__device__ __forceinline__ void dequant_raw(const Raw<MODE>& r, int s, int half, uint32_t* o) {
    if constexpr (MODE == 13) {
#pragma unroll
        for (int sb = 0; sb < 2; ++sb) {
            const __half2 sc = subscale_h2(r.hdr.x, r.hdr.y, (s & 3) * 2 + sb);
            word_f16(r.q[2 * sb].x, sc, o + 16 * sb + 0);
            word_f16(r.q[2 * sb].y, sc, o + 16 * sb + 4);
            word_f16(r.q[2 * sb + 1].x, sc, o + 16 * sb + 8);
            word_f16(r.q[2 * sb + 1].y, sc, o + 16 * sb + 12);
        }
    } else {
        const __half2 sc = subscale_h2(r.hdr.x, r.hdr.y, (s & 3) * 2 + half);
        word_f16(r.q[0].x, sc, o + 0);
        word_f16(r.q[0].y, sc, o + 4);
        word_f16(r.q[1].x, sc, o + 8);
        word_f16(r.q[1].y, sc, o + 12);
    }
}

struct Item {
    int bucket, p0, n, rt;
};

__device__ __forceinline__ Item get_item(const TcArgs& a, int item) {
    const int t = item / a.row_tiles;
    const TcTile tl = a.tiles[t];
    return Item{tl.bucket, tl.p0, tl.n, item - t * a.row_tiles};
}

template <int MODE, bool A_TMEM>
__global__ void __launch_bounds__(kThreads, 1)
expert_tc_kernel(const __grid_constant__ CUtensorMap bmap, const TcArgs a) {
    using C = Cfg<MODE>;
    constexpr int kBStage = C::kNMax * 128;                        // bytes
    constexpr int kAStage = A_TMEM ? 0 : C::kMats * 128 * 128;     // bytes
    extern __shared__ uint8_t smem_raw[];
    // 128-byte-swizzled operand tiles need 1024-byte aligned shared-memory addresses
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* bst = smem;                                   // [kStages][kBStage]
    uint8_t* ast = smem + kStages * kBStage;               // [kStages][kAStage] (smem A)
    uint64_t* bars = reinterpret_cast<uint64_t*>(ast + kStages * kAStage);
    uint64_t* full = bars;                 // [kStages]
    uint64_t* empty = bars + kStages;      // [kStages]
    uint64_t* accf = bars + 2 * kStages;   // [2]
    uint64_t* acce = accf + 2;             // [2]
    uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(acce + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_base_p + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = a.counters[a.counter_idx] * a.row_tiles;
    const int nst = a.K / 64;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], kProdWarps * 32 + 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], 128);
        }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) tmem_alloc(tmem_base_p, kTmemCols);
    if (warp == kTmaWarp && lane == 0) tma_prefetch_desc(&bmap);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base_p;
    const uint32_t a_col0 = 256;  // A stages start at TMEM column 256

    if (warp < kProdWarps) {
        // ---------------- producers: IQ4_XS -> fp16 A operand ----------------
        const int q = warp & 3;
        const int sel = warp >> 2;  // gemm13: 0 = W1 (gate), 1 = W3 (up); gemm2: K half
        const int row_in_tile = q * 32 + lane;
        const int total = ((n_items - static_cast<int>(blockIdx.x)) + gridDim.x - 1) / gridDim.x;
        const int total_st = total > 0 ? total * nst : 0;
        auto row_ptr = [&](int it) -> const uint8_t* {
            const Item x = get_item(a, static_cast<int>(blockIdx.x) + it * gridDim.x);
            const uint8_t* w = MODE == 13 ? (sel == 0 ? a.tabs.w1[x.bucket] : a.tabs.w3[x.bucket])
                                          : a.tabs.w2[x.bucket];
            return w + static_cast<size_t>(x.rt * 128 + row_in_tile) * a.row_bytes;
        };
        Raw<MODE> cur, nxt;
        const uint8_t* rp = total_st > 0 ? row_ptr(0) : nullptr;
        if (total_st > 0) load_raw<MODE>(nxt, rp, 0, sel);
        for (int g = 0; g < total_st; ++g) {
            const int it = g / nst, s = g - it * nst;
            cur = nxt;
            if (g + 1 < total_st) {
                const int it1 = (g + 1) / nst, s1 = (g + 1) - it1 * nst;
                if (s1 == 0) rp = row_ptr(it1);
                load_raw<MODE>(nxt, rp, s1, sel);
            }
            const int slot = g % kStages;
            const uint32_t ph = (g / kStages) & 1;
            if (!mbar_wait(&empty[slot], ph ^ 1, abort)) break;
            if constexpr (MODE == 13) {
                uint32_t v[32];
                dequant_raw<MODE>(cur, s, sel, v);
                if constexpr (A_TMEM) {
                    tmem_st32(tmem + (static_cast<uint32_t>(q * 32) << 16) +
                                  a_col0 + slot * C::kAColsPerStage + sel * 32, v);
                    tmem_wait_st();
                } else {
                    uint8_t* rowp = ast + slot * kAStage + sel * 128 * 128 + row_in_tile * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        *reinterpret_cast<uint4*>(rowp + ((c ^ (row_in_tile & 7)) << 4)) =
                            make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                }
            } else {
                uint32_t v[16];
                dequant_raw<MODE>(cur, s, sel, v);
                if constexpr (A_TMEM) {
                    tmem_st16(tmem + (static_cast<uint32_t>(q * 32) << 16) +
                                  a_col0 + slot * C::kAColsPerStage + sel * 16, v);
                    tmem_wait_st();
                } else {
                    uint8_t* rowp = ast + slot * kAStage + row_in_tile * 128;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int cc = sel * 4 + c;
                        *reinterpret_cast<uint4*>(rowp + ((cc ^ (row_in_tile & 7)) << 4)) =
                            make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                    }
                }
            }
            if constexpr (A_TMEM) tc_fence_before(); else fence_proxy_async_smem();
            mbar_arrive(&full[slot]);
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int g = 0, it = 0;
            for (int item = blockIdx.x; item < n_items && !*abort; item += gridDim.x, ++it) {
                const Item x = get_item(a, item);
                const int N = (x.n + 15) & ~15;
                const uint32_t idesc = idesc_f16(128, N);
                const int b = it & 1;
                if (!mbar_wait(&acce[b], ((it >> 1) & 1) ^ 1, abort)) break;
                tc_fence_after();
                bool ok = true;
                for (int s = 0; s < nst; ++s, ++g) {
                    const int slot = g % kStages;
                    if (!mbar_wait(&full[slot], (g / kStages) & 1, abort)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t bbase = smem_u32(bst + slot * kBStage);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t bdesc = sw128_desc(bbase + 32 * j);
                        const uint32_t accum = (s | j) != 0;
#pragma unroll
                        for (int m = 0; m < C::kMats; ++m) {
                            const uint32_t d = tmem + b * C::kAccStride + m * 64;
                            if constexpr (A_TMEM) {
                                const uint32_t at = tmem + a_col0 + slot * C::kAColsPerStage + m * 32 + 8 * j;
                                mma_ts(d, at, bdesc, idesc, accum);
                            } else {
                                const uint32_t aa = smem_u32(ast + slot * kAStage + m * 128 * 128) + 32 * j;
                                mma_ss(d, sw128_desc(aa), bdesc, idesc, accum);
                            }
                        }
                    }
                    mma_commit(&empty[slot]);
                }
                if (!ok) break;
                mma_commit(&accf[b]);
            }
        }
        __syncwarp();
    } else if (warp == kTmaWarp) {
        // ---------------- B operand loads (TMA) ----------------
        if (lane == 0) {
            int g = 0;
            for (int item = blockIdx.x; item < n_items && !*abort; item += gridDim.x) {
                const Item x = get_item(a, item);
                const int nbox = (x.n + kBoxRows - 1) / kBoxRows;
                bool ok = true;
                for (int s = 0; s < nst; ++s, ++g) {
                    const int slot = g % kStages;
                    if (!mbar_wait(&empty[slot], ((g / kStages) & 1) ^ 1, abort)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[slot], nbox * kBoxRows * 128);
                    for (int i = 0; i < nbox; ++i)
                        tma_load_2d(bst + slot * kBStage + i * kBoxRows * 128, &bmap, s * 64,
                                    x.p0 + i * kBoxRows, &full[slot]);
                }
                if (!ok) break;
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue ----------------
        const int q = warp & 3;
        const int row = q * 32 + lane;
        int it = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
            const Item x = get_item(a, item);
            const int b = it & 1;
            if (!mbar_wait(&accf[b], (it >> 1) & 1, abort)) break;
            tc_fence_after();
            const int feat = x.rt * 128 + row;
            const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * C::kAccStride;
            for (int c0 = 0; c0 < x.n; c0 += 16) {
                uint32_t g[16];
                tmem_ld16(tl + c0, g);
                if constexpr (MODE == 13) {
                    uint32_t u[16];
                    tmem_ld16(tl + 64 + c0, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        if (c0 + t < x.n) {
                            const int p = x.p0 + c0 + t;
                            const int e = a.sexp[p];
                            const float gv = ldexpf(__uint_as_float(g[t]), e);
                            const float uv = ldexpf(__uint_as_float(u[t]), e);
                            a.out[static_cast<size_t>(p) * a.out_ld + feat] = silu_f(gv) * uv;
                        }
                    }
                } else {
                    tmem_wait_ld();
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        if (c0 + t < x.n) {
                            const int p = x.p0 + c0 + t;
                            a.out[static_cast<size_t>(p) * a.out_ld + feat] =
                                ldexpf(__uint_as_float(g[t]), a.sexp[p]);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acce[b]);
        }
    }

    __syncthreads();
    if (*abort) {
        if (threadIdx.x == 0) set_dev_error(a.status, kDevTimeout);
        // let in-flight TMA loads and MMAs drain before TMEM is released
        for (int i = 0; i < 200; ++i) __nanosleep(1000);
    }
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
}

// ---- activation conversion: one warp per slot row ------------------------------------------
// dst[p][perm(k)] = fp16(src_row[k] * 2^-e), e chosen so max|row| * 2^-e < 2^15; sexp[p] = e.
__global__ void __launch_bounds__(256)
convert_rows_kernel(const float* __restrict__ src, const int* __restrict__ gather, int n_rows,
                    int len, __half* __restrict__ dst, int* __restrict__ sexp) {
    const int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (p >= n_rows) return;
    const int r = gather ? gather[p] : p;
    const float* s = src + static_cast<size_t>(r) * len;
    float mx = 0.f;
    for (int i = lane * 4; i < len; i += 128) {
        const float4 v = *reinterpret_cast<const float4*>(s + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    mx = warp_max(mx);
    int e = 0;
    if (mx > 0.f) { frexpf(mx, &e); e -= 15; }
    if (lane == 0) sexp[p] = e;
    __half* d = dst + static_cast<size_t>(p) * len;
    // chunk c (8 halves): stage c/8, sub-block (c%8)/4, word c%4 -> k = 64*(c/8)+32*((c%8)/4)+4*(c%4)
    for (int c = lane; c < len / 8; c += 32) {
        const int kb = 64 * (c >> 3) + 32 * ((c & 7) >> 2) + 4 * (c & 3);
        const float4 lo = *reinterpret_cast<const float4*>(s + kb);
        const float4 hi = *reinterpret_cast<const float4*>(s + kb + 16);
        __half2 o[4];
        o[0] = __floats2half2_rn(ldexpf(lo.x, -e), ldexpf(hi.x, -e));
        o[1] = __floats2half2_rn(ldexpf(lo.y, -e), ldexpf(hi.y, -e));
        o[2] = __floats2half2_rn(ldexpf(lo.z, -e), ldexpf(hi.z, -e));
        o[3] = __floats2half2_rn(ldexpf(lo.w, -e), ldexpf(hi.w, -e));
        *reinterpret_cast<uint4*>(d + 8 * c) = *reinterpret_cast<uint4*>(o);
    }
}

template <int MODE, bool A_TMEM>
size_t tc_smem_bytes() {
    using C = Cfg<MODE>;
    const size_t b = static_cast<size_t>(kStages) * C::kNMax * 128;
    const size_t as = A_TMEM ? 0 : static_cast<size_t>(kStages) * C::kMats * 128 * 128;
    size_t total = 1024 + b + as + 256;
    return total < 140 * 1024 ? 140 * 1024 : total;  // > half the SM: one CTA (and TMEM owner) per SM
}

template <int MODE, bool A_TMEM>
void launch_tc(const CUtensorMap& bmap, const TcArgs& args, int n_cta, cudaStream_t s) {
    const size_t smem = tc_smem_bytes<MODE, A_TMEM>();
    cudaFuncSetAttribute(expert_tc_kernel<MODE, A_TMEM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    expert_tc_kernel<MODE, A_TMEM><<<n_cta, kThreads, smem, s>>>(bmap, args);
}

}  // namespace

int tc_max_n(int mode) { return mode == 13 ? Cfg<13>::kNMax : Cfg<2>::kNMax; }

void launch_convert_rows(const float* src, const int* gather, int n_rows, int len, __half* dst,
                         int* sexp, cudaStream_t s) {
    convert_rows_kernel<<<(n_rows * 32 + 255) / 256, 256, 0, s>>>(src, gather, n_rows, len, dst, sexp);
}

void launch_tc13(const Layer& L, const CUtensorMap& xmap, const Workspace& ws, int max_items,
                 int sm_count, bool a_tmem, cudaStream_t s) {
    TcArgs a{L.tables(), ws.tiles13, ws.counters, 1, static_cast<int>(L.spec.inter) / 128,
             static_cast<int>(L.spec.hidden), static_cast<int>(L.spec.hidden / kQK) * kBlockBytes,
             ws.xexp, ws.h, static_cast<int>(L.spec.inter), ws.status};
    const int grid = max_items < sm_count ? (max_items > 0 ? max_items : 1) : sm_count;
    if (a_tmem) launch_tc<13, true>(xmap, a, grid, s);
    else launch_tc<13, false>(xmap, a, grid, s);
}

void launch_tc2(const Layer& L, const CUtensorMap& hmap, const Workspace& ws, int max_items,
                int sm_count, bool a_tmem, cudaStream_t s) {
    TcArgs a{L.tables(), ws.tiles2, ws.counters, 2, static_cast<int>(L.spec.hidden) / 128,
             static_cast<int>(L.spec.inter), static_cast<int>(L.spec.inter / kQK) * kBlockBytes,
             ws.hexp, ws.ypart, static_cast<int>(L.spec.hidden), ws.status};
    const int grid = max_items < sm_count ? (max_items > 0 ? max_items : 1) : sm_count;
    if (a_tmem) launch_tc<2, true>(hmap, a, grid, s);
    else launch_tc<2, false>(hmap, a, grid, s);
}

// 2D tensor map over an fp16 [rows][cols] row-major matrix, box 16 rows x 64 cols, 128B swizzle.
bool make_fp16_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return false;
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, kBoxRows};
    const cuuint32_t estr[2] = {1, 1};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace moe
