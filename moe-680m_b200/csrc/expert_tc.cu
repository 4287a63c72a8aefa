// Grouped IQ4_XS expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM), for buckets
// of several tokens (prefill, batched decode): the roles of moe-680m's w1_w3_fused.comp
// (gate/up) and w2.comp / w2_scatter.comp (down), regrouped by expert bucket.
//
// Formulation: D[feature][token] = W[feature][:] . X[token][:].  The expert's output features
// are the MMA M dimension (128-row tiles) and the bucket's tokens the N dimension (16..kNMax),
// so a bucket of a few tokens still fills 128-row MMAs, and one dequantised weight tile serves
// up to kNMax tokens.  The gate/up product is one GEMM over W1 and W3 stacked ([2I][H]: feature
// tiles 0..I/128-1 read W1, the rest W3); SiLU(g)*u is applied by the next conversion kernel.
//
// One persistent CTA per SM (warp-specialised; 27 warps with the default 16 producer warps),
// looping over work items (token tile of one bucket x 128-row feature tile):
//   TMA-A warp  raw IQ4_XS bytes of the item's 128 weight rows, 512 K (two 136-byte blocks per
//               row) per tensor-map load, into a 2-deep shared-memory ring;
//   producer warps (16, or 8 with MOE_B200_TC_PRODUCER_WARPS=8) dequantise from that ring
//               (a shared-memory table of kvalues_iq4nl half2 per qs byte, fp16 scale per
//               32-weight sub-block) and
//               store the fp16 A operand into TMEM (tcgen05.st; 128 K per pipeline stage) or
//               128-byte-swizzled shared memory (64 K per stage); the warps of one 32-row
//               quarter take turns by stage;
//   TMA-B warp  fp16 activations of the tile's slots (pre-scaled per slot by a power of two, K
//               permuted as below), one 16/32/64/112-row box per 64 K, 4 stages in flight;
//   MMA warp    allocates TMEM; one elected lane issues tcgen05.mma (M=128, N=16..kNMax, K=16)
//               and tcgen05.commit;
//   8 epilogue warps (two per TMEM lane quarter): TMEM -> registers, undo the activation
//               scale, store f32 out[slot][feature] (gate/up pre-activations, or the unweighted
//               down output).
// Every stage costs one handshake per role (full / empty barriers, one arrival per warp), and
// that fixed cost, not memory or the tensor pipe, paced the 64-K stages (measured: with the
// dequantisation, MMAs and operand loads all stubbed out the kernel kept most of its time), so
// a stage covers 128 K: two 64-K sub-slots in TMEM and two B boxes.
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

#include <cstdlib>

#include "moe_common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

#ifdef MOE_TC_TRACE
// Debug timeline (builds with -DMOE_TC_TRACE only): %globaltimer stamps of CTA 0's roles.
// Rows: 0 MMA full-wait done (per stage), 1 producer warp 0 empty-wait done (per stage),
// 2 TMA-B empty-wait done (per stage), 3 TMA-A rempty-wait done (per chunk),
// 4 epilogue accf-wait done (per item), 5 epilogue done (per item), 6 MMA acce-wait done.
// Bank 0: gate/up launch, bank 1: down launch.
__device__ unsigned long long g_tc_trace[2][8][1024];
#define TC_TRACE(row, idx)                                                                     \
    do {                                                                                       \
        if (blockIdx.x == 0 && (idx) < 1024)                                                   \
            g_tc_trace[a.counter_idx == 1 ? 0 : 1][row][idx] = tc::globaltimer_ns();          \
    } while (0)
#else
#define TC_TRACE(row, idx) do {} while (0)
#endif

namespace {

using namespace tc;

#ifndef MOE_TC_EPI_WARPS
#define MOE_TC_EPI_WARPS 8
#endif
// Warp roles: producers 0..PW-1, then MMA, TMA-B, TMA-A, and eight epilogue warps.
template <int PW>
struct Roles {
    static constexpr int kProd = PW;
    static constexpr int kMma = PW, kTmaB = PW + 1, kTmaA = PW + 2, kEpi0 = PW + 3;
    static constexpr int kEpiWarps = MOE_TC_EPI_WARPS;  // 4: one per 32-lane TMEM quarter; 8: two
    static constexpr int kThreads = (PW + 3 + kEpiWarps) * 32;
    static constexpr int kParts = PW / 4;          // producer warps per 32-row quarter
};
constexpr int kTmemCols = 512;
constexpr int kNMax = 112;          // tokens per tile (B stages of 112 rows leave shared memory for the
                                    // dequantisation table)
constexpr int kAccStride = 128;     // TMEM columns per accumulator buffer
constexpr int kACol0 = 256;         // TMEM column of A stage 0 (32 columns per stage)
constexpr int kRawRowBytes = 2 * kBlockBytes;      // 512 K of one weight row
#ifndef MOE_TC_L2_AHEAD
#define MOE_TC_L2_AHEAD 0   // raw chunks prefetched into L2 ahead of their tensor-map load (0: none; measured fastest)
#endif
#ifndef MOE_TC_RAW_BOX
#define MOE_TC_RAW_BOX 128
#endif
constexpr int kRawBoxRows = MOE_TC_RAW_BOX;        // rows per raw tensor-map box
#ifndef MOE_TC_RAW_ELEM
#define MOE_TC_RAW_ELEM 8
#endif
constexpr int kRawElem = MOE_TC_RAW_ELEM;          // bytes per element of the raw tensor map
constexpr int kRawBytes = 128 * kRawRowBytes;      // one raw A chunk (34,816 bytes)
constexpr int kStagesPerChunk = 8;                 // 512 K / 64 K
constexpr int kBStageBytes = kNMax * 128;
// rows of B box i (16, 32, 64, kNMax): the smallest covering the tile is loaded
__host__ __device__ constexpr int box_rows(int i) { return i < 3 ? 16 << i : kNMax; }
constexpr int kAStageBytes = 128 * 128;            // smem-A variant
constexpr int kKvTabBytes = 256 * 32 * 4;          // kv half2 per qs byte, one copy per lane (bank)

// Pipeline depth.  With A in TMEM (columns 256..511): 4 stages of 128 K (MOE_TC_SUB = 2 sub-slots
// of 64 K; MOE_TC_SUB=1 gives MOE_TC_STAGES stages of 64 K) and a 2-chunk raw ring (raw rings of
// 2, 3 and 4 chunks measured alike); with A in shared memory, 4 stages of 64 K and 2 chunks.
#ifndef MOE_TC_STAGES
#define MOE_TC_STAGES 6
#endif
#ifndef MOE_TC_RAW
#define MOE_TC_RAW 2
#endif
#ifndef MOE_TC_EPI_SLEEP
#define MOE_TC_EPI_SLEEP 0
#endif
#ifndef MOE_TC_SUB
#define MOE_TC_SUB 2
#endif
template <bool A_TMEM>
struct Layout {
    // 64-K sub-slots per pipeline stage (one barrier handshake per stage)
    static constexpr int kSub = A_TMEM ? MOE_TC_SUB : 1;
    static constexpr int kStages = A_TMEM ? (kSub == 4 ? 2 : kSub == 2 ? 4 : MOE_TC_STAGES) : 4;
    static constexpr int kRaw = A_TMEM ? MOE_TC_RAW : 2;
    static constexpr size_t kBSt = static_cast<size_t>(kSub) * kBStageBytes;  // B bytes per stage
    static constexpr size_t kB = 0;
    static constexpr size_t kA = kB + static_cast<size_t>(kStages) * kBSt;
    static constexpr size_t kR = kA + (A_TMEM ? 0 : static_cast<size_t>(kStages) * kAStageBytes);
    static constexpr size_t kT = kR + static_cast<size_t>(kRaw) * kRawBytes;  // dequantisation table
    static constexpr size_t kBars = kT + kKvTabBytes;
    static constexpr size_t kTotal = kBars + 256 + 1024;  // + barriers, + alignment slack
};

struct TcArgs {
    ExpertTables tabs;         // per-expert weight pointers (W1, W3, W2)
    int row_bytes;             // IQ4_XS bytes per row of the item's matrix
    const CUtensorMap* wmaps;  // [3][E+1] raw IQ4_XS maps: W1, W3, W2
    int n_buckets;             // E + 1
    int mat0;                  // matrix of feature tile 0 (0 = W1, 2 = W2)
    int rt_per_mat;            // feature tiles per matrix (I/128 for W1/W3, H/128 for W2)
    int n_rt;                  // feature tiles per item row (2*I/128 or H/128)
    const TcTile* tiles;
    const int* counters;       // counters[counter_idx] = number of token tiles
    int counter_idx;
    int K;                     // contraction length (multiple of 512)
    const int* sexp;           // per-slot power-of-two exponent of the B operand scale
    float* out;                // [S][out_ld] f32
    int out_ld;
    int* status;
};

// ---- dequantisation ---------------------------------------------------------------------------
// kvalues_iq4nl[n] from the packed kv+128 byte tables.
__device__ __forceinline__ int kv_value(uint32_t n) {
    const uint32_t w = n < 4 ? kKvT0 : n < 8 ? kKvT1 : n < 12 ? kKvT2 : kKvT3;
    return static_cast<int>((w >> (8 * (n & 3))) & 0xFFu) - 128;
}

// One qs word -> 4 packed fp16x2 by table: word (b * 32 + lane) of the table holds the half2
// {kv[b & 15], kv[b >> 4]} of qs byte b, one copy per lane so that the 32 lanes of a warp read
// 32 different banks whatever their bytes; tl = table address + 4 * lane.  The same values as
// word_f16 (kv * scale, rounded once), with most of the work on the load and FMA pipes instead
// of the byte-permute (ALU) pipe, which bounded the dequantisation.
__device__ __forceinline__ void word_tab(uint32_t q, __half2 scale, uint32_t tl, uint32_t* o) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t off = i == 0 ? (q << 7) & 0x7F80u : (q >> (8 * i - 7)) & 0x7F80u;
        uint32_t m;
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(m) : "r"(tl + off));
        __half2 v = __hmul2(*reinterpret_cast<const __half2*>(&m), scale);
        o[i] = *reinterpret_cast<uint32_t*>(&v);
    }
}

__device__ __forceinline__ __half2 subscale_h2(uint32_t h0, uint32_t h1, int ib) {
    const __half d = __ushort_as_half(static_cast<unsigned short>(h0 & 0xFFFFu));
    const int ls = static_cast<int>(((h1 >> (4 * ib)) & 0xFu) | (((h0 >> (16 + 2 * ib)) & 3u) << 4));
    return __half2half2(__hmul(d, __int2half_rn(ls - 32)));
}

__device__ __forceinline__ uint2 lds64(const uint8_t* p) {
    return *reinterpret_cast<const uint2*>(p);
}

struct Item {
    int bucket, p0, n, rt;
};

__device__ __forceinline__ Item get_item(const TcArgs& a, int item) {
    const int t = item / a.n_rt;
    const TcTile tl = a.tiles[t];
    return Item{tl.bucket, tl.p0, tl.n, item - t * a.n_rt};
}

template <bool A_TMEM, int PW>
__global__ void __launch_bounds__(Roles<PW>::kThreads, 1)
expert_tc_kernel(const __grid_constant__ BMaps bmap, const TcArgs a) {
    using R = Roles<PW>;
    constexpr int kProdWarps = R::kProd, kMmaWarp = R::kMma, kTmaBWarp = R::kTmaB, kTmaAWarp = R::kTmaA;
    using Lay = Layout<A_TMEM>;
    constexpr int kRaw = Lay::kRaw;
    constexpr int kStages = Lay::kStages;
    constexpr int kSub = Lay::kSub;
    constexpr int kSPC = kStagesPerChunk / kSub;  // pipeline stages per raw chunk
    static_assert(kSub == 1 || A_TMEM, "multi-slot stages need A in TMEM");
    // A producer warp waits on the slot of its own previous stage; with fewer slots than warps
    // per row quarter it would wait on a slot another warp has not filled yet and the barrier
    // parity would alias.
    static_assert(kStages >= R::kParts, "MMA ring must have at least one slot per producer warp of a quarter");
    extern __shared__ uint8_t smem_raw[];
    // 128-byte-swizzled operand tiles need 1024-byte aligned shared-memory addresses
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* bst = smem + Lay::kB;
    uint8_t* ast = smem + Lay::kA;
    uint8_t* rst = smem + Lay::kR;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::kBars);
    uint32_t* kvtab = reinterpret_cast<uint32_t*>(smem + Lay::kT);
    uint64_t* full = bars;                    // [kStages]  A stored + B landed
    uint64_t* empty = full + kStages;         // [kStages]  MMAs of the stage done
    uint64_t* rfull = empty + kStages;        // [kRaw]     raw A chunk landed
    uint64_t* rempty = rfull + kRaw;          // [kRaw]     raw A chunk consumed
    uint64_t* accf = rempty + kRaw;           // [2]
    uint64_t* acce = accf + 2;                // [2]
    uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(acce + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_base_p + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = a.counters[a.counter_idx] * a.n_rt;
    const int nchunk = a.K / 512;
    const int nst = nchunk * kSPC;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 4 + 1);  // one arrival per row-quarter producer warp + TMA-B
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kRaw; ++i) {
            mbar_init(&rfull[i], 1);
            mbar_init(&rempty[i], kProdWarps);  // one arrival per producer warp
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], R::kEpiWarps);  // one arrival per epilogue warp
        }
        *abort = 0;
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < kKvTabBytes / 4; i += blockDim.x) {
        const uint32_t b = static_cast<uint32_t>(i) >> 5;
        const __half lo = __int2half_rn(kv_value(b & 15u)), hi = __int2half_rn(kv_value(b >> 4));
        const __half2 h = __halves2half2(lo, hi);
        kvtab[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    if (warp == kMmaWarp) tmem_alloc(tmem_base_p, kTmemCols);
    if (warp == kTmaBWarp && lane < 4) tma_prefetch_desc(&bmap.m[lane]);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base_p;

    if (warp < kProdWarps) {
        // ---------------- producers: raw IQ4_XS (smem) -> fp16 A operand ----------------
        // Warp (q, part) builds whole 64-K stages of rows 32q..32q+31 for the stages g with
        // g % kParts == part, so kParts stages per row quarter are in flight at once and the
        // fixed per-stage latency (store, completion wait, barrier) overlaps across warps.
        constexpr int kParts = R::kParts;
        const int q = warp & 3;
        const int part = warp >> 2;
        const int row = q * 32 + lane;
        const uint32_t ktab = smem_u32(kvtab) + 4u * lane;
        // dequantise one 64-K stage (header + 32 qs bytes of this thread's row), wait for the
        // slot, store the fp16 A operand, signal the MMA warp
        auto produce = [&](int g, int h, uint2 hdr, const uint32_t (&qw)[8], int ib0) -> bool {
            const int slot = g % kStages;
            uint32_t v[32];
            const __half2 s0 = subscale_h2(hdr.x, hdr.y, ib0);
            const __half2 s1 = subscale_h2(hdr.x, hdr.y, ib0 + 1);
#pragma unroll
            for (int i = 0; i < 8; ++i) word_tab(qw[i], i < 4 ? s0 : s1, ktab, v + 4 * i);
            if (warp == 0 && lane == 0) TC_TRACE(7, g);
            if (h == 0 && !mbar_wait_warp(&empty[slot], ((g / kStages) & 1) ^ 1, abort)) return false;
            if (warp == 0 && lane == 0) TC_TRACE(1, g);
            if constexpr (A_TMEM) {
                tmem_st32(tmem + (static_cast<uint32_t>(q * 32) << 16) + kACol0 + (slot * kSub + h) * 32, v);
                if (h != kSub - 1) return true;
                tmem_wait_st();
                tc_fence_before();
            } else if constexpr (!A_TMEM) {
                uint8_t* rowp = ast + slot * kAStageBytes + row * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4*>(rowp + ((c ^ (row & 7)) << 4)) =
                        make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[slot]);
            return true;
        };
        int g = 0, rc = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            bool ok = true;
            for (int kc = 0; kc < nchunk && ok; ++kc, ++rc) {
                const int rs = rc % kRaw;
                if (!mbar_wait_warp(&rfull[rs], (rc / kRaw) & 1, abort)) { ok = false; break; }
                if (warp == 0 && lane == 0) TC_TRACE(5, 512 + rc);
                const uint8_t* raw = rst + rs * kRawBytes + row * kRawRowBytes;
                for (int sc = 0; sc < kSPC && ok; ++sc, ++g) {
                    if (g % kParts != part) continue;
                    for (int h = 0; h < kSub; ++h) {
                        const int os = sc * kSub + h;  // 64-K sub-stage within the chunk
                        const uint8_t* blk = raw + (os >> 2) * kBlockBytes;
                        const int ib0 = (os & 3) * 2;
                        const uint2 hdr = lds64(blk);
                        uint32_t qw[8];
#pragma unroll
                        for (int i = 0; i < 8; i += 2) {
                            const uint2 qq = lds64(blk + 8 + ib0 * 16 + i * 4);
                            qw[i] = qq.x;
                            qw[i + 1] = qq.y;
                        }
                        if (!produce(g, h, hdr, qw, ib0)) { ok = false; break; }
                    }
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&rempty[rs]);
            }
            if (!ok) break;
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer (whole warp loops, one elected lane issues) ----------------
        int g = 0, it = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
            const Item x = get_item(a, item);
            const uint32_t idesc = idesc_f16(128, (x.n + 15) & ~15);
            const int b = it & 1;
            if (!mbar_wait_warp(&acce[b], ((it >> 1) & 1) ^ 1, abort)) break;
            if (lane == 0) TC_TRACE(6, it);
            tc_fence_after();
            const uint32_t d = tmem + b * kAccStride;
            bool ok = true;
            for (int s = 0; s < nst; ++s, ++g) {
                const int slot = g % kStages;
                if (!mbar_wait_warp(&full[slot], (g / kStages) & 1, abort)) { ok = false; break; }
                if (lane == 0) TC_TRACE(0, g);
                tc_fence_after();
                const uint32_t bbase = smem_u32(bst + slot * Lay::kBSt);
                if (elect_one()) {
#pragma unroll
                    for (int j = 0; j < 4 * kSub; ++j) {
                        const uint64_t bdesc = sw128_desc(bbase + (j >> 2) * kBStageBytes + 32 * (j & 3));
                        const uint32_t accum = (s | j) != 0;
                        if constexpr (A_TMEM) {
                            mma_ts(d, tmem + kACol0 + slot * 32 * kSub + 8 * j, bdesc, idesc, accum);
                        } else {
                            const uint32_t aa = smem_u32(ast + slot * kAStageBytes) + 32 * j;
                            mma_ss(d, sw128_desc(aa), bdesc, idesc, accum);
                        }
                    }
                    mma_commit(&empty[slot]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (elect_one()) mma_commit(&accf[b]);
            __syncwarp();
        }
    } else if (warp == kTmaBWarp) {
        // ---------------- B operand loads ----------------
        if (lane == 0) {
            int g = 0;
            for (int item = blockIdx.x; item < n_items && !*abort; item += gridDim.x) {
                const Item x = get_item(a, item);
                // one box per stage: 16, 32, 64 or 128 rows, the smallest covering the tile
                const int bsel = x.n <= 16 ? 0 : x.n <= 32 ? 1 : x.n <= 64 ? 2 : 3;
                const CUtensorMap* bm = &bmap.m[bsel];
                const uint32_t bbytes = static_cast<uint32_t>(box_rows(bsel)) * 128u;
                bool ok = true;
                for (int s = 0; s < nst; ++s, ++g) {
                    const int slot = g % kStages;
                    if (!mbar_wait(&empty[slot], ((g / kStages) & 1) ^ 1, abort)) { ok = false; break; }
                    TC_TRACE(2, g);
                    mbar_arrive_expect_tx(&full[slot], bbytes * kSub);
                    for (int h = 0; h < kSub; ++h)
                        tma_load_2d(bst + slot * Lay::kBSt + h * kBStageBytes, bm, (s * kSub + h) * 64, x.p0,
                                    &full[slot]);
                }
                if (!ok) break;
            }
        }
        __syncwarp();
    } else if (warp == kTmaAWarp) {
        // ---------------- raw A loads: tensor-map boxes into the raw ring ----------------
        // Optionally, tiles are prefetched into L2 MOE_TC_L2_AHEAD chunks before their load
        // (off by default: the prefetches compete with the loads and measured slower).
        if (lane == 0) {
            const int my_items = (n_items - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                 static_cast<int>(gridDim.x);
            const int total_rc = my_items > 0 ? my_items * nchunk : 0;
            auto chunk_src = [&](int c, const CUtensorMap*& wm, int& row0, int& kc) {
                const int it = c / nchunk;
                kc = c - it * nchunk;
                const Item x = get_item(a, static_cast<int>(blockIdx.x) + it * static_cast<int>(gridDim.x));
                const int mat = a.mat0 + x.rt / a.rt_per_mat;
                row0 = (x.rt % a.rt_per_mat) * 128;
                wm = a.wmaps + mat * a.n_buckets + x.bucket;
            };
            for (int c = 0; c < MOE_TC_L2_AHEAD && c < total_rc; ++c) {
                const CUtensorMap* wm; int row0, kc;
                chunk_src(c, wm, row0, kc);
                for (int r = 0; r < 128; r += kRawBoxRows)
                    tma_prefetch_l2_2d(wm, kc * (kRawRowBytes / kRawElem), row0 + r);
            }
            for (int rc = 0; rc < total_rc && !*abort; ++rc) {
                const int rs = rc % kRaw;
                if (!mbar_wait(&rempty[rs], ((rc / kRaw) & 1) ^ 1, abort)) break;
                TC_TRACE(3, rc);
                if (rc + MOE_TC_L2_AHEAD < total_rc) {
                    const CUtensorMap* wp; int prow, pkc;
                    chunk_src(rc + MOE_TC_L2_AHEAD, wp, prow, pkc);
                    for (int r = 0; r < 128; r += kRawBoxRows)
                        tma_prefetch_l2_2d(wp, pkc * (kRawRowBytes / kRawElem), prow + r);
                }
                const CUtensorMap* wm; int row0, kc;
                chunk_src(rc, wm, row0, kc);
                mbar_arrive_expect_tx(&rfull[rs], kRawBytes);
                for (int r = 0; r < 128; r += kRawBoxRows)
                    tma_load_2d(rst + rs * kRawBytes + r * kRawRowBytes, wm, kc * (kRawRowBytes / kRawElem),
                                row0 + r, &rfull[rs]);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue ----------------
        // Two warps per TMEM lane quarter, each taking alternate 16-column chunks.
        const int ew = warp - R::kEpi0;
        const int q = warp & 3;
        const int sub = ew >> 2;
        const int row = q * 32 + lane;
        int it = 0;
        constexpr int kStep = 16 * (R::kEpiWarps / 4);  // columns between a warp's chunks
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
            const Item x = get_item(a, item);
            const int b = it & 1;
            // activation exponents of the tile's tokens, read before the accumulator is ready:
            // lane j holds token j + 32 i in ex[i]; a chunk's 16 tokens lie in one group of 32
            int ex[(kNMax + 31) / 32];
#pragma unroll
            for (int i = 0; i < (kNMax + 31) / 32; ++i) {
                const int t = lane + 32 * i;
                ex[i] = t < x.n ? __ldg(a.sexp + x.p0 + t) : 0;
            }
            if (!mbar_wait_warp(&accf[b], (it >> 1) & 1, abort, MOE_TC_EPI_SLEEP)) break;
            if (ew == 0 && lane == 0) TC_TRACE(4, it);
            tc_fence_after();
            const int feat = x.rt * 128 + row;
            const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * kAccStride;
            float* __restrict__ out = a.out + feat;
            for (int c0 = sub * 16; c0 < x.n; c0 += 2 * kStep) {
                // two chunks per TMEM wait: c0 and c0 + kStep
                const int c1 = c0 + kStep;
                uint32_t v[2][16];
                tmem_ld16(tl + c0, v[0]);
                if (c1 < x.n) tmem_ld16(tl + c1, v[1]);
                tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int cc = h == 0 ? c0 : c1;
                    if (cc >= x.n) break;
                    const int gi = cc >> 5;
                    int eg = ex[0];
#pragma unroll
                    for (int i = 1; i < (kNMax + 31) / 32; ++i)
                        if (gi == i) eg = ex[i];
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const int e = __shfl_sync(0xffffffffu, eg, (cc & 31) + t);
                        if (cc + t < x.n)
                            out[static_cast<size_t>(x.p0 + cc + t) * a.out_ld] =
                                __uint_as_float(v[h][t]) * __int_as_float((127 + e) << 23);  // * 2^e
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[b]);
            if (ew == 0 && lane == 0) TC_TRACE(5, it);
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

// ---- activation conversion: one warp per slot row --------------------------------------------
// Power-of-two row scale: e such that max|row| * 2^-e < 2^15 (fp16 max 65504).
__device__ __forceinline__ int row_exp(float mx) {
    int e = 0;
    if (mx > 0.f) { frexpf(mx, &e); e -= 15; }
    return max(-100, min(100, e));
}

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }


// chunk c (8 halves): stage c/8, sub-block (c%8)/4, word c%4 -> k = 64*(c/8)+32*((c%8)/4)+4*(c%4)
__device__ __forceinline__ int chunk_k(int c) { return 64 * (c >> 3) + 32 * ((c & 7) >> 2) + 4 * (c & 3); }

__device__ __forceinline__ float4 swiglu4(float4 g, float4 u) {
    return make_float4(silu_f(g.x) * u.x, silu_f(g.y) * u.y, silu_f(g.z) * u.z, silu_f(g.w) * u.w);
}

// Two permuted chunks of 8 halves (chunks c0, c1) from four float4 (lo, hi of each), scaled.
__device__ __forceinline__ uint4 pack_chunk(float4 lo, float4 hi, float sc) {
    __half2 o[4];
    o[0] = __floats2half2_rn(lo.x * sc, hi.x * sc);
    o[1] = __floats2half2_rn(lo.y * sc, hi.y * sc);
    o[2] = __floats2half2_rn(lo.z * sc, hi.z * sc);
    o[3] = __floats2half2_rn(lo.w * sc, hi.w * sc);
    return *reinterpret_cast<uint4*>(o);
}

__device__ __forceinline__ float absmax4(float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// Largest value of v over a group of `warps` consecutive warps starting at warp w0 (red: one
// float per warp of the block).  Every thread of the group gets the result.
__device__ __forceinline__ float group_max(float v, float* red, int w0, int warps) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warps == 1) return v;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = 0.f;
    for (int w = 0; w < warps; ++w) m = fmaxf(m, red[w0 + w]);
    return m;
}

// One CTA of len/16 threads per token: x[t] -> fp16(x * 2^-e) in the permuted K order, written
// to the rows of all the token's slots (slot_pos[t][0..ns)); sexp[p] = e for those slots.
// Each thread holds its two chunks (16 values) in registers: the row is read once.
__global__ void __launch_bounds__(1024)
convert_x_kernel(const IoArgs* __restrict__ io, const int* __restrict__ slot_pos, int M, int ns,
                 int len, __half* __restrict__ dst, int* __restrict__ sexp) {
    __shared__ int pos[kMaxTopK + 1];
    __shared__ float red[32];
    const int t = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    if (t >= M) return;
    if (tid <= kMaxTopK) pos[tid] = tid < ns ? slot_pos[static_cast<size_t>(t) * ns + tid] : -1;
    __syncthreads();
    bool any = false;
#pragma unroll
    for (int j = 0; j <= kMaxTopK; ++j) any |= pos[j] >= 0;
    if (!any) return;  // a token without slots (expert-parallel padding rows): row not read
    const float* s = io->x + static_cast<size_t>(t) * len;
    const int c0 = tid, c1 = tid + nt;
    const float4 l0 = *reinterpret_cast<const float4*>(s + chunk_k(c0));
    const float4 h0 = *reinterpret_cast<const float4*>(s + chunk_k(c0) + 16);
    const float4 l1 = *reinterpret_cast<const float4*>(s + chunk_k(c1));
    const float4 h1 = *reinterpret_cast<const float4*>(s + chunk_k(c1) + 16);
    const float mx = group_max(fmaxf(fmaxf(absmax4(l0), absmax4(h0)), fmaxf(absmax4(l1), absmax4(h1))), red, 0,
                               nt >> 5);
    const int e = row_exp(mx);
    const float sc = pow2f(-e);
    if (tid < ns && pos[tid] >= 0) sexp[pos[tid]] = e;
    const uint4 v0 = pack_chunk(l0, h0, sc), v1 = pack_chunk(l1, h1, sc);
#pragma unroll
    for (int j = 0; j <= kMaxTopK; ++j) {
        if (pos[j] < 0) continue;
        __half* d = dst + static_cast<size_t>(pos[j]) * len;
        *reinterpret_cast<uint4*>(d + 8 * c0) = v0;
        *reinterpret_cast<uint4*>(d + 8 * c1) = v1;
    }
}

// gu[p] = [g (I) | u (I)] f32 -> h = silu(g) * u -> dst[p][perm(k)] = fp16(h * 2^-e); sexp[p] = e.
// I/16 threads per slot row (rows per CTA: 256 / (I/16)), two chunks each, held in registers.
__global__ void __launch_bounds__(256)
convert_h_kernel(const float* __restrict__ gu, int n_rows, const int* __restrict__ n_used, int I,
                 __half* __restrict__ dst, int* __restrict__ sexp) {
    __shared__ float red[8];
    const int T = I / 16, tid = threadIdx.x;
    const int r = tid / T, c0 = tid - r * T, c1 = c0 + T;
    const int p = blockIdx.x * (blockDim.x / T) + r;
    const int used = min(n_rows, *n_used);  // slot rows past the buckets' total are unused
    const bool live = p < used;
    const float* g = gu + static_cast<size_t>(live ? p : 0) * 2 * I;
    const float* u = g + I;
    float4 l0 = make_float4(0.f, 0.f, 0.f, 0.f), h0 = l0, l1 = l0, h1 = l0;
    if (live) {
        const int k0 = chunk_k(c0), k1 = chunk_k(c1);
        l0 = swiglu4(*reinterpret_cast<const float4*>(g + k0), *reinterpret_cast<const float4*>(u + k0));
        h0 = swiglu4(*reinterpret_cast<const float4*>(g + k0 + 16), *reinterpret_cast<const float4*>(u + k0 + 16));
        l1 = swiglu4(*reinterpret_cast<const float4*>(g + k1), *reinterpret_cast<const float4*>(u + k1));
        h1 = swiglu4(*reinterpret_cast<const float4*>(g + k1 + 16), *reinterpret_cast<const float4*>(u + k1 + 16));
    }
    const int wpr = T >> 5;  // warps per row
    const float mx = group_max(fmaxf(fmaxf(absmax4(l0), absmax4(h0)), fmaxf(absmax4(l1), absmax4(h1))), red,
                               r * wpr, wpr);
    if (!live) return;
    const int e = row_exp(mx);
    if (c0 == 0) sexp[p] = e;
    const float sc = pow2f(-e);
    __half* d = dst + static_cast<size_t>(p) * I;
    *reinterpret_cast<uint4*>(d + 8 * c0) = pack_chunk(l0, h0, sc);
    *reinterpret_cast<uint4*>(d + 8 * c1) = pack_chunk(l1, h1, sc);
}

template <bool A_TMEM, int PW>
void launch_tc_pw(const BMaps& bmap, const TcArgs& args, int n_cta, cudaStream_t s) {
    const size_t smem = Layout<A_TMEM>::kTotal;
    cudaFuncSetAttribute(expert_tc_kernel<A_TMEM, PW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    expert_tc_kernel<A_TMEM, PW><<<n_cta, Roles<PW>::kThreads, smem, s>>>(bmap, args);
}

int producer_warps() {
    static int pw = [] {
        const char* e = std::getenv("MOE_B200_TC_PRODUCER_WARPS");
        return (e && std::atoi(e) == 8) ? 8 : (e && std::atoi(e) == 12) ? 12 : 16;
    }();
    return pw;
}

template <bool A_TMEM>
void launch_tc(const BMaps& bmap, const TcArgs& args, int n_cta, cudaStream_t s) {
#if MOE_TC_SUB == 4
    launch_tc_pw<A_TMEM, 8>(bmap, args, n_cta, s);
#else
    if (producer_warps() == 8) launch_tc_pw<A_TMEM, 8>(bmap, args, n_cta, s);
    else if (producer_warps() == 12) launch_tc_pw<A_TMEM, 12>(bmap, args, n_cta, s);
    else launch_tc_pw<A_TMEM, 16>(bmap, args, n_cta, s);
#endif
}

static_assert(Layout<true>::kTotal <= 227 * 1024, "smem budget (A in TMEM)");
static_assert(Layout<false>::kTotal <= 227 * 1024, "smem budget (A in smem)");
static_assert(Layout<true>::kTotal > 114 * 1024, "one CTA (and TMEM owner) per SM");
static_assert(Layout<false>::kTotal > 114 * 1024, "one CTA (and TMEM owner) per SM");

}  // namespace

int tc_max_n(int) { return kNMax; }

bool tc_supported(int hidden, int inter) {
    // conversion kernels: hidden / 16 threads per token (<= 1024), inter / 16 per slot row (<= 256)
    return hidden % 512 == 0 && inter % 512 == 0 && hidden <= 16384 && inter <= 4096;
}

void launch_convert_x(const IoArgs* x, const int* slot_pos, int M, int ns, int len, __half* dst,
                      int* sexp, cudaStream_t s) {
    convert_x_kernel<<<M, len / 16, 0, s>>>(x, slot_pos, M, ns, len, dst, sexp);
}

void launch_convert_h(const float* gu, int n_rows, const int* n_used, int inter, __half* dst, int* sexp,
                      cudaStream_t s) {
    const int per_cta = 256 / (inter / 16);
    convert_h_kernel<<<(n_rows + per_cta - 1) / per_cta, per_cta * (inter / 16), 0, s>>>(gu, n_rows, n_used, inter,
                                                                                        dst, sexp);
}

void launch_tc13(const Layer& L, const BMaps& xmap, const Workspace& ws, int max_items,
                 int sm_count, bool a_tmem, cudaStream_t s) {
    const int I = static_cast<int>(L.spec.inter);
    TcArgs a{L.tables(), static_cast<int>(L.spec.hidden / kQK) * kBlockBytes, L.wmaps,
             static_cast<int>(L.spec.n_experts) + 1, 0, I / 128, 2 * I / 128,
             ws.tiles13, ws.counters, 1, static_cast<int>(L.spec.hidden), ws.xexp, ws.h, 2 * I,
             ws.status};
    const int grid = max_items < sm_count ? (max_items > 0 ? max_items : 1) : sm_count;
    if (a_tmem) launch_tc<true>(xmap, a, grid, s);
    else launch_tc<false>(xmap, a, grid, s);
}

void launch_tc2(const Layer& L, const BMaps& hmap, const Workspace& ws, int max_items,
                int sm_count, bool a_tmem, cudaStream_t s) {
    const int H = static_cast<int>(L.spec.hidden);
    TcArgs a{L.tables(), static_cast<int>(L.spec.inter / kQK) * kBlockBytes, L.wmaps,
             static_cast<int>(L.spec.n_experts) + 1, 2, H / 128, H / 128, ws.tiles2,
             ws.counters, 2, static_cast<int>(L.spec.inter), ws.hexp, ws.ypart, H, ws.status};
    const int grid = max_items < sm_count ? (max_items > 0 ? max_items : 1) : sm_count;
    if (a_tmem) launch_tc<true>(hmap, a, grid, s);
    else launch_tc<false>(hmap, a, grid, s);
}

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return encode;
}

// 2D tensor maps over an fp16 [rows][cols] row-major matrix, boxes of 16/32/64/112 rows x 64
// cols, 128B swizzle.
bool make_fp16_tmaps(BMaps* m, const void* base, uint64_t rows, uint64_t cols) {
    auto encode = tmap_encoder();
    if (!encode) return false;
    for (int i = 0; i < 4; ++i) {
        const cuuint64_t dims[2] = {cols, rows};
        const cuuint64_t strides[1] = {cols * 2};
        const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows(i))};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&m->m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

// 2D tensor map over an f32 [rows][cols] row-major matrix, box box_rows x 32 cols, 128B swizzle.
bool make_f32_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto encode = tmap_encoder();
    if (!encode || (cols * 4) % 16 != 0) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {32, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2D tensor map over the raw bytes of an IQ4_XS matrix [rows][row_bytes], viewed as 8-byte
// elements (the 16-bit view measured several times slower per box), box 128 rows x 272 bytes
// (two blocks = 512 weights of K), no swizzle.
bool make_iq4_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes) {
    auto encode = tmap_encoder();
    if (!encode || row_bytes % 16 != 0) return false;
    const cuuint64_t dims[2] = {row_bytes / kRawElem, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {kRawRowBytes / kRawElem, kRawBoxRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = kRawElem == 8 ? CU_TENSOR_MAP_DATA_TYPE_UINT64
                                 : kRawElem == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32
                                                 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    return encode(m, dt, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

#ifdef MOE_TC_TRACE
extern "C" int moe_debug_tc_trace(unsigned long long* out) {
    return cudaMemcpyFromSymbol(out, g_tc_trace, sizeof(g_tc_trace)) == cudaSuccess ? 0 : -2;
}
extern "C" int moe_debug_tc_trace_clear() {
    static unsigned long long zero[2][8][1024];
    return cudaMemcpyToSymbol(g_tc_trace, zero, sizeof(zero)) == cudaSuccess ? 0 : -2;
}
#endif

}  // namespace moe
