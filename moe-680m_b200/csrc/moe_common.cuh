// Shared device helpers of the MoE-layer library: IQ4_XS block access and decode, warp
// reductions, streaming loads.
//
// IQ4_XS (GGUF ggml type 23) block of 256 weights, 136 bytes:
//   +0 f16 d | +2 u16 scales_h | +4 u8 scales_l[4] | +8 u8 qs[128]
// Sub-block ib (0..7) covers weights 32*ib .. 32*ib+31 with the 6-bit scale
//   ls = (scales_l[ib/2] >> 4*(ib%2) & 15) | ((scales_h >> 2*ib & 3) << 4)
// and weight 32*ib + j (j < 16) = d*(ls-32)*kvalues_iq4nl[qs[16*ib+j] & 15],
//     weight 32*ib + 16 + j     = d*(ls-32)*kvalues_iq4nl[qs[16*ib+j] >> 4].
// (The reference decodes a private 36-byte block in shaders/common.glsl:59-86; this library
// implements the GGUF block named by the contract.)
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace moe {

constexpr int kQK = 256;          // weights per block
constexpr int kBlockBytes = 136;  // bytes per block
constexpr int kSubPerBlock = 8;   // 32-weight sub-blocks per block
constexpr int kMaxTopK = 8;
constexpr int kMaxExperts = 256;
constexpr uint32_t kNoExpert = 0xFFFFFFFFu;  // expert id of an empty routed slot

// kvalues_iq4nl + 128 as unsigned bytes, packed 4 per word (entries 0-3, 4-7, 8-11, 12-15):
// {-127,-104,-83,-65, -49,-35,-22,-10, 1,13,25,38, 53,69,89,113} + 128
constexpr uint32_t kKvT0 = 0x3F2D1801u;  // 1, 24, 45, 63
constexpr uint32_t kKvT1 = 0x766A5D4Fu;  // 79, 93, 106, 118
constexpr uint32_t kKvT2 = 0xA6998D81u;  // 129, 141, 153, 166
constexpr uint32_t kKvT3 = 0xF1D9C5B5u;  // 181, 197, 217, 241
// float with bits 0x4B000000 | b equals 2^23 + b; subtracting 2^23 + 128 yields b - 128 = kv.
constexpr float kKvMagicOffset = 8388736.0f;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}

// Table lookup of 4 nibbles (the low 16 bits of `sel`) -> 4 bytes kv+128.
// Bits 0-2 of each nibble index an 8-entry half table, bit 3 picks the half.
__device__ __forceinline__ uint32_t kv_lookup4(uint32_t nib7, uint32_t pick) {
    const uint32_t lo = prmt(kKvT0, kKvT1, nib7);
    const uint32_t hi = prmt(kKvT2, kKvT3, nib7);
    return prmt(lo, hi, pick);
}

// Decode the 8 nibbles of one qs word q (bytes b0..b3) into kv+128 bytes.
// r0 = [kv(b0 lo), kv(b0 hi), kv(b1 lo), kv(b1 hi)], r1 = same for b2, b3.
__device__ __forceinline__ void kv_lookup8(uint32_t q, uint32_t& r0, uint32_t& r1) {
    const uint32_t nib7 = q & 0x77777777u;
    const uint32_t pick = ((q >> 1) & 0x44444444u) | 0x32103210u;
    r0 = kv_lookup4(nib7, pick);
    r1 = kv_lookup4(nib7 >> 16, pick >> 16);
}

// Byte i of r (a kv+128 byte) -> exact float kv.
template <int I>
__device__ __forceinline__ float kv_float(uint32_t r) {
    return __uint_as_float(prmt(r, 0x4B000000u, 0x7440u | I)) - kKvMagicOffset;
}

// Sub-block scale d*(ls-32) from the block header words (h0 = bytes 0..3, h1 = bytes 4..7).
__device__ __forceinline__ float iq4_subscale(uint32_t h0, uint32_t h1, int ib) {
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(h0 & 0xFFFFu)));
    const uint32_t ls = ((h1 >> (4 * ib)) & 0xFu) | (((h0 >> (16 + 2 * ib)) & 3u) << 4);
    return d * static_cast<float>(static_cast<int>(ls) - 32);
}

// Streaming 8-byte load that skips L1 allocation (weights are read once).
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// One sub-block of a row: 8-byte block header + 16 bytes of nibbles.
struct SubBlk {
    uint2 hdr;
    uint2 q01;
    uint2 q23;
};

// Load sub-block `sb` (0-based along the row) of a row starting at `row`.
__device__ __forceinline__ SubBlk load_subblk(const uint8_t* row, int sb) {
    const uint8_t* blk = row + (sb >> 3) * kBlockBytes;
    SubBlk s;
    s.hdr = ldg_stream_u2(blk);
    const uint8_t* q = blk + 8 + (sb & 7) * 16;
    s.q01 = ldg_stream_u2(q);
    s.q23 = ldg_stream_u2(q + 8);
    return s;
}

// Dot of one IQ4_XS word (8 weights: j0..j0+3 low nibbles, j0+16..j0+19 high nibbles) with
// x (xa = x[j0..j0+3], xb = x[j0+16..j0+19]).
__device__ __forceinline__ float dot_word(uint32_t q, float4 xa, float4 xb, float acc) {
    uint32_t r0, r1;
    kv_lookup8(q, r0, r1);
    acc = fmaf(kv_float<0>(r0), xa.x, acc);
    acc = fmaf(kv_float<1>(r0), xb.x, acc);
    acc = fmaf(kv_float<2>(r0), xa.y, acc);
    acc = fmaf(kv_float<3>(r0), xb.y, acc);
    acc = fmaf(kv_float<0>(r1), xa.z, acc);
    acc = fmaf(kv_float<1>(r1), xb.z, acc);
    acc = fmaf(kv_float<2>(r1), xa.w, acc);
    acc = fmaf(kv_float<3>(r1), xb.w, acc);
    return acc;
}

// Unscaled dot of a sub-block's 32 codes with 32 activations at xs (16-byte aligned, f32).
__device__ __forceinline__ float dot_subblk(const SubBlk& s, const float* xs) {
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    float acc = 0.f;
    acc = dot_word(s.q01.x, x4[0], x4[4], acc);
    acc = dot_word(s.q01.y, x4[1], x4[5], acc);
    acc = dot_word(s.q23.x, x4[2], x4[6], acc);
    acc = dot_word(s.q23.y, x4[3], x4[7], acc);
    return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// Padded activation layout in shared memory: 32-float sub-block s at float offset 36*s, so
// lanes reading consecutive sub-blocks with 16-byte loads hit distinct banks.
__host__ __device__ constexpr int padded_len(int n) { return (n / 32) * 36; }
__device__ __forceinline__ int padded_idx(int k) { return (k >> 5) * 36 + (k & 31); }

// Device-side error codes written to the status word.
enum DevErr : int { kDevOk = 0, kDevBadExpert = 1, kDevBadToken = 2, kDevOverflow = 3, kDevTimeout = 4 };

__device__ __forceinline__ void set_dev_error(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

}  // namespace moe
