/*
 * CPU oracle and CPU baseline of the MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm load this
 * library, and only as the checker or the timed CPU restatement; the product path never does.
 *
 * A plain-C (OpenMP) restatement of moe-680m's MoE layer (paths in the moe-680m tree), with
 * the contract's semantics where the reference has known defects (same list as
 * oracle/moe_oracle.py):
 *   router      shaders/router.comp:21-60 (f32 weight), bias added to the logits
 *   softmax     shaders/router_topk.comp:36-60, src/router.rs:23-35
 *   top-k       shaders/router_topk.comp:67-85 (descending, ties -> lower index)
 *   bucketing   src/router.rs:55-97 (stable; shared expert in its own bucket E)
 *   experts     shaders/w1_w3_fused(_m1).comp, shaders/silu_mult.comp, shaders/w2.comp:
 *               g = W1 x, u = W3 x, h = silu(g) u, y = W2 h, silu from shaders/common.glsl:106
 *   combine     shaders/moe_combine.comp:32-45 / w2_scatter.comp:67-86:
 *               out = resid + scale * (sum_k p_k y_k + gate * y_shared)
 *   decode      GGUF IQ4_XS (ggml type 23), the format the contract names; the reference's
 *               shaders/common.glsl:59-86 decodes a private 36-byte block instead.
 * Accumulation is double (acc64 = 1, the parity oracle) or float (acc64 = 0, the loop
 * structure and precision of the reference shaders, used as the timed CPU baseline).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 256
#define BLK 136

static const int8_t KV[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                              1, 13, 25, 38, 53, 69, 89, 113};

static float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) bits = s;
        else { /* subnormal: value m * 2^-24 */
            float v = (float)m * (1.0f / 16777216.0f);
            memcpy(&bits, &v, 4);
            bits |= s;
        }
    } else if (e == 31) bits = s | 0x7f800000u | (m << 13);
    else bits = s | ((e + 112) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Decode one block into 256 floats (exact). */
static void decode_block(const uint8_t* b, float* out) {
    uint16_t dh, sh;
    memcpy(&dh, b, 2);
    memcpy(&sh, b + 2, 2);
    const float d = f16_to_f32(dh);
    for (int ib = 0; ib < 8; ++ib) {
        const int ls = ((b[4 + ib / 2] >> (4 * (ib % 2))) & 0xf) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
        const uint8_t* q = b + 8 + 16 * ib;
        for (int j = 0; j < 16; ++j) {
            out[32 * ib + j] = dl * (float)KV[q[j] & 0xf];
            out[32 * ib + 16 + j] = dl * (float)KV[q[j] >> 4];
        }
    }
}

void oracle_dequant_iq4xs(const uint8_t* src, int64_t n_blocks, float* dst) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n_blocks; ++i) decode_block(src + i * BLK, dst + i * QK);
}

static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint16_t f32_to_f16_rn(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t m = x & 0x7fffffu;
    if (e <= 0 || e >= 31) return (uint16_t)sign; /* values used here are normal f16 */
    uint32_t h = ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
    return (uint16_t)(sign | h);
}

/* C twin of the library's synthetic IQ4_XS generator (moe_synth_iq4xs). */
void oracle_synth_iq4xs(uint8_t* dst, uint64_t key, uint64_t block_start, uint64_t n_blocks) {
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < (int64_t)n_blocks; ++b) {
        uint64_t w[17];
        for (int i = 0; i < 17; ++i) w[i] = splitmix64(key + ((uint64_t)b + block_start) * 17 + i);
        volatile float u = (float)(uint32_t)(w[0] >> 40) * (1.0f / 16777216.0f);
        volatile float p = 0.015f * u;
        volatile float v = 0.005f + p;
        const uint16_t d = f32_to_f16_rn(v);
        w[0] = (w[0] & ~0xffffull) | d;
        memcpy(dst + (uint64_t)b * BLK, w, BLK);
    }
}

typedef struct oracle_layer {
    int32_t hidden, inter, n_experts, top_k;
    int32_t has_shared, has_gate;
    float scale;
    const float* router_w;  /* [E][H] */
    const float* router_bias; /* [E] or NULL */
    const float* gate_w;    /* [H] or NULL */
    const uint8_t* const* w1; /* [E+1] (index E: shared) */
    const uint8_t* const* w3;
    const uint8_t* const* w2;
} oracle_layer;

/* Router + softmax + top-k for M tokens. ids/w: [M][k]; gate: [M]; logits (optional) [M][E]. */
void oracle_route(const oracle_layer* L, const float* x, int M, int acc64, int32_t* ids,
                  float* w, float* gate, float* logits_out) {
    const int H = L->hidden, E = L->n_experts, k = L->top_k;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < M; ++t) {
        float lg[256], p[256];
        const float* xt = x + (size_t)t * H;
        for (int e = 0; e < E; ++e) {
            const float* wr = L->router_w + (size_t)e * H;
            float v;
            if (acc64) {
                double a = 0.0;
                for (int i = 0; i < H; ++i) a += (double)xt[i] * (double)wr[i];
                v = (float)a;
            } else {
                float a = 0.f;
                for (int i = 0; i < H; ++i) a += xt[i] * wr[i];
                v = a;
            }
            if (L->router_bias) v += L->router_bias[e];
            lg[e] = v;
            if (logits_out) logits_out[(size_t)t * E + e] = v;
        }
        float mx = -INFINITY;
        for (int e = 0; e < E; ++e) mx = lg[e] > mx ? lg[e] : mx;
        float s = 0.f;
        for (int e = 0; e < E; ++e) { p[e] = expf(lg[e] - mx); s += p[e]; }
        for (int e = 0; e < E; ++e) p[e] = s > 0.f ? p[e] / s : 0.f;
        /* strict '>' insertion: descending, earlier (lower) index wins ties */
        int bi[8];
        float bv[8];
        for (int j = 0; j < k; ++j) { bi[j] = 0; bv[j] = -1.f; }
        for (int e = 0; e < E; ++e) {
            for (int j = 0; j < k; ++j) {
                if (p[e] > bv[j]) {
                    for (int s2 = k - 1; s2 > j; --s2) { bv[s2] = bv[s2 - 1]; bi[s2] = bi[s2 - 1]; }
                    bv[j] = p[e];
                    bi[j] = e;
                    break;
                }
            }
        }
        for (int j = 0; j < k; ++j) { ids[(size_t)t * k + j] = bi[j]; w[(size_t)t * k + j] = bv[j]; }
        float g = 1.f;
        if (L->has_gate && L->gate_w) {
            double a = 0.0;
            for (int i = 0; i < H; ++i) a += (double)xt[i] * (double)L->gate_w[i];
            g = (float)(1.0 / (1.0 + exp(-a)));
        }
        gate[t] = g;
    }
}

/* Stable bucketing (src/router.rs:55-97).  ranges [E+2], tokens/weights [S], pos [M][ns]. */
void oracle_bucket(const int32_t* ids, const float* w, const float* gate, int M, int E, int k,
                   int has_shared, int32_t* ranges, int32_t* tokens, float* weights, int32_t* pos) {
    const int nb = E + 1, ns = k + (has_shared ? 1 : 0);
    int32_t* cnt = (int32_t*)calloc((size_t)nb, sizeof(int32_t));
    for (int t = 0; t < M; ++t)
        for (int j = 0; j < k; ++j) cnt[ids[(size_t)t * k + j]]++;
    if (has_shared) cnt[E] += M;
    ranges[0] = 0;
    for (int e = 0; e < nb; ++e) ranges[e + 1] = ranges[e] + cnt[e];
    for (int e = 0; e < nb; ++e) cnt[e] = ranges[e];
    for (int t = 0; t < M; ++t) {
        for (int j = 0; j < k; ++j) {
            const int e = ids[(size_t)t * k + j];
            const int p = cnt[e]++;
            tokens[p] = t;
            weights[p] = w[(size_t)t * k + j];
            pos[(size_t)t * ns + j] = p;
        }
        if (has_shared) {
            const int p = cnt[E]++;
            tokens[p] = t;
            weights[p] = gate ? gate[t] : 1.f;
            pos[(size_t)t * ns + k] = p;
        }
    }
    free(cnt);
}

static double silu_d(double v) { return v / (1.0 + exp(-v)); }
static float silu_f(float v) { return v / (1.0f + expf(-v)); }

/* Full layer.  out [M][H] (float; also out64 [M][H] if non-NULL).  ids/w/gate optional
 * outputs of the routing ([M][k], [M][k], [M]).  nthreads <= 0: OpenMP default. */
int oracle_moe_forward(const oracle_layer* L, const float* x, const float* resid, int M,
                       int acc64, int nthreads, float* out, double* out64, int32_t* ids_out,
                       float* w_out, float* gate_out) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
    const int H = L->hidden, I = L->inter, E = L->n_experts, k = L->top_k;
    const int ns = k + (L->has_shared ? 1 : 0);
    const size_t S = (size_t)M * ns;
    int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * M * k);
    float* w = (float*)malloc(sizeof(float) * M * k);
    float* gate = (float*)malloc(sizeof(float) * M);
    int32_t* ranges = (int32_t*)malloc(sizeof(int32_t) * (E + 2));
    int32_t* tokens = (int32_t*)malloc(sizeof(int32_t) * S);
    float* sw = (float*)malloc(sizeof(float) * S);
    int32_t* pos = (int32_t*)malloc(sizeof(int32_t) * S);
    double* h = (double*)malloc(sizeof(double) * S * I);
    double* y = (double*)malloc(sizeof(double) * S * H);
    if (!ids || !w || !gate || !ranges || !tokens || !sw || !pos || !h || !y) return -1;
    oracle_route(L, x, M, acc64, ids, w, gate, NULL);
    oracle_bucket(ids, w, gate, M, E, k, L->has_shared, ranges, tokens, sw, pos);
    const int nbh = H / QK, nbi = I / QK;
    for (int e = 0; e <= E; ++e) {
        const int p0 = ranges[e], p1 = ranges[e + 1];
        if (p1 <= p0) continue;
        const uint8_t* w1 = L->w1[e];
        const uint8_t* w3 = L->w3[e];
        const uint8_t* w2 = L->w2[e];
#pragma omp parallel
        {
            float* r1 = (float*)malloc(sizeof(float) * (H > I ? H : I));
            float* r3 = (float*)malloc(sizeof(float) * H);
#pragma omp for schedule(static)
            for (int j = 0; j < I; ++j) {
                for (int b = 0; b < nbh; ++b) {
                    decode_block(w1 + ((size_t)j * nbh + b) * BLK, r1 + b * QK);
                    decode_block(w3 + ((size_t)j * nbh + b) * BLK, r3 + b * QK);
                }
                for (int p = p0; p < p1; ++p) {
                    const float* xt = x + (size_t)tokens[p] * H;
                    if (acc64) {
                        double g = 0, u = 0;
                        for (int i = 0; i < H; ++i) { g += (double)r1[i] * xt[i]; u += (double)r3[i] * xt[i]; }
                        h[(size_t)p * I + j] = silu_d(g) * u;
                    } else {
                        float g = 0, u = 0;
                        for (int i = 0; i < H; ++i) { g += r1[i] * xt[i]; u += r3[i] * xt[i]; }
                        h[(size_t)p * I + j] = (double)(silu_f(g) * u);
                    }
                }
            }
#pragma omp for schedule(static)
            for (int n = 0; n < H; ++n) {
                for (int b = 0; b < nbi; ++b) decode_block(w2 + ((size_t)n * nbi + b) * BLK, r1 + b * QK);
                for (int p = p0; p < p1; ++p) {
                    const double* hp = h + (size_t)p * I;
                    if (acc64) {
                        double a = 0;
                        for (int i = 0; i < I; ++i) a += (double)r1[i] * hp[i];
                        y[(size_t)p * H + n] = a;
                    } else {
                        float a = 0;
                        for (int i = 0; i < I; ++i) a += r1[i] * (float)hp[i];
                        y[(size_t)p * H + n] = a;
                    }
                }
            }
            free(r1);
            free(r3);
        }
    }
#pragma omp parallel for schedule(static)
    for (int t = 0; t < M; ++t) {
        for (int n = 0; n < H; ++n) {
            double a = 0;
            for (int s = 0; s < ns; ++s) {
                const int p = pos[(size_t)t * ns + s];
                a += (double)sw[p] * y[(size_t)p * H + n];
            }
            const double r = (resid ? (double)resid[(size_t)t * H + n] : 0.0) + (double)L->scale * a;
            if (out) out[(size_t)t * H + n] = (float)r;
            if (out64) out64[(size_t)t * H + n] = r;
        }
    }
    if (ids_out) memcpy(ids_out, ids, sizeof(int32_t) * M * k);
    if (w_out) memcpy(w_out, w, sizeof(float) * M * k);
    if (gate_out) memcpy(gate_out, gate, sizeof(float) * M);
    free(ids); free(w); free(gate); free(ranges); free(tokens); free(sw); free(pos); free(h); free(y);
    return 0;
}
