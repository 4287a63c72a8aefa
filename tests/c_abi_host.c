/* A host program in plain C11 that drives the library only through include/moe_b200.h, the
 * way a non-Python host (the reference's Rust engine through its FFI crate) would: context and
 * arena, synthetic IQ4_XS weights, one layer, routing, forwards at M = 1 and M = 64 (the fused
 * single-token kernel and the bucketed tensor-core path), the LM-head projection, and the error
 * path.  Exit status 0 and a final "c host ok" line on success.
 *
 * Build: cc -std=c11 -Wall -Wextra -Werror -I include tests/c_abi_host.c \
 *           -L moe-680m_b200/lib -lmoe_b200 -lm -o c_abi_host */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "moe_b200.h"

#define H 2048u
#define I 512u
#define E 256u
#define K 8u

static moe_ctx* g_ctx;
static uint64_t g_top = 256;

static void die(const char* what, int rc) {
    char msg[512] = {0};
    moe_last_error(g_ctx, msg, sizeof msg);
    fprintf(stderr, "%s failed (%d): %s\n", what, rc, msg);
    exit(1);
}

#define CHECK(call)                        \
    do {                                   \
        int rc_ = (call);                  \
        if (rc_ != MOE_OK) die(#call, rc_); \
    } while (0)

static uint64_t arena_alloc(uint64_t bytes) {
    const uint64_t off = g_top;
    g_top = (g_top + bytes + 255) / 256 * 256;
    return off;
}

static uint64_t g_rng = 0x9E3779B97F4A7C15ull;
static float uniform_pm1(void) { /* xorshift64*, uniform in [-1, 1) */
    g_rng ^= g_rng >> 12;
    g_rng ^= g_rng << 25;
    g_rng ^= g_rng >> 27;
    return (float)((g_rng * 0x2545F4914F6CDD1Dull) >> 40) / 8388608.0f - 1.0f;
}

static uint64_t upload_random(size_t n, float amp) {
    float* h = malloc(n * sizeof(float));
    for (size_t i = 0; i < n; ++i) h[i] = amp * uniform_pm1();
    const uint64_t off = arena_alloc(n * sizeof(float));
    CHECK(moe_arena_upload(g_ctx, off, h, n * sizeof(float)));
    free(h);
    return off;
}

static uint64_t synth_matrix(uint64_t key, uint32_t rows, uint32_t cols) {
    const uint64_t blocks = (uint64_t)rows * (cols / 256);
    const uint64_t off = arena_alloc(blocks * 136);
    CHECK(moe_synth_iq4xs(g_ctx, off, key, 0, blocks));
    return off;
}

static int forward_and_check(uint32_t id, uint32_t m) {
    const size_t n = (size_t)m * H;
    const uint64_t x = upload_random(n, 1.0f);
    const uint64_t out = arena_alloc(n * sizeof(float));
    float* a = malloc(n * sizeof(float));
    float* b = malloc(n * sizeof(float));
    CHECK(moe_forward(g_ctx, id, x, x, out, m));
    CHECK(moe_sync(g_ctx));
    CHECK(moe_arena_download(g_ctx, out, a, n * sizeof(float)));
    CHECK(moe_forward(g_ctx, id, x, x, out, m));
    CHECK(moe_sync(g_ctx));
    CHECK(moe_arena_download(g_ctx, out, b, n * sizeof(float)));
    /* the same rows from host memory through the asynchronous entry point */
    float* xh = malloc(n * sizeof(float));
    float* c = malloc(n * sizeof(float));
    CHECK(moe_arena_download(g_ctx, x, xh, n * sizeof(float)));
    CHECK(moe_forward_host(g_ctx, id, xh, c, m, 1));
    CHECK(moe_sync(g_ctx));
    int bad = 0;
    if (memcmp(a, c, n * sizeof(float)) != 0) bad = 1;
    free(xh);
    free(c);
    double s = 0.0;
    for (size_t i = 0; i < n; ++i) {
        if (!isfinite(a[i])) bad = 1;
        s += fabs((double)a[i]);
    }
    if (memcmp(a, b, n * sizeof(float)) != 0) bad = 1; /* deterministic reruns */
    printf("forward M=%u: mean |out| %.4f%s\n", m, s / (double)n, bad ? " MISMATCH" : "");
    free(a);
    free(b);
    return bad;
}

int main(void) {
    int rc = moe_ctx_create(0, 2ull << 30, &g_ctx);
    if (rc != MOE_OK) die("moe_ctx_create", rc);
    if (moe_abi_version() != MOE_B200_ABI_VERSION) {
        fprintf(stderr, "ABI version %d, header %d\n", moe_abi_version(), MOE_B200_ABI_VERSION);
        return 1;
    }
    moe_layer_spec spec;
    memset(&spec, 0, sizeof spec);
    spec.hidden = H;
    spec.inter = I;
    spec.n_experts = E;
    spec.top_k = K;
    spec.flags = MOE_F_SHARED | MOE_F_SHARED_GATE;
    spec.scale = 1.0f;
    spec.router_w = upload_random((size_t)E * H, 0.02f);
    spec.shared_gate = upload_random(H, 0.02f);
    uint64_t w1[E], w3[E], w2[E];
    for (uint32_t e = 0; e < E; ++e) {
        w1[e] = synth_matrix(1000u + 3u * e, I, H);
        w3[e] = synth_matrix(1001u + 3u * e, I, H);
        w2[e] = synth_matrix(1002u + 3u * e, H, I);
    }
    spec.shared_w1 = synth_matrix(7u, I, H);
    spec.shared_w3 = synth_matrix(8u, I, H);
    spec.shared_w2 = synth_matrix(9u, H, I);
    uint32_t id = 0;
    CHECK(moe_layer_create(g_ctx, &spec, w1, w3, w2, &id));

    /* routing records on the host (do_route's RoutingOutput) */
    const uint32_t mr = 4;
    const uint64_t xr = upload_random((size_t)mr * H, 1.0f);
    uint16_t routed[4 * K];
    float weights[4 * K], gate[4];
    CHECK(moe_do_route(g_ctx, id, xr, mr, routed, weights, gate));
    int bad = 0;
    for (uint32_t t = 0; t < mr; ++t) {
        float sum = 0.f;
        for (uint32_t s = 0; s < K; ++s) {
            if (routed[t * K + s] >= E) bad = 1;
            if (s > 0 && weights[t * K + s] > weights[t * K + s - 1]) bad = 1; /* descending */
            sum += weights[t * K + s];
        }
        if (!(sum > 0.f && sum <= 1.0001f) || !(gate[t] > 0.f && gate[t] < 1.f)) bad = 1;
    }
    printf("route: token 0 experts %u %u %u ... weights %.4f %.4f ...%s\n", routed[0], routed[1], routed[2],
           weights[0], weights[1], bad ? " BAD" : "");

    bad |= forward_and_check(id, 1);
    bad |= forward_and_check(id, 64);

    /* LM head: 4096-row vocabulary, greedy id */
    const uint32_t vocab = 4096;
    const uint64_t wv = synth_matrix(77u, vocab, H);
    const uint64_t xv = upload_random(H, 1.0f);
    const uint64_t lv = arena_alloc((uint64_t)vocab * sizeof(float));
    const uint64_t iv = arena_alloc(256);
    CHECK(moe_vocab_logits(g_ctx, wv, vocab, H, xv, 1, lv, iv));
    CHECK(moe_sync(g_ctx));
    float* lg = malloc(vocab * sizeof(float));
    uint32_t tok = 0;
    CHECK(moe_arena_download(g_ctx, lv, lg, vocab * sizeof(float)));
    CHECK(moe_arena_download(g_ctx, iv, &tok, sizeof tok));
    uint32_t best = 0;
    for (uint32_t n = 1; n < vocab; ++n)
        if (lg[n] > lg[best]) best = n;
    if (tok != best) bad = 1;
    printf("lm head: token %u (host argmax %u)\n", tok, best);
    free(lg);

    /* error path: offset 0 is the missing-tensor sentinel */
    rc = moe_forward(g_ctx, id, 0, 0, lv, 1);
    char msg[256] = {0};
    moe_last_error(g_ctx, msg, sizeof msg);
    if (rc != MOE_E_INVALID || msg[0] == 0) bad = 1;
    printf("error path: %d \"%s\"\n", rc, msg);

    moe_ctx_destroy(g_ctx);
    if (bad) {
        fprintf(stderr, "c host FAILED\n");
        return 1;
    }
    printf("c host ok\n");
    return 0;
}
