/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * This library replaces the Vulkan MoE dispatch of moe-680m (paths below are relative to the
 * moe-680m source tree).  The reference binds its compute through ash/Vulkan
 * (src/device.rs, src/pipeline.rs) and records the MoE layer in
 * InferenceEngine::record_and_submit_moe (src/inference.rs:663-766), with routing from
 * do_route (src/inference.rs:622-659) and the router tail of record_and_submit_layer
 * (src/inference.rs:598-616).  Every argument of those kernels is a u64 byte offset into one
 * device arena (PushConstants, src/inference.rs:15-51), offset 0 meaning "missing tensor"
 * (src/memory.rs:33, :234).  This ABI keeps that model: a context owns (or wraps) one device
 * arena and every tensor argument is a byte offset into it; offset 0 is invalid.
 *
 * Conventions
 *  - Every call returns MOE_OK (0) or a negative MOE_E* status; moe_last_error() gives text.
 *  - Calls are stream-ordered on the context's stream (moe_set_stream) and asynchronous
 *    unless stated otherwise; moe_sync() is the fence wait of the reference
 *    (src/inference.rs:169-182).  A context is not thread-safe (the reference serialises its
 *    engine behind a Mutex, src/server.rs:95).
 *  - Weights are GGUF IQ4_XS (ggml type 23): rows of 136-byte blocks of 256 weights, row-major
 *    [out_features][in_features], blocks along in_features.
 *  - Activations are f32 row-major [M][hidden].
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 1

/* status codes */
#define MOE_OK 0
#define MOE_E_INVALID (-1)     /* bad argument (offset 0, out of arena, bad shape) */
#define MOE_E_CUDA (-2)        /* a CUDA runtime call failed */
#define MOE_E_OOM (-3)         /* device allocation failed */
#define MOE_E_UNSUPPORTED (-4) /* shape or device outside what this build supports */
#define MOE_E_DEVICE (-5)      /* a kernel reported an error status (bounds / bad index) */

typedef struct moe_ctx moe_ctx;

/* Layer flags */
#define MOE_F_SHARED 1u      /* layer has a shared expert (always active, own bucket) */
#define MOE_F_SHARED_GATE 2u /* shared expert weighted by sigmoid(g . x); else weight 1.0 */
#define MOE_F_EXPERT_SUBSET 4u /* expert-parallel rank: experts whose w1, w3 and w2 offsets are all
                                  0 are held by another rank; such a layer only serves moe_route
                                  and moe_forward_topk, and nothing may be routed to a missing
                                  expert (no counterpart in the single-device reference) */

#define MOE_F_REF36 8u   /* expert weights in the reference's own format: 36-byte blocks of 32 weights
                            (shaders/common.glsl:59-86), each matrix stored [in][out] with weight
                            (k, n) at flat index k*out + n (shaders/w1_w3_fused_m1.comp:46-47,
                            w2_scatter_m1.comp:41): W1/W3 [hidden][inter], W2 [inter][hidden],
                            hidden*inter/32*36 bytes each.  A compatibility path (CUDA cores, f32,
                            K-split grouped GEMV); hidden and inter multiples of 512 */

/* Expert id of an empty routed entry in a routing record (skipped by bucketing). */
#define MOE_NO_EXPERT 0xFFFFFFFFu

/* Per-layer description: the scalar half of LayerWeights (src/memory.rs:201-223) plus the
 * ModelConfig fields the MoE kernels read.  Offsets are arena byte offsets. */
typedef struct moe_layer_spec {
    uint32_t hidden;      /* H, multiple of 256 */
    uint32_t inter;       /* I (expert and shared intermediate), multiple of 256 */
    uint32_t n_experts;   /* E, 1..256 */
    uint32_t top_k;       /* k, 1..8 */
    uint32_t flags;       /* MOE_F_* */
    float scale;          /* global combine scale (1.0; 1/9 reproduces the reference) */
    uint64_t router_w;    /* f32 [E][H]  (ffn_gate; src/memory.rs:212) */
    uint64_t router_bias; /* f32 [E] added to the logits, or 0 */
    uint64_t shared_gate; /* f32 [H] (MOE_F_SHARED_GATE), else 0 */
    uint64_t shared_w1;   /* IQ4_XS [I][H] (shared_expert.w1; src/memory.rs:251) */
    uint64_t shared_w3;   /* IQ4_XS [I][H] */
    uint64_t shared_w2;   /* IQ4_XS [H][I] */
} moe_layer_spec;

/* ---- context and arena (replaces DeviceContext::init / allocate_uma, src/device.rs:20,217) */

/* Create a context on CUDA device `device` owning a fresh arena of `arena_bytes`. */
int moe_ctx_create(int device, uint64_t arena_bytes, moe_ctx** out);
/* Create a context over caller-owned device memory [base, base+bytes) (not freed by us). */
int moe_ctx_create_external(int device, void* base, uint64_t bytes, moe_ctx** out);
void moe_ctx_destroy(moe_ctx* ctx);
/* Copy into / out of the arena (replaces the host memcpy of load_weights_from_tensors,
 * src/memory.rs:297-321, and the coherent-mapping writes of src/inference.rs:685-699).
 * Upload is stream-ordered; download waits for the stream and the copy. */
int moe_arena_upload(moe_ctx* ctx, uint64_t off, const void* host, uint64_t n);
int moe_arena_download(moe_ctx* ctx, uint64_t off, void* host, uint64_t n);
/* Device address of arena offset `off` (for interop; no ownership transfer). */
int moe_arena_ptr(moe_ctx* ctx, uint64_t off, void** dptr);
/* Use `stream` (a cudaStream_t, or NULL for the context's own stream) for later calls. */
int moe_set_stream(moe_ctx* ctx, void* stream);
/* Wait for all work queued on the context's stream (the reference's fence wait). */
int moe_sync(moe_ctx* ctx);
/* Copy the last error message of this context (or of context creation if ctx is NULL). */
int moe_last_error(const moe_ctx* ctx, char* buf, size_t n);
int moe_abi_version(void);

/* ---- layers (replaces LayerWeights::from_registry, src/memory.rs:227-290) ---------------- */

/* Register one MoE layer.  w1/w3/w2 are host arrays of E arena offsets (the flat
 * expert_w{1,2,3}[layer*E + e] tables of LayerWeights, one layer's slice).  Every offset is
 * validated (non-zero, 256-byte aligned, inside the arena).  Returns a layer id >= 0. */
int moe_layer_create(moe_ctx* ctx, const moe_layer_spec* spec, const uint64_t* w1,
                     const uint64_t* w3, const uint64_t* w2, uint32_t* layer_id);

/* Pre-size the internal workspace for batches of up to max_tokens tokens (call before CUDA
 * graph capture; forward calls otherwise grow it on demand). */
int moe_reserve(moe_ctx* ctx, uint32_t layer_id, uint32_t max_tokens);

/* ---- routing (router.comp + router_topk.comp + router.rs::route_single) ------------------ */

/* Router projection, 256-way softmax and top-k for M tokens of x (f32 [M][H] at x_off).
 * Writes M records of (k+1) x {u32 expert_id, f32 weight} at topk_off: entry 0 is the shared
 * expert {E, gate} (gate = sigmoid(g.x), or 1.0), entries 1..k the routed experts by
 * descending probability, ties to the lower expert index (the 72-byte record of
 * shaders/router_topk.comp:87-92 with the shared id made distinct from expert 0). */
int moe_route(moe_ctx* ctx, uint32_t layer_id, uint64_t x_off, uint32_t M, uint64_t topk_off);

/* do_route (src/inference.rs:622-659): moe_route into the workspace, wait, and return
 * RoutingOutput rows on the host: routed[M][k] expert ids and weights[M][k]
 * (src/router.rs:4-8).  `shared_gate` (M floats) may be NULL. */
int moe_do_route(moe_ctx* ctx, uint32_t layer_id, uint64_t x_off, uint32_t M,
                 uint16_t* routed, float* weights, float* shared_gate);

/* ---- bucketing (src/router.rs:55-97 build_expert_batches) -------------------------------- */

/* Bucket M routing records (format of moe_route) by expert.  Outputs (arena offsets):
 *   ranges   i32 [E+2]  bucket e = [ranges[e], ranges[e+1]); bucket E is the shared expert
 *   tokens   i32 [S]    token index per slot, ascending inside each bucket (stable)
 *   weights  f32 [S]    routing weight per slot (shared: the gate)
 *   slot_pos i32 [M][k+1] sorted position of each token's slot (slot k = shared)
 * with S = M*(k + has_shared). */
int moe_bucket(moe_ctx* ctx, uint32_t n_experts, uint32_t top_k, int has_shared,
               uint64_t topk_off, uint32_t M, uint64_t ranges_off, uint64_t tokens_off,
               uint64_t weights_off, uint64_t slot_pos_off);

/* Allocation-free variant of moe_bucket, with no counterpart in the reference: for callers that
 * cannot allocate device memory (an engine that sized one arena up front, or code where
 * cudaMalloc is not allowed), since moe_bucket's context grows its workspace with cudaMalloc.
 * Same inputs and outputs as moe_bucket, given as device pointers on the current device, and
 * launched on `stream` (a cudaStream_t, NULL = legacy default stream).  Its scratch is a fixed
 * file-scope device array of about 190 KB that every GPU loading the library keeps until exit;
 * M is limited to 8192 tokens (larger M returns MOE_E_UNSUPPORTED), E to 256, top_k to 8.
 * The first call in a CUDA context looks up the array's device address in that context; make
 * that first call before any stream capture.  All calls on a device share the array: calls that
 * may run concurrently on the GPU race and must be ordered by the caller.  Asynchronous;
 * argument failures are reported only by the return code.  Nothing is checked on the device:
 * a routed expert id outside [0, E) (other than MOE_NO_EXPERT) is dropped -- its slot gets
 * slot_pos -1 and no bucket position -- and no error is reported. */
int moe_bucket_static(uint32_t n_experts, uint32_t top_k, int has_shared, const void* topk,
                      uint32_t M, int32_t* ranges, int32_t* tokens, float* weights,
                      int32_t* slot_pos, void* stream);

/* ---- the MoE layer (record_and_submit_moe, src/inference.rs:663-766) --------------------- */

/* out = resid + scale * (sum_j w_j * E_j(x) + gate * S(x)), E_j(x) = W2 (silu(W1 x) * W3 x),
 * for M tokens: router, top-k, bucketing, grouped experts and combine, all on the device.
 * resid_off may equal x_off; out_off may equal resid_off (in-place residual update). */
int moe_forward(moe_ctx* ctx, uint32_t layer_id, uint64_t x_off, uint64_t resid_off,
                uint64_t out_off, uint32_t M);

/* moe_forward from and to host memory, asynchronously: x_host[M][H] f32 goes to the device on a
 * copy stream, the layer runs on the context's stream, out_host[M][H] comes back on a second
 * copy stream; out = (add_residual ? x : 0) + MoE(x).  The call returns before any of it has
 * run, so a caller serving successive batches overlaps one batch's copies with another's layer:
 * the library keeps three device staging slots and orders every copy and launch with events
 * (a slot is reused only after its previous layer call and result copy are done).  x_host must
 * stay unchanged and out_host unread until moe_sync returns; pinned host memory (cudaHostAlloc /
 * cudaHostRegister) is needed for the copies to overlap anything.  Not capturable in a CUDA
 * graph (it launches the layer's own graph).  Replaces the reference's upload / submit / fence /
 * read-back sequence around record_and_submit_moe (src/inference.rs:663-766 with the staging
 * copies of src/memory.rs:297). */
int moe_forward_host(moe_ctx* ctx, uint32_t layer_id, const float* x_host, float* out_host, uint32_t M,
                     int add_residual);

/* Declare that layer next_id runs after layer_id (-1: none).  The single-token kernel of
 * layer_id then prefetches next_id's router weight and shared expert into L2 while it finishes,
 * so a layer stack decodes with those reads served from L2 (no counterpart in the reference,
 * whose layers run as separate submissions).  Set it before capturing a CUDA graph. */
int moe_layer_set_next(moe_ctx* ctx, uint32_t layer_id, int32_t next_id);

/* The layer with its pre-norm and residual, as one step of the reference's layer loop
 * (src/inference.rs:474-482, 588-596 with attention replaced by identity):
 *   out = x + scale * MoE(RMSNorm(x)),  RMSNorm(x) = x / sqrt(mean(x^2) + eps) (no gain).
 * For one token the normalisation runs inside the fused decode kernel (one launch); otherwise
 * an RMSNorm launch precedes the layer.  out_off must differ from x_off. */
int moe_forward_norm(moe_ctx* ctx, uint32_t layer_id, uint64_t x_off, uint64_t out_off, uint32_t M,
                     float eps);

/* record_and_submit_moe with host routing (RoutingOutput rows as returned by moe_do_route):
 * experts and combine only; routed[M][k] ids, weights[M][k], shared_gate[M] (NULL: 1.0). */
int moe_forward_routed(moe_ctx* ctx, uint32_t layer_id, uint64_t x_off, uint64_t resid_off,
                       uint64_t out_off, uint32_t M, const uint16_t* routed,
                       const float* weights, const float* shared_gate);

/* Experts and combine from device routing records (format of moe_route, M records of k+1
 * entries at topk_off; routed entries equal to MOE_NO_EXPERT are skipped).  The expert-parallel
 * building block: a rank runs its own experts on the rows dispatched to it (MOE_FT_UNSCALED,
 * resid 0 -> one partial row per received row).  An entry 0 with id MOE_NO_EXPERT drops that
 * row's shared expert. */
#define MOE_FT_NO_SHARED 1u   /* leave out the shared expert */
#define MOE_FT_SHARED_ONLY 2u /* only the shared expert (routed entries ignored) */
#define MOE_FT_UNSCALED 4u    /* combine scale 1 instead of the layer's scale */
int moe_forward_topk(moe_ctx* ctx, uint32_t layer_id, uint64_t x_off, uint64_t resid_off,
                     uint64_t out_off, uint32_t M, uint64_t topk_off, uint32_t flags);

/* ---- expert-parallel prefill (no counterpart in the single-device reference) -------------
 * Rank r of n_ranks (1..8) owns experts [r*E/n, (r+1)*E/n).  Every rank sends each peer a block
 * of `capacity` rows (capacity >= the largest per-rank token count), so the all-to-alls have
 * fixed, equal splits and need no host synchronisation.  Per layer and batch:
 *   moe_route -> moe_ep_dispatch -> all-to-all of the send rows and records (NCCL, by the
 *   caller) -> moe_forward_topk(received n_ranks*capacity rows, MOE_FT_UNSCALED, resid 0) ->
 *   all-to-all of the partial rows back -> moe_ep_combine.
 * A token's shared expert runs on its own rank (its record to itself keeps entry 0). */

/* Bytes of the dispatch plan of M tokens over n_ranks ranks (arena offset 256-aligned). */
uint64_t moe_ep_plan_bytes(uint32_t M, uint32_t n_ranks);

/* Builds the plan and the send buffers (n_ranks blocks of `capacity` rows: f32 rows of x and
 * (top_k+1)-entry records) from M routing records and rows x (f32 [M][H]).  Block d holds, in
 * token order, the tokens routed to at least one of rank d's experts (and every token in block
 * my_rank), each record keeping only rank d's experts; unused rows carry empty records.
 * Asynchronous on the context's stream. */
int moe_ep_dispatch(moe_ctx* ctx, uint32_t n_experts, uint32_t top_k, uint32_t n_ranks, uint32_t my_rank,
                    uint32_t capacity, uint64_t topk_off, uint64_t x_off, uint32_t M, uint32_t H,
                    uint64_t plan_off, uint64_t send_x_off, uint64_t send_topk_off);

/* out[t] = resid[t] + scale * (sum over the ranks t was sent to, ascending, of its returned
 * partial row).  y_back holds the returned blocks in send layout (n_ranks*capacity rows);
 * resid_off may be 0. */
int moe_ep_combine(moe_ctx* ctx, uint32_t n_ranks, uint32_t capacity, uint32_t H, uint32_t M,
                   uint64_t plan_off, uint64_t y_back_off, uint64_t resid_off, uint64_t out_off, float scale);

/* ---- expert parallelism over NCCL, no Python (one process per GPU) ---------------------- *
 * The C-level form of the expert-parallel layer: rank r of N holds routed experts
 * [r*E/N, (r+1)*E/N) (a layer created with MOE_F_EXPERT_SUBSET, or a full layer), the router and
 * the shared expert, and its own M_r tokens.  NCCL is loaded at run time (libnccl.so.2; the copy
 * already in the process when there is one).  Not thread-safe, like the rest of the context. */

/* Write a new NCCL unique id (128 bytes) to out[0..n); rank 0 makes it and the caller passes it
 * to every rank out of band. */
int moe_ep_unique_id(void* out, size_t n);
/* Join the n_ranks-rank group (blocks until every rank has called it; 1 <= n_ranks <= 8).
 * Replaces an earlier group of this context. */
int moe_ep_init(moe_ctx* ctx, const void* unique_id, uint32_t n_ranks, uint32_t rank);
/* out = resid + scale * MoE(x) for this rank's M tokens (M may be 0) through the group: route,
 * per-rank blocks of `capacity` rows, NCCL all-to-all, this rank's experts, all-to-all back,
 * combine.  Every rank must call it with the same layer shape and the same capacity
 * (>= the largest M of any rank).  A rank whose own token arguments are invalid (offsets, or
 * M > capacity) still completes the exchange as a rank without tokens, serving its experts to
 * the others, and then returns MOE_E_INVALID; a rank that cannot grow its workspace returns NaN
 * partial rows to the others and MOE_E_OOM, so one rank's bad call never leaves the others
 * waiting.  The exchange buffers keep the largest capacity asked for;
 * buffers replaced by a larger request stay allocated until the context is destroyed, so a
 * graph captured earlier stays valid.  Stream-ordered on the context's stream; capturable in a
 * CUDA graph after one eager call (which sizes the buffers). */
int moe_forward_ep(moe_ctx* ctx, uint32_t layer_id, uint64_t x_off, uint64_t resid_off, uint64_t out_off,
                   uint32_t M, uint32_t capacity);

/* Abort the group's NCCL communicator (ncclCommAbort), from any thread: a host watchdog that
 * finds a peer rank dead or stuck calls it so that this rank's blocked NCCL work ends with an
 * error instead of waiting forever (NCCL's GPU-side waits have no time limit; the peer
 * transport's waits give up after 1 s on their own).  Afterwards moe_forward_ep fails with
 * MOE_E_CUDA until moe_ep_init forms a new group.  Like the reference's Vulkan fence wait
 * (src/inference.rs:169-182) there is no counterpart for a lost peer in the reference. */
int moe_ep_abort(moe_ctx* ctx);

/* How the rank blocks travel (set identically on every rank, before moe_forward_ep):
 *   MOE_EP_TRANSPORT_PEER (default): the dispatch kernel stores rows and records straight into
 *     the owner ranks' receive buffers and the combine kernel reads the partial rows from the
 *     expert ranks' output buffers, over NVLink through CUDA IPC mappings of the context's
 *     exchange buffers, with per-step flags (bounded waits) in place of collectives; falls back
 *     to NCCL on every rank when any rank cannot map its peers;
 *   MOE_EP_TRANSPORT_NCCL: grouped ncclSend/ncclRecv all-to-alls of whole capacity blocks. */
#define MOE_EP_TRANSPORT_NCCL 0
#define MOE_EP_TRANSPORT_PEER 1
int moe_ep_set_transport(moe_ctx* ctx, int transport);
/* The transport of the current exchange buffers (-1 before the first moe_forward_ep). */
int moe_ep_transport(moe_ctx* ctx, int* transport);

/* Expert-product kernels used by moe_forward / moe_forward_routed (a tuning and diagnostic
 * knob; the default picks by batch size: CUDA-core grouped GEMV for M <= 8, tcgen05 grouped
 * GEMM otherwise). */
#define MOE_PATH_AUTO 0
#define MOE_PATH_GEMV 1        /* CUDA cores, exact f32 dequantisation and accumulation */
#define MOE_PATH_TC_SMEM_A 2   /* tcgen05, fp16 operands, dequantised weights in shared memory */
#define MOE_PATH_TC_TMEM_A 3   /* tcgen05, fp16 operands, dequantised weights in tensor memory */
int moe_set_path(moe_ctx* ctx, int path);

/* ---- stack glue (rms_norm.comp + residual_add.comp, src/inference.rs:474-482, :588-596) -- */

/* y = x / sqrt(mean(x^2) + eps), per token, no gain (shaders/rms_norm.comp:36-58). */
int moe_rms_norm(moe_ctx* ctx, uint64_t x_off, uint64_t y_off, uint32_t M, uint32_t H, float eps);

/* ---- tracing ----------------------------------------------------------------------------- */

/* Per-stage device time of the MoE calls, from CUDA events recorded on the context's stream
 * around every kernel stage (the reference has no timing; its only trace is MOE_DEBUG logging,
 * src/main.rs:21-28).  While enabled, each moe_forward / moe_forward_routed waits for its own
 * completion to read its events, so enable it only for measurement runs. */
typedef struct moe_stage_stat {
    char name[24];       /* "router", "topk", "bucket", "gemv13", "gemv2", "combine", ... */
    uint32_t calls;      /* launches of this stage since the last reset */
    float total_ms;      /* summed device time */
} moe_stage_stat;

/* Enable (1) or disable (0) stage timing; either resets the accumulated statistics. */
int moe_profile(moe_ctx* ctx, int enable);
/* Copy up to `max` stage statistics; *n receives the number of stages. */
int moe_profile_read(moe_ctx* ctx, moe_stage_stat* out, int max, int* n);
/* Number of kernels this context has launched since creation. */
int moe_launch_count(moe_ctx* ctx, uint64_t* n);

/* ---- vocabulary projection (LM head) -------------------------------------------------- */

/* logits[m][n] = sum_h x[m][h] * W[n][h] for m < M, n < V: the LM head / MTP output-head
 * projection of src/inference.rs:319-330 and :355-360 (shaders/attn_output.comp with
 * M = 1, N = vocab), which the reference follows with a greedy argmax on the host
 * (sampling::sample -> util::argmax, src/util.rs:66-76).
 *   w_off      IQ4_XS matrix [V][H] in GGUF row layout (V rows of H/256 blocks), 16-byte aligned
 *   x_off      f32 [M][H] activations (the final hidden state)
 *   logits_off f32 [M][V] output, or 0 to skip writing logits
 *   ids_off    u32 [M] output: per row the lowest index of the largest logit (NaN and -inf
 *              never win; 0 when no logit exceeds -inf), or 0 to skip the argmax
 * 1 <= M <= 8, 512 <= H <= 4096 with H % 512 == 0 (else MOE_E_UNSUPPORTED).  Activations are
 * rounded to 16-bit fixed point per row (relative step 2^-15 of the row's largest magnitude);
 * a row with a non-finite value gives NaN logits.  Stream-ordered on the context's stream;
 * capturable in a CUDA graph after one eager call on the device. */
int moe_vocab_logits(moe_ctx* ctx, uint64_t w_off, uint32_t V, uint32_t H, uint64_t x_off, uint32_t M,
                     uint64_t logits_off, uint64_t ids_off);

/* y[i] = silu(g[i]) * u[i] for i < n (u_off 0: y = silu(g)), silu(v) = v / (1 + e^-v), f32, in place
 * allowed (y_off == g_off): shaders/silu_mult.comp with gate and up at their own offsets; the
 * MTP head (src/inference.rs:335-360) is moe_vocab_logits(w1, V = H) -> moe_silu_mul ->
 * moe_vocab_logits(w2, V = vocab). */
int moe_silu_mul(moe_ctx* ctx, uint64_t g_off, uint64_t u_off, uint64_t y_off, uint64_t n);

/* ---- weight utilities ------------------------------------------------------------------ */

/* Decode n_blocks IQ4_XS blocks at src_off into f32 [n_blocks*256] at dst_off (exact; the
 * dequant_iq4_xs primitive of shaders/common.glsl:59-86 for the GGUF block format). */
int moe_dequant_iq4xs(moe_ctx* ctx, uint64_t src_off, uint64_t n_blocks, uint64_t dst_off);

/* Decode n_blocks of the reference's own 36-byte weight blocks (shaders/common.glsl:59-86:
 * 32 weights, f16 scales for weights 0-15 and 16-31, 5-bit codes, w = (q - 8) * d, subnormal
 * scales flushed to zero) into f32 at dst_off (128 bytes per block), bit-exact with the shipped
 * shaders' decode.  For checking or converting weights stored in that format. */
int moe_dequant_ref36(moe_ctx* ctx, uint64_t src_off, uint64_t n_blocks, uint64_t dst_off);

/* Fill n_blocks synthetic IQ4_XS blocks at dst_off (seeded counter-based generator: block b
 * is 17 little-endian words splitmix64(key + 17*(block_start+b) + i), then its f16 d is
 * replaced by f16(0.005 + 0.015*u), u = (word0 >> 40) * 2^-24).  Benchmark/test input only. */
int moe_synth_iq4xs(moe_ctx* ctx, uint64_t dst_off, uint64_t key, uint64_t block_start,
                    uint64_t n_blocks);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
