/*
 * sosob200.h -- C ABI of the B200 (sm_100a) quantized decode hot path.
 *
 * Drop-in boundary for demonodojo/soso's `trait GpuDispatch`
 * (crates/soso-llm-core/src/gpu.rs:338-737): a Rust `impl GpuDispatch` binds
 * these symbols with `extern "C"`.  Plain pointers and sizes only.
 *
 * Two layers:
 *   sb_*   -- the GpuDispatch surface.  Host buffers, weights resident per key
 *             (uploaded on first sight, like CudaGpu's `pesos` map,
 *             crates/soso-llm-api/src/cuda.rs:290, :2364-2376).  Return value:
 *             1 = handled (outputs fully written), 0 = declined (the caller
 *             computes on its own path), <0 = error (sb_last_error()).
 *   sbk_*  -- the kernels themselves on DEVICE pointers, enqueued on a
 *             caller-provided cudaStream_t (passed as void*); no host sync.
 *             Return value: 0 = enqueued, <0 = rejected (bad shape / dtype /
 *             alignment; nothing was launched).
 *
 * Weight layouts are the reference's on-disk bytes, unchanged:
 *   Q8_0 (.som)  36 B / 32 weights: f32 scale + 32 i8   (crates/sosomodel/src/layout.rs:57-59)
 *   Q4_K (GGML) 144 B / 256: f16 d, f16 dmin, 12 B 6-bit scales/mins, 128 B nibbles (layout.rs:63-64)
 *   Q6_K (GGML) 210 B / 256: ql[128] qh[64] i8 sc[16] f16 d  (crates/gguf2som/src/lib.rs:1639-1661)
 * Matrices are row-major [rows = out][cols = in]; each row is a whole number
 * of blocks (crates/sosomodel/src/dequant.rs:47-63).
 */
#ifndef SOSOB200_H
#define SOSOB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* sosomodel dtype codes (crates/sosomodel/src/layout.rs:8-12).  SB_DTYPE_Q6_K
 * is an extension: the reference stores no Q6_K tensors (gguf2som converts
 * them to Q8_0, crates/gguf2som/src/lib.rs:1592-1610). */
#define SB_DTYPE_F32  1
#define SB_DTYPE_Q8_0 2
#define SB_DTYPE_Q4_K 3
#define SB_DTYPE_Q6_K 13
/* Q6_K repacked for the device (no counterpart in the reference): the same
 * 210-byte blocks, regrouped per row into groups of 8 blocks laid out as
 * planes [ql 8x128][qh 8x64][scales 8x16][d 8x2] (a last partial group of m
 * blocks the same way with m, padded to 16 bytes), so rows and fields are
 * 16-byte aligned for TMA.  Made by sbk_q6k_pack; the host-buffer calls (sb_*)
 * repack Q6_K weights this way when they upload them. */
#define SB_DTYPE_Q6_K_P 14
/* Q8_0 with every row padded to a multiple of 16 bytes (zeros after the last block) so
 * rows start 16-byte aligned for TMA; the same 36-byte blocks.  Rows of a multiple of 128
 * weights need no padding (SB_DTYPE_Q8_0 rows are read as they are).  Made by sbk_q80_pad;
 * the host-buffer calls (sb_*) hold Q8_0 weights this way.  No counterpart in the reference. */
#define SB_DTYPE_Q8_0_R 15

/* Mirror of `TensorView { bytes, dtype, elems }` (crates/soso-llm-core/src/layer.rs:26-31). */
typedef struct {
    const uint8_t *bytes;
    size_t len;
    uint8_t dtype;
    size_t elems;
} sb_view;

/* Mirror of `MatvecOp` (crates/soso-llm-core/src/gpu.rs:189-196). */
typedef struct {
    const char *key;
    const sb_view *view;
    size_t rows, cols;
    const float *x;
    float *out;
} sb_matvec_op;

/* Mirror of `GpuStats` (crates/soso-llm-core/src/gpu.rs:17-36) without the cost model's
 * per-stretch averages (ewma_ns / samples, sched.rs): launches, time and bytes of the host
 * calls; the per-step transfers of the device-resident decode (embedding row up, position
 * and control words up, logits down, new KV rows down, steps), as CudaGpu counts them
 * (crates/soso-llm-api/src/cuda/decode.rs:790-937); expert-pool hits and misses (always 0:
 * every expert is resident, nothing is streamed). */
typedef struct {
    uint64_t launches;
    uint64_t total_ns;
    uint64_t bytes_up;
    uint64_t bytes_down;
    uint64_t decode_embed_up;
    uint64_t decode_control_up;
    uint64_t decode_logits_down;
    uint64_t decode_kv_down;
    uint64_t decode_steps;
    uint64_t stream_hits;
    uint64_t stream_misses;
} sb_stats;

typedef struct sb_ctx sb_ctx;

/* ---- GpuDispatch surface (host buffers) -------------------------------- */

/* `CudaGpu::nueva` (crates/soso-llm-api/src/cuda.rs:440): one context per device. */
int sb_create(int device, sb_ctx **out);
void sb_destroy(sb_ctx *ctx);
/* `GpuDispatch::available` (gpu.rs:339). */
int sb_available(const sb_ctx *ctx);
/* `GpuDispatch::dtype_soportado` (gpu.rs:343-345). */
int sb_dtype_supported(const sb_ctx *ctx, uint8_t dtype);
/* `GpuDispatch::matvec` (gpu.rs:432-440): out[0..rows] = W . x. */
int sb_matvec(sb_ctx *ctx, const char *key, const sb_view *w, size_t rows, size_t cols, const float *x,
              float *out);
/* `GpuDispatch::matmul` (gpu.rs:443-455): out[n x rows] = X[n x cols] . W^T. */
int sb_matmul(sb_ctx *ctx, const char *key, const sb_view *w, size_t rows, size_t cols, size_t n,
              const float *x, float *out);
/* `GpuDispatch::matvec_lote` (gpu.rs:694-701): independent matvecs, one wait; done[i] = 1 when ops[i] ran. */
int sb_matvec_batch(sb_ctx *ctx, sb_matvec_op *ops, size_t nops, uint8_t *done);
/* `GpuDispatch::rmsnorm` (gpu.rs:733-736): x *= rsqrt(mean(x^2) + eps) * w, in place. */
int sb_rmsnorm(sb_ctx *ctx, float *x, const float *w, size_t n, float eps);
/* `GpuDispatch::gemma_subir` (gpu.rs:364-368): make a tensor resident under its key (quantized
 * matrices in their matvec form, F32 as they are) for the block calls below.  1 = resident,
 * 0 = declined (dtype, shape; remembered), <0 = error. */
int sb_upload(sb_ctx *ctx, const char *key, const sb_view *w, size_t rows, size_t cols);
/* `GpuDispatch::router_topk` (gpu.rs:477-494): for each of n tokens xs[t] (h floats), router
 * logits against the f32 matrix w [n_exp x h] (resident under key), softmax, stable top-k
 * and renormalisation (topk_softmax, gemm.rs:62-91); idx / wts [n x top_k] in rank order.
 * 1 = done, 0 = declined, <0 = error. */
int sb_router_topk(sb_ctx *ctx, const char *key, const float *w, const float *xs, size_t n, size_t h, size_t n_exp,
                   size_t top_k, int32_t *idx, float *wts);
/* Mirror of `ExpertoBloque` (gpu.rs:175-187): one expert of a block, its three matrices
 * (keys of ffn_gate, ffn_up, ffn_down; a view may be NULL or of dtype 0 when the caller
 * expects the tensor resident already), the tokens (indices within the block) that chose
 * it, whether it is a shared expert, and for each of those tokens its weight's index
 * token * top_k + rank in `weights`. */
typedef struct {
    const char *keys[3];
    const sb_view *views[3];
    const uint32_t *tokens;
    size_t n_tokens;
    int shared;
    const uint32_t *dests;
} sb_expert_block;
/* `GpuDispatch::expertos_bloque` (gpu.rs:457-475): the experts of a block of n tokens
 * (xs [n x h]): per expert, for its tokens, down(silu(gate . x) * (up . x)) with gate / up
 * [ffn x h] and down [h x ffn]; sum [n x h] receives per token the weighted sum, in rank
 * order, of the experts resolved here (done[i] = 1), the others are the caller's.  The
 * experts' tokens are grouped on the device: one tensor-core GEMM launch for every gate and
 * up, one for the downs (f16 operands, f32 sums; Q4_K / Q8_0 matrices, h and ffn multiples
 * of 64, at least 256).  1 = ran, 0 = declined (nothing done), <0 = error. */
int sb_experts(sb_ctx *ctx, const float *xs, size_t n, size_t h, size_t ffn, size_t top_k, const float *weights,
               sb_expert_block *exps, size_t n_exps, float *sum, uint8_t *done);
/* `GpuDispatch::atencion_prefill` (gpu.rs:496-517): causal attention of a block of n tokens
 * at positions seq_before .. seq_before + n - 1 on the device, over the layer's f16 KV rows
 * mirrored from the host: k / v [seq_before + n][kv_heads * hd] with the block's rows
 * already appended; *valid_rows = leading rows the device mirror already holds, counted up
 * to seq_before (the rest go up; set to seq_before + n).  q / out [n][heads * hd] (q roped).
 * Softmax of q.k / sqrt(hd) in f32 per query row (attn.rs:73-140), q.k exact to f32
 * rounding, the softmax weights multiplied with V in f16.  1 = done, 0 = declined (hd not a
 * multiple of 8 or above 256, heads / kv_heads above 64), <0 = error. */
int sb_attention_prefill(sb_ctx *ctx, uint32_t layer, const float *q, float *out, size_t n, size_t seq_before,
                         size_t heads, size_t kv_heads, size_t hd, const uint16_t *k, const uint16_t *v,
                         size_t *valid_rows);
/* Number of resident weight tensors (`CudaGpu::residentes`, used by cuda_matvec.rs:138). */
/* Mirror of `MoeCapa` (gpu.rs:294-335) and its `MoeNormas` (:279-289): one MoE layer of a
 * block of n tokens at positions pos0.. on the device (Qwen3-MoE-style: GQA with optional
 * QK-norm, NeoX RoPE, softmax top-k router in f32, SwiGLU experts).  hidden [n][h] in and
 * out (host); the attention matrices resident under key_q/k/v/o and the experts under
 * `{prefix}.E{nn}.ffn_{gate,up,down}` (nn at least two digits), made resident by sb_upload
 * (gemma_subir).  attn_norm / ffn_norm [h], q_norm / k_norm [head_dim] (qk_norm), router
 * [n_exp x h] f32, rope_factors [head_dim / 2] or NULL: needed at a layer's first call, may
 * be NULL after (sb_moe_ready).  cont: the input rows are the previous layer's output still
 * on the device (sb_moe_pending), hidden is not read; chain: leave the output on the device
 * for the next layer (hidden is not written; sb_moe_flush brings it down).  streamed != 0
 * means the caller could supply experts on demand (ModoMoe::Flujo); this backend only runs
 * layers whose experts are all resident.  evicted: KV rows dropped ahead of the layer's cache
 * (0: sliding-window layers are declined). */
typedef struct {
    uint32_t layer;
    size_t pos0, n;
    float *hidden;
    size_t h, heads, kv_heads, head_dim, ffn, n_exp, top_k, window, ctx_max;
    float eps, theta, scale;
    int qk_norm;
    float rope_mscale;
    int cont, chain;
    const char *key_q, *key_k, *key_v, *key_o, *prefix;
    const float *attn_norm, *q_norm, *k_norm, *ffn_norm, *router, *rope_factors;
    int streamed;
    size_t evicted;
} sb_moe_layer_args;
/* `GpuDispatch::moe_capa` (gpu.rs:424-429; CudaGpu's moe_ejecutar,
 * crates/soso-llm-api/src/cuda/capa/moe.rs:316): the layer on the block path (tcgen05 GEMMs,
 * the tensor-core prefill attention, experts grouped on the device), its f16 KV cache of
 * ctx_max rows held on the device across calls (rows [0, pos0) must be there; a smaller pos0
 * rewinds).  1 = done, 0 = declined (remembered: sb_moe_can turns 0), <0 = error. */
int sb_moe_layer(sb_ctx *ctx, sb_moe_layer_args *args);
/* `moe_lista` (gpu.rs:385-389): the layer's norms, router and expert tables are held. */
int sb_moe_ready(sb_ctx *ctx, uint32_t layer);
/* `moe_puede` (gpu.rs:379-383): 0 once the layer was declined or discarded. */
int sb_moe_can(sb_ctx *ctx, uint32_t layer);
/* `moe_pendiente` (gpu.rs:391-395): the device holds, not yet brought down, the output of
 * that layer for n tokens from pos0. */
int sb_moe_pending(sb_ctx *ctx, uint32_t layer, size_t pos0, size_t n);
/* `moe_volcar` (gpu.rs:397-401): the pending output down into hidden (len floats, at least
 * the pending rows), then no longer pending; nothing to do without one. */
int sb_moe_flush(sb_ctx *ctx, float *hidden, size_t len);
/* `moe_descartar` (gpu.rs:370-373): drop the layer's device state; not tried again. */
int sb_moe_discard(sb_ctx *ctx, uint32_t layer);

size_t sb_resident_count(const sb_ctx *ctx);
/* `GpuDispatch::stats` (gpu.rs:350-352). */
int sb_get_stats(const sb_ctx *ctx, sb_stats *out);
/* Thread-local description of the last error. */
const char *sb_last_error(void);

/* ---- whole-token decode (device-resident model, one CUDA graph per token) -- */

/* Mirror of `MatDec` (gpu.rs:92-98): one matrix of the model, rows = out, cols = in. */
typedef struct {
    const char *key;
    sb_view view;
    size_t rows, cols;
} sb_mat;

/* Mirror of `MoeDec` (gpu.rs:130-137): router [n_exp x hidden], experts[3*e + {0,1,2}] =
 * gate, up, down of expert e; optional shared expert (3 matrices) with an optional
 * sigmoid gate row [hidden] (layer.rs:1883-1907). */
typedef struct {
    size_t n_exp, top_k, ffn;
    sb_mat router;
    const sb_mat *experts;
    const sb_mat *shared;
    const float *shared_gate;
} sb_moe_plan;

/* Multi-head latent attention of one layer (arch.rs:51-202, attn.rs:306-404): q_down
 * [q_rank x hidden], q_up [heads*(qk_nope+qk_rope) x q_rank], kv_down [kv_rank x hidden],
 * k_up [kv_heads*(qk_nope+qk_rope) x kv_rank], v_up [kv_heads*v_dim x kv_rank]; q rows per
 * head are nope then rope.  The layer's KV cache is the reference's latent cache
 * ([ctx][kv_rank] f16, kv.rs:293-315) plus the rope keys [ctx][kv_heads][qk_rope] f32. */
typedef struct {
    size_t q_rank, kv_rank, qk_nope, qk_rope, v_dim;
    sb_mat q_down, q_up, kv_down, k_up, v_up;
} sb_mla_plan;

/* One layer: `CapaDec` (gpu.rs:138-148) with GQA attention (`GatedDec`, gpu.rs:113-122;
 * bias and QK-norm as layer.rs:1146-1181, RoPE as layer.rs:1184-1193) and a dense SwiGLU
 * FFN (layer.rs:1352-1389) or, when moe != NULL, a MoE FFN. */
typedef struct {
    size_t heads, kv_heads, head_dim;
    float theta;
    int neox;
    const float *q_norm, *k_norm; /* [head_dim] each, or NULL */
    const float *qkv_bias;        /* [heads*hd + 2*kv_heads*hd] stacked q|k|v, or NULL */
    const float *norm_attn, *norm_ffn;
    sb_mat q, k, v, o;
    sb_mat gate, up, down;
    const sb_moe_plan *moe;
    const sb_mla_plan *mla; /* when set: MLA attention (q, k, v unused; o = attn_output) */
    /* YaRN RoPE of this layer (layer.rs:1184-1193 takes it on full-attention layers), as
     * the reference's GPU rope takes it (gm_rope, gemma_capa.cu:99-125): head_dim/2
     * divisors of the pair frequencies (yarn_factores, gemm.rs:1413-1428) and the mscale
     * that multiplies cos and sin (> 0); NULL = plain RoPE.  GQA layers only. */
    const float *rope_factors;
    float rope_mscale;
} sb_layer_plan;

/* `DecodePlan` (gpu.rs:150-158) plus the embedding table (for device-side greedy
 * decoding; view.bytes may be NULL) and the KV context length to allocate. */
typedef struct {
    const sb_layer_plan *layers;
    size_t n_layers;
    size_t hidden, vocab, ctx;
    float eps;
    const float *final_norm;
    sb_mat lm_head;
    sb_mat embed;
} sb_decode_plan;

/* `GpuDispatch::decode_preparar` (gpu.rs:654-657): weights resident, KV caches
 * (f16, [ctx][kv_heads*head_dim] per layer, kv.rs:21-56) and buffers allocated, the
 * per-token CUDA graphs captured.  1 = ready, 0 = the plan has something this
 * backend does not run, <0 = error.  Resets the KV caches. */
int sb_decode_prepare(sb_ctx *ctx, const sb_decode_plan *plan);
/* `GpuDispatch::decode_token` (gpu.rs:675-684): one token from its embedding row
 * (host f32[hidden]) at position pos; logits (host f32[vocab]) out, and when
 * kv_rows != NULL the new f16 K and V rows of every layer, in layer order
 * ([k | v] per layer).  1 = done, 0 = not prepared, <0 = error. */
int sb_decode_token(sb_ctx *ctx, const float *embed, size_t pos, float *logits, uint16_t *kv_rows);
/* n greedy steps entirely on the device (graph per token, no host round trip):
 * positions pos .. pos+n-1; the token fed at step i is prompt[i] while i < n_prompt,
 * else the argmax of the previous step (runtime.rs:2021-2028).  tokens_out[i] = the
 * argmax produced at step i.  Needs plan.embed.  1 = done, 0 = not prepared, <0 = error. */
int sb_decode_greedy(sb_ctx *ctx, const int32_t *prompt, size_t n_prompt, size_t pos, size_t n, int32_t *tokens_out);

/* Mirror of `EstadoCapaDec` (gpu.rs:166-173) for the layers this backend runs (it has no
 * Gated DeltaNet state): the host's copy of one layer's cache, rows from position 0 --
 * K and V, f16 [rows][kv_heads*head_dim], of an attention layer (LayerKv, kv.rs:21-56), or
 * the latent rows, f16 [rows][kv_rank], of an MLA layer in k with v NULL (kv.rs:293-315)
 * -- and how many leading rows the device already holds. */
typedef struct {
    const uint16_t *k;
    const uint16_t *v;
    size_t *valid_rows;
} sb_layer_state;
/* `GpuDispatch::decode_subir_estado` (gpu.rs:664-668; CudaGpu's decode_subir_estado_impl,
 * crates/soso-llm-api/src/cuda/decode.rs:629-660): for every layer the rows
 * [min(*valid_rows, pos), pos) go up and *valid_rows becomes pos, so the next step can run
 * at position pos.  An MLA layer's rope keys are formed again from its latent rows, exactly
 * as the decode step forms them.  n_layers must be the plan's.  1 = done, 0 = not prepared
 * (or a tensor-parallel engine), <0 = error. */
int sb_decode_upload_state(sb_ctx *ctx, const sb_layer_state *layers, size_t n_layers, size_t pos);
/* Rows [0, rows) of every layer's cache, in the sb_layer_state layout, down into k / v (v
 * NULL for an MLA layer), and when hidden != NULL the hidden vector the last step left
 * (f32[hidden], before the output norm: the Runtime::hidden that Runtime::exportar_kv stores
 * with the rows, crates/soso-llm-core/src/runtime.rs:544-556).  The reference's
 * decode_bajar_estado (gpu.rs:686-690) brings back only Gated DeltaNet state, because its
 * host mirrors the KV rows through decode_token; steps run by sb_decode_greedy have no host
 * mirror, so the rows come down here.  1 = done, 0 = not prepared (or tensor-parallel),
 * <0 = error. */
typedef struct {
    uint16_t *k;
    uint16_t *v;
} sb_layer_rows;
int sb_decode_download_state(sb_ctx *ctx, const sb_layer_rows *layers, size_t n_layers, size_t rows, float *hidden);
/* The experts every MoE layer chose at the last decode step, in layer order, top_k IDs each
 * in rank order (the order topk_softmax ranks them, crates/soso-llm-core/src/gemm.rs:77-91):
 * a trace for checking a step against a CPU run, where a near-tie of two router logits can
 * let the two sides pick different experts.  No counterpart in the reference.  idx holds
 * at least the sum of the MoE layers' top_k.  1 = written, 0 = no decode prepared, <0 = error. */
int sb_decode_routes(sb_ctx *ctx, int32_t *idx, size_t n);
/* The same for the decode step at position pos (any step run since sb_decode_prepare, by
 * sb_decode_token or sb_decode_greedy, prompt steps included; positions the block prefill ran
 * hold no trace), and, when gaps != NULL, per MoE layer the router-logit gap between its
 * k-th choice and the best expert it did not choose (gaps holds at least the number of MoE
 * layers): a small gap marks a near-tie that another summation order may break the other
 * way.  No counterpart in the reference.  1 = written, 0 = no decode step yet, <0 = error. */
int sb_decode_route_trace(sb_ctx *ctx, size_t pos, int32_t *idx, size_t n, float *gaps, size_t n_gaps);

/* Block prefill of a prompt on the prepared model: tokens[0..n) at positions pos0 .. pos0+n-1
 * through every layer at once -- the reference's prompt path over forward_layer_block
 * (crates/soso-llm-core/src/layer.rs:1433) with its GPU offload of the block's matrix
 * products, expert groups and attention (GpuDispatch::matmul / expertos_bloque /
 * router_topk / atencion_prefill, gpu.rs:443-530) -- then the logits of the last token
 * (runtime.rs:1976-2019).  Every matrix product is a tcgen05 GEMM over the n tokens with
 * f16 operands and f32 sums (the precision of the reference's f16 mma.sync prefill,
 * lxdde/ports/nouveau/matvec_iq.cu:731-816); a MoE layer groups the block's (token,
 * choice) pairs by expert on the device and runs one grouped GEMM over every routed
 * expert.  The KV caches of those positions are filled where the decode step puts them:
 * decoding goes on with sb_decode_greedy / sb_decode_token at pos0 + n.  logits
 * (host f32[vocab]) and next (the argmax, ties to the last index) may be NULL.  Needs
 * plan.embed.  1 = done, 0 = not prepared, a tensor-parallel engine, or a plan with a
 * layer the block path does not take (expert matrices other than Q4_K / Q8_0, other
 * matrices other than Q4_K / Q8_0 / Q6_K, widths not multiples of 64), <0 = error. */
int sb_decode_prefill(sb_ctx *ctx, const int32_t *tokens, size_t n, size_t pos0, float *logits, int32_t *next);

/* ---- tensor-parallel groups (no counterpart in the reference, whose multi-machine mode
 * is a TCP layer pipeline, crates/soso-llm-core/src/pipeline.rs) -------------------------
 * One process per GPU of one node.  Each rank creates its group exchange area, the ranks
 * swap the returned CUDA IPC handles over their own host channel (soso_b200 uses
 * torch.distributed), each opens the others', and then sb_decode_prepare shards the plan
 * it is given (the full model) across the group: attention heads and FFN rows of the
 * dense layers (column shards of attn_output / ffn_down, whose partial sums every rank
 * adds in rank order inside the next matvec's input preparation) and vocabulary rows of
 * the output matrix (the greedy token is the largest of the ranks' maxima).  With a group
 * of world > 1, sb_decode_prepare returns before its warm-up token: call
 * sb_decode_finish on every rank after a host barrier; only sb_decode_greedy runs. */
size_t sb_group_handle_bytes(void);
/* The consuming side of an exchange point on its own: wait, bounded by `limit` spins of about
 * 100 ns, until the n counters cnt[0..n) (device memory) reach target; *ok (device int) = 1,
 * or 0 when the limit ran out, which also leaves 0x91 in the device error word
 * (sbk_take_device_error) -- how a rank learns that a peer never published, without a trap
 * and with the context still usable.  limit <= 2^26 (the limit every exchange wait of the
 * decode kernels uses).  No counterpart in the reference. */
int sbk_exchange_wait(const unsigned *cnt, int n, unsigned target, unsigned limit, int *ok, void *stream);
int sb_group_create(sb_ctx *ctx, int rank, int world, void *handle_out);
int sb_group_open(sb_ctx *ctx, const void *handles /* world x sb_group_handle_bytes(), rank order */);
int sb_decode_finish(sb_ctx *ctx);

/* ---- kernels on device pointers --------------------------------------- */

/* Bytes per row for (dtype, cols), 0 if cols is not a whole number of blocks
 * (`sosomodel::dequant::row_bytes`, crates/sosomodel/src/dequant.rs:53-63). */
size_t sbk_row_bytes(uint8_t dtype, size_t cols);

/* The .som container of the reference's model directories (manifest.som, index.som,
 * shards/): host functions, no device.  sb_crc32c: CRC-32C (Castagnoli) of n bytes, the
 * checksum every .som header carries (sosomodel::crc32c, crates/sosomodel/src/lib.rs:32-34).
 * sb_som_payload: 1 and the payload / its length / the version when the header's magic,
 * length and CRC agree (parse_som, lib.rs:88-104; shard != 0: verify_shard,
 * index.rs:118-139, payload at byte 64 from shard version 2), else 0. */
uint32_t sb_crc32c(const void *data, size_t n);
int sb_som_payload(const void *file, size_t file_len, int shard, const void **payload, size_t *len,
                   uint32_t *version);

/* y[rows] = W[rows x cols] . x[cols] for dtype Q8_0 / Q4_K / Q6_K / Q6_K_P.  Replaces
 * `gm_matvec_q4k` / `gm_matvec_q80` (lxdde/ports/nouveau/gemma_capa.cu:433,:501)
 * and the CPU `gemm::matvec_q4_k` / `matvec_q8_0` (crates/soso-llm-core/src/gemm.rs:295,:402).
 * w must be 16-byte aligned.  pdl != 0 launches with programmatic dependent
 * launch so the weight stream overlaps the previous kernel on the stream. */
int sbk_matvec(uint8_t dtype, const void *w, size_t rows, size_t cols, const float *x, float *y, int pdl,
               void *stream);

/* One device-pointer matvec of a batch. */
typedef struct {
    const void *w;
    size_t rows, cols;
    const float *x;
    float *y;
} sbk_mv_op;

/* Repack rows x cols Q6_K weights (reference layout, device memory) into
 * SB_DTYPE_Q6_K_P at dst (sbk_row_bytes(SB_DTYPE_Q6_K_P, cols) * rows bytes,
 * 16-byte aligned).  No counterpart in the reference, which converts Q6_K to
 * Q8_0 on import instead (crates/gguf2som/src/lib.rs:1592-1610). */
int sbk_q6k_pack(const void *src, size_t rows, size_t cols, void *dst, void *stream);
/* Copy rows x cols Q8_0 weights (reference layout, device memory) to SB_DTYPE_Q8_0_R at dst
 * (sbk_row_bytes(SB_DTYPE_Q8_0_R, cols) * rows bytes, 16-byte aligned). */
int sbk_q80_pad(const void *src, size_t rows, size_t cols, void *dst, void *stream);

/* Independent matvecs of one dtype in as few launches as possible (Q4_K: one
 * launch per 40 matrices, their weight streams split across all SMs as one) --
 * the device-pointer form of `GpuDispatch::matvec_lote` (gpu.rs:694-701) and of
 * the reference's `Lote` batches (crates/soso-llm-core/src/layer.rs:571-641). */
int sbk_matvec_batch(uint8_t dtype, const sbk_mv_op *ops, size_t n, int pdl, void *stream);

/* How the input vector of a fused batch is formed as the kernel reads it, so the
 * step that produces it costs no launch of its own (a = every op's x, which must
 * be the same vector for the whole batch):
 *   SBK_XS_NORM    h = a (+ res when res != NULL) and x = rmsnorm(h) * norm_w
 *                  (gemm::rmsnorm, crates/soso-llm-core/src/gemm.rs:93-100, after the
 *                  residual add add_f32, gemm.rs:265); when h_out != NULL it receives h
 *                  (the new residual stream; must not alias a or res)
 *   SBK_XS_SWIGLU  x = silu(a) * res  (swiglu_inplace, gemm.rs:210-226; a = gate, res = up)
 * Replaces the reference's separate rmsnorm / residual-add / SwiGLU passes between
 * matvecs (layer.rs:1284-1389). */
enum { SBK_XS_PLAIN = 0, SBK_XS_NORM = 1, SBK_XS_SWIGLU = 2 };
typedef struct {
    const float *res;
    const float *norm_w;
    float *h_out;
    float eps;
    int mode;
    /* SBK_XS_NORM after a MoE FFN: with ny > 0 the residual is a weighted set of
     * vectors, h = (sum over i = 0..ny-1, in order, of yw[i] * ys[i*ystride ..]) + a
     * (the expert combine of layer.rs:1922-1933, then add_assign_f32 :1389); res unused.
     * ny <= 16; yw is read on the device (it may be written by an earlier kernel). */
    const float *ys;
    const float *yw;
    int ny, ystride;
} sbk_xsrc;
/* sbk_matvec_batch with the input formed as *xs says (dtype Q4_K or Q6_K_P; 16-byte
 * aligned vectors).  Returns -5 for a dtype without the fused input forms. */
int sbk_matvec_batch_x(uint8_t dtype, const sbk_mv_op *ops, size_t n, const sbk_xsrc *xs, int pdl, void *stream);

/* Batched prefill GEMM on the tcgen05 tensor cores: y[n x rows] = x[n x cols] . W^T for
 * Q4_K weights (device pointers, x and y f32, row-major).  W is dequantised to 16-bit
 * operands in shared memory tile by tile, x is rounded likewise (into ws), accumulation is
 * f32 in tensor memory.  Replaces the reference's block-prefill GEMM iq_matmul_mma
 * (lxdde/ports/nouveau/matvec_iq.cu:731-816, :966; f16 mma.sync) and the CPU
 * matvec_q4_k_batch (crates/soso-llm-core/src/gemm.rs:495-546) behind
 * GpuDispatch::matmul (crates/soso-llm-core/src/gpu.rs:443-455).  ws: at least
 * sbk_matmul_ws_bytes(n, cols) bytes, 16-byte aligned (X as 16-bit operands, then ~21 MB
 * for the partial sums when too few output tiles make the GEMM split K into slices).
 * -5: dtype not supported. */
size_t sbk_matmul_ws_bytes(size_t n, size_t cols);
/* prec: SBK_PREC_BF16 (weights and x as bf16, 8 significant bits) or SBK_PREC_F16 (as f16,
 * 11 bits: the precision of the reference's f16 mma.sync prefill). */
enum { SBK_PREC_BF16 = 0, SBK_PREC_F16 = 1 };
int sbk_matmul(uint8_t dtype, const void *w, size_t rows, size_t cols, size_t n, const float *x, float *y, void *ws,
               int prec, int pdl, void *stream);

/* RMSNorm of `rows` rows of n floats, `gemm::rmsnorm` (crates/soso-llm-core/src/gemm.rs:93-100),
 * optionally fused with the residual add `add_f32` (gemm.rs:265): with res != NULL,
 * h_out = x + res and y = rmsnorm(h_out) * w; else y = rmsnorm(x) * w.  y may alias x.
 * Replaces `gm_rmsnorm_rows` / `rmsnorm_rows_f32` (gemma_capa.cu:81-96, rmsnorm_rows.cu:13-38). */
int sbk_rmsnorm(const float *x, const float *res, float *h_out, const float *w, float *y, size_t rows, size_t n,
                float eps, void *stream);

/* ---- decode-step kernels (device pointers; `pos` / `token` read from device memory,
 * so a captured CUDA graph serves every step) ---------------------------------- */

/* On the stacked [q | k | v] vector of one token: optional bias (add_optional_bias,
 * crates/soso-llm-core/src/layer.rs:1146-1163), optional per-head QK-norm
 * (layer.rs:1164-1181), RoPE (rope_cabezas, gemm.rs:1452-1491; neox != 0 pairs
 * (i, i+d/2), else (2i, 2i+1)), then K/V appended as f16 rows at *pos of the
 * [ctx][kv_heads*head_dim] caches (LayerKv::append_f16, kv.rs:258-275, with the
 * reference's f32->f16 rounding, f16.rs:10-37).  q is roped in place.
 * Replaces gm_rope + gm_kv_append (lxdde/ports/nouveau/gemma_capa.cu:99-141). */
int sbk_rope_kv_append(float *qkv, const float *bias, const float *qnorm, const float *knorm, uint16_t *kcache,
                       uint16_t *vcache, const int32_t *pos, size_t heads, size_t kv_heads, size_t head_dim,
                       size_t ctx, float theta, float eps, int neox, int pdl, void *stream);
/* The same with gm_rope's frequency factors (lxdde/ports/nouveau/gemma_capa.cu:99-125),
 * how the reference runs YaRN on the GPU: factors[head_dim/2] (device, or NULL) divide
 * the pair frequencies -- the divisors of yarn_factores, crates/soso-llm-core/src/
 * gemm.rs:1413-1428 -- and mscale (> 0; 1 + 0.1 ln(factor) for YaRN) multiplies cos and
 * sin.  factors NULL and mscale 1 are sbk_rope_kv_append exactly. */
int sbk_rope_kv_append_yarn(float *qkv, const float *bias, const float *qnorm, const float *knorm, uint16_t *kcache,
                            uint16_t *vcache, const int32_t *pos, size_t heads, size_t kv_heads, size_t head_dim,
                            size_t ctx, float theta, float eps, int neox, const float *factors, float mscale,
                            int pdl, void *stream);

/* Workspace bytes for sbk_attn_decode (zero-filled before first use; left zeroed). */
size_t sbk_attn_ws_bytes(size_t heads, size_t kv_heads, size_t head_dim, size_t ctx);
/* GQA decode attention of one token over positions 0..*pos of the f16 caches:
 * softmax(q.k / sqrt(hd)) . v per query head, kv head = head / (heads/kv_heads)
 * (attention_decode_f16_tiled_scalar, crates/soso-llm-core/src/attn.rs:73-140; split
 * into chunks merged like combinar_trozos, attn_grupo.rs:171-203).  head_dim 128.
 * Replaces mo_attn_split + mo_attn_combine (gemma_capa.cu:765-926). */
int sbk_attn_decode(const float *q, const uint16_t *kcache, const uint16_t *vcache, float *out, const int32_t *pos,
                    size_t heads, size_t kv_heads, size_t head_dim, size_t ctx, void *ws, int pdl, void *stream);
/* sbk_rope_kv_append and sbk_attn_decode in one launch: on the stacked, unroped
 * [q | k | v] vector, bias / QK-norm / RoPE as sbk_rope_kv_append, this token's K/V
 * rows appended at *pos (f16, the reference's rounding), then attention over
 * positions 0..*pos.  qkv is not modified (the roped q lives in shared memory).
 * Workspace as sbk_attn_decode.  Replaces gm_rope + gm_kv_append + mo_attn_split +
 * mo_attn_combine (gemma_capa.cu:99-141, :765-926); the CPU order is layer.rs:1146-1282. */
int sbk_attn_rope_decode(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                         uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos, size_t heads,
                         size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox, void *ws,
                         int pdl, void *stream);
/* The same with YaRN: factors / mscale as sbk_rope_kv_append_yarn (gm_rope's frequency
 * divisors, gemma_capa.cu:99-125); factors NULL is sbk_attn_rope_decode exactly. */
int sbk_attn_rope_decode_yarn(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                              uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos, size_t heads,
                              size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                              const float *factors, float mscale, void *ws, int pdl, void *stream);

/* out = silu(gate) * up, elementwise (`swiglu_inplace`, crates/soso-llm-core/src/gemm.rs:210-226). */
int sbk_swiglu(const float *gate, const float *up, float *out, size_t n, int pdl, void *stream);

/* Router: softmax over n_exp logits, stable top-k by weight, renormalised
 * (gemm::topk_softmax, crates/soso-llm-core/src/gemm.rs:62-91); idx/wts in rank
 * order.  Replaces mo_router (gemma_capa.cu:586-639). */
int sbk_router_topk(const float *logits, size_t n_exp, size_t top_k, int32_t *idx, float *wts, int pdl, void *stream);

/* Workspace bytes for sbk_argmax (zero-filled before first use; left zeroed). */
size_t sbk_argmax_ws_bytes(void);
/* Greedy token: index of the maximum, ties to the LAST index like
 * Runtime::argmax (crates/soso-llm-core/src/runtime.rs:2021-2028). */
int sbk_argmax(const float *v, size_t n, int32_t *out, void *ws, int pdl, void *stream);

/* MLA decode in the absorbed form (mathematically the reference's re-expansion,
 * attention_decode_mla_latent, crates/soso-llm-core/src/attn.rs:306-404; the reference
 * has no GPU kernel for MLA).  sbk_mla_absorb, kv_rank / 64 CTAs per head: appends this token's
 * latent row c (f16, the reference's rounding) at *pos, its rope keys
 * rope_pos(W_kr . c) per kv head, the roped q slice qr[heads][qk_rope] and the absorbed
 * query qt[heads][kv_rank] = W_kn^T q_nope (W_kn, W_kr = head's nope / rope rows of the
 * Q4_K k_up).  sbk_mla_attn: cbar[heads][kv_rank] = sum_t softmax_t(qt.c_t + qr.kr_t) c_t
 * / scaled by 1/sqrt(qk_nope+qk_rope); the output of a head is then W_v,h . cbar_h.
 * heads <= 16, kv_rank a multiple of 512 (<= 1024), qk_nope <= 256, qk_rope even (<= 128).  ws: at least
 * sbk_mla_ws_bytes(heads, kv_rank), zero-filled before first use (left zeroed). */
size_t sbk_mla_ws_bytes(size_t heads, size_t kv_rank);
int sbk_mla_absorb(const float *q, const float *c, const void *k_up, uint8_t k_up_dtype, uint16_t *latent,
                   float *krope, float *qt, float *qr, const int32_t *pos, size_t heads, size_t kv_heads,
                   size_t kv_rank, size_t qk_nope, size_t qk_rope, size_t ctx, float theta, int pdl, void *stream);
int sbk_mla_attn(const float *qt, const float *qr, const uint16_t *latent, const float *krope, float *cbar,
                 const int32_t *pos, size_t heads, size_t kv_heads, size_t kv_rank, size_t qk_nope, size_t qk_rope,
                 size_t ctx, void *ws, int pdl, void *stream);

/* One embedding row (dtype F32 / Q8_0 / Q4_K / Q6_K) dequantised exactly
 * (Runtime::embed_token, crates/soso-llm-core/src/runtime.rs:787-802). */
int sbk_embed_row(const void *table, uint8_t dtype, size_t vocab, size_t hidden, const int32_t *token, float *out,
                  int pdl, void *stream);

/* y = W . x for Q4_K weights, like sbk_matvec(SB_DTYPE_Q4_K, ...) and with the
 * same results, for callers that must not allocate device memory (a host engine
 * that owns a fixed memory budget, or code that may run while a CUDA graph is
 * being captured in global mode, where an allocation breaks the capture).  No
 * counterpart in the reference.  Its scratch is a fixed 96 KiB array compiled
 * into the library (held by every GPU that loads it until exit), so it takes
 * rows <= 262144 (returns -8 beyond that), cols <= 8192, and no cudaMalloc,
 * cudaFree or allocating library call is made.  The first call on a device
 * looks the array's device address up (cudaGetSymbolAddress): make it before
 * any stream capture.  All calls share the array and it keeps the last call's
 * contents: calls that overlap on the GPU race, so serialise them. */
int sbk_matvec_q4k_noalloc(const void *w, size_t rows, size_t cols, const float *x, float *y, void *stream);

/* Number of SMs the kernels size their grids for. */
int sbk_num_sms(int device);

/* Device-side error word (bounded waits that gave up set it); read-and-clear. */
int sbk_take_device_error(int device, uint32_t *code);

#ifdef __cplusplus
}
#endif

#endif /* SOSOB200_H */
