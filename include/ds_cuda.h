/*
 * ds_cuda.h — C ABI of the B200 (sm_100a) implementation of ds-ocr's
 * MoE-decoder hot path. It fills the slot the reference's Metal offload
 * (ds_metal.h) occupies and adds CUDA entry points with the signatures of
 * the ds_kernels / ds_quantize functions the hot path calls.
 *
 * Conventions
 *  - Plain C types only: pointers, sizes, ints. No CUDA or torch types.
 *  - Every call returns an int status: >= 0 success (token ids are >= 0),
 *    negative = error (DS_CUDA_E*). ds_cuda_last_error() describes the last
 *    failure of a context. Nothing fails silently (unlike the reference's
 *    void Metal calls, ds_metal.m:263,318,439).
 *  - Host-pointer calls are synchronous, like the Metal ones
 *    (waitUntilCompleted, ds_metal.m:425-427): inputs are copied to the
 *    device, outputs copied back before return.
 *  - Weights are copied to HBM once and looked up by HOST pointer, interior
 *    pointers included (the Metal context wraps host buffers and translates
 *    pointers into the expert block, ds_metal.m:56-86). A weight not
 *    registered beforehand is registered on first use with the size the call
 *    implies (the Metal get_wbuf wraps on demand the same way).
 *  - "_dev" entry points take DEVICE pointers and a stream (cudaStream_t
 *    passed as void*, NULL = the context's stream) and only enqueue work.
 *  - One context per device; a context is not thread-safe (the Metal one
 *    is not either: shared scratch per context).
 *  - Shape limits: hidden dimensions a multiple of 16 and <= 2048, expert
 *    intermediate a multiple of 16, top_k <= 6 with shared experts (<= 8
 *    without), <= 256 routed experts. DS_CUDA_EINVAL otherwise.
 *
 * This library has no CPU fallback: without a usable CUDA device
 * ds_cuda_init returns NULL and ds_cuda_is_available returns 0.
 */
#ifndef DS_CUDA_H
#define DS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DS_CUDA_OK 0
#define DS_CUDA_EINVAL (-1)     /* bad argument or unsupported shape */
#define DS_CUDA_ENOTREG (-2)    /* pointer not inside a registered weight */
#define DS_CUDA_ECUDA (-3)      /* CUDA runtime / launch error */
#define DS_CUDA_ENOMEM (-4)     /* device allocation failed */
#define DS_CUDA_ESTATE (-5)     /* call not valid in the current state */
#define DS_CUDA_ENCCL (-6)      /* NCCL error */
#define DS_CUDA_ETIMEOUT (-7)   /* a bounded device-side wait gave up */

typedef struct ds_cuda_ctx ds_cuda_ctx_t;

/* Same memory layout as the reference's ds_int4_block_t
 * (ds_quantize.h:30-37): per-row asymmetric INT8, stored q - 128. */
typedef struct {
    int8_t *qweight; /* [out_dim, in_dim] row-major */
    float *scale;    /* [out_dim] */
    float *offset;   /* [out_dim] (row minimum) */
    int out_dim;
    int in_dim;
    size_t bytes;
} ds_cuda_int8_block_t;

/* ---------------------------------------------------------------------
 * Lifecycle — ds_metal_init / ds_metal_free / ds_metal_is_available
 * (ds_metal.h:37-46).
 * --------------------------------------------------------------------- */
ds_cuda_ctx_t *ds_cuda_init(int device);
void ds_cuda_free(ds_cuda_ctx_t *ctx);
int ds_cuda_is_available(const ds_cuda_ctx_t *ctx);
const char *ds_cuda_last_error(const ds_cuda_ctx_t *ctx);
/* The context's CUDA stream (cudaStream_t) as an opaque pointer. */
void *ds_cuda_stream(ds_cuda_ctx_t *ctx);
int ds_cuda_synchronize(ds_cuda_ctx_t *ctx);

/* Numerics switches of the reference:
 *  simulate_bf16 — ds_bf16_simulate_python (ds_ocr.c:27, main.c:106): BF16
 *                  round-trip of expert intermediates (ds_kernels.c:333-356).
 *  renorm_topk   — divide the top-k router weights by their sum. The
 *                  reference code does NOT (ds_moe_decoder.c:157-183); default 0. */
int ds_cuda_set_numerics(ds_cuda_ctx_t *ctx, int simulate_bf16, int renorm_topk);

/* ---------------------------------------------------------------------
 * Weight registration — ds_metal_register_bf16 / _f32 /
 * _register_expert_block (ds_metal.h:52-66). The host range is copied to
 * HBM once; later calls passing any pointer inside it use the device copy.
 * --------------------------------------------------------------------- */
int ds_cuda_register_bf16(ds_cuda_ctx_t *ctx, const uint16_t *data, size_t n);
int ds_cuda_register_f32(ds_cuda_ctx_t *ctx, const float *data, size_t n);
int ds_cuda_register_expert_block(ds_cuda_ctx_t *ctx, const void *block_ptr, size_t block_bytes);
/* Registers the three arrays of an INT8 block (the --int4 path,
 * ds_quantize.h:30-37; quantised by ds_int4_quantize_bf16 on the host). */
int ds_cuda_register_int8_block(ds_cuda_ctx_t *ctx, const ds_cuda_int8_block_t *block);
/* Drops the registration whose host range starts at host_ptr and frees its
 * HBM copy. Registrations are keyed by host address, so a caller that frees
 * or reuses a registered host buffer must unregister it first (the
 * reference's weights are mmap'd for the context's lifetime and never are). */
int ds_cuda_unregister(ds_cuda_ctx_t *ctx, const void *host_ptr);
/* Device address of a registered host pointer (NULL if unregistered). */
const void *ds_cuda_device_ptr(ds_cuda_ctx_t *ctx, const void *host_ptr);
/* Bytes of HBM held by registered weights. */
size_t ds_cuda_registered_bytes(const ds_cuda_ctx_t *ctx);

/* ---------------------------------------------------------------------
 * Decode MoE — ds_metal_moe_experts / ds_metal_shared_experts
 * (ds_metal.h:96-128). moe_experts WRITES output = sum_k w_k expert_k(x);
 * shared_experts ADDS its result into output.
 * --------------------------------------------------------------------- */
int ds_cuda_moe_experts(ds_cuda_ctx_t *ctx, const float *x, const uint16_t **gate_up_ptrs,
                        const uint16_t **down_ptrs, const float *top_weights, int top_k,
                        int hidden, int inter, float *output);
int ds_cuda_shared_experts(ds_cuda_ctx_t *ctx, const float *x, const uint16_t *gate_up_bf16,
                           const uint16_t *down_bf16, int hidden, int shared_inter, float *output);

/* ds_expert_forward_fused (ds_kernels.h:209-214) and
 * ds_expert_forward_fused_int4 (ds_quantize.h:69-75) without the caller
 * scratch buffers (scratch lives in the context). */
int ds_cuda_expert_forward_fused(ds_cuda_ctx_t *ctx, float *out, const float *x,
                                 const uint16_t *gate_up_fused_bf16, const uint16_t *down_bf16,
                                 int hidden, int intermediate);
int ds_cuda_expert_forward_fused_int4(ds_cuda_ctx_t *ctx, float *out, const float *x,
                                      const ds_cuda_int8_block_t *gate_up_int4,
                                      const ds_cuda_int8_block_t *down_int4, int hidden,
                                      int intermediate);

/* Whole moe_forward (ds_moe_decoder.c:131-333) for one token: router
 * matvec, softmax + top-k, routed experts, combine, shared experts.
 *   router_bf16   [n_experts x hidden]
 *   expert_block  [n_experts x (2*inter x hidden)] then shared [(2*shared_inter) x hidden]
 *                 (the contiguous block of ds_ocr.c:696-768)
 *   down_bf16     [n_experts x (hidden x inter)] contiguous
 *   shared_down   [hidden x shared_inter]
 * top_idx / top_w (optional, may be NULL) receive the routing decision. */
int ds_cuda_moe_layer(ds_cuda_ctx_t *ctx, const float *x, float *out, const uint16_t *router_bf16,
                      const uint16_t *expert_block, const uint16_t *down_bf16,
                      const uint16_t *shared_down_bf16, int hidden, int inter, int shared_inter,
                      int n_experts, int top_k, int *top_idx, float *top_w);
/* Same with INT8 experts: per-expert blocks laid out contiguously
 * (gu: [E][2I x H] q, [E][2I] scale/offset; dn: [E][H x I], [E][H]). */
int ds_cuda_moe_layer_int8(ds_cuda_ctx_t *ctx, const float *x, float *out, const uint16_t *router_bf16,
                           const int8_t *gu_q, const float *gu_scale, const float *gu_off,
                           const int8_t *dn_q, const float *dn_scale, const float *dn_off,
                           const int8_t *sgu_q, const float *sgu_scale, const float *sgu_off,
                           const int8_t *sdn_q, const float *sdn_scale, const float *sdn_off,
                           int hidden, int inter, int shared_inter, int n_experts, int top_k,
                           int *top_idx, float *top_w);
/* Device-pointer form of ds_cuda_moe_layer_int8 (the reference's int4
 * branch of moe_forward, ds_moe_decoder.c:237-243, 269-278): every pointer
 * is device memory, the work is enqueued on `stream` (NULL = the context's
 * stream) and nothing is copied to or from the host; d_top_idx / d_top_w
 * may be NULL. */
int ds_cuda_moe_layer_int8_dev(ds_cuda_ctx_t *ctx, const float *d_x, float *d_out, const uint16_t *d_router,
                               const int8_t *d_gu_q, const float *d_gu_scale, const float *d_gu_off,
                               const int8_t *d_dn_q, const float *d_dn_scale, const float *d_dn_off,
                               const int8_t *d_sgu_q, const float *d_sgu_scale, const float *d_sgu_off,
                               const int8_t *d_sdn_q, const float *d_sdn_scale, const float *d_sdn_off,
                               int hidden, int inter, int shared_inter, int n_experts, int top_k,
                               int *d_top_idx, float *d_top_w, void *stream);

/* ---------------------------------------------------------------------
 * LM head — ds_metal_lm_head_argmax (ds_metal.h:146-150) and
 * ds_argmax_matvec_bf16 (ds_kernels.h:239-240). Returns the token id
 * (lowest id wins ties) or a negative error. *logit (optional) receives its
 * logit.
 * --------------------------------------------------------------------- */
int ds_cuda_lm_head_argmax(ds_cuda_ctx_t *ctx, const float *x, const uint16_t *W_bf16, int hidden,
                           int vocab);
int ds_cuda_argmax_matvec_bf16(ds_cuda_ctx_t *ctx, const float *x, const uint16_t *W_bf16, int in_dim,
                               int out_dim, float *logit);
/* B independent inputs x[B x in_dim] (the reference loops). B = 2..64 with
 * in_dim % 64 == 0 is one tensor-core pass over W (the inputs split into two
 * BF16 planes, F32 accumulation); other shapes run one matvec per input. */
int ds_cuda_argmax_matvec_bf16_batch(ds_cuda_ctx_t *ctx, const float *x, const uint16_t *W_bf16,
                                     int in_dim, int out_dim, int batch, int *tokens, float *logits);
/* Same on device buffers (W registered, d_W its device copy), enqueued on
 * `stream` (NULL: the context's stream). */
int ds_cuda_argmax_matvec_bf16_batch_dev(ds_cuda_ctx_t *ctx, const float *d_x, const uint16_t *d_W, int in_dim,
                                         int out_dim, int batch, int *d_tokens, float *d_logits, void *stream);

/* ds_metal_matvec_bf16 (ds_metal.h:168-174): y = W x (+ bias). */
int ds_cuda_matvec_bf16(ds_cuda_ctx_t *ctx, float *y, const float *x, const uint16_t *W_bf16,
                        const float *bias, int in_dim, int out_dim);

/* ---------------------------------------------------------------------
 * INT8 quantisation on the device, bit-identical to ds_int4_quantize_bf16
 * (ds_quantize.c:49-81). W is host BF16 [out_dim x in_dim]; q/scale/offset
 * receive the host result.
 * --------------------------------------------------------------------- */
int ds_cuda_int8_quantize_bf16(ds_cuda_ctx_t *ctx, const uint16_t *W_bf16, int out_dim, int in_dim,
                               int8_t *qweight, float *scale, float *offset);

/* ---------------------------------------------------------------------
 * Device-pointer entry points (enqueue only).
 * --------------------------------------------------------------------- */
int ds_cuda_argmax_matvec_bf16_dev(ds_cuda_ctx_t *ctx, const float *d_x, const uint16_t *d_W,
                                   int in_dim, int out_dim, int *d_token, float *d_logit, void *stream);
int ds_cuda_moe_layer_dev(ds_cuda_ctx_t *ctx, const float *d_x, float *d_out,
                          const uint16_t *d_router, const uint16_t *d_expert_block,
                          const uint16_t *d_down, const uint16_t *d_shared_down, int hidden, int inter,
                          int shared_inter, int n_experts, int top_k, int *d_top_idx, float *d_top_w,
                          void *stream);

/* ds_cuda_moe_experts_noalloc — no counterpart in the reference.
 * The routed-expert chain of ds_cuda_moe_experts (output = sum_k
 * top_weights[k] * expert_k(x), no shared expert) for callers that cannot
 * allocate device memory at the point of the call, e.g. a plugin handed
 * device buffers by its host framework, or a process whose device memory is
 * fixed after start-up. It creates no context and allocates nothing: x,
 * the weights and output are DEVICE pointers the caller owns (gate-up and
 * down are host arrays of top_k device pointers; top_weights is a host
 * array), and the SwiGLU activations live in a static 48 KB device array
 * the library holds on every GPU that loads it until the process exits.
 * Limits: top_k <= 8, hidden and inter multiples of 8 and <= 2048,
 * top_k * inter <= 12288 (the scratch); larger sizes return DS_CUDA_EINVAL with a message
 * on stderr. Work is enqueued on `stream` (NULL = the legacy default stream)
 * of the current device. The first call on a device looks up the array's
 * device address; make that first call before any stream capture. All
 * calls share the one array, so calls that overlap on the GPU (different
 * streams, or different host threads) race; serialise them. */
int ds_cuda_moe_experts_noalloc(const float *d_x, const uint16_t *const *d_gate_up,
                                const uint16_t *const *d_down, const float *top_weights, int top_k,
                                int hidden, int inter, float *d_output, void *stream);

/* ---------------------------------------------------------------------
 * Decoder — the single-token greedy decode step of ds_decoder_forward
 * (ds_moe_decoder.c:911-1264, decoder_layer_forward :339-474) on the GPU,
 * with the KV cache resident in HBM. One call = input RMSNorm, QKV, RoPE,
 * KV append, attention, O-proj + residual, post-attention RMSNorm, dense
 * FFN (layer < first_dense) or MoE, residual, for every layer; final
 * RMSNorm; argmax LM head. Engine 0 runs the step as one CUDA graph of
 * per-phase kernels chained with programmatic dependent launch.
 * --------------------------------------------------------------------- */
typedef struct {
    int hidden, n_layers, n_heads, head_dim; /* head_dim must be 128 */
    int dense_inter, moe_inter, n_experts, n_shared, top_k, vocab, first_dense;
    float rms_eps, rope_theta;
    int kv_max;   /* KV capacity in tokens (the reference allocates 4096, ds_ocr.c:861) */
    int use_int8; /* 1: MoE layers use the INT8 blocks (the --int4 path) */
    int engine;   /* 0: a CUDA graph of per-phase kernels per token (default; any
                        supported shape, INT8);
                     1: one persistent kernel per call (BF16, hidden 1280) */
} ds_cuda_decoder_config_t;

/* The fields of the reference's ds_dec_layer_t (ds_ocr.h:282-342) the
 * decode step reads. Host pointers; copied to HBM at create. */
typedef struct {
    const uint16_t *wq, *wk, *wv, *wo;        /* [heads*head_dim x hidden], wo [hidden x heads*head_dim] */
    const float *input_norm, *post_attn_norm; /* [hidden] */
    const uint16_t *dense_gate, *dense_up;    /* dense layers: [dense_inter x hidden] */
    const uint16_t *dense_down;               /* [hidden x dense_inter] */
    const uint16_t *router;                   /* MoE layers: [n_experts x hidden] */
    const uint16_t *expert_block;             /* [E x 2I x H] + shared [2S x H] (ds_ocr.c:696-768) */
    const uint16_t *down;                     /* [E x H x I] */
    const uint16_t *shared_down;              /* [H x S] */
    /* INT8 copies (use_int8), contiguous per kind as in ds_cuda_moe_layer_int8 */
    const int8_t *gu_q; const float *gu_scale, *gu_off;
    const int8_t *dn_q; const float *dn_scale, *dn_off;
    const int8_t *sgu_q; const float *sgu_scale, *sgu_off;
    const int8_t *sdn_q; const float *sdn_scale, *sdn_off;
} ds_cuda_layer_weights_t;

/* Returns a model handle > 0. lm_head is [vocab x hidden] BF16, also used
 * as the token embedding table (tied, as in the reference's V2 config). */
int ds_cuda_decoder_create(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg,
                           const ds_cuda_layer_weights_t *layers, const float *final_norm,
                           const uint16_t *lm_head);
int ds_cuda_decoder_destroy(ds_cuda_ctx_t *ctx, int model);
/* Writes KV rows [pos0, pos0+n) of one layer from F32 [n x heads*head_dim]
 * arrays (the reference's F32 cache rows, ds_moe_decoder.c:45-53). */
int ds_cuda_decoder_load_kv(ds_cuda_ctx_t *ctx, int model, int layer, int pos0, int n, const float *k,
                            const float *v);
/* kv_cache_len: the position the next token is written at. */
int ds_cuda_decoder_set_len(ds_cuda_ctx_t *ctx, int model, int kv_len);
int ds_cuda_decoder_get_len(ds_cuda_ctx_t *ctx, int model);
/* ds_decoder_forward: one step on input_embed [hidden]; returns the greedy
 * token. final_x (optional) receives the final RMS-normed hidden state,
 * logit (optional) the winning logit. Advances kv_cache_len by one. */
int ds_cuda_decoder_forward(ds_cuda_ctx_t *ctx, int model, const float *input_embed, float *final_x,
                            float *logit);
/* n_steps greedy steps without host round trips: step 0 consumes
 * first_embed (NULL: the embedding of the previous step's token), each
 * next step the embedding row of the previous token. tokens[n_steps]. */
int ds_cuda_decoder_generate(ds_cuda_ctx_t *ctx, int model, const float *first_embed, int n_steps,
                             int *tokens);
/* Enqueue n_steps greedy steps on `stream` from the device-resident state
 * (no host copies; for timing). */
int ds_cuda_decoder_generate_dev(ds_cuda_ctx_t *ctx, int model, int n_steps, void *stream);
/* Kernel launches one decode step issues with engine 0; 0 with the
 * persistent engine (one launch per forward/generate call). */
int ds_cuda_decoder_launches_per_step(ds_cuda_ctx_t *ctx, int model);

/* LM-head selection settings, the reference's ctx->repeat_penalty,
 * no_repeat_ngram_size and temperature (ds_ocr.h; set from main.c:132-134,
 * read by ds_decoder_forward at ds_moe_decoder.c:1021-1263). Defaults 1, 0,
 * 0 (greedy argmax). repeat_penalty > 1: the history tokens' logits are
 * divided (positive) or multiplied (negative) by it; no_repeat_ngram_size
 * n > 0: a token that would complete an n-gram already in the history is
 * banned; temperature > 0: softmax sampling with the uniforms given by
 * ds_cuda_decoder_set_uniforms. Engine 0 only (EINVAL with engine 1).
 * Forward and generate then return the selected token (and its penalised
 * logit). */
int ds_cuda_decoder_set_sampling(ds_cuda_ctx_t *ctx, int model, float repeat_penalty, int no_repeat_ngram_size,
                                 float temperature);
/* The generated-token history (ctx->token_history, ds_ocr.h:433-435): every
 * decode step appends its token, as the reference's generation loop does
 * (ds_ocr.c:2245-2248). set replaces it (n <= kv_max + 512); get copies up
 * to cap tokens and returns the length. */
int ds_cuda_decoder_set_history(ds_cuda_ctx_t *ctx, int model, const int *tokens, int n);
int ds_cuda_decoder_get_history(ds_cuda_ctx_t *ctx, int model, int *tokens, int cap);
/* Uniforms for temperature sampling, consumed one per sampled step in order
 * (the reference draws (float)rand() / RAND_MAX, ds_moe_decoder.c:1251).
 * Forward/generate return DS_CUDA_ESTATE when too few are left. */
int ds_cuda_decoder_set_uniforms(ds_cuda_ctx_t *ctx, int model, const float *u, int n);
/* V3's reference sliding-window decode attention (R-SWA): the reference's
 * cfg->sliding_window_size and ctx->prefill_token_count (ds_ocr.h:438),
 * read at ds_moe_decoder.c:409-436. With W > 0 and the query at or past
 * prefill_token_count P, each step attends rows [0, P) and then
 * [max(P, len - W), len) through the same sequential softmax. 0 disables
 * (full causal attention). Engine 0 only. */
int ds_cuda_decoder_set_window(ds_cuda_ctx_t *ctx, int model, int sliding_window_size, int prefill_token_count);
/* The token embedding table the decode loop takes the next input from (the
 * reference's tok_embeddings_bf16, ds_ocr.c:2272-2279), [vocab x hidden]
 * BF16 host pointer (registered on first use). Default: the LM head (tied). */
int ds_cuda_decoder_set_embeddings(ds_cuda_ctx_t *ctx, int model, const uint16_t *embed_tokens);

/* Whole-decoder prefill, ds_decoder_prefill (ds_moe_decoder.c:480-905):
 * n_tokens input embeddings (F32 [n_tokens x hidden]) at positions len ..
 * len + n_tokens - 1 through every layer on the tensor cores (QKV, O-proj,
 * dense FFN and MoE as split-BF16 GEMMs, the exact sequential-softmax
 * attention per query), their K/V rows written to the cache. Returns the
 * first generated token (LM-head argmax of the last row's final RMSNorm);
 * final_x / logit (optional) receive that row and its logit. Decoding then
 * continues at len + n_tokens with the token's embedding staged (forward
 * takes an explicit embedding; generate with first_embed NULL uses it), and
 * the token is appended to the history. BF16 expert weights required. */
int ds_cuda_decoder_prefill(ds_cuda_ctx_t *ctx, int model, const float *embeds, int n_tokens, float *final_x,
                            float *logit);
/* The same on device embeddings, enqueued on `stream` (NULL: the context's)
 * without host copies. */
int ds_cuda_decoder_prefill_dev(ds_cuda_ctx_t *ctx, int model, const float *d_embeds, int n_tokens, void *stream);
/* Cache rows [pos0, pos0 + n) of one layer as F32 [n x heads*head_dim]. */
int ds_cuda_decoder_get_kv(ds_cuda_ctx_t *ctx, int model, int layer, int pos0, int n, float *k, float *v);

/* ---------------------------------------------------------------------
 * Weight ingest from a safetensors checkpoint (the reference's
 * ds_safetensors.c reader and ds_ocr.c:608-757 decoder loader).
 * --------------------------------------------------------------------- */
/* A decoder model from `path`: a directory holding model.safetensors or
 * model-*.safetensors shards (read in name order), or one file. Tensors are
 * looked up by the reference's names (model.layers.N.self_attn.q_proj.weight,
 * ...mlp.experts.E.gate_proj.weight, model.embed_tokens.weight,
 * lm_head.weight (absent: tied), model.norm.weight, ...), checked against cfg,
 * copied into HBM once; the expert blocks are assembled on the device, the
 * INT8 copies (cfg->use_int8) quantised there. Returns a model handle as
 * ds_cuda_decoder_create; DS_CUDA_EINVAL names a missing or mis-shaped
 * tensor. The files are unmapped before it returns. */
int ds_cuda_decoder_create_from_safetensors(ds_cuda_ctx_t *ctx, const char *path,
                                            const ds_cuda_decoder_config_t *cfg);
/* Host-only probes of a checkpoint (no device): number of tensors over all
 * shards (< 0 on a bad file); metadata of one tensor (1 found, 0 absent,
 * < 0 bad file): dtype as the reference's safetensor_dtype_t (F32 0, F16 1,
 * BF16 2, I32 3, I64 4, BOOL 5, other -1), dims, and the byte offset and
 * size within its file's data section. The message of the last failure. */
int ds_cuda_safetensors_count(const char *path);
int ds_cuda_safetensors_find(const char *path, const char *name, int *dtype, int *ndim, int64_t *shape8,
                             size_t *data_offset, size_t *data_size);
const char *ds_cuda_safetensors_error(void);

/* ---------------------------------------------------------------------
 * Multi-stream decoder — ds_decoder_forward for up to 64 independent
 * streams at once (each with its own KV cache and position; the reference
 * runs streams one at a time). One step advances every stream by one token;
 * the linear layers run on the tensor cores with the weights read once per
 * step for all streams. Same configuration and layer structs as the
 * single-stream decoder (BF16 experts; use_int8 and engine are ignored).
 * Greedy with causal attention unless set_sampling / set_window say
 * otherwise.
 * --------------------------------------------------------------------- */
int ds_cuda_batch_decoder_create(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg,
                                 const ds_cuda_layer_weights_t *layers, const float *final_norm,
                                 const uint16_t *lm_head, int n_streams);
int ds_cuda_batch_decoder_destroy(ds_cuda_ctx_t *ctx, int model);
/* KV rows [pos0, pos0+n) of one layer of one stream (F32 [n x heads*head_dim]). */
int ds_cuda_batch_decoder_load_kv(ds_cuda_ctx_t *ctx, int model, int stream, int layer, int pos0, int n,
                                  const float *k, const float *v);
int ds_cuda_batch_decoder_set_len(ds_cuda_ctx_t *ctx, int model, int stream, int kv_len);
/* One step: embeds [n_streams x hidden] (NULL: the embeddings of the
 * previous step's tokens); tokens [n_streams]; final_x [n_streams x hidden]
 * (optional) receives the final RMS-normed hidden states. */
int ds_cuda_batch_decoder_forward(ds_cuda_ctx_t *ctx, int model, const float *embeds, int *tokens,
                                  float *final_x);
/* n_steps steps; tokens [n_steps x n_streams]. */
int ds_cuda_batch_decoder_generate(ds_cuda_ctx_t *ctx, int model, const float *first_embeds, int n_steps,
                                   int *tokens);
/* n_steps steps enqueued on `stream` from the device state (a CUDA graph
 * per step; no host copies). */
int ds_cuda_batch_decoder_generate_dev(ds_cuda_ctx_t *ctx, int model, int n_steps, void *stream);
/* LM-head selection settings for every stream, as
 * ds_cuda_decoder_set_sampling (ds_moe_decoder.c:1021-1263, the reference's
 * per-context repeat_penalty, no_repeat_ngram_size and temperature, applied
 * here to each stream against its own history). Needs hidden % 256 == 0
 * when any setting is on. */
int ds_cuda_batch_decoder_set_sampling(ds_cuda_ctx_t *ctx, int model, float repeat_penalty,
                                       int no_repeat_ngram_size, float temperature);
/* One stream's generated-token history (the reference's per-context
 * ctx->token_history, ds_ocr.h:433-435); every step appends each stream's
 * token (ds_ocr.c:2245-2248). set replaces it (n <= kv_max + 512); get
 * copies up to cap tokens and returns the length. */
int ds_cuda_batch_decoder_set_history(ds_cuda_ctx_t *ctx, int model, int stream, const int *tokens, int n);
int ds_cuda_batch_decoder_get_history(ds_cuda_ctx_t *ctx, int model, int stream, int *tokens, int cap);
/* Uniforms for temperature sampling (the reference's (float)rand() /
 * RAND_MAX, ds_moe_decoder.c:1251): u [n_streams x n], row s consumed by
 * stream s in order, one per sampled step; every stream restarts at its
 * first. Steps return DS_CUDA_ESTATE when too few are left. */
int ds_cuda_batch_decoder_set_uniforms(ds_cuda_ctx_t *ctx, int model, const float *u, int n);
/* V3's reference sliding-window decode attention (ds_moe_decoder.c:409-436)
 * for every stream: window W (0 disables) and each stream's prefill length
 * prefill_token_counts[n_streams] (the reference's per-context
 * ctx->prefill_token_count, ds_ocr.h:438). */
int ds_cuda_batch_decoder_set_window(ds_cuda_ctx_t *ctx, int model, int sliding_window_size,
                                     const int *prefill_token_counts);

/* ---------------------------------------------------------------------
 * Batched MoE prefill — the MoE block of ds_decoder_prefill for n tokens
 * (ds_moe_decoder.c:630-809): per token RMSNorm(post_attn_norm), router
 * softmax/top-k (fast exp, strict '>', weights = probabilities unless the
 * renorm numerics flag is set), shared expert and routed experts grouped by
 * expert, then x += routed + shared. The reference runs F32 sgemm on
 * widened BF16 weights; here the GEMMs run on the tensor cores with the
 * activations split into two BF16 planes (F32-class accuracy).
 * Shapes: hidden % 256 == 0, moe_inter and n_shared*moe_inter % 128 == 0,
 * n_experts <= 256, top_k <= 8.
 * Weights are the layer's host pointers (registered on first use, as
 * elsewhere in this ABI); router may be NULL when logits are given.
 * logits [n_tokens x n_experts] (optional) replace xn W_r^T (the scores
 * before the softmax). top_idx / top_w [n_tokens x top_k] (optional)
 * receive the routing.
 * --------------------------------------------------------------------- */
int ds_cuda_prefill_moe(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg,
                        const ds_cuda_layer_weights_t *layer, float *x, int n_tokens, const float *logits,
                        int *top_idx, float *top_w);
/* Same on device buffers, enqueued on `stream` (NULL: the context's stream);
 * no synchronisation. A device-side wait that gave up is reported by the
 * next ds_cuda_prefill_check. */
int ds_cuda_prefill_moe_dev(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg,
                            const ds_cuda_layer_weights_t *layer, float *d_x, int n_tokens, const float *d_logits,
                            int *d_top_idx, float *d_top_w, void *stream);
/* The three stages of ds_cuda_prefill_moe_dev on caller buffers, for
 * expert-parallel prefill, where the caller moves rows between devices
 * between the stages (no counterpart in the reference, which runs on one
 * host):
 *  route:   RMSNorm of d_x [n x H] into two BF16 planes d_xn_hi/lo [n x H]
 *           (v = hi + lo), and the routing d_top_idx / d_top_w [n x top_k].
 *  experts: for each pair p = (row d_pair_row[p] of d_rows_hi/lo, rows
 *           rows_ld elements apart (a multiple of 8), expert d_pair_expert[p])
 *           the routed expert's output d_y[p] [H]; pairs whose expert is
 *           outside [0, n_experts) are skipped. d_pair_row NULL means
 *           row = p / top_k. Also the shared expert of d_sh_hi/lo
 *           [n_shared_rows x H] into d_ys.
 *  combine: d_x[s] += sum over k, in ascending expert order, of
 *           w[s,k] * y_k, plus d_ys[s] (ds_moe_decoder.c:785-800), where y_k
 *           is row s*top_k + k of d_y, or row d_y_row[s*top_k + k] if given. */
int ds_cuda_prefill_route_dev(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg,
                              const ds_cuda_layer_weights_t *layer, const float *d_x, int n_tokens,
                              const float *d_logits, uint16_t *d_xn_hi, uint16_t *d_xn_lo, int *d_top_idx,
                              float *d_top_w, void *stream);
int ds_cuda_prefill_experts_dev(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg,
                                const ds_cuda_layer_weights_t *layer, const uint16_t *d_rows_hi,
                                const uint16_t *d_rows_lo, int rows_ld, int n_rows, const int *d_pair_row,
                                const int *d_pair_expert, int n_pairs, float *d_y, const uint16_t *d_sh_hi,
                                const uint16_t *d_sh_lo, int n_shared_rows, float *d_ys, void *stream);
int ds_cuda_prefill_combine_dev(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg, float *d_x,
                                int n_tokens, const int *d_top_idx, const float *d_top_w, const float *d_y,
                                const int *d_y_row, const float *d_ys, void *stream);
/* Expert-parallel bookkeeping (no counterpart in the reference). Ranks own
 * contiguous blocks of experts_per_rank experts (n_ranks <= 8, top_k <= 7).
 * A payload row is [hi plane H | lo plane H | 8 int32 meta] as uint16_t, row
 * pitch 2*H + 16; meta = the top_k expert ids served at the destination (-1
 * for the others, -1 padding) and, in the last slot, the offset of the
 * row's first (row, expert) pair within that destination's pairs.
 *  dispatch: plans sending each token once to every rank owning one of its
 *            experts (rank ascending, token ascending) and packs those rows
 *            into d_payload (capacity n_tokens * min(top_k, n_ranks) rows);
 *            d_send_tok[i] = token of row i; d_counts[0..G) rows and
 *            d_counts[G..2G) (token, expert) pairs per destination rank;
 *            d_inv[s*top_k + k] = row of that pair's output in the stream
 *            that comes back (rank, token, k ascending).
 *  pairs:    for n_rows received payload rows (recv_counts [n_ranks], a HOST
 *            array, rows per source rank in rank order, each source's rows
 *            one destination section of its dispatch) the compact
 *            row-major (row, expert) pairs; d_counts[0..G) pairs per source
 *            rank, d_counts[G] all pairs. */
int ds_cuda_ep_dispatch_dev(ds_cuda_ctx_t *ctx, int n_tokens, int top_k, int n_ranks, int experts_per_rank,
                            const int *d_top_idx, const uint16_t *d_xn_hi, const uint16_t *d_xn_lo, int hidden,
                            uint16_t *d_payload, int *d_send_tok, int *d_counts, int *d_inv, void *stream);
int ds_cuda_ep_pairs_dev(ds_cuda_ctx_t *ctx, int n_rows, int top_k, int n_ranks, const int *recv_counts,
                         const uint16_t *d_payload, int hidden, int *d_pair_row, int *d_pair_expert, int *d_counts,
                         void *stream);
/* Expert-parallel prefill through the C ABI (no counterpart in the
 * reference, which runs ds_decoder_prefill's MoE block, ds_moe_decoder.c:
 * 630-809, on one host). One process per GPU; each context joins a group of
 * `world` ranks (1..8) sharing a 128-byte id that rank 0 makes with
 * ds_cuda_ep_unique_id and hands to the others out of band (as for NCCL).
 * The library loads NCCL at run time (libnccl.so.2, or $DS_CUDA_NCCL_LIB).
 * ds_cuda_prefill_moe_ep then runs one MoE layer on this rank's n_tokens
 * rows of d_x (updated in place; the ranks' rows together are the batch,
 * in rank order): routing, the token rows sent once to each rank owning one
 * of their experts (experts in contiguous blocks of n_experts / world), the
 * shared expert on local rows while the rows travel, the routed experts,
 * the outputs sent back, and the combine — the same arithmetic as
 * ds_cuda_prefill_moe_dev, so the result is bit-identical to one GPU. Every
 * rank must call it for every layer (it synchronises its stream twice per
 * call to size the transfers). d_logits / d_top_idx / d_top_w as in
 * ds_cuda_prefill_moe_dev. */
int ds_cuda_ep_unique_id(ds_cuda_ctx_t *ctx, void *id128);
int ds_cuda_ep_init(ds_cuda_ctx_t *ctx, int rank, int world, const void *id128);
int ds_cuda_ep_free(ds_cuda_ctx_t *ctx);
int ds_cuda_prefill_moe_ep(ds_cuda_ctx_t *ctx, const ds_cuda_decoder_config_t *cfg,
                           const ds_cuda_layer_weights_t *layer, float *d_x, int n_tokens, const float *d_logits,
                           int *d_top_idx, float *d_top_w, void *stream);
/* The multi-stream decode GEMM on its own (no counterpart in the
 * reference): d_y [n x N] = d_x [n x K] . d_W^T (+ d_resid), n <= 64 token
 * rows, K % 64 == 0, on the tensor cores with the inputs split into two
 * BF16 planes. d_W is the device copy of a registered weight. */
int ds_cuda_skinny_matmul_dev(ds_cuda_ctx_t *ctx, const float *d_x, int n, int K, const uint16_t *d_W, int N,
                              const float *d_resid, float *d_y, void *stream);
/* Synchronises the context's stream and reports DS_CUDA_ETIMEOUT if a
 * prefill kernel's bounded wait gave up since the last check. */
int ds_cuda_prefill_check(ds_cuda_ctx_t *ctx);
/* Stage timing (no counterpart in the reference): while enabled, prefill
 * calls record CUDA events between their six kernels; stage_ms returns the
 * last call's durations (norm+route, plan, scatter, gate/up GEMM, down GEMM,
 * combine) in ms[6]. */
int ds_cuda_prefill_timing(ds_cuda_ctx_t *ctx, int enable);
int ds_cuda_prefill_stage_ms(ds_cuda_ctx_t *ctx, float *ms);

/* ---------------------------------------------------------------------
 * Host-side synthetic data (seeded, counter-based: value i of a stream
 * depends only on (seed, i)); used to build the benchmark workloads.
 * normal_bf16: RNE-rounded N(mean, std); normal_f32: F32 N(mean, std);
 * normal_f32_bf16exact: F32 values that are exactly BF16-representable.
 * --------------------------------------------------------------------- */
void ds_synth_normal_bf16(uint16_t *out, size_t n, uint64_t seed, float mean, float stddev);
void ds_synth_normal_f32(float *out, size_t n, uint64_t seed, float mean, float stddev);
void ds_synth_normal_f32_bf16exact(float *out, size_t n, uint64_t seed, float mean, float stddev);

#ifdef __cplusplus
}
#endif
#endif /* DS_CUDA_H */
