/*
 * ref_harness.c — drives the UNMODIFIED reference sources (compiled from
 * the reference tree by oracle/Makefile) on caller-supplied synthetic
 * weights, so that the restated oracle and the CUDA path can be checked
 * against the reference's own code.
 *
 * Test infrastructure only (oracle/_ref/libdsref.so): the product never
 * links or loads this file.
 *
 * The reference's decode-path functions are `static` in ds_moe_decoder.c
 * (moe_forward :131, decoder_layer_forward :339), so this translation unit
 * includes that file to reach them. The decoder context is built by hand
 * the way alloc_decoder_buffers (ds_ocr.c:847-961) builds it, with the
 * expert layout of load_all_weights (ds_ocr.c:696-768).
 */
#include "ds_safetensors.h"
#include "ds_moe_decoder.c"
#include "ds_quantize.h"
#include <cblas.h>

int ds_verbose = 0;
int ds_bf16_simulate_python = 0;

void ref_set_threads(int n) {
    ds_set_threads(n);
    openblas_set_num_threads(n < 1 ? 1 : n);
}
int ref_get_threads(void) { return ds_get_threads(); }
void ref_set_simulate(int on) { ds_bf16_simulate_python = on ? 1 : 0; }

/* Per-layer weight pointers, in this fixed order (see ref_ctx_set_layer). */
enum {
    RW_WQ = 0, RW_WK, RW_WV, RW_WO, RW_IN_NORM, RW_POST_NORM,
    RW_DENSE_GATE, RW_DENSE_UP, RW_DENSE_DOWN,
    RW_ROUTER, RW_EXPERT_BLOCK, RW_DOWN, RW_SHARED_DOWN,
    RW_COUNT
};

int ref_layer_slot_count(void) { return RW_COUNT; }

void *ref_ctx_new(int n_layers, int kv_max, int vocab) {
    ds_ctx_t *ctx = (ds_ctx_t *)calloc(1, sizeof(ds_ctx_t));
    if (!ctx) return NULL;
    ds_config_t *cfg = &ctx->config;
    cfg->model_version = 2;
    cfg->sliding_window_size = 0;
    cfg->dec_hidden = DS_DEC_HIDDEN;
    cfg->dec_layers = n_layers;
    cfg->dec_heads = DS_DEC_HEADS;
    cfg->dec_kv_heads = DS_DEC_KV_HEADS;
    cfg->dec_head_dim = DS_DEC_HEAD_DIM;
    cfg->dec_intermediate = DS_DEC_INTERMEDIATE;
    cfg->dec_moe_inter = DS_DEC_MOE_INTER;
    cfg->dec_n_routed_experts = DS_DEC_NUM_EXPERTS;
    cfg->dec_n_shared_experts = DS_DEC_SHARED_EXPERTS;
    cfg->dec_top_k = DS_DEC_TOP_K;
    cfg->dec_first_k_dense = DS_DEC_FIRST_K_DENSE;
    cfg->vocab_size = vocab;
    cfg->dec_rms_norm_eps = 1e-6f;
    cfg->dec_rope_theta = 10000.0f;

    int hidden = cfg->dec_hidden, head_dim = cfg->dec_head_dim;
    int kv_dim = cfg->dec_kv_heads * head_dim;
    int inter = cfg->dec_intermediate, moe_inter = cfg->dec_moe_inter;
    int shared_inter = cfg->dec_n_shared_experts * moe_inter;

    ctx->kv_cache_max = kv_max;
    ctx->kv_cache_len = 0;
    int stride = (kv_dim + 15) & ~15;
    size_t kv_total = (size_t)n_layers * kv_max * stride * sizeof(float);
    if (posix_memalign((void **)&ctx->kv_cache_k, 64, kv_total) != 0) return NULL;
    if (posix_memalign((void **)&ctx->kv_cache_v, 64, kv_total) != 0) return NULL;
    memset(ctx->kv_cache_k, 0, kv_total);
    memset(ctx->kv_cache_v, 0, kv_total);
    ctx->_kv_row_stride = stride;

#define RA(n) (float *)calloc((size_t)(n), sizeof(float))
    ctx->dec_x = RA(hidden); ctx->dec_x_norm = RA(hidden);
    ctx->dec_q = RA(kv_dim); ctx->dec_k = RA(kv_dim); ctx->dec_v = RA(kv_dim);
    ctx->dec_attn_out = RA(kv_dim); ctx->dec_proj_out = RA(hidden);
    ctx->dec_expert_out = RA(hidden); ctx->dec_shared_out = RA(hidden);
    ctx->dec_layer_out = RA(hidden);
    ctx->dec_gate_scores = RA(cfg->dec_n_routed_experts);
    ctx->dec_logits = RA(vocab);
    ctx->token_history_cap = kv_max + 512;
    ctx->token_history = (int *)calloc(ctx->token_history_cap, sizeof(int));
    ctx->dec_dense_gate = RA(inter); ctx->dec_dense_up = RA(inter);
    ctx->dec_dense_swiglu = RA(inter); ctx->dec_dense_out = RA(hidden);
    ctx->moe_expert_gate_buf = RA(moe_inter); ctx->moe_expert_up_buf = RA(moe_inter);
    ctx->moe_expert_gate_up_buf = RA(2 * moe_inter);
    ctx->moe_expert_hidden_buf = RA(moe_inter);
    ctx->moe_expert_outputs = RA(cfg->dec_top_k * hidden);
    ctx->moe_shared_gate_buf = RA(shared_inter); ctx->moe_shared_up_buf = RA(shared_inter);
    ctx->moe_shared_gate_up_buf = RA(2 * shared_inter);
    ctx->moe_shared_swiglu_buf = RA(shared_inter);
    ctx->moe_shared_out_buf = RA(hidden);
#undef RA

    ctx->rope_cache_cap = kv_max;
    ctx->rope_cache_cos = (float *)malloc((size_t)kv_max * head_dim * sizeof(float));
    ctx->rope_cache_sin = (float *)malloc((size_t)kv_max * head_dim * sizeof(float));
    int *pos = (int *)malloc(kv_max * sizeof(int));
    for (int i = 0; i < kv_max; i++) pos[i] = i;
    ds_compute_rope_neox(ctx->rope_cache_cos, ctx->rope_cache_sin, pos, kv_max,
                         head_dim, cfg->dec_rope_theta);
    free(pos);

    ctx->max_new_tokens = 4096;
    ctx->temperature = 0.0f;
    ctx->repeat_penalty = 1.0f;
    ctx->no_repeat_ngram_size = 0;
    ctx->metal_ctx = NULL;
    return ctx;
}

void ref_ctx_set_layer(void *vctx, int l, void **w) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ds_config_t *cfg = &ctx->config;
    ds_dec_layer_t *ly = &ctx->decoder.layers[l];
    int hidden = cfg->dec_hidden, moe_inter = cfg->dec_moe_inter;
    int shared_inter = cfg->dec_n_shared_experts * moe_inter;
    ly->wq_weight_bf16 = (uint16_t *)w[RW_WQ];
    ly->wk_weight_bf16 = (uint16_t *)w[RW_WK];
    ly->wv_weight_bf16 = (uint16_t *)w[RW_WV];
    ly->wo_weight_bf16 = (uint16_t *)w[RW_WO];
    ly->input_norm = (float *)w[RW_IN_NORM];
    ly->post_attn_norm = (float *)w[RW_POST_NORM];
    ly->q_norm_weight = NULL;
    ly->k_norm_weight = NULL;
    ly->dense_gate_weight_bf16 = (uint16_t *)w[RW_DENSE_GATE];
    ly->dense_up_weight_bf16 = (uint16_t *)w[RW_DENSE_UP];
    ly->dense_down_weight_bf16 = (uint16_t *)w[RW_DENSE_DOWN];
    ly->gate_weight_bf16 = (uint16_t *)w[RW_ROUTER];
    uint16_t *block = (uint16_t *)w[RW_EXPERT_BLOCK];
    uint16_t *down = (uint16_t *)w[RW_DOWN];
    if (block) {
        size_t fused = (size_t)2 * moe_inter * hidden;
        ly->expert_block_bf16 = block;
        ly->expert_block_size = ((size_t)cfg->dec_n_routed_experts * fused +
                                 (size_t)2 * shared_inter * hidden) * sizeof(uint16_t);
        for (int e = 0; e < cfg->dec_n_routed_experts; e++) {
            uint16_t *p = block + (size_t)e * fused;
            ly->experts[e].gate_up_fused_bf16 = p;
            ly->experts[e].gate_weight_bf16 = p;
            ly->experts[e].up_weight_bf16 = p + (size_t)moe_inter * hidden;
            ly->experts[e].down_weight_bf16 = down + (size_t)e * hidden * moe_inter;
        }
        uint16_t *sp = block + (size_t)cfg->dec_n_routed_experts * fused;
        ly->shared_gate_up_fused_bf16 = sp;
        ly->shared_gate_weight_bf16 = sp;
        ly->shared_up_weight_bf16 = sp + (size_t)shared_inter * hidden;
        ly->shared_down_weight_bf16 = (uint16_t *)w[RW_SHARED_DOWN];
    }
}

void ref_ctx_set_head(void *vctx, const float *final_norm, const uint16_t *lm_head) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ctx->decoder.norm = (float *)final_norm;
    ctx->decoder.lm_head_bf16 = (uint16_t *)lm_head;
    ctx->decoder.tok_embeddings_bf16 = (uint16_t *)lm_head;
}

/* The --int4 switch (main.c:137-140) calls ds_quantize_moe_int4
 * (ds_ocr.c:781-841), which lives in ds_ocr.c with the whole model loader;
 * its loop is repeated here over the reference's ds_int4_quantize_bf16:
 * every routed expert's gate_up [2I x H] and down [H x I], the shared
 * gate_up [2S x H] and down [H x S]; dense layers are skipped. */
int ref_ctx_quantize(void *vctx) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ds_config_t *cfg = &ctx->config;
    int mi = cfg->dec_moe_inter, h = cfg->dec_hidden;
    int si = cfg->dec_n_shared_experts * mi;
    ctx->int4_enabled = 1;
    for (int l = 0; l < cfg->dec_layers; l++) {
        ds_dec_layer_t *ly = &ctx->decoder.layers[l];
        if (l >= cfg->dec_first_k_dense) {
            for (int e = 0; e < cfg->dec_n_routed_experts; e++) {
                if (ly->experts[e].gate_up_fused_bf16)
                    ds_int4_quantize_bf16(&ly->experts_int4[e].gate_up_fused,
                                          ly->experts[e].gate_up_fused_bf16, 2 * mi, h);
                if (ly->experts[e].down_weight_bf16)
                    ds_int4_quantize_bf16(&ly->experts_int4[e].down_weight,
                                          ly->experts[e].down_weight_bf16, h, mi);
            }
            if (ly->shared_gate_up_fused_bf16)
                ds_int4_quantize_bf16(&ly->shared_gate_up_int4, ly->shared_gate_up_fused_bf16, 2 * si, h);
            if (ly->shared_down_weight_bf16)
                ds_int4_quantize_bf16(&ly->shared_down_int4, ly->shared_down_weight_bf16, h, si);
        }
        ly->int4_enabled = 1;
    }
    return 0;
}

/* Copy one quantised block out: which 0 = expert gate_up, 1 = expert down,
 * 2 = shared gate_up, 3 = shared down. */
int ref_ctx_int8_block(void *vctx, int l, int which, int e,
                       int8_t *q, float *scale, float *off) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ds_dec_layer_t *ly = &ctx->decoder.layers[l];
    ds_int4_block_t *b = NULL;
    if (which == 0) b = &ly->experts_int4[e].gate_up_fused;
    else if (which == 1) b = &ly->experts_int4[e].down_weight;
    else if (which == 2) b = &ly->shared_gate_up_int4;
    else b = &ly->shared_down_int4;
    if (!b->qweight) return -1;
    memcpy(q, b->qweight, (size_t)b->out_dim * b->in_dim);
    memcpy(scale, b->scale, (size_t)b->out_dim * sizeof(float));
    memcpy(off, b->offset, (size_t)b->out_dim * sizeof(float));
    return 0;
}

void ref_ctx_kv_set(void *vctx, int l, int pos0, int n, const float *k, const float *v) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    int kv_dim = ctx->config.dec_kv_heads * ctx->config.dec_head_dim;
    for (int i = 0; i < n; i++) {
        memcpy(ds_kv_k_row(ctx, l, pos0 + i), k + (size_t)i * kv_dim, kv_dim * sizeof(float));
        memcpy(ds_kv_v_row(ctx, l, pos0 + i), v + (size_t)i * kv_dim, kv_dim * sizeof(float));
    }
}

void ref_ctx_kv_get(void *vctx, int l, int pos0, int n, float *k, float *v) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    int kv_dim = ctx->config.dec_kv_heads * ctx->config.dec_head_dim;
    for (int i = 0; i < n; i++) {
        memcpy(k + (size_t)i * kv_dim, ds_kv_k_row(ctx, l, pos0 + i), kv_dim * sizeof(float));
        memcpy(v + (size_t)i * kv_dim, ds_kv_v_row(ctx, l, pos0 + i), kv_dim * sizeof(float));
    }
}

void ref_ctx_set_len(void *vctx, int len) { ((ds_ctx_t *)vctx)->kv_cache_len = len; }
int ref_ctx_get_len(void *vctx) { return ((ds_ctx_t *)vctx)->kv_cache_len; }

/* One greedy decode step (ds_decoder_forward, ds_moe_decoder.c:911).
 * If final_x is non-NULL it receives the final RMS-normed hidden state that
 * fed the LM head. */
int ref_decoder_step(void *vctx, const float *embed, float *final_x, float *logit) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    int tok = ds_decoder_forward(ctx, embed);
    int hidden = ctx->config.dec_hidden;
    const float *x = (ctx->config.dec_layers % 2 == 0) ? ctx->dec_x : ctx->dec_layer_out;
    if (final_x) memcpy(final_x, x, hidden * sizeof(float));
    if (logit) *logit = ds_bf16_dot_row(x, ctx->decoder.lm_head_bf16, hidden, tok);
    return tok;
}

/* Sampling settings read by ds_decoder_forward's LM head
 * (ds_moe_decoder.c:1021-1263); the CLI sets them from its flags
 * (main.c:132-134). */
void ref_ctx_set_sampling(void *vctx, float repeat_penalty, int no_repeat_ngram_size, float temperature) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ctx->repeat_penalty = repeat_penalty;
    ctx->no_repeat_ngram_size = no_repeat_ngram_size;
    ctx->temperature = temperature;
}

/* Replace the generated-token history (ds_ctx_t.token_history). */
int ref_ctx_set_history(void *vctx, const int *tokens, int n) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    if (n < 0 || n > ctx->token_history_cap) return -1;
    if (n) memcpy(ctx->token_history, tokens, (size_t)n * sizeof(int));
    ctx->token_history_len = n;
    return 0;
}

int ref_ctx_get_history(void *vctx, int *out, int cap) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    int n = ctx->token_history_len < cap ? ctx->token_history_len : cap;
    if (n > 0) memcpy(out, ctx->token_history, (size_t)n * sizeof(int));
    return ctx->token_history_len;
}

/* One step of the generation loop: ds_decoder_forward, then the produced
 * token appended to the history as ds_ocr.c:2245-2248 does. */
int ref_decoder_step_gen(void *vctx, const float *embed) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    int tok = ds_decoder_forward(ctx, embed);
    if (ctx->token_history_len < ctx->token_history_cap) ctx->token_history[ctx->token_history_len++] = tok;
    return tok;
}

/* V3's reference sliding-window attention: cfg->sliding_window_size and
 * ctx->prefill_token_count, read by decoder_layer_forward
 * (ds_moe_decoder.c:409-436). */
void ref_ctx_set_window(void *vctx, int sliding_window_size, int prefill_token_count) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ctx->config.sliding_window_size = sliding_window_size;
    ctx->prefill_token_count = prefill_token_count;
}

/* The reference's safetensors reader (ds_safetensors.c) on a checkpoint
 * directory: tensor count, and one tensor's metadata (1 found, 0 absent,
 * -1 the directory did not open). */
int ref_st_count(const char *dir) {
    multi_safetensors_t *ms = multi_safetensors_open(dir);
    if (!ms) return -1;
    int n = 0;
    for (int s = 0; s < ms->num_shards; s++) n += ms->shards[s]->num_tensors;
    multi_safetensors_close(ms);
    return n;
}

int ref_st_find(const char *dir, const char *name, int *dtype, int *ndim, int64_t *shape8, size_t *off,
                size_t *size) {
    multi_safetensors_t *ms = multi_safetensors_open(dir);
    if (!ms) return -1;
    safetensors_file_t *sf = NULL;
    const safetensor_t *t = multi_safetensors_find(ms, name, &sf);
    int found = t != NULL;
    if (t) {
        *dtype = t->dtype;
        *ndim = t->ndim;
        for (int i = 0; i < t->ndim && i < 8; i++) shape8[i] = t->shape[i];
        *off = t->data_offset;
        *size = t->data_size;
    }
    multi_safetensors_close(ms);
    return found;
}

/* ds_decoder_prefill (ds_moe_decoder.c:480-905) on T input embeddings at
 * the current cache length; returns the first generated token, the strict
 * '>' argmax of the logits it leaves in ctx->dec_logits (the generation
 * loop's pick, ds_ocr.c), and its logit. */
int ref_decoder_prefill(void *vctx, const float *embeds, int T, float *logit) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ds_decoder_prefill(ctx, embeds, T);
    const float *lg = ctx->dec_logits;
    int tok = 0;
    float best = lg[0];
    for (int i = 1; i < ctx->config.vocab_size; i++)
        if (lg[i] > best) { best = lg[i]; tok = i; }
    if (logit) *logit = best;
    return tok;
}

/* Seeds the C library generator that the temperature path draws from. */
void ref_srand(unsigned seed) { srand(seed); }

/* One decoder layer (decoder_layer_forward, ds_moe_decoder.c:339): writes the
 * K/V row at kv_cache_len, attends over kv_cache_len+1 keys. */
void ref_layer_forward(void *vctx, int l, const float *x, float *out) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    decoder_layer_forward(ctx, x, out, l, ctx->kv_cache_len);
}

/* moe_forward (ds_moe_decoder.c:131) on layer l; x is the post-attention
 * RMS-normed hidden state. */
void ref_moe_forward(void *vctx, int l, float *out, const float *x) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    mlp_forward(out, x, &ctx->decoder.layers[l], &ctx->config, NULL, l,
                ctx->dec_dense_gate, ctx->dec_dense_up, ctx->dec_dense_swiglu,
                ctx->moe_expert_gate_buf, ctx->moe_expert_up_buf,
                ctx->moe_expert_gate_up_buf, ctx->moe_expert_hidden_buf,
                ctx->moe_shared_gate_buf, ctx->moe_shared_up_buf,
                ctx->moe_shared_gate_up_buf, ctx->moe_shared_swiglu_buf,
                ctx->moe_shared_out_buf, ctx->moe_expert_outputs);
}

int ref_argmax(const float *x, const uint16_t *W, int in_dim, int out_dim, float *val) {
    int tok = ds_argmax_matvec_bf16(x, W, in_dim, out_dim);
    if (val) *val = ds_bf16_dot_row(x, W, in_dim, tok);
    return tok;
}

void ref_matvec(float *y, const float *x, const uint16_t *W, int in_dim, int out_dim) {
    ds_linear_nobias_bf16(y, x, W, 1, in_dim, out_dim);
}

void ref_rms_norm(float *out, const float *x, const float *w, int rows, int hidden) {
    ds_rms_norm(out, x, w, rows, hidden, 1e-6f);
}

int ref_quantize(const uint16_t *W, int out_dim, int in_dim, int8_t *q, float *scale, float *off) {
    ds_int4_block_t b;
    if (ds_int4_quantize_bf16(&b, W, out_dim, in_dim) != 0) return -1;
    memcpy(q, b.qweight, (size_t)out_dim * in_dim);
    memcpy(scale, b.scale, out_dim * sizeof(float));
    memcpy(off, b.offset, out_dim * sizeof(float));
    ds_int4_block_free(&b);
    return 0;
}

void ref_int8_matvec(float *y, const float *x, const int8_t *q, const float *scale,
                     const float *off, int out_dim, int in_dim) {
    ds_int4_block_t b;
    memset(&b, 0, sizeof(b));
    b.qweight = (int8_t *)q; b.scale = (float *)scale; b.offset = (float *)off;
    b.out_dim = out_dim; b.in_dim = in_dim;
    ds_int4_matvec(y, x, &b);
}

float ref_fast_expf(float x) { return ds_fast_expf(x); }

/*
 * Batched MoE prefill block for one MoE layer: the reference's own steps at
 * ds_moe_decoder.c:598-801, restated here as a callable (they sit inline in
 * ds_decoder_prefill) and run on the reference's kernels:
 *   x_norm = RMSNorm(x; post_attn_norm)                 (:598)
 *   scores = x_norm · W_r^T   (cblas via ds_linear_nobias_bf16, :644)
 *            — or the caller's logits when logits != NULL (benchmark
 *            config 4 overrides the router logits)
 *   softmax (fast exp) + strict-> top-k per token        (:652-686)
 *   shared = down(SwiGLU(gate, up))  batched sgemm       (:695-710)
 *   per expert e, tokens in order: gather → gate, up sgemm → SwiGLU →
 *            down sgemm → scatter-add w·out               (:719-791)
 *   x += routed + shared                                  (:794-801)
 * Optional outputs: top-k indices and weights per token.
 */
void ref_prefill_moe(void *vctx, int l, float *x, int seq_len, const float *logits,
                     int *top_idx_out, float *top_w_out) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    ds_config_t *cfg = &ctx->config;
    ds_dec_layer_t *layer = &ctx->decoder.layers[l];
    int hidden = cfg->dec_hidden;
    int n_experts = cfg->dec_n_routed_experts;
    int top_k = cfg->dec_top_k;
    int moe_inter = cfg->dec_moe_inter;
    int shared_inter = cfg->dec_n_shared_experts * moe_inter;

    float *x_norm = (float *)malloc((size_t)seq_len * hidden * sizeof(float));
    ds_rms_norm(x_norm, x, layer->post_attn_norm, seq_len, hidden, cfg->dec_rms_norm_eps);

    float *gate_scores = (float *)malloc((size_t)seq_len * n_experts * sizeof(float));
    if (logits)
        memcpy(gate_scores, logits, (size_t)seq_len * n_experts * sizeof(float));
    else
        ds_linear_nobias_bf16(gate_scores, x_norm, layer->gate_weight_bf16,
                              seq_len, hidden, n_experts);

    int *all_idx = (int *)malloc((size_t)seq_len * top_k * sizeof(int));
    float *all_w = (float *)malloc((size_t)seq_len * top_k * sizeof(float));
    for (int s = 0; s < seq_len; s++) {
        float *sc = gate_scores + (size_t)s * n_experts;
        float max_s = -1e30f;
        for (int e = 0; e < n_experts; e++) if (sc[e] > max_s) max_s = sc[e];
        float sum_exp = 0.0f;
        for (int e = 0; e < n_experts; e++) { sc[e] = ds_fast_expf(sc[e] - max_s); sum_exp += sc[e]; }
        float inv = 1.0f / sum_exp;
        for (int e = 0; e < n_experts; e++) sc[e] *= inv;
        int *ti = all_idx + (size_t)s * top_k;
        float *tw = all_w + (size_t)s * top_k;
        for (int k = 0; k < top_k; k++) {
            int best = -1; float bs = -1e30f;
            for (int e = 0; e < n_experts; e++) {
                int already = 0;
                for (int j = 0; j < k; j++) if (ti[j] == e) { already = 1; break; }
                if (already) continue;
                if (sc[e] > bs) { bs = sc[e]; best = e; }
            }
            ti[k] = best; tw[k] = bs;
        }
    }
    if (top_idx_out) memcpy(top_idx_out, all_idx, (size_t)seq_len * top_k * sizeof(int));
    if (top_w_out) memcpy(top_w_out, all_w, (size_t)seq_len * top_k * sizeof(float));

    float *s_gate = (float *)malloc((size_t)seq_len * shared_inter * sizeof(float));
    float *s_up = (float *)malloc((size_t)seq_len * shared_inter * sizeof(float));
    float *s_sw = (float *)malloc((size_t)seq_len * shared_inter * sizeof(float));
    float *shared_out = (float *)malloc((size_t)seq_len * hidden * sizeof(float));
    ds_linear_nobias_bf16(s_gate, x_norm, layer->shared_gate_weight_bf16, seq_len, hidden, shared_inter);
    ds_linear_nobias_bf16(s_up, x_norm, layer->shared_up_weight_bf16, seq_len, hidden, shared_inter);
    ds_swiglu_direct(s_sw, s_gate, s_up, seq_len, shared_inter);
    ds_linear_nobias_bf16(shared_out, s_sw, layer->shared_down_weight_bf16, seq_len, shared_inter, hidden);
    free(s_gate); free(s_up); free(s_sw);

    int *count = (int *)calloc(n_experts, sizeof(int));
    for (int s = 0; s < seq_len; s++)
        for (int k = 0; k < top_k; k++) count[all_idx[(size_t)s * top_k + k]]++;
    int **tok = (int **)malloc(n_experts * sizeof(int *));
    for (int e = 0; e < n_experts; e++) { tok[e] = (int *)malloc((count[e] + 1) * sizeof(int)); count[e] = 0; }
    for (int s = 0; s < seq_len; s++)
        for (int k = 0; k < top_k; k++) { int e = all_idx[(size_t)s * top_k + k]; tok[e][count[e]++] = s; }

    float *routed = (float *)calloc((size_t)seq_len * hidden, sizeof(float));
    for (int e = 0; e < n_experts; e++) {
        int n = count[e];
        if (n == 0) continue;
        float *xe = (float *)malloc((size_t)n * hidden * sizeof(float));
        for (int i = 0; i < n; i++)
            memcpy(xe + (size_t)i * hidden, x_norm + (size_t)tok[e][i] * hidden, hidden * sizeof(float));
        float *g = (float *)malloc((size_t)n * moe_inter * sizeof(float));
        float *u = (float *)malloc((size_t)n * moe_inter * sizeof(float));
        float *sw = (float *)malloc((size_t)n * moe_inter * sizeof(float));
        float *eo = (float *)malloc((size_t)n * hidden * sizeof(float));
        ds_linear_nobias_bf16(g, xe, layer->experts[e].gate_weight_bf16, n, hidden, moe_inter);
        ds_linear_nobias_bf16(u, xe, layer->experts[e].up_weight_bf16, n, hidden, moe_inter);
        ds_swiglu_direct(sw, g, u, n, moe_inter);
        ds_linear_nobias_bf16(eo, sw, layer->experts[e].down_weight_bf16, n, moe_inter, hidden);
        for (int i = 0; i < n; i++) {
            int s = tok[e][i];
            float w = 0.0f;
            for (int k = 0; k < top_k; k++)
                if (all_idx[(size_t)s * top_k + k] == e) { w = all_w[(size_t)s * top_k + k]; break; }
            float *dst = routed + (size_t)s * hidden;
            const float *src = eo + (size_t)i * hidden;
            for (int j = 0; j < hidden; j++) dst[j] += w * src[j];
        }
        free(xe); free(g); free(u); free(sw); free(eo);
    }
    for (size_t i = 0; i < (size_t)seq_len * hidden; i++) x[i] += routed[i] + shared_out[i];

    free(routed); free(shared_out);
    for (int e = 0; e < n_experts; e++) free(tok[e]);
    free(tok); free(count); free(all_idx); free(all_w); free(gate_scores); free(x_norm);
}

void ref_ctx_free(void *vctx) {
    ds_ctx_t *ctx = (ds_ctx_t *)vctx;
    if (!ctx) return;
    for (int l = 0; l < ctx->config.dec_layers; l++) {
        ds_dec_layer_t *ly = &ctx->decoder.layers[l];
        for (int e = 0; e < DS_MAX_EXPERTS; e++) {
            ds_int4_block_free(&ly->experts_int4[e].gate_up_fused);
            ds_int4_block_free(&ly->experts_int4[e].down_weight);
        }
        ds_int4_block_free(&ly->shared_gate_up_int4);
        ds_int4_block_free(&ly->shared_down_int4);
    }
    free(ctx->kv_cache_k); free(ctx->kv_cache_v);
    free(ctx->dec_x); free(ctx->dec_x_norm); free(ctx->dec_q); free(ctx->dec_k); free(ctx->dec_v);
    free(ctx->dec_attn_out); free(ctx->dec_proj_out); free(ctx->dec_expert_out);
    free(ctx->dec_shared_out); free(ctx->dec_layer_out); free(ctx->dec_gate_scores);
    free(ctx->dec_logits); free(ctx->token_history); free(ctx->lm_head_f32);
    free(ctx->dec_dense_gate); free(ctx->dec_dense_up); free(ctx->dec_dense_swiglu); free(ctx->dec_dense_out);
    free(ctx->moe_expert_gate_buf); free(ctx->moe_expert_up_buf); free(ctx->moe_expert_gate_up_buf);
    free(ctx->moe_expert_hidden_buf); free(ctx->moe_expert_outputs);
    free(ctx->moe_shared_gate_buf); free(ctx->moe_shared_up_buf); free(ctx->moe_shared_gate_up_buf);
    free(ctx->moe_shared_swiglu_buf); free(ctx->moe_shared_out_buf);
    free(ctx->rope_cache_cos); free(ctx->rope_cache_sin);
    free(ctx);
}
