/*
 * ds_oracle.c — CPU restatement of ds-ocr's MoE-decoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see ds_oracle.h): the checker for the CUDA path,
 * never part of the product. Each function names the reference lines it
 * restates; paths are relative to the reference project root.
 *
 * Built with -ffp-contract=off so that every fused multiply-add below is an
 * explicit fmaf() where the reference's gcc -O3 -march=native build fuses.
 */
#include "ds_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

/* ds_kernels.h:296-302 — Schraudolph (1999) exp; the reference's compiler
 * fuses 12102203*x + 1064866805 into one FMA (verified against the compiled
 * reference in tests/test_oracle_vs_ref.py). */
float orc_fast_expf(float x) {
    if (x < -88.0f) return 0.0f;
    if (x > 88.0f) return 1e38f;
    union { uint32_t i; float f; } u;
    u.i = (uint32_t)fmaf(12102203.0f, x, 1064866805.0f);
    return u.f;
}

/* ds_kernels.c:2464-2492 — F32 -> BF16 -> F32, rounding half away on the
 * magnitude: (u + 0x8000) & 0xFFFF0000. */
float orc_bf16_roundtrip(float x) {
    union { uint32_t i; float f; } u;
    u.f = x;
    u.i = (u.i + 0x8000u) & 0xFFFF0000u;
    return u.f;
}

static inline float bf16f(uint16_t h) {
    union { uint32_t i; float f; } u;
    u.i = ((uint32_t)h) << 16;
    return u.f;
}

/* One BF16-row x F32-vector dot in the reference's AVX-512 order
 * (ds_kernels_avx.c:25-155): 16 lanes, two accumulators for even/odd
 * 16-column halves of each 32-column step, then a 16-wide tail. */
static float dot_bf16(const uint16_t *w, const float *x, int n) {
    float a0[16], a1[16];
    for (int l = 0; l < 16; l++) { a0[l] = 0.0f; a1[l] = 0.0f; }
    int k = 0;
    for (; k + 32 <= n; k += 32)
        for (int l = 0; l < 16; l++) {
            a0[l] = fmaf(bf16f(w[k + l]), x[k + l], a0[l]);
            a1[l] = fmaf(bf16f(w[k + 16 + l]), x[k + 16 + l], a1[l]);
        }
    for (; k + 16 <= n; k += 16)
        for (int l = 0; l < 16; l++) a0[l] = fmaf(bf16f(w[k + l]), x[k + l], a0[l]);
    float s = 0.0f;
    for (int l = 0; l < 16; l++) s += a0[l] + a1[l];
    for (; k < n; k++) s = fmaf(bf16f(w[k]), x[k], s);
    return s;
}

/* ds_linear_nobias_bf16 at seq_len 1 (ds_kernels.c:917-927 -> :820-828 ->
 * ds_bf16_matvec_fused_avx): y[o] = sum_k bf16(W[o,k]) * x[k]. */
void orc_matvec_bf16(float *y, const float *x, const uint16_t *W, int in_dim, int out_dim) {
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; o++) y[o] = dot_bf16(W + (size_t)o * in_dim, x, in_dim);
}

float orc_dot_bf16_row(const float *x, const uint16_t *W, int in_dim, int row) {
    return dot_bf16(W + (size_t)row * in_dim, x, in_dim);
}

/* ds_argmax_matvec_bf16 (ds_kernels.c:1013-1099, ds_kernels_avx.c:157-249):
 * argmax over rows of W.x, strict '>' so the lowest index wins ties. */
int orc_argmax_bf16(const float *x, const uint16_t *W, int in_dim, int out_dim, float *val) {
    int best = 0;
    float best_val = -1e30f;
    for (int o = 0; o < out_dim; o++) {
        float s = dot_bf16(W + (size_t)o * in_dim, x, in_dim);
        if (s > best_val) { best_val = s; best = o; }
    }
    if (val) *val = best_val;
    return best;
}

/* Router softmax + top-k, ds_moe_decoder.c:157-183 (prefill copy :652-686):
 * max, fast-exp, sequential sum, multiply by 1/sum; then k selection passes,
 * strict '>', skipping chosen experts. Weights are the raw probabilities;
 * renorm=1 divides them by their sum (what the docs describe, not the code). */
void orc_router_topk(const float *logits, int n_experts, int top_k, int renorm,
                     int *idx, float *w) {
    float p[256];
    float mx = -1e30f;
    for (int e = 0; e < n_experts; e++) if (logits[e] > mx) mx = logits[e];
    float sum = 0.0f;
    for (int e = 0; e < n_experts; e++) { p[e] = orc_fast_expf(logits[e] - mx); sum += p[e]; }
    float inv = 1.0f / sum;
    for (int e = 0; e < n_experts; e++) p[e] *= inv;
    for (int k = 0; k < top_k; k++) {
        int best = -1;
        float bs = -1e30f;
        for (int e = 0; e < n_experts; e++) {
            int taken = 0;
            for (int j = 0; j < k; j++) if (idx[j] == e) { taken = 1; break; }
            if (taken) continue;
            if (p[e] > bs) { bs = p[e]; best = e; }
        }
        idx[k] = best;
        w[k] = bs;
    }
    if (renorm) {
        float s = 0.0f;
        for (int k = 0; k < top_k; k++) s += w[k];
        for (int k = 0; k < top_k; k++) w[k] /= s;
    }
}

/* ds_swiglu_direct, non-Apple branch (ds_kernels.c:1770-1773):
 * out = (g / (1 + fast_exp(-g))) * u. */
void orc_swiglu(float *out, const float *g, const float *u, int n) {
    for (int j = 0; j < n; j++) out[j] = (g[j] / (1.0f + orc_fast_expf(-g[j]))) * u[j];
}

static void trunc_arr(float *a, int n) { for (int i = 0; i < n; i++) a[i] = orc_bf16_roundtrip(a[i]); }

/* ds_expert_forward_fused (ds_kernels.c:322-357): gate_up matvec, split,
 * [trunc], SwiGLU, [trunc], down matvec, [trunc]. */
void orc_expert_fused(float *out, const float *x, const uint16_t *gu, const uint16_t *down,
                      int hidden, int inter, int simulate) {
    float *gub = (float *)malloc((size_t)2 * inter * sizeof(float));
    float *h = (float *)malloc((size_t)inter * sizeof(float));
    orc_matvec_bf16(gub, x, gu, hidden, 2 * inter);
    if (simulate) trunc_arr(gub, 2 * inter);
    orc_swiglu(h, gub, gub + inter, inter);
    if (simulate) trunc_arr(h, inter);
    orc_matvec_bf16(out, h, down, inter, hidden);
    if (simulate) trunc_arr(out, hidden);
    free(gub); free(h);
}

/* int8_quantize_row / ds_int4_quantize_bf16 (ds_quantize.c:29-81): per row
 * min, max, scale = max((max-min)/255, 1e-10), q = clamp(roundf((w-min) *
 * (1/scale)), 0, 255) - 128; offset = min. */
int orc_int8_quantize(const uint16_t *W, int out_dim, int in_dim,
                      int8_t *q, float *scale, float *off) {
    if (!W || out_dim <= 0 || in_dim <= 0) return -1;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < out_dim; r++) {
        const uint16_t *row = W + (size_t)r * in_dim;
        float mn = 1e30f, mx = -1e30f;
        for (int c = 0; c < in_dim; c++) {
            float v = bf16f(row[c]);
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        float s = (mx - mn) / 255.0f;
        if (s < 1e-10f) s = 1e-10f;
        scale[r] = s;
        off[r] = mn;
        float inv = 1.0f / s;
        for (int c = 0; c < in_dim; c++) {
            int v = (int)roundf((bf16f(row[c]) - mn) * inv);
            if (v < 0) v = 0;
            if (v > 255) v = 255;
            q[(size_t)r * in_dim + c] = (int8_t)(v - 128);
        }
    }
    return 0;
}

/* int8_matvec_generic (ds_quantize.c:154-169): the rows are split over
 * OpenMP threads; each row's dot and x-sum come from orc_int8_rows
 * (int8_dot.c), compiled with the reference build's flags so its FMA
 * contraction matches the reference's on the build host. */
void orc_int8_rows(float *y, const float *x, const int8_t *q, const float *scale,
                   const float *off, int row0, int row1, int in_dim);

void orc_int8_matvec(float *y, const float *x, const int8_t *q, const float *scale,
                     const float *off, int out_dim, int in_dim) {
#pragma omp parallel
    {
        int nt = omp_get_num_threads(), t = omp_get_thread_num();
        int per = (out_dim + nt - 1) / nt;
        int r0 = t * per, r1 = r0 + per < out_dim ? r0 + per : out_dim;
        if (r0 < r1) orc_int8_rows(y, x, q, scale, off, r0, r1, in_dim);
    }
}

/* ds_expert_forward_fused_int4 (ds_quantize.c:301-321). */
void orc_expert_fused_int8(float *out, const float *x,
                           const int8_t *guq, const float *gus, const float *guo,
                           const int8_t *dnq, const float *dns, const float *dno,
                           int hidden, int inter, int simulate) {
    float *gub = (float *)malloc((size_t)2 * inter * sizeof(float));
    float *h = (float *)malloc((size_t)inter * sizeof(float));
    orc_int8_matvec(gub, x, guq, gus, guo, 2 * inter, hidden);
    if (simulate) trunc_arr(gub, 2 * inter);
    orc_swiglu(h, gub, gub + inter, inter);
    if (simulate) trunc_arr(h, inter);
    orc_int8_matvec(out, h, dnq, dns, dno, hidden, inter);
    if (simulate) trunc_arr(out, hidden);
    free(gub); free(h);
}

/* moe_forward (ds_moe_decoder.c:131-333), CPU branches: router matvec,
 * softmax/top-k, routed experts in top-k order, ds_expert_combine
 * (ds_kernels.c:359-371: out = 0; out += w_k y_k for k = 0..K-1), then the
 * shared expert (fused BF16 branch :287-317, or INT8 branch :269-278) added
 * with ds_vec_add. */
void orc_moe_forward(float *out, const float *x, const orc_layer_t *ly, const orc_dims_t *d,
                     int use_int8, int *idx_out, float *w_out) {
    int H = d->hidden, I = d->moe_inter, S = d->n_shared * d->moe_inter, E = d->n_experts;
    int K = d->top_k;
    float scores[256];
    int idx[64];
    float w[64];
    orc_matvec_bf16(scores, x, ly->router, H, E);
    orc_router_topk(scores, E, K, d->renorm_topk, idx, w);
    if (idx_out) memcpy(idx_out, idx, K * sizeof(int));
    if (w_out) memcpy(w_out, w, K * sizeof(float));

    float *y = (float *)malloc((size_t)K * H * sizeof(float));
    size_t fused = (size_t)2 * I * H;
    for (int k = 0; k < K; k++) {
        int e = idx[k];
        if (use_int8)
            orc_expert_fused_int8(y + (size_t)k * H, x,
                                  ly->gu_q + (size_t)e * fused, ly->gu_scale + (size_t)e * 2 * I,
                                  ly->gu_off + (size_t)e * 2 * I,
                                  ly->dn_q + (size_t)e * H * I, ly->dn_scale + (size_t)e * H,
                                  ly->dn_off + (size_t)e * H, H, I, d->simulate_bf16);
        else
            orc_expert_fused(y + (size_t)k * H, x, ly->expert_block + (size_t)e * fused,
                             ly->down + (size_t)e * H * I, H, I, d->simulate_bf16);
    }
    for (int i = 0; i < H; i++) out[i] = 0.0f;
    for (int k = 0; k < K; k++)
        for (int i = 0; i < H; i++) out[i] = fmaf(w[k], y[(size_t)k * H + i], out[i]);

    float *sh = (float *)malloc((size_t)H * sizeof(float));
    if (use_int8)
        orc_expert_fused_int8(sh, x, ly->sgu_q, ly->sgu_scale, ly->sgu_off,
                              ly->sdn_q, ly->sdn_scale, ly->sdn_off, H, S, d->simulate_bf16);
    else
        orc_expert_fused(sh, x, ly->expert_block + (size_t)E * fused, ly->shared_down, H, S,
                         d->simulate_bf16);
    for (int i = 0; i < H; i++) out[i] = out[i] + sh[i];
    free(y); free(sh);
}

/* ds_rms_norm (ds_kernels.c:1387-1471): inv = 1/sqrtf(sum(x^2)/n + eps);
 * out = (x * w) * inv. */
void orc_rms_norm(float *out, const float *x, const float *w, int n, float eps) {
    float a[16];
    for (int l = 0; l < 16; l++) a[l] = 0.0f;
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 16; l++) a[l] = fmaf(x[i + l], x[i + l], a[l]);
    float ss = 0.0f;
    for (int l = 0; l < 16; l++) ss += a[l];
    for (; i < n; i++) ss = fmaf(x[i], x[i], ss);
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int j = 0; j < n; j++) out[j] = (x[j] * w[j]) * inv;
}

/* ds_residual_rms_norm (ds_kernels.c:1544-1618): out = x + r; norm_out =
 * RMSNorm(out). */
void orc_residual_rms_norm(float *out, float *norm_out, const float *x, const float *r,
                           const float *w, int n, float eps) {
    for (int i = 0; i < n; i++) out[i] = x[i] + r[i];
    orc_rms_norm(norm_out, out, w, n, eps);
}

/* ds_compute_rope_neox (ds_kernels.c:2399-2424) with the positions 0..max-1
 * table of alloc_decoder_buffers (ds_ocr.c:925-941). */
void orc_rope_table(float *cos_t, float *sin_t, int max_pos, int head_dim, float theta) {
    int half = head_dim / 2;
    for (int s = 0; s < max_pos; s++) {
        float pos = (float)s;
        for (int d = 0; d < half; d++) {
            float freq = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
            float ang = pos * freq;
            float c = cosf(ang), sn = sinf(ang);
            cos_t[(size_t)s * head_dim + d] = c;
            cos_t[(size_t)s * head_dim + d + half] = c;
            sin_t[(size_t)s * head_dim + d] = sn;
            sin_t[(size_t)s * head_dim + d + half] = sn;
        }
    }
}

/* ds_apply_rope_neox (ds_kernels.c:2426-2458), split-half rotation. */
void orc_apply_rope(float *vec, const float *c, const float *s, int n_heads, int head_dim) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        float *v = vec + (size_t)h * head_dim;
        for (int d = 0; d < half; d++) {
            float x1 = v[d], x2 = v[d + half];
            v[d] = x1 * c[d] - x2 * s[d];
            v[d + half] = x1 * s[d + half] + x2 * c[d + half];
        }
    }
}

static float dot_f32(const float *a, const float *b, int n) {
    float acc[16];
    for (int l = 0; l < 16; l++) acc[l] = 0.0f;
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 16; l++) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = 0.0f;
    for (int l = 0; l < 16; l++) s += acc[l];
    for (; i < n; i++) s = fmaf(a[i], b[i], s);
    return s;
}

/* Decode attention, MHA fast path of ds_causal_attention_aligned
 * (ds_kernels.c:2181-2249 / worker :2124-2159): per head, a sequential
 * online softmax over keys 0..n_keys-1 with fast exp:
 *   s > m : corr = fexp(m - s); sum = sum*corr + 1; o = o*corr + v; m = s
 *   else  : wt = fexp(s - m);   sum += wt;         o += wt*v
 * then o *= 1/sum. */
void orc_attention_decode(float *out, const float *q, const float *K, const float *V,
                          int n_keys, int n_heads, int head_dim, int kv_stride, float scale) {
#pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; h++) {
        const float *qh = q + (size_t)h * head_dim;
        float *o = out + (size_t)h * head_dim;
        float m = -1e30f, sum = 0.0f;
        for (int d = 0; d < head_dim; d++) o[d] = 0.0f;
        for (int j = 0; j < n_keys; j++) {
            const float *kr = K + (size_t)j * kv_stride + (size_t)h * head_dim;
            const float *vr = V + (size_t)j * kv_stride + (size_t)h * head_dim;
            float s = dot_f32(qh, kr, head_dim) * scale;
            if (s > m) {
                float corr = orc_fast_expf(m - s);
                sum = fmaf(sum, corr, 1.0f);
                for (int d = 0; d < head_dim; d++) o[d] = fmaf(o[d], corr, vr[d]);
                m = s;
            } else {
                float wt = orc_fast_expf(s - m);
                sum += wt;
                for (int d = 0; d < head_dim; d++) o[d] = fmaf(vr[d], wt, o[d]);
            }
        }
        if (sum > 0.0f) {
            float inv = 1.0f / sum;
            for (int d = 0; d < head_dim; d++) o[d] *= inv;
        }
    }
}

/* dense_ffn_forward (ds_moe_decoder.c:75-105): separate gate and up
 * matvecs, SwiGLU, down. */
static void dense_ffn(float *out, const float *x, const orc_layer_t *ly, const orc_dims_t *d) {
    int H = d->hidden, D = d->inter_dense;
    float *g = (float *)malloc((size_t)D * sizeof(float));
    float *u = (float *)malloc((size_t)D * sizeof(float));
    float *h = (float *)malloc((size_t)D * sizeof(float));
    orc_matvec_bf16(g, x, ly->dense_gate, H, D);
    orc_matvec_bf16(u, x, ly->dense_up, H, D);
    orc_swiglu(h, g, u, D);
    orc_matvec_bf16(out, h, ly->dense_down, D, H);
    free(g); free(u); free(h);
}

/* Reference sliding-window attention of V3 decode (R-SWA,
 * ds_moe_decoder.c:409-436 -> ds_rswa_attention_aligned,
 * ds_kernels.c:2255-2314): with window W > 0 and the query at or past the
 * prefill length P, the keys are [0, P) then [max(P, n - W), n), through the
 * same sequential softmax; when the two ranges touch, plain causal. The
 * rows are gathered into a compact copy and attended in that order. */
static void attention_rswa(float *out, const float *q, const float *K, const float *V, int n, int nh, int hd,
                           int stride, float scale, int window, int ref_len, int pos) {
    int ws = ref_len > n - window ? ref_len : n - window;
    if (window <= 0 || pos < ref_len || ws <= ref_len) {
        orc_attention_decode(out, q, K, V, n, nh, hd, stride, scale);
        return;
    }
    int m = ref_len + (n - ws);
    float *Kc = (float *)malloc((size_t)m * stride * sizeof(float));
    float *Vc = (float *)malloc((size_t)m * stride * sizeof(float));
    memcpy(Kc, K, (size_t)ref_len * stride * sizeof(float));
    memcpy(Vc, V, (size_t)ref_len * stride * sizeof(float));
    memcpy(Kc + (size_t)ref_len * stride, K + (size_t)ws * stride, (size_t)(n - ws) * stride * sizeof(float));
    memcpy(Vc + (size_t)ref_len * stride, V + (size_t)ws * stride, (size_t)(n - ws) * stride * sizeof(float));
    orc_attention_decode(out, q, Kc, Vc, m, nh, hd, stride, scale);
    free(Kc);
    free(Vc);
}

/* ds_decoder_forward (ds_moe_decoder.c:911-1264) greedy branch with
 * decoder_layer_forward (:339-474) per layer: input RMSNorm, QKV matvecs,
 * RoPE at `pos`, K/V stored (F32) at row `pos`, attention over pos+1 keys,
 * O-proj, residual + post-attention RMSNorm, dense FFN (layer <
 * first_dense) or MoE, residual add; final RMSNorm; argmax LM head.
 * KV layout [layer][kv_max][H] F32. Returns the token; final_x receives
 * the normed hidden state, logit its LM-head logit. */
int orc_decoder_step(const orc_layer_t *layers, const orc_dims_t *d,
                     const float *final_norm, const uint16_t *lm_head,
                     float *kv_k, float *kv_v, int kv_max, int pos,
                     const float *cos_t, const float *sin_t, int use_int8,
                     const float *embed, float *final_x, float *logit) {
    return orc_decoder_step_swa(layers, d, final_norm, lm_head, kv_k, kv_v, kv_max, pos, cos_t, sin_t, use_int8,
                                embed, final_x, logit, 0, 0);
}

int orc_decoder_step_swa(const orc_layer_t *layers, const orc_dims_t *d,
                         const float *final_norm, const uint16_t *lm_head,
                         float *kv_k, float *kv_v, int kv_max, int pos,
                         const float *cos_t, const float *sin_t, int use_int8,
                         const float *embed, float *final_x, float *logit, int window, int ref_len) {
    int H = d->hidden, hd = d->head_dim, nh = d->n_heads, qd = nh * hd;
    float *x = (float *)malloc((size_t)H * sizeof(float));
    float *xn = (float *)malloc((size_t)H * sizeof(float));
    float *q = (float *)malloc((size_t)qd * sizeof(float));
    float *k = (float *)malloc((size_t)qd * sizeof(float));
    float *v = (float *)malloc((size_t)qd * sizeof(float));
    float *att = (float *)malloc((size_t)qd * sizeof(float));
    float *proj = (float *)malloc((size_t)H * sizeof(float));
    float *o = (float *)malloc((size_t)H * sizeof(float));
    float *mlp = (float *)malloc((size_t)H * sizeof(float));
    memcpy(x, embed, (size_t)H * sizeof(float));
    float scale = 1.0f / sqrtf((float)hd);
    for (int l = 0; l < d->n_layers; l++) {
        const orc_layer_t *ly = &layers[l];
        orc_rms_norm(xn, x, ly->input_norm, H, d->eps);
        orc_matvec_bf16(q, xn, ly->wq, H, qd);
        orc_matvec_bf16(k, xn, ly->wk, H, qd);
        orc_matvec_bf16(v, xn, ly->wv, H, qd);
        orc_apply_rope(q, cos_t + (size_t)pos * hd, sin_t + (size_t)pos * hd, nh, hd);
        orc_apply_rope(k, cos_t + (size_t)pos * hd, sin_t + (size_t)pos * hd, nh, hd);
        float *Kl = kv_k + (size_t)l * kv_max * qd;
        float *Vl = kv_v + (size_t)l * kv_max * qd;
        memcpy(Kl + (size_t)pos * qd, k, (size_t)qd * sizeof(float));
        memcpy(Vl + (size_t)pos * qd, v, (size_t)qd * sizeof(float));
        attention_rswa(att, q, Kl, Vl, pos + 1, nh, hd, qd, scale, window, ref_len, pos);
        orc_matvec_bf16(proj, att, ly->wo, qd, H);
        orc_residual_rms_norm(o, xn, x, proj, ly->post_norm, H, d->eps);
        if (l < d->first_dense) dense_ffn(mlp, xn, ly, d);
        else orc_moe_forward(mlp, xn, ly, d, use_int8, NULL, NULL);
        for (int i = 0; i < H; i++) x[i] = o[i] + mlp[i];
    }
    orc_rms_norm(x, x, final_norm, H, d->eps);
    float val;
    int tok = orc_argmax_bf16(x, lm_head, H, d->vocab, &val);
    if (final_x) memcpy(final_x, x, (size_t)H * sizeof(float));
    if (logit) *logit = val;
    free(x); free(xn); free(q); free(k); free(v); free(att); free(proj); free(o); free(mlp);
    return tok;
}

/* Row-major F32 x BF16^T product for the prefill restatement:
 * Y[n x out] = X[n x in] . W[out x in]^T (the reference does this with
 * cblas_sgemm on a widened copy of W, ds_kernels.c:625-653). */
static void gemm_bf16(float *Y, const float *X, const uint16_t *W, int n, int in_dim, int out_dim) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int r = 0; r < n; r++)
        for (int o = 0; o < out_dim; o++)
            Y[(size_t)r * out_dim + o] = dot_bf16(W + (size_t)o * in_dim, X + (size_t)r * in_dim, in_dim);
}

/* Prefill MoE block of ds_decoder_prefill (ds_moe_decoder.c:598-801):
 * x_norm = RMSNorm(x; post_attn_norm); router logits (caller-supplied when
 * `logits` is non-NULL); per-token softmax/top-k; shared expert with
 * separate gate and up products; routed experts grouped by expert, tokens
 * in order, outputs scattered with their weight in ascending expert order;
 * x += routed + shared. No BF16 truncation on this path. */
void orc_prefill_moe(const orc_layer_t *ly, const orc_dims_t *d, float *x, int seq_len,
                     const float *logits, int *idx_out, float *w_out) {
    int H = d->hidden, I = d->moe_inter, S = d->n_shared * d->moe_inter, E = d->n_experts;
    int K = d->top_k;
    size_t fused = (size_t)2 * I * H;
    float *xn = (float *)malloc((size_t)seq_len * H * sizeof(float));
    for (int s = 0; s < seq_len; s++)
        orc_rms_norm(xn + (size_t)s * H, x + (size_t)s * H, ly->post_norm, H, d->eps);
    float *lg = (float *)malloc((size_t)seq_len * E * sizeof(float));
    if (logits) memcpy(lg, logits, (size_t)seq_len * E * sizeof(float));
    else gemm_bf16(lg, xn, ly->router, seq_len, H, E);
    int *idx = (int *)malloc((size_t)seq_len * K * sizeof(int));
    float *w = (float *)malloc((size_t)seq_len * K * sizeof(float));
    for (int s = 0; s < seq_len; s++)
        orc_router_topk(lg + (size_t)s * E, E, K, d->renorm_topk, idx + (size_t)s * K, w + (size_t)s * K);
    if (idx_out) memcpy(idx_out, idx, (size_t)seq_len * K * sizeof(int));
    if (w_out) memcpy(w_out, w, (size_t)seq_len * K * sizeof(float));

    const uint16_t *sgu = ly->expert_block + (size_t)E * fused;
    float *sg = (float *)malloc((size_t)seq_len * S * sizeof(float));
    float *su = (float *)malloc((size_t)seq_len * S * sizeof(float));
    float *sh = (float *)malloc((size_t)seq_len * H * sizeof(float));
    gemm_bf16(sg, xn, sgu, seq_len, H, S);
    gemm_bf16(su, xn, sgu + (size_t)S * H, seq_len, H, S);
    for (int s = 0; s < seq_len; s++)
        orc_swiglu(sg + (size_t)s * S, sg + (size_t)s * S, su + (size_t)s * S, S);
    gemm_bf16(sh, sg, ly->shared_down, seq_len, S, H);

    float *routed = (float *)calloc((size_t)seq_len * H, sizeof(float));
#pragma omp parallel for schedule(dynamic)
    for (int s = 0; s < seq_len; s++) {
        float g[4096], u[4096], y[4096];
        const float *xs = xn + (size_t)s * H;
        for (int e = 0; e < E; e++) {
            float we = 0.0f;
            int hit = 0;
            for (int k = 0; k < K; k++)
                if (idx[(size_t)s * K + k] == e) { we = w[(size_t)s * K + k]; hit = 1; break; }
            if (!hit) continue;
            const uint16_t *gu = ly->expert_block + (size_t)e * fused;
            for (int i = 0; i < I; i++) {
                g[i] = dot_bf16(gu + (size_t)i * H, xs, H);
                u[i] = dot_bf16(gu + (size_t)(I + i) * H, xs, H);
            }
            orc_swiglu(g, g, u, I);
            const uint16_t *dn = ly->down + (size_t)e * H * I;
            for (int j = 0; j < H; j++) y[j] = dot_bf16(dn + (size_t)j * I, g, I);
            float *dst = routed + (size_t)s * H;
            for (int j = 0; j < H; j++) dst[j] = fmaf(we, y[j], dst[j]);
        }
    }
    for (size_t i = 0; i < (size_t)seq_len * H; i++) x[i] += routed[i] + sh[i];
    free(xn); free(lg); free(idx); free(w); free(sg); free(su); free(sh); free(routed);
}

/* LM-head token selection of ds_decoder_forward with the sampling settings
 * (ds_moe_decoder.c:1021-1263), on the final RMS-normed hidden state xn.
 * hist = the generated tokens so far (ds_ocr.c:2245-2248), in order.
 * temperature <= 0, fast path (:1033-1099): argmax; best value recomputed
 *   by a row dot; repetition penalty rp > 1 applied once to the winner if it
 *   is in the history, then every history token other than the current
 *   winner is scored, penalised and taken on a strict '>' (:1044-1066);
 *   n-gram blocking (:1071-1094): if the winner would complete an n-gram
 *   already in the history, fall through to the full path.
 * full path (:1101-1263): all logits; the penalty once per history
 *   OCCURRENCE (:1186-1198); tokens that complete a seen n-gram set to -1e30
 *   (:1205-1230); strict '>' argmax; temperature > 0: softmax with expf and
 *   a double sum, sampled with the uniform r by a sequential F32 cumulative
 *   sum (:1241-1260).
 * Returns the token; *val = the selected value (penalised logit, before
 * temperature); *full = 1 when the full path ran. */
static float orc_penalise(float v, float rp) { return v > 0 ? v / rp : v * rp; }

static int orc_banned(const int *hist, int len, int ngram, int tok) {
    if (ngram <= 0 || len < ngram - 1) return 0;
    int p = ngram - 1;
    for (int i = 0; i <= len - p - 1; i++) {
        int m = 1;
        for (int j = 0; j < p; j++)
            if (hist[i + j] != hist[len - p + j]) { m = 0; break; }
        if (m && hist[i + p] == tok) return 1;
    }
    return 0;
}

int orc_lm_select(const float *xn, const uint16_t *W, int H, int V, const int *hist, int len, float rp,
                  int ngram, float temperature, float r, float *val, int *full) {
    if (full) *full = 0;
    if (temperature <= 0.0f) {
        int best = orc_argmax_bf16(xn, W, H, V, NULL);
        float bv = orc_dot_bf16_row(xn, W, H, best);
        if (rp > 1.0f && len > 0) {
            for (int i = 0; i < len; i++)
                if (hist[i] == best) { bv = orc_penalise(bv, rp); break; }
            for (int i = 0; i < len; i++) {
                int t = hist[i];
                if (t >= 0 && t < V && t != best) {
                    float v = orc_penalise(orc_dot_bf16_row(xn, W, H, t), rp);
                    if (v > bv) { bv = v; best = t; }
                }
            }
        }
        if (!orc_banned(hist, len, ngram, best)) {
            if (val) *val = bv;
            return best;
        }
    }
    if (full) *full = 1;
    float *lg = (float *)malloc((size_t)V * sizeof(float));
    orc_matvec_bf16(lg, xn, W, H, V);
    if (rp > 1.0f)
        for (int i = 0; i < len; i++)
            if (hist[i] >= 0 && hist[i] < V) lg[hist[i]] = orc_penalise(lg[hist[i]], rp);
    if (ngram > 0 && len >= ngram - 1) {
        int p = ngram - 1;
        for (int i = 0; i <= len - p - 1; i++) {
            int m = 1;
            for (int j = 0; j < p; j++)
                if (hist[i + j] != hist[len - p + j]) { m = 0; break; }
            if (m && hist[i + p] >= 0 && hist[i + p] < V) lg[hist[i + p]] = -1e30f;
        }
    }
    int tok = 0;
    float best = lg[0];
    for (int i = 1; i < V; i++)
        if (lg[i] > best) { best = lg[i]; tok = i; }
    if (val) *val = best;
    if (temperature > 0.0f) {
        double sum = 0.0;
        for (int i = 0; i < V; i++) {
            lg[i] = expf((lg[i] - best) / temperature);
            sum += lg[i];
        }
        float inv = (float)(1.0 / sum);
        float cum = 0.0f;
        tok = V - 1;
        for (int i = 0; i < V; i++) {
            cum += lg[i] * inv;
            if (cum >= r) { tok = i; break; }
        }
    }
    free(lg);
    return tok;
}

/* ds_decoder_prefill (ds_moe_decoder.c:480-905) for T tokens at positions
 * pos0 .. pos0+T-1 (no BF16 truncation): per layer input RMSNorm of every
 * row, Q/K/V GEMMs, RoPE per position, K/V rows stored (F32), causal
 * attention (ds_causal_attention_heads_aligned, ds_kernels.c:2061-2114: the
 * decode rule per query over keys 0 .. pos0+t), O-proj GEMM and residual,
 * then the dense FFN (layer < first_dense: post-attention RMSNorm, gate/up
 * GEMMs, SwiGLU, down GEMM, residual) or the MoE block (orc_prefill_moe).
 * The first generated token is the argmax of the LM head on the final
 * RMSNorm of the last row (:877-891); *logit = its value, last_x = that
 * normed row. Returns the token. */
int orc_decoder_prefill(const orc_layer_t *layers, const orc_dims_t *d, const float *final_norm,
                        const uint16_t *lm_head, float *kv_k, float *kv_v, int kv_max, int pos0,
                        const float *cos_t, const float *sin_t, const float *embeds, int T, float *last_x,
                        float *logit) {
    int H = d->hidden, hd = d->head_dim, nh = d->n_heads, qd = nh * hd, D = d->inter_dense;
    float *x = (float *)malloc((size_t)T * H * sizeof(float));
    float *xn = (float *)malloc((size_t)T * H * sizeof(float));
    float *Q = (float *)malloc((size_t)T * qd * sizeof(float));
    float *K = (float *)malloc((size_t)T * qd * sizeof(float));
    float *V = (float *)malloc((size_t)T * qd * sizeof(float));
    float *att = (float *)malloc((size_t)T * qd * sizeof(float));
    float *proj = (float *)malloc((size_t)T * H * sizeof(float));
    memcpy(x, embeds, (size_t)T * H * sizeof(float));
    float scale = 1.0f / sqrtf((float)hd);
    for (int l = 0; l < d->n_layers; l++) {
        const orc_layer_t *ly = &layers[l];
        for (int t = 0; t < T; t++) orc_rms_norm(xn + (size_t)t * H, x + (size_t)t * H, ly->input_norm, H, d->eps);
        gemm_bf16(Q, xn, ly->wq, T, H, qd);
        gemm_bf16(K, xn, ly->wk, T, H, qd);
        gemm_bf16(V, xn, ly->wv, T, H, qd);
        float *Kl = kv_k + (size_t)l * kv_max * qd;
        float *Vl = kv_v + (size_t)l * kv_max * qd;
        for (int t = 0; t < T; t++) {
            int p = pos0 + t;
            orc_apply_rope(Q + (size_t)t * qd, cos_t + (size_t)p * hd, sin_t + (size_t)p * hd, nh, hd);
            orc_apply_rope(K + (size_t)t * qd, cos_t + (size_t)p * hd, sin_t + (size_t)p * hd, nh, hd);
            memcpy(Kl + (size_t)p * qd, K + (size_t)t * qd, (size_t)qd * sizeof(float));
            memcpy(Vl + (size_t)p * qd, V + (size_t)t * qd, (size_t)qd * sizeof(float));
        }
#pragma omp parallel for schedule(dynamic, 4)
        for (int t = 0; t < T; t++)
            orc_attention_decode(att + (size_t)t * qd, Q + (size_t)t * qd, Kl, Vl, pos0 + t + 1, nh, hd, qd, scale);
        gemm_bf16(proj, att, ly->wo, T, qd, H);
        for (size_t i = 0; i < (size_t)T * H; i++) x[i] += proj[i];
        if (l < d->first_dense) {
            float *g = (float *)malloc((size_t)T * D * sizeof(float));
            float *u = (float *)malloc((size_t)T * D * sizeof(float));
            float *mo = (float *)malloc((size_t)T * H * sizeof(float));
            for (int t = 0; t < T; t++)
                orc_rms_norm(xn + (size_t)t * H, x + (size_t)t * H, ly->post_norm, H, d->eps);
            gemm_bf16(g, xn, ly->dense_gate, T, H, D);
            gemm_bf16(u, xn, ly->dense_up, T, H, D);
            for (int t = 0; t < T; t++) orc_swiglu(g + (size_t)t * D, g + (size_t)t * D, u + (size_t)t * D, D);
            gemm_bf16(mo, g, ly->dense_down, T, D, H);
            for (size_t i = 0; i < (size_t)T * H; i++) x[i] += mo[i];
            free(g); free(u); free(mo);
        } else {
            orc_prefill_moe(ly, d, x, T, NULL, NULL, NULL);
        }
    }
    float *lx = (float *)malloc((size_t)H * sizeof(float));
    orc_rms_norm(lx, x + (size_t)(T - 1) * H, final_norm, H, d->eps);
    float val;
    int tok = orc_argmax_bf16(lx, lm_head, H, d->vocab, &val);
    if (last_x) memcpy(last_x, lx, (size_t)H * sizeof(float));
    if (logit) *logit = val;
    free(lx); free(x); free(xn); free(Q); free(K); free(V); free(att); free(proj);
    return tok;
}
