/*
 * ds_oracle.h — CPU restatement of ds-ocr's MoE-decoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py load liboracle.so, and only as the checker.
 * The product (libds_cuda.so, the ds_ocr_b200 package) never links it.
 *
 * Parity pin: every function here is checked against the reference itself,
 * compiled unmodified from its own sources into oracle/_ref/libdsref.so
 * (tests/test_oracle_vs_ref.py), and against the golden vectors that
 * tests/golden/make_golden.py generated from that library.
 *
 * Numerics follow the reference: BF16 weights widened exactly (u16 << 16),
 * F32 accumulation, Schraudolph fast exp with the product-add fused (gcc
 * -O3 -march=native contracts it into one FMA), strict '>' comparisons so
 * the lowest index wins ties. Summation order is 16 interleaved lanes, the
 * reference's AVX-512 order; lane-combine order differs, so dot products
 * agree to a few ulp, not bit-for-bit.
 */
#ifndef DS_ORACLE_H
#define DS_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int hidden, n_heads, head_dim, inter_dense, moe_inter;
    int n_experts, n_shared, top_k, vocab, n_layers, first_dense;
    float eps, theta;
    int simulate_bf16;   /* ds_bf16_simulate_python */
    int renorm_topk;     /* 0 = reference behaviour (raw softmax probabilities) */
} orc_dims_t;

/* Weights of one decoder layer. Expert layout as ds_ocr.c:696-768:
 * expert_block = [E x gate_up_fused (2I x H)] [shared gate_up (2S x H)];
 * down = [E x (H x I)]; shared_down = H x S. int8 pointers may be NULL. */
typedef struct {
    const uint16_t *wq, *wk, *wv, *wo;
    const float *input_norm, *post_norm;
    const uint16_t *dense_gate, *dense_up, *dense_down;
    const uint16_t *router, *expert_block, *down, *shared_down;
    const int8_t *gu_q;  const float *gu_scale,  *gu_off;   /* [E][2I x H], [E][2I] */
    const int8_t *dn_q;  const float *dn_scale,  *dn_off;   /* [E][H x I],  [E][H]  */
    const int8_t *sgu_q; const float *sgu_scale, *sgu_off;  /* [2S x H], [2S] */
    const int8_t *sdn_q; const float *sdn_scale, *sdn_off;  /* [H x S],  [H]  */
} orc_layer_t;

float orc_fast_expf(float x);
float orc_bf16_roundtrip(float x);
void orc_matvec_bf16(float *y, const float *x, const uint16_t *W, int in_dim, int out_dim);
float orc_dot_bf16_row(const float *x, const uint16_t *W, int in_dim, int row);
int orc_argmax_bf16(const float *x, const uint16_t *W, int in_dim, int out_dim, float *val);
void orc_router_topk(const float *logits, int n_experts, int top_k, int renorm,
                     int *idx, float *w);
void orc_swiglu(float *out, const float *g, const float *u, int n);
void orc_expert_fused(float *out, const float *x, const uint16_t *gu, const uint16_t *down,
                      int hidden, int inter, int simulate);
int orc_int8_quantize(const uint16_t *W, int out_dim, int in_dim,
                      int8_t *q, float *scale, float *off);
void orc_int8_matvec(float *y, const float *x, const int8_t *q, const float *scale,
                     const float *off, int out_dim, int in_dim);
void orc_expert_fused_int8(float *out, const float *x,
                           const int8_t *guq, const float *gus, const float *guo,
                           const int8_t *dnq, const float *dns, const float *dno,
                           int hidden, int inter, int simulate);
void orc_moe_forward(float *out, const float *x, const orc_layer_t *ly, const orc_dims_t *d,
                     int use_int8, int *idx_out, float *w_out);
void orc_rms_norm(float *out, const float *x, const float *w, int n, float eps);
void orc_residual_rms_norm(float *out, float *norm_out, const float *x, const float *r,
                           const float *w, int n, float eps);
void orc_rope_table(float *cos_t, float *sin_t, int max_pos, int head_dim, float theta);
void orc_apply_rope(float *vec, const float *c, const float *s, int n_heads, int head_dim);
void orc_attention_decode(float *out, const float *q, const float *K, const float *V,
                          int n_keys, int n_heads, int head_dim, int kv_stride, float scale);
int orc_decoder_step(const orc_layer_t *layers, const orc_dims_t *d,
                     const float *final_norm, const uint16_t *lm_head,
                     float *kv_k, float *kv_v, int kv_max, int pos,
                     const float *cos_t, const float *sin_t, int use_int8,
                     const float *embed, float *final_x, float *logit);
int orc_decoder_prefill(const orc_layer_t *layers, const orc_dims_t *d, const float *final_norm,
                        const uint16_t *lm_head, float *kv_k, float *kv_v, int kv_max, int pos0,
                        const float *cos_t, const float *sin_t, const float *embeds, int T, float *last_x,
                        float *logit);
int orc_lm_select(const float *xn, const uint16_t *W, int H, int V, const int *hist, int len, float rp,
                  int ngram, float temperature, float r, float *val, int *full);
/* orc_decoder_step with V3's reference sliding-window attention: window
 * W > 0 and prefill length ref_len (ds_moe_decoder.c:409-436). */
int orc_decoder_step_swa(const orc_layer_t *layers, const orc_dims_t *d,
                         const float *final_norm, const uint16_t *lm_head,
                         float *kv_k, float *kv_v, int kv_max, int pos,
                         const float *cos_t, const float *sin_t, int use_int8,
                         const float *embed, float *final_x, float *logit, int window, int ref_len);
void orc_prefill_moe(const orc_layer_t *ly, const orc_dims_t *d, float *x, int seq_len,
                     const float *logits, int *idx_out, float *w_out);

#ifdef __cplusplus
}
#endif
#endif
