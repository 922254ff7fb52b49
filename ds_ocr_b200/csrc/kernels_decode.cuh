// kernels_decode.cuh — argument blocks and launchers of the decode-step
// kernels (kernels_decode.cu).
#pragma once
#include "kernels_moe.cuh"
#include "launch.h"

namespace ds {

struct QkvArgs {
    const float *x, *norm_w;
    float eps;
    int hidden;
    const uint16_t *w[3];        // Wq, Wk, Wv [n_heads*head_dim x hidden]
    const float *cos_t, *sin_t;  // [kv_max][head_dim]
    const int *d_pos;
    float *q_out;
    uint16_t *k_hi, *k_lo, *v_hi, *v_lo;  // this layer's cache, [head][kv_max][head_dim]
    int kv_max, n_heads, head_dim;
    int pos_ready;  // 1: *d_pos was written by a kernel that completed before the predecessor's dependent part
    const void *pf[3];  // weights a later kernel of the step reads (e.g. the dense FFN), asked of L2 before the
    size_t pf_bytes[3]; //   dependency wait, split over the CTAs (null / 0: none)
};

struct AttnArgs {
    const float *q;
    const uint16_t *k_hi, *k_lo, *v_hi, *v_lo;  // this layer: [head][kv_max][128]
    int kv_max, n_heads;
    const int *d_pos;  // keys 0..pos are attended (pos written by qkv_rope_kernel)
    int lo_start;      // rows below lo_start are exact BF16 (lo plane is zero)
    float scale;
    float *out;        // [n_heads * 128]
    // several independent streams (grid.y = stream): per-stream offsets of
    // q/out (elements), of the KV planes (elements) and d_pos[stream];
    // lo_starts (optional) per stream. Zero strides: one stream.
    long long kv_stream_stride;
    int q_stride;
    const int *lo_starts;
    // V3 reference sliding-window attention (0: off): window W, prefill
    // length P
    int swa_window, swa_ref;
    const int *swa_refs;  // per stream P (several streams; null: swa_ref)
};

// Router folded into the O-projection (optional): logits_e =
// (sum_r Wr[e][r] g[r] y[r]) * inv(y), y = the O-proj + residual output. Each
// CTA adds the terms of its 16 output rows (and their squares) into `part`;
// the last CTA sums the parts in CTA order, scales by the RMS of y and runs
// softmax/top-k (ds_moe_decoder.c:140-183 on the post-attention RMSNorm).
struct RouterFold {
    const uint16_t *Wr;    // [E x rows] BF16, null = no router
    const float *g;        // post-attention norm weight [rows]
    float eps;
    int E, top_k, renorm;
    float *part;           // [(E + 1) x rf_pstride(gridDim.x)]: column e's terms contiguous
    unsigned *ticket;      // zero between launches
    float *scores;         // [E] (for inspection)
    int *d_idx;
    float *d_wt;
    int no_tail;           // 1: only write the parts (the MoE-step kernel reduces them)
};

struct MvArgs {
    const uint16_t *W;
    const float *x, *norm_w;
    float eps;
    const float *bias, *resid;
    float *y;
    int rows, n;
    RouterFold rf;
};

cudaError_t launch_qkv_rope(const QkvArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_attn_decode(const AttnArgs &a, cudaStream_t st, bool pdl, int n_streams = 1);
// batch 1, causal: the cluster-exchange kernel (attn_step.cu)
cudaError_t launch_attn_step(const AttnArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_matvec_res(const MvArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, int n, float eps, cudaStream_t st, bool pdl);
cudaError_t launch_decode_advance(const uint16_t *E, int hidden, const int *d_tok, int *d_pos, int *tok_log,
                                  float *x_out, cudaStream_t st, bool pdl, int *hist = nullptr, int *hist_len = nullptr,
                                  int hist_cap = 0);

// Whole-decoder prefill kernels (prefill_full.cu).
cudaError_t launch_pd_split(const float *x, int M, int H, const float *nw, float eps, uint16_t *hi, uint16_t *lo,
                            cudaStream_t st);
cudaError_t launch_pd_rope_kv(const float *qkv, int T, int NH, int HD, int p0, const float *cos_t, const float *sin_t,
                              float *q, uint16_t *k_hi, uint16_t *k_lo, uint16_t *v_hi, uint16_t *v_lo, int kv_max,
                              cudaStream_t st);
cudaError_t launch_pd_add(float *x, const float *y, size_t n, cudaStream_t st);
// The prefill attention on the tensor cores (attn_prefill_tc.cu); head_dim 128.
bool attn_prefill_tc_ok(int head_dim, int kv_max, int n_heads);
cudaError_t launch_attn_prefill_tc(const float *q, const uint16_t *k_hi, const uint16_t *k_lo,
                                   const uint16_t *v_hi, const uint16_t *v_lo, int kv_max, int n_heads, int p0, int T,
                                   int q_stride, float scale, float *out, unsigned *err, cudaStream_t st);
cudaError_t launch_attn_prefill(const float *q, const uint16_t *k_hi, const uint16_t *k_lo, const uint16_t *v_hi,
                                const uint16_t *v_lo, int kv_max, int n_heads, int p0, int T, int lo_start,
                                int q_stride, float scale, float *out, cudaStream_t st);
cudaError_t launch_pd_finish(const uint16_t *E, int H, const int *tok, float *x_out, int *pos, int p_next,
                             int *tok_log, int *hist, int *hist_len, int hist_cap, cudaStream_t st);

// LM-head token selection with the sampling settings (select.cu).
struct SelectArgs {
    const uint16_t *W;   // LM head [V x H]
    const float *x;      // final RMS-normed hidden state [H]
    int H, V;
    const int *hist;     // generated tokens so far
    const int *hist_len;
    int cap;             // history capacity
    float *hval;         // [cap] history tokens' logits
    float *bval;         // the argmax winner's logit
    float *logits;       // [V]
    int *tok;            // in: the argmax winner; out: the selected token
    float *val;          // out: the selected value
    int *full;           // the full-logits path runs
    float rp;            // repetition penalty (> 1 enables)
    int ngram;           // no-repeat n-gram size (> 0 enables)
    float temperature;   // > 0: sampling
    const float *unif;   // caller-supplied uniforms, one per sampling step
    int *unif_pos;
    // several independent streams (grid.y = stream; 0 or 1: one stream).
    // Stream s reads x + s * x_ld, hist + s * cap, unif + s * unif_ld,
    // logits + s * V, hval + s * cap and entry s of hist_len, bval, tok,
    // val, full and unif_pos.
    int n_streams;
    int x_ld, unif_ld;
};
cudaError_t launch_select(const SelectArgs &a, cudaStream_t st);

}  // namespace ds
