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
};

struct MvArgs {
    const uint16_t *W;
    const float *x, *norm_w;
    float eps;
    const float *bias, *resid;
    float *y;
    int rows, n;
};

cudaError_t launch_qkv_rope(const QkvArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_attn_decode(const AttnArgs &a, cudaStream_t st, bool pdl, int n_streams = 1);
cudaError_t launch_matvec_res(const MvArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, int n, float eps, cudaStream_t st, bool pdl);
cudaError_t launch_decode_advance(const uint16_t *E, int hidden, const int *d_tok, int *d_pos, int *tok_log,
                                  float *x_out, cudaStream_t st, bool pdl);

}  // namespace ds
