// mega.h — parameter block of the persistent decode kernel (mega.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace ds {

struct MegaLayer {
    const uint16_t *wq, *wk, *wv, *wo;
    const float *in_norm, *post_norm;
    int dense;
    const uint16_t *dgate, *dup, *ddown;
    const uint16_t *router, *block, *down, *sdown;
    uint16_t *k_hi, *k_lo, *v_hi, *v_lo;  // this layer's cache, [head][kv_max][128]
    int lo_start;                         // rows below are exact BF16 (lo plane zero)
};

struct MegaParams {
    int H, NH, HD, D, I, E, S, K, V, L, kv_max;
    float eps, scale;
    int simulate, renorm;
    const MegaLayer *layers;  // device array [L]
    const float *final_norm;
    const uint16_t *lm_head;  // [V x H]
    const uint16_t *embed;    // [V x H] token embeddings (the LM head when tied)
    const float *cos_t, *sin_t;
    // activations and cross-CTA exchange buffers (device)
    float *xa, *xb, *q;
    float *att_sc;    // [NH][kv_max] attention scores
    float *att_part;  // [NH][G][HD] partial outputs
    float *att_sum;   // [NH]
    float *h;         // [max(K*I + S, D)]
    float *rscore;    // [E]
    unsigned long long *slot;  // [2] argmax keys (ping-pong per step)
    unsigned *bar;             // [0] arrive count, [1] generation, [2] error flag
    int *pos, *tok, *tok_log;
    float *val, *final_x;      // final_x optional (last step's normed hidden state)
    long long *trace;          // optional: CTA 0 / last CTA phase timestamps (clock64)
    int trace_cap;
    int n_steps;
    int first_from_token;      // 1: step 0 input = embedding of *tok; 0: xa holds it
};

// Launches the persistent kernel (cooperative, one CTA per SM); `dparams`
// points to a MegaParams in device memory.
cudaError_t launch_mega(const MegaParams *dparams, int grid, cudaStream_t st);
// CTAs per SM the kernel fits (0 = it cannot run on this device).
int mega_grid(int device);
size_t mega_smem_bytes();

}  // namespace ds
