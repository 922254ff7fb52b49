// moe_step.h — the fused batch-1 MoE block kernel (moe_step.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ds {

struct MoeStepArgs {
    int H, I, S, E, K;       // hidden, expert inter, shared inter (n_shared * I), experts, top_k
    int simulate, renorm;    // BF16 truncation (ds_bf16_simulate_python); renormalised top-k weights
    float eps;
    const float *x;          // residual stream after attention [H]
    const float *norm_w;     // post-attention RMSNorm weight [H]
    const float *rpart;      // router terms of the O-projection CTAs [nparts][E + 1] (last column: sum x^2)
    int nparts;
    const uint16_t *block;   // expert block: E x [gate (I); up (I)] x H, then shared [gate (S); up (S)] x H
    const uint16_t *down;    // routed down projections [E][H][I]
    const uint16_t *sdown;   // shared down projection [H][S]
    float *h;                // SwiGLU outputs [K*I + S] (global: every CTA reads all of it)
    float *out;              // x + MoE(x) [H]
    int *d_idx;              // routing, published by CTA 0 (for inspection)
    float *d_wt, *scores;
    unsigned long long *bar; // launch counter (every CTA adds 1 per launch; only ever incremented)
    unsigned long long *done;// [K + 1] completion counters: routed slot k's h rows, then the shared rows
    unsigned *err;           // set when a bounded wait gives up
    const void *pf[3];       // the next layer's Q, K, V weights: asked of L2 once this CTA's stream is done
    size_t pf_bytes;         // bytes of each (0: none)
    size_t a_bytes, d_bytes; // shared-memory regions (set by the launcher)
    int ncta[8];             // CTAs contributing to each routed slot (set by the launcher)
};

struct DenseStepArgs {
    int H, D;                // hidden, dense intermediate
    float eps;
    const float *x;          // residual stream after attention [H]
    const float *norm_w;     // post-attention RMSNorm weight [H]
    const uint16_t *gate, *up, *down;  // [D x H], [D x H], [H x D]
    float *h;                // SwiGLU outputs [D]
    float *out;              // x + FFN(x) [H]
    unsigned long long *bar; // grid-barrier counter (only ever incremented)
    unsigned *err;
    const void *pf[3];       // the next layer's Q, K, V weights (see MoeStepArgs)
    size_t pf_bytes;
};

bool dense_step_supported(int H, int D, int sms);
cudaError_t launch_dense_step(DenseStepArgs a, int grid, cudaStream_t st, bool pdl);
bool moe_step_supported(int H, int I, int S, int E, int K, int sms);
size_t moe_step_smem(int H, int I, int S, int K, int grid);
cudaError_t launch_moe_step(MoeStepArgs a, int grid, cudaStream_t st, bool pdl);

}  // namespace ds
