// prefill.h — host entry points of the tensor-core prefill (prefill.cu)
// used by the whole-decoder prefill (decoder.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "ctx.h"

struct PfShape {
    int H, I, S, E, K;
    float eps;
    int logits_ld = 0;  // row stride of caller-supplied logits (0: E)
};

// One MoE prefill layer on device buffers: d_x [M x H] += MoE(RMSNorm(d_x)).
int prefill_moe_enqueue(ds_cuda_ctx *c, const PfShape &g, const float *d_norm, const uint16_t *d_router,
                        const uint16_t *d_block, const uint16_t *d_down, const uint16_t *d_sdown, float *d_x, int M,
                        const float *d_logits, int *d_idx_out, float *d_w_out, cudaStream_t st);

// Dense split-BF16 GEMM (mode 1: y = A.B^T; mode 0: SwiGLU planes of
// [gate; up] B); shapes in prefill.cu.
int pf_dense_gemm(ds_cuda_ctx *c, int mode, const uint16_t *a_hi, const uint16_t *a_lo, int M, int K,
                  const uint16_t *B, int N, float *y, int y_ld, uint16_t *h_hi, uint16_t *h_lo, cudaStream_t st);

// DS_CUDA_ETIMEOUT if a bounded device-side wait of the prefill kernels gave up.
int prefill_check_flag(ds_cuda_ctx *c);
