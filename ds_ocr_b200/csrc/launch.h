// launch.h — internal host-side launchers of the ds_cuda kernels (C++ only,
// not part of the C ABI).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "kernels_moe.cuh"

namespace ds {

cudaError_t launch_ex(const void *func, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      void **args);

cudaError_t launch_argmax_bf16(const uint16_t *W, const float *x, int rows, int n, unsigned long long *slot,
                               unsigned *ticket, int *tok, float *val, cudaStream_t st, bool pdl,
                               const float *norm_w = nullptr, float eps = 0.f);
bool st_stages_ok(int n);
cudaError_t launch_argmax_tma(const uint16_t *W, const float *x, int rows, int n, unsigned long long *slot,
                              unsigned *ticket, int *tok, float *val, cudaStream_t st, bool pdl, const float *norm_w,
                              float eps, unsigned *err);
cudaError_t launch_router(const uint16_t *Wr, const float *x, int E, int n, float *scores, unsigned *ticket,
                          int top_k, int renorm, int *d_idx, float *d_wt, cudaStream_t st, bool pdl,
                          const float *norm_w = nullptr, float eps = 0.f);
cudaError_t launch_router_select(const float *scores, int E, int top_k, int renorm, int *d_idx, float *d_wt,
                                 cudaStream_t st, bool pdl);
cudaError_t launch_moe_gate_up(const MoeArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_moe_down(const MoeArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_matvec_bf16(const uint16_t *W, const float *x, const float *bias, float *y, int rows, int n,
                               cudaStream_t st, bool pdl);
cudaError_t launch_quantize_int8(const uint16_t *W, int rows, int n, int8_t *q, float *scale, float *off,
                                 cudaStream_t st);

}  // namespace ds
