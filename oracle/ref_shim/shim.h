/* Force-included (gcc -include) when compiling the unmodified reference
 * sources on x86. ds_kernels.c:59-60 names the dispatch function-pointer
 * typedefs that ds_kernels_impl.h:44-49 only declares inside its ARM branch;
 * this header supplies the same two typedefs so the x86 build compiles.
 * Test infrastructure only: nothing in the product links this. */
#ifndef DS_REF_SHIM_H
#define DS_REF_SHIM_H
#include <stdint.h>
#ifndef __ARM_NEON
typedef void (*ds_bf16_matvec_fused_fn_t)(float *y, const float *x,
                                           const uint16_t *W_bf16,
                                           const float *bias, int in_dim, int out_dim);
typedef void (*ds_argmax_bf16_range_fn_t)(const float *x, const uint16_t *W_bf16,
                                            int in_dim, int start, int end,
                                            int *best_out, float *best_val_out);
#endif
#endif
