// batch.cu — batched argmax LM head (B independent inputs over one weight).
#include "ctx.h"

// Batches of 2..64 with in_dim % 64 == 0 run as one tensor-core pass over W
// (lmhead_tc.cu); otherwise each input row gets its own argmax launch (and
// slot), back to back on one stream so the shared ticket is reused safely.
int batch_argmax_enqueue(ds_cuda_ctx *c, const float *d_x, const uint16_t *d_W, int in_dim, int out_dim, int batch,
                         int *d_tok, float *d_val, cudaStream_t st) {
    if (batch > 512) return ctx_fail(c, DS_CUDA_EINVAL, "argmax batch > 512");
    if (batch >= 2 && batch <= 64 && in_dim % 64 == 0)
        return lmhead_tc_enqueue(c, d_x, d_W, in_dim, out_dim, batch, d_tok, d_val, st);
    for (int b = 0; b < batch; b++) {
        cudaError_t e = ds::launch_argmax_bf16(d_W, d_x + (size_t)b * in_dim, out_dim, in_dim, c->d_slots + b,
                                               c->d_tickets + 0, d_tok + b, d_val + b, st, false);
        if (e != cudaSuccess) return ctx_cuda(c, e, "argmax batch launch");
    }
    return DS_CUDA_OK;
}

