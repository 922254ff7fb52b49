// ctx.h — the ds_cuda context (opaque to C callers) and internal helpers.
#pragma once
#include <cstdint>
#include <map>
#include <vector>
#include <string>
#include <cuda_runtime.h>
#include "ds_cuda.h"
#include "launch.h"

struct Reg {
    uintptr_t host;
    size_t bytes;
    void *dev;
};

struct DecoderModel;  // decoder.cu

struct ds_cuda_ctx {
    int device = 0;
    int sm_count = 0;
    bool ok = false;
    cudaStream_t stream = nullptr;
    std::string err;
    std::map<uintptr_t, Reg> regs;  // keyed by host base address
    size_t reg_bytes = 0;
    int simulate = 0, renorm = 0;
    // device scratch
    unsigned *d_tickets = nullptr;          // [64] grid-completion tickets (self-resetting)
    unsigned long long *d_slots = nullptr;  // [512] argmax slots (self-resetting)
    int *d_tok = nullptr;                   // [512]
    float *d_val = nullptr;                 // [512]
    float *d_scores = nullptr;              // [256] router logits
    int *d_idx = nullptr;                   // [64] top-k indices
    float *d_wt = nullptr;                  // [64] top-k weights
    float *d_x = nullptr, *d_out = nullptr, *d_h = nullptr;
    size_t x_cap = 0, out_cap = 0, h_cap = 0;
    void *d_tmp = nullptr;
    size_t tmp_cap = 0;
    // tensor-core batched LM head: split input planes, error flag
    void *d_lt_planes = nullptr;
    size_t lt_planes_cap = 0;
    void *d_lt_err = nullptr;
    // multi-stream GEMM standalone entry: planes + tile list
    void *d_sk_scratch = nullptr;
    size_t sk_scratch_cap = 0;
    // pinned staging
    void *pin = nullptr;
    size_t pin_cap = 0;
    // batched-prefill workspace (prefill.cu) and optional per-stage timing
    void *prefill = nullptr;
    bool prefill_timing = false;
    // expert-parallel state (ep_nccl.cu): communicator, stream, buffers
    void *ep = nullptr;
    cudaEvent_t prefill_ev[7] = {};
    // decoder models owned by this context
    std::map<int, DecoderModel *> models;
    int next_model = 1;
    // host address ranges reserved (no access, no memory) as the keys of
    // weights built directly in HBM (ingest.cu); released with the context
    std::vector<std::pair<void *, size_t>> key_ranges;
};

int ctx_fail(ds_cuda_ctx *c, int code, const char *fmt, ...);
int ctx_cuda(ds_cuda_ctx *c, cudaError_t e, const char *what);
int ctx_grow(ds_cuda_ctx *c, void **p, size_t *cap, size_t need);
int ctx_pinned(ds_cuda_ctx *c, size_t need);
int ctx_register(ds_cuda_ctx *c, const void *p, size_t bytes);
// Registers device memory the context takes ownership of under a fresh
// reserved host key range of the same size; returns the key (or null).
void *ctx_adopt(ds_cuda_ctx *c, void *dev, size_t bytes);
const void *ctx_lookup(ds_cuda_ctx *c, const void *p, size_t bytes, bool auto_register);
void ctx_release_models(ds_cuda_ctx *c);
void prefill_release(ds_cuda_ctx *c);
void ep_release(ds_cuda_ctx *c);
void ctx_release_batch_models(ds_cuda_ctx *c);
int moe_layer_enqueue(ds_cuda_ctx *c, ds::MoeArgs &a, const uint16_t *d_router, int n_experts, int *d_idx,
                      float *d_wt, cudaStream_t st, bool pdl);
int lmhead_tc_enqueue(ds_cuda_ctx *c, const float *d_x, const uint16_t *d_W, int in_dim, int out_dim, int batch,
                      int *d_tok, float *d_val, cudaStream_t st);
int batch_argmax_enqueue(ds_cuda_ctx *c, const float *d_x, const uint16_t *d_W, int in_dim, int out_dim, int batch,
                         int *d_tok, float *d_val, cudaStream_t st);
