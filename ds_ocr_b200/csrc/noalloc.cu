// noalloc.cu — ds_cuda_moe_experts_noalloc: the routed-expert MoE chain
// (gate_up + SwiGLU, then down + weighted combine) for callers that cannot
// allocate device memory.
//
// Some hosts cannot call cudaMalloc at the point where they run the expert
// chain: a plugin that only receives device buffers from its host framework,
// code running while another component owns the allocator, or a process whose
// memory budget is fixed after start-up. This entry point takes the caller's
// input, weights and output as device pointers, creates no context, and keeps
// its one scratch buffer (the SwiGLU activations between the two kernels) in
// the file-scope array below, which every GPU that loads this library holds
// until the process exits.
#include <atomic>
#include <cstdio>

#include "ds_cuda.h"
#include "launch.h"

using namespace ds;

// Largest top_k * inter the scratch holds: 12288 floats (48 KB), enough for
// the decoder's 6 routed experts of up to 2048 rows each. The kernels alone
// accept top_k <= 8 and inter <= 2048, so 8 experts of inter > 1536 are
// refused by this bound.
constexpr int NOALLOC_MAX_H = 12288;

static __device__ __align__(256) float g_noalloc_h[NOALLOC_MAX_H];

// Device address of g_noalloc_h per device, resolved on the first call made
// with that device current (the host-side name is only a stand-in). Atomic:
// host threads making their first calls at once each store the same value.
static std::atomic<float *> g_noalloc_ptr[64];

static int noalloc_fail(int code, const char *msg) {
    fprintf(stderr, "ds_cuda_moe_experts_noalloc: %s\n", msg);
    return code;
}

extern "C" int ds_cuda_moe_experts_noalloc(const float *d_x, const uint16_t *const *d_gate_up,
                                           const uint16_t *const *d_down, const float *top_weights, int top_k,
                                           int hidden, int inter, float *d_output, void *stream) {
    if (!d_x || !d_output || top_k <= 0 || !d_gate_up || !d_down || !top_weights)
        return noalloc_fail(DS_CUDA_EINVAL, "null argument or top_k <= 0");
    if (top_k > 8 || inter <= 0 || inter % 8 || inter > 2048 || hidden <= 0 || hidden % 8 || hidden > 2048)
        return noalloc_fail(DS_CUDA_EINVAL, "unsupported shape (top_k <= 8, hidden and inter multiples of 8, <= 2048)");
    if (top_k * inter > NOALLOC_MAX_H)
        return noalloc_fail(DS_CUDA_EINVAL, "top_k * inter exceeds the 12288-float static scratch");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return noalloc_fail(DS_CUDA_ECUDA, "no current CUDA device (or device index >= 64)");
    float *scratch = g_noalloc_ptr[dev].load(std::memory_order_acquire);
    if (!scratch) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_h);
        if (e != cudaSuccess || !p) return noalloc_fail(DS_CUDA_ECUDA, cudaGetErrorString(e));
        scratch = (float *)p;
        g_noalloc_ptr[dev].store(scratch, std::memory_order_release);
    }
    MoeArgs a = {};
    a.hidden = hidden;
    a.inter = inter;
    a.top_k = top_k;
    for (int k = 0; k < top_k; k++) {
        if (!d_gate_up[k] || !d_down[k]) return noalloc_fail(DS_CUDA_EINVAL, "null expert weight pointer");
        a.gu[k].w = d_gate_up[k];
        a.dn[k].w = d_down[k];
        a.wt[k] = top_weights[k];
    }
    a.x = d_x;
    a.h = scratch;  // fully written by gate_up before down reads it: nothing to clear
    a.out = d_output;
    a.out_mode = 0;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = launch_moe_gate_up(a, st, false);
    if (e == cudaSuccess) e = launch_moe_down(a, st, false);
    if (e != cudaSuccess) return noalloc_fail(DS_CUDA_ECUDA, cudaGetErrorString(e));
    return DS_CUDA_OK;
}
