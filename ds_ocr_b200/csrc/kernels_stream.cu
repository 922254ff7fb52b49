// kernels_stream.cu — weight streaming through the TMA engine.
//
// A batch-1 matvec reads every weight byte once, so its speed is the number
// of bytes in flight per SM. Register-held loads cap that at roughly
// (warps x loads per lane x 16 B); here one producer thread per CTA keeps a
// ring of shared-memory stages filled with cp.async.bulk copies (completion
// tracked by mbarriers) while 16 consumer warps compute from shared memory,
// so each SM keeps ~100-200 KB of weights in flight independent of
// registers (16 consumers: the per-row wait/dot/reduce chains of 8 were the
// limit at 0.71 of the copy bandwidth). The CTA owns a contiguous range of row tiles, so the DRAM
// stream of each SM is sequential.
#include "kernels_moe.cuh"
#include "launch.h"

namespace ds {

constexpr int ST_ROWS = 16;       // rows per tile (one per consumer warp)
constexpr int ST_CONSUMERS = 16;  // consumer warps
constexpr int ST_THREADS = 32 * (ST_CONSUMERS + 1);
constexpr int ST_SMEM_BUDGET = 200 * 1024;

__host__ __device__ constexpr int st_stages(int n) {
    return (ST_SMEM_BUDGET / (ST_ROWS * n * 2)) < 8 ? (ST_SMEM_BUDGET / (ST_ROWS * n * 2)) : 8;
}

// Argmax LM head over TMA-streamed tiles (same contract as
// argmax_bf16_kernel: ds_argmax_matvec_bf16, ds_kernels.c:1013-1099).
template <int CPL>
__global__ void __launch_bounds__(ST_THREADS) argmax_tma_kernel(const uint16_t *__restrict__ W,
                                                                const float *__restrict__ x, int rows, int n,
                                                                unsigned long long *slot, unsigned *ticket,
                                                                int *tok_out, float *val_out, const float *norm_w,
                                                                float eps, unsigned *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[8], empty[8];
    __shared__ unsigned long long cta_best;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    TraceScope tr;
    const int S = st_stages(n);
    const uint32_t row_b = (uint32_t)n * 2, stage_b = ST_ROWS * row_b;
    const int tiles = (rows + ST_ROWS - 1) / ST_ROWS;
    const int t0 = (int)((long long)tiles * blockIdx.x / gridDim.x);
    const int t1 = (int)((long long)tiles * (blockIdx.x + 1) / gridDim.x);
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ST_CONSUMERS);
        }
        cta_best = 0ull;
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == ST_CONSUMERS) {
        // producer: weights do not depend on the predecessor kernel, so the
        // stream starts before griddepcontrol.wait
        if (lane == 0) {
            for (int t = t0, i = 0; t < t1; t++, i++) {
                int s = i % S;
                if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, err)) break;
                int r0 = t * ST_ROWS;
                uint32_t bytes = (uint32_t)min(ST_ROWS, rows - r0) * row_b;
                mbar_expect_tx(&full[s], bytes);
                bulk_g2s_stream(smem + (size_t)s * stage_b, W + (size_t)r0 * n, bytes, &full[s]);
            }
        }
        return;
    }
    pdl_wait();
    pdl_launch();
    tr.waited();
    // block_rms_inv needs every thread of the block: consumers only here, so
    // compute the norm with the consumer warps through named barrier 1
    float inv = 1.f;
    if (norm_w) {
        __shared__ float red[ST_CONSUMERS + 1];
        float ss = 0.f;
        for (int i = threadIdx.x; i < n; i += 32 * ST_CONSUMERS) ss = __fmaf_rn(x[i], x[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        asm volatile("bar.sync 1, %0;" :: "r"(32 * ST_CONSUMERS) : "memory");
        if (threadIdx.x == 0) {
            float t = 0.f;
            for (int w = 0; w < ST_CONSUMERS; w++) t = __fadd_rn(t, red[w]);
            red[ST_CONSUMERS] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)n), eps)));
        }
        asm volatile("bar.sync 1, %0;" :: "r"(32 * ST_CONSUMERS) : "memory");
        inv = red[ST_CONSUMERS];
    }
    XRegBF16<CPL> xr;
    xr.load_norm(x, norm_w, inv, n, lane);
    const int nch = n >> 3;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int t = t0, i = 0; t < t1; t++, i++) {
        int s = i % S;
        if (!mbar_wait(&full[s], (i / S) & 1, err)) break;
        int r = t * ST_ROWS + warp;
        if (r < rows) {
            const uint16_t *row = reinterpret_cast<const uint16_t *>(smem + (size_t)s * stage_b) + (size_t)warp * n;
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < CPL; c++) {
                int ch = lane + 32 * c;
                if (ch < nch) {
                    uint4 w = *reinterpret_cast<const uint4 *>(row + 8 * ch);
                    acc = dot8_bf16(w, xr.v[c][0], xr.v[c][1], acc);
                }
            }
            acc = warp_sum(acc);
            if (acc > best) { best = acc; bi = r; }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (lane == 0 && bi != 0x7fffffff) atomicMax(&cta_best, argmax_key(best, (uint32_t)bi));
    asm volatile("bar.sync 1, %0;" :: "r"(32 * ST_CONSUMERS) : "memory");
    if (threadIdx.x == 0) {
        if (cta_best) atomicMax(slot, cta_best);
        __threadfence();
        unsigned tk = atomicAdd(ticket, 1u);
        if (tk == gridDim.x - 1) {
            __threadfence();
            unsigned long long k = atomicExch(slot, 0ull);
            *tok_out = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
            *val_out = f32_from_ordered((uint32_t)(k >> 32));
            *ticket = 0u;
        }
    }
    tr.done(8);
}

bool st_stages_ok(int n) { return n % 8 == 0 && n <= 2048 && st_stages(n) >= 2; }

cudaError_t launch_argmax_tma(const uint16_t *W, const float *x, int rows, int n, unsigned long long *slot,
                              unsigned *ticket, int *tok, float *val, cudaStream_t st, bool pdl, const float *norm_w,
                              float eps, unsigned *err) {
    if (n % 8 || n > 2048 || st_stages(n) < 2) return cudaErrorInvalidValue;
    int dev, sms;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int tiles = (rows + ST_ROWS - 1) / ST_ROWS;
    int grid = min(tiles, sms);
    size_t smem = (size_t)st_stages(n) * ST_ROWS * n * 2;
    void *args[] = {&W, &x, &rows, &n, &slot, &ticket, &tok, &val, &norm_w, &eps, &err};
#define ST_CASE(C)                                                                                               \
    {                                                                                                            \
        const void *f = (const void *)argmax_tma_kernel<C>;                                                      \
        static int set_##C = 0;                                                                                  \
        if (set_##C < (int)smem) {                                                                               \
            cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, ST_SMEM_BUDGET);               \
            set_##C = ST_SMEM_BUDGET;                                                                            \
        }                                                                                                        \
        return launch_ex(f, grid, ST_THREADS, smem, st, pdl, args);                                              \
    }
    int c = (n / 8 + 31) / 32;
    if (c <= 4) ST_CASE(4)
    if (c <= 5) ST_CASE(5)
    ST_CASE(8)
#undef ST_CASE
}

}  // namespace ds

DS_TRACE_TU(stream)
