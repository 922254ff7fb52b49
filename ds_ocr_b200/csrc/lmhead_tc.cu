// lmhead_tc.cu — batched argmax LM head on the tensor cores:
// ds_argmax_matvec_bf16 (ds_kernels.c:1013-1099) for up to 64 independent
// inputs over one weight matrix, token = argmax_v W[v,:] x_b (lowest index
// wins ties), logit = that maximum.
//
// The reference loops over the inputs (one matvec each). At B = 64 the 21
// GFLOP of F32 CUDA-core work would be compute-bound; here it is one pass
// over W (331 MB at vocab 129280 x 1280) with the products on tcgen05:
//   * the inputs are split into BF16 planes hi = bf16(x), lo = bf16(x - hi)
//     and stacked as the 128 rows of the B operand (rows 0..63 hi, 64..127
//     lo), so one M=128, N=128 MMA per K step gives W x_hi and W x_lo for a
//     128-row vocab tile; logit = acc_hi + acc_lo (F32-class accuracy);
//   * W tiles stream through a 6-stage TMA ring; the 2 x 64 KB of split
//     inputs per vocab tile come from L2;
//   * the accumulator is double-buffered in tensor memory; each epilogue
//     thread owns one vocab row of the tile and keeps a running (max, index)
//     per input across all its tiles; one CTA reduction and one 64-bit
//     atomicMax per input at the end; the last CTA decodes the winners.
#include "ctx.h"
#include "tmap.h"
#include "umma.cuh"

namespace ds {

constexpr int LT_BM = 128;  // vocab rows per tile
constexpr int LT_BN = 128;  // 64 inputs x (hi, lo)
constexpr int LT_B = 64;    // max inputs
constexpr int LT_STAGES = 6;
constexpr int LT_THREADS = 192;
constexpr int LT_STAGE_BYTES = (LT_BM + LT_BN) * 64 * 2;
constexpr int LT_SMEM = LT_STAGES * LT_STAGE_BYTES + 1024;

struct LtArgs {
    CUtensorMap w;  // [V x K] BF16, box 64 x 128
    CUtensorMap x;  // [128 x K] BF16 planes, box 64 x 128
    int V, K, B;
    unsigned long long *slot;  // [B] packed (ordered value, ~index), zero on entry
    unsigned *ticket;          // zero on entry; reset by the last CTA
    int *tok;
    float *val;
    unsigned *err;
};

// x [B x K] F32 -> planes [128 x K]: rows 0..B-1 hi, 64..64+B-1 lo, rest 0.
__global__ void lt_split_kernel(const float *__restrict__ x, int B, int K, uint16_t *planes) {
    const int r = blockIdx.y;  // 0..63
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x) {
        uint16_t hi = 0, lo = 0;
        if (r < B) split_bf16(x[(size_t)r * K + k], hi, lo);
        planes[(size_t)r * K + k] = hi;
        planes[(size_t)(r + LT_B) * K + k] = lo;
    }
}

__global__ void __launch_bounds__(LT_THREADS, 1) lt_argmax_kernel(const __grid_constant__ LtArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[LT_STAGES], empty[LT_STAGES], acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_base;
    __shared__ float red_v[4][LT_B];
    __shared__ int red_i[4][LT_B];
    __shared__ bool last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (p.V + LT_BM - 1) / LT_BM;
    const int nk = p.K / 64;
    if (threadIdx.x == 0) {
        for (int s = 0; s < LT_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(&drain, 1);
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(&tmem_base, 2 * LT_BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % LT_STAGES, r = it / LT_STAGES;
                    if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + s * LT_STAGE_BYTES;
                    mbar_expect_tx(&full[s], LT_STAGE_BYTES);
                    tma_load_2d(st, &p.w, kb * 64, t * LT_BM, &full[s]);
                    tma_load_2d(st + LT_BM * 128, &p.x, kb * 64, 0, &full[s]);
                }
            }
            for (int i = max(0, it - LT_STAGES); i < it; i++)
                mbar_wait(&full[i % LT_STAGES], (i / LT_STAGES) & 1, p.err);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(LT_BM, LT_BN);
            int it = 0, ti = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ti++) {
                const int b = ti & 1, u = ti >> 1;
                if (u > 0 && !mbar_wait(&acc_empty[b], (u - 1) & 1, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + b * LT_BN;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % LT_STAGES, r = it / LT_STAGES;
                    if (!mbar_wait(&full[s], r & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t *st = smem + s * LT_STAGE_BYTES;
                    const uint64_t ad = sw128_desc(st), bd = sw128_desc(st + LT_BM * 128);
#pragma unroll
                    for (int j = 0; j < 4; j++) umma_bf16(d, ad + 2 * j, bd + 2 * j, idesc, (kb | j) != 0);
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&acc_full[b]);
            }
            umma_commit(&drain);
            mbar_wait(&drain, 0, p.err);
        }
    } else {
        // epilogue: thread = one vocab row of each tile; running best per input
        const int q = warp & 3;
        const int row = q * 32 + lane;
        // running best value per input, and the CTA-local tile count of the
        // row that holds it (16 bits, two per register; 0xffff = none)
        float best[LT_B];
        uint32_t bti[LT_B / 2];
#pragma unroll
        for (int c = 0; c < LT_B; c++) best[c] = -INFINITY;
#pragma unroll
        for (int c = 0; c < LT_B / 2; c++) bti[c] = 0xffffffffu;
        int ti = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ti++) {
            const int b = ti & 1, u = ti >> 1;
            if (!mbar_wait(&acc_full[b], u & 1, p.err)) break;
            tc_fence_after();
            const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + b * LT_BN;
            const int v = t * LT_BM + row;
#pragma unroll
            for (int c0 = 0; c0 < LT_B; c0 += 16) {
                float h[16], l[16];
                tmem_ld16(tb + c0, h);
                tmem_ld16(tb + LT_B + c0, l);
                if (v < p.V) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const float s = __fadd_rn(h[j], l[j]);
                        if (s > best[c0 + j]) {  // rows only grow: ties keep the lower index
                            best[c0 + j] = s;
                            const int c = c0 + j, sh = (c & 1) * 16;
                            bti[c >> 1] = (bti[c >> 1] & ~(0xffffu << sh)) | ((uint32_t)ti << sh);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        // reduce over the warp's 32 rows, per input
#pragma unroll
        for (int c = 0; c < LT_B; c++) {
            float bv = best[c];
            const uint32_t tc = (bti[c >> 1] >> ((c & 1) * 16)) & 0xffffu;
            int bi = tc == 0xffffu ? 0x7fffffff : (int)((blockIdx.x + tc * gridDim.x) * LT_BM + row);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) {
                red_v[q][c] = bv;
                red_i[q][c] = bi;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < p.B) {
        const int c = threadIdx.x;
        float bv = red_v[0][c];
        int bi = red_i[0][c];
        for (int w = 1; w < 4; w++)
            if (red_v[w][c] > bv || (red_v[w][c] == bv && red_i[w][c] < bi)) {
                bv = red_v[w][c];
                bi = red_i[w][c];
            }
        if (bi != 0x7fffffff) atomicMax(&p.slot[c], argmax_key(bv, (uint32_t)bi));
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last && threadIdx.x < p.B) {
        __threadfence();
        const unsigned long long k = atomicExch(&p.slot[threadIdx.x], 0ull);
        const uint32_t ord = (uint32_t)(k >> 32);
        const uint32_t bits = (ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord;
        p.tok[threadIdx.x] = k ? (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull)) : -1;
        p.val[threadIdx.x] = __uint_as_float(bits);
    }
    if (last && threadIdx.x == 0) *p.ticket = 0u;
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * LT_BN);
    }
}

}  // namespace ds

using namespace ds;

// Tensor-core batched argmax: B <= 64 inputs d_x [B x in_dim] (device),
// d_W [out_dim x in_dim] BF16 (device), in_dim % 64 == 0. Returns
// DS_CUDA_EINVAL when the shape does not fit (the caller then uses the
// CUDA-core path).
int lmhead_tc_enqueue(ds_cuda_ctx *c, const float *d_x, const uint16_t *d_W, int in_dim, int out_dim, int batch,
                      int *d_tok, float *d_val, cudaStream_t st) {
    if (batch <= 0 || batch > LT_B || in_dim % 64 || in_dim <= 0 || out_dim <= 0) return DS_CUDA_EINVAL;
    void *planes = c->d_lt_planes;
    size_t need = (size_t)2 * LT_B * in_dim * 2;
    if (ctx_grow(c, &c->d_lt_planes, &c->lt_planes_cap, need) < 0) return DS_CUDA_ENOMEM;
    planes = c->d_lt_planes;
    if (!c->d_lt_err) {
        if (cudaMalloc(&c->d_lt_err, 4) != cudaSuccess) return ctx_fail(c, DS_CUDA_ENOMEM, "lm head error flag");
        cudaMemsetAsync(c->d_lt_err, 0, 4, st);
    }
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(lt_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LT_SMEM);
        attr = true;
    }
    lt_split_kernel<<<dim3((in_dim + 255) / 256, LT_B), 256, 0, st>>>(d_x, batch, in_dim, (uint16_t *)planes);
    LtArgs a;
    memset(&a, 0, sizeof a);
    if (!tmap_bf16(&a.w, d_W, in_dim, out_dim, LT_BM) || !tmap_bf16(&a.x, planes, in_dim, 2 * LT_B, LT_BN))
        return ctx_fail(c, DS_CUDA_ECUDA, "lm head: tensor map encoding failed");
    a.V = out_dim;
    a.K = in_dim;
    a.B = batch;
    a.slot = c->d_slots;        // zero between uses (the last CTA resets them)
    a.ticket = c->d_tickets + 2;
    a.tok = d_tok;
    a.val = d_val;
    a.err = (unsigned *)c->d_lt_err;
    const int tiles = (out_dim + LT_BM - 1) / LT_BM;
    const int grid = tiles < c->sm_count ? tiles : c->sm_count;
    lt_argmax_kernel<<<grid, LT_THREADS, LT_SMEM, st>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DS_CUDA_OK : ctx_cuda(c, e, "lm head tensor-core launch");
}
