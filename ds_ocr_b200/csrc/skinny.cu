// skinny.cu — tcgen05 GEMM for up to 64 token rows against BF16 weights
// (multi-stream decode): warp 0 streams weight tiles (A, 128 rows) and the
// split token planes (B, 64 hi + 64 lo rows) with TMA through a 6-stage ring,
// warp 1 issues M=128, N=128, K=16 MMAs into a double-buffered tensor-memory
// accumulator, warps 2-5 add the hi and lo columns and write outputs.
// MODE 0: Y = x.W (+ residual). MODE 1: SwiGLU over a tile of 64 gate rows
// and the matching 64 up rows, written as the next GEMM's split planes.
#include <cstring>
#include <vector>
#include "ctx.h"
#include "skinny.cuh"
#include "tmap.h"
#include "umma.cuh"

namespace ds {

constexpr int SK_STAGES = 6;
constexpr int SK_THREADS = 192;
constexpr int SK_A_BYTES = 128 * 128;  // 128 rows x 64 BF16
constexpr int SK_STAGE_BYTES = 2 * SK_A_BYTES;
constexpr int SK_XCH = 64 * 65 * 4;    // SwiGLU gate exchange
constexpr int SK_SMEM = SK_STAGES * SK_STAGE_BYTES + SK_XCH + 1024;

// Named barrier of the 4 epilogue warps; the _or form also ORs a flag over
// them (so a wait that gave up on one thread stops all four warps together).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool epi_bar_or(bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
                 "bar.red.or.pred po, 1, 128, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
                 : "=r"(r) : "r"((uint32_t)v) : "memory");
    return r != 0;
}

template <int MODE>
__global__ void __launch_bounds__(SK_THREADS, 1) sk_gemm_kernel(const __grid_constant__ SkGemm p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *xch = reinterpret_cast<float *>(smem + SK_STAGES * SK_STAGE_BYTES);
    __shared__ uint64_t full[SK_STAGES], empty[SK_STAGES], acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = *p.n_tiles;
    if (threadIdx.x == 0) {
        for (int s = 0; s < SK_STAGES; s++) {
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
    if (warp == 1) tmem_alloc(&tmem_base, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const SkTile tl = p.tiles[t];
                const CUtensorMap *am = &p.a[tl.amap];
                const CUtensorMap *am2 = &p.a[MODE == 1 ? tl.amap2 : tl.amap];
                const CUtensorMap *bm = &p.b[tl.kind];
                const int r2 = MODE == 1 ? tl.a_row2 : tl.a_row + 64;
                for (int kb = 0; kb < tl.kb; kb++, it++) {
                    const int s = it % SK_STAGES, r = it / SK_STAGES;
                    if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + s * SK_STAGE_BYTES;
                    const int kx = (tl.k0 + kb) * 64;
                    mbar_expect_tx(&full[s], SK_STAGE_BYTES);
                    tma_load_2d(st, am, kx, tl.a_row, &full[s]);
                    tma_load_2d(st + SK_A_BYTES / 2, am2, kx, r2, &full[s]);
                    tma_load_2d(st + SK_A_BYTES, bm, kx, tl.b_row, &full[s]);
                    tma_load_2d(st + SK_A_BYTES + SK_A_BYTES / 2, bm, kx, p.lo_off[tl.kind] + tl.b_row, &full[s]);
                }
            }
            for (int i = max(0, it - SK_STAGES); i < it; i++)
                mbar_wait(&full[i % SK_STAGES], (i / SK_STAGES) & 1, p.err);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(128, 128);
            int it = 0, ti = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ti++) {
                const int b = ti & 1, u = ti >> 1;
                if (u > 0 && !mbar_wait(&acc_empty[b], (u - 1) & 1, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + b * 128;
                const int nk = p.tiles[t].kb;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % SK_STAGES, r = it / SK_STAGES;
                    if (!mbar_wait(&full[s], r & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t *st = smem + s * SK_STAGE_BYTES;
                    const uint64_t ad = sw128_desc(st), bd = sw128_desc(st + SK_A_BYTES);
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
        const int q = warp & 3;
        const int row = q * 32 + lane;  // accumulator lane = weight row of the tile
        int ti = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ti++) {
            const int b = ti & 1, u = ti >> 1;
            bool bad = !mbar_wait(&acc_full[b], u & 1, p.err);
            // the four warps leave together (SwiGLU exchange buffer, split-K
            // hand-over)
            bad = epi_bar_or(bad);
            if (bad) break;
            tc_fence_after();
            const SkTile tl = p.tiles[t];
            const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + b * 128;
            if (MODE == 0) {
                const int col = tl.out_col + row;
                const bool cv = col < p.out_n[tl.amap];
                float *out = p.out[tl.amap];
                const float *res = p.resid[tl.amap];
                const int ld = p.out_ld[tl.amap];
                if (tl.nsplit <= 1) {
#pragma unroll 1
                    for (int c0 = 0; c0 < SK_TOK; c0 += 16) {
                        float h[16], l[16];
                        tmem_ld16(tb + c0, h);
                        tmem_ld16(tb + SK_TOK + c0, l);
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const int tok = c0 + j;
                            if (cv && tok < tl.n_tok) {
                                const size_t o = (size_t)(tl.b_row + tok) * ld + col;
                                float v = __fadd_rn(h[j], l[j]);
                                if (res) v = __fadd_rn(res[o], v);
                                out[o] = v;
                            }
                        }
                    }
                } else {
                    // split K: this part to the part buffer ([tok][row]: a
                    // warp's stores are contiguous); the reader sums the parts
                    float *mine = p.ws + ((size_t)tl.otile * p.max_split + tl.split) * SK_TOK * 128 + row;
#pragma unroll 1
                    for (int c0 = 0; c0 < SK_TOK; c0 += 16) {
                        float h[16], l[16];
                        tmem_ld16(tb + c0, h);
                        tmem_ld16(tb + SK_TOK + c0, l);
#pragma unroll
                        for (int j = 0; j < 16; j++) mine[(size_t)(c0 + j) * 128] = __fadd_rn(h[j], l[j]);
                    }
                }
            } else {
                // lanes 0..63: gate rows -> exchange buffer; lanes 64..127:
                // up rows, kept in registers until the gates are in
                float uv[SK_TOK];
#pragma unroll
                for (int c0 = 0; c0 < SK_TOK; c0 += 16) {
                    float h[16], l[16];
                    tmem_ld16(tb + c0, h);
                    tmem_ld16(tb + SK_TOK + c0, l);
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const float v = __fadd_rn(h[j], l[j]);
                        if (row < 64) xch[row * 65 + c0 + j] = v;
                        uv[c0 + j] = v;
                    }
                }
                epi_bar();
                if (row >= 64) {
                    const int i = row - 64;
#pragma unroll
                    for (int tok = 0; tok < SK_TOK; tok++) {
                        if (tok < tl.n_tok) {
                            uint16_t hi, lo;
                            split_bf16(swiglu(xch[i * 65 + tok], uv[tok]), hi, lo);
                            const size_t o = (size_t)(tl.b_row + tok) * p.h_ld[tl.kind] + tl.out_col + i;
                            p.h_hi[tl.kind][o] = hi;
                            p.h_lo[tl.kind][o] = lo;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// x [n x K] F32 (optionally RMS-normalised with w: (x * w) * inv) -> planes
// [2*lo_off x K]: hi rows 0..n-1, lo rows lo_off..lo_off+n-1. One block of
// 128 threads per row; K % 4 == 0. With `parts` the row is first assembled
// from a split-K GEMM's parts (+ resid) and written to x_out.
struct SkParts {
    const float *ws;
    int max_split, nsplit;
    const float *resid;
    float *x_out;
};

__global__ void __launch_bounds__(128) sk_split_kernel(const float *__restrict__ x, int n, int K, int x_ld,
                                                       const float *__restrict__ w, float eps, uint16_t *planes,
                                                       int lo_off, float *normed, SkParts parts) {
    __shared__ float part[4];
    const int r = blockIdx.x;
    if (r >= n) return;
    const float *xr = x + (size_t)r * x_ld;
    if (parts.ws) {
        // assemble the row, then read it back like a plain input
        for (int c = threadIdx.x * 4; c < K; c += 512) {
            float4 v;
            v.x = sk_part_sum(parts.ws, parts.max_split, parts.nsplit, r, c);
            v.y = sk_part_sum(parts.ws, parts.max_split, parts.nsplit, r, c + 1);
            v.z = sk_part_sum(parts.ws, parts.max_split, parts.nsplit, r, c + 2);
            v.w = sk_part_sum(parts.ws, parts.max_split, parts.nsplit, r, c + 3);
            if (parts.resid) {
                const float4 q = *reinterpret_cast<const float4 *>(parts.resid + (size_t)r * K + c);
                v.x = __fadd_rn(q.x, v.x);
                v.y = __fadd_rn(q.y, v.y);
                v.z = __fadd_rn(q.z, v.z);
                v.w = __fadd_rn(q.w, v.w);
            }
            *reinterpret_cast<float4 *>(parts.x_out + (size_t)r * K + c) = v;
        }
        __syncthreads();
        xr = parts.x_out + (size_t)r * K;
    }
    float inv = 1.f;
    if (w) {
        float ss = 0.f;
        for (int c = threadIdx.x * 4; c < K; c += 512) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c);
            ss = __fmaf_rn(v.x, v.x, ss);
            ss = __fmaf_rn(v.y, v.y, ss);
            ss = __fmaf_rn(v.z, v.z, ss);
            ss = __fmaf_rn(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        ss = __fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3]));
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
    }
    for (int c = threadIdx.x * 4; c < K; c += 512) {
        float4 v = *reinterpret_cast<const float4 *>(xr + c);
        if (w) {
            const float4 g = *reinterpret_cast<const float4 *>(w + c);
            v.x = __fmul_rn(__fmul_rn(v.x, g.x), inv);
            v.y = __fmul_rn(__fmul_rn(v.y, g.y), inv);
            v.z = __fmul_rn(__fmul_rn(v.z, g.z), inv);
            v.w = __fmul_rn(__fmul_rn(v.w, g.w), inv);
        }
        if (normed) *reinterpret_cast<float4 *>(normed + (size_t)r * K + c) = v;
        uint16_t h[4], l[4];
        split_bf16(v.x, h[0], l[0]);
        split_bf16(v.y, h[1], l[1]);
        split_bf16(v.z, h[2], l[2]);
        split_bf16(v.w, h[3], l[3]);
        *reinterpret_cast<uint2 *>(planes + (size_t)r * K + c) =
            make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
        *reinterpret_cast<uint2 *>(planes + (size_t)(lo_off + r) * K + c) =
            make_uint2((uint32_t)l[0] | ((uint32_t)l[1] << 16), (uint32_t)l[2] | ((uint32_t)l[3] << 16));
    }
}

}  // namespace ds

using namespace ds;

void sk_set_attrs() {
    static bool done = false;
    if (done) return;
    cudaFuncSetAttribute(sk_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM);
    cudaFuncSetAttribute(sk_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM);
    done = true;
}

cudaError_t sk_gemm_launch(int mode, const SkGemm &g, int grid, cudaStream_t st) {
    sk_set_attrs();
    if (mode == 0) sk_gemm_kernel<0><<<grid, SK_THREADS, SK_SMEM, st>>>(g);
    else sk_gemm_kernel<1><<<grid, SK_THREADS, SK_SMEM, st>>>(g);
    return cudaGetLastError();
}

cudaError_t sk_split_launch(const float *x, int n, int K, int x_ld, const float *w, float eps, uint16_t *planes,
                            int lo_off, float *normed, cudaStream_t st, const float *ws, int max_split, int nsplit,
                            const float *resid, float *x_out) {
    if (n <= 0) return cudaSuccess;
    SkParts parts = {ws, max_split, nsplit, resid, x_out};
    sk_split_kernel<<<n, 128, 0, st>>>(x, n, K, x_ld, w, eps, planes, lo_off, normed, parts);
    return cudaGetLastError();
}

// out [n x N] = resid + the split-K parts (the standalone GEMM entry's reader).
__global__ void sk_reduce_kernel(const float *ws, int max_split, int nsplit, int n, int N, const float *resid,
                                 float *out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * N) return;
    const int tok = i / N, f = i - tok * N;
    const float v = sk_part_sum(ws, max_split, nsplit, tok, f);
    out[i] = resid ? __fadd_rn(resid[i], v) : v;
}

// Y [n x N] = x [n x K] . W^T on the tensor cores (n <= 64, K % 128 == 0),
// optionally + resid [n x N]; a standalone entry of the multi-stream GEMM.
extern "C" int ds_cuda_skinny_matmul_dev(ds_cuda_ctx_t *c, const float *d_x, int n, int K, const uint16_t *d_W,
                                         int N, const float *d_resid, float *d_y, void *stream) {
    if (!c || !c->ok || n <= 0 || n > SK_TOK || K <= 0 || K % 64 || N <= 0 || !d_x || !d_W || !d_y)
        return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    const size_t plane_bytes = ((size_t)2 * SK_TOK * K * 2 + 255) & ~size_t(255);
    const int otiles = (N + 127) / 128;
    // split K so that the parts cover the SMs
    int nsplit = c->sm_count / otiles;
    nsplit = nsplit < 1 ? 1 : (nsplit > SK_MAX_SPLIT ? SK_MAX_SPLIT : nsplit);
    const int ntiles_max = otiles * nsplit;
    const size_t tile_bytes = ((size_t)ntiles_max * sizeof(SkTile) + 16 + 255) & ~size_t(255);
    const size_t ws_bytes = nsplit > 1 ? (size_t)otiles * SK_MAX_SPLIT * 128 * SK_TOK * 4 : 0;
    if (otiles > 1000) return ctx_fail(c, DS_CUDA_EINVAL, "skinny_matmul: N too large");
    // [0, 4 KB): the tile count; then planes, tiles, split-K parts
    const size_t head = 4096;
    const size_t need = head + plane_bytes + tile_bytes + ws_bytes;
    const bool fresh = need > c->sk_scratch_cap;
    if (ctx_grow(c, &c->d_sk_scratch, &c->sk_scratch_cap, need) < 0) return DS_CUDA_ENOMEM;
    uint8_t *base = (uint8_t *)c->d_sk_scratch;
    int *nt = (int *)(base + head - 16);
    uint16_t *planes = (uint16_t *)(base + head);
    SkTile *tiles = (SkTile *)(base + head + plane_bytes);
    float *ws = (float *)(base + head + plane_bytes + tile_bytes);
    if (fresh) cudaMemsetAsync(base, 0, c->sk_scratch_cap, st);
    else cudaMemsetAsync(planes, 0, plane_bytes, st);
    cudaError_t e = sk_split_launch(d_x, n, K, K, nullptr, 0.f, planes, SK_TOK, nullptr, st, nullptr, 0, 0, nullptr,
                                    nullptr);
    if (e != cudaSuccess) return ctx_cuda(c, e, "skinny split");
    std::vector<SkTile> ht;
    for (int t = 0; t < otiles; t++) sk_push_split(ht, SkTile{0, t * 128, 0, 0, 0, 0, n, t * 128, K / 64}, nsplit, t);
    const int ntiles = (int)ht.size();
    // pageable sources: the copies are staged before the calls return
    cudaMemcpyAsync(tiles, ht.data(), ntiles * sizeof(SkTile), cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(nt, &ntiles, sizeof(int), cudaMemcpyHostToDevice, st);
    SkGemm g;
    memset(&g, 0, sizeof g);
    if (!tmap_bf16(&g.a[0], d_W, K, N, 64) || !tmap_bf16(&g.b[0], planes, K, 2 * SK_TOK, 64))
        return ctx_fail(c, DS_CUDA_ECUDA, "skinny: tensor map encoding failed");
    g.lo_off[0] = SK_TOK;
    g.tiles = tiles;
    g.n_tiles = nt;
    g.out[0] = d_y;
    g.resid[0] = d_resid;
    g.out_ld[0] = N;
    g.out_n[0] = N;
    g.ws = ws;
    g.max_split = SK_MAX_SPLIT;
    g.err = (unsigned *)c->d_lt_err;
    if (!g.err) {
        if (cudaMalloc(&c->d_lt_err, 4) != cudaSuccess) return ctx_fail(c, DS_CUDA_ENOMEM, "skinny error flag");
        cudaMemsetAsync(c->d_lt_err, 0, 4, st);
        g.err = (unsigned *)c->d_lt_err;
    }
    e = sk_gemm_launch(0, g, ntiles < c->sm_count ? ntiles : c->sm_count, st);
    if (e == cudaSuccess && nsplit > 1)
        sk_reduce_kernel<<<(n * N + 255) / 256, 256, 0, st>>>(ws, SK_MAX_SPLIT, nsplit, n, N, d_resid, d_y);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? DS_CUDA_OK : ctx_cuda(c, e, "skinny gemm launch");
}
