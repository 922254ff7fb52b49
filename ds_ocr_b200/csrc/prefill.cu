// prefill.cu — batched MoE prefill block of ds_decoder_prefill
// (ds_moe_decoder.c:630-809) for n tokens at once, on the 5th-generation
// tensor cores.
//
// Per MoE layer the reference computes, for x [n x H] (F32):
//   xn = RMSNorm(x)                                  (:598, ds_rms_norm)
//   logits = xn W_r^T; softmax (fast exp); top-6     (:643-686, no renorm)
//   shared = down_s(SwiGLU(xn Wg_s^T, xn Wu_s^T))    (:688-712, sgemm)
//   per expert e, over its tokens (ascending e):     (:714-791)
//     y = down_e(SwiGLU(X_e Wg_e^T, X_e Wu_e^T)); routed[s] += w * y
//   x += routed + shared                              (:794-800)
// with BF16 weights widened exactly to F32 and F32 GEMMs (cblas_sgemm).
//
// B200 design:
//   * activations are split into two BF16 planes, hi = bf16(v) and
//     lo = bf16(v - hi), so hi + lo carries 16 significant bits; the weights
//     are exact in BF16. Each GEMM runs A_hi*B + A_lo*B into one F32
//     accumulator (tcgen05.mma kind::f16, accumulator in tensor memory):
//     twice the tensor work of a plain BF16 GEMM, F32-class accuracy.
//   * routing groups token copies by expert into contiguous row segments
//     (counting sort), so every expert's A operand is a plain 2-D TMA tile.
//   * one persistent grouped-GEMM kernel per stage walks a device-built tile
//     list (routed expert tiles and shared-expert tiles together): warp 0
//     streams A_hi/A_lo/B tiles with TMA into a 3-stage ring, warp 1 issues
//     the MMAs, warps 2-5 drain the accumulator (two tensor-memory buffers,
//     so the epilogue of one tile overlaps the main loop of the next).
//   * gate/up tiles hold 128 gate rows and the matching 128 up rows, so the
//     SwiGLU runs in the epilogue and writes the down GEMM's split A planes.
//   * the down GEMM writes each routed (token, slot) row; a combine kernel
//     sums a token's 6 rows in ascending expert order (the reference's
//     accumulation order) and adds the shared expert and the residual.
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <vector>
#include <cuda.h>
#include "ctx.h"
#include "umma.cuh"
#include "tmap.h"
#include "route.cuh"
#include "prefill.h"

namespace ds {

constexpr int PF_BM = 128;  // tile rows (tokens) = tensor-memory lanes
constexpr int PF_BK = 64;   // K per stage: one 128-byte swizzle row of BF16
constexpr int PF_BN = 256;  // accumulator columns per tile
constexpr int PF_STAGES = 3;
constexpr int PF_THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int PF_A_BYTES = PF_BM * PF_BK * 2;
constexpr int PF_B_BYTES = PF_BN * PF_BK * 2;
constexpr int PF_STAGE_BYTES = 2 * PF_A_BYTES + PF_B_BYTES;
constexpr int PF_SMEM = PF_STAGES * PF_STAGE_BYTES + 1024;
constexpr int PF_MAXE = 256;

struct PfTile {
    int kind;   // 0: routed expert, 1: shared expert
    int e;      // expert (kind 0)
    int a_row;  // first row of the tile in the A planes
    int rows;   // valid rows (<= 128)
    int n0;     // first output column (gate/up: first gate row)
};

struct PfGemm {
    CUtensorMap a_hi[2], a_lo[2], b[2];  // [kind]
    const PfTile *tiles;
    const int *n_tiles;
    int k_blocks[2];
    int b_base[2], b_group_rows[2], b_half[2];
    uint16_t *h_hi[2], *h_lo[2];  // gate/up epilogue outputs
    int h_ld[2];
    float *y[2];                  // down epilogue outputs
    const int *slot_of;           // routed: output row of each sorted position
    int y_ld;
    unsigned *err;
};

// ---------------------------------------------------------------------------
// Grouped split-BF16 GEMM. MODE 0: gate/up + SwiGLU; MODE 1: down.
// ---------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(PF_THREADS, 1) pf_gemm_kernel(const __grid_constant__ PfGemm p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[PF_STAGES], empty[PF_STAGES], acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = *p.n_tiles;
    if (threadIdx.x == 0) {
        for (int s = 0; s < PF_STAGES; s++) {
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
    if (warp == 1) tmem_alloc(&tmem_base, 2 * PF_BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // producer: A_hi, A_lo and B tiles of every k block of every tile
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const PfTile tl = p.tiles[t];
                const int kind = tl.kind;
                const int brow = p.b_base[kind] + tl.e * p.b_group_rows[kind] + tl.n0;
                for (int kb = 0; kb < p.k_blocks[kind]; kb++, it++) {
                    const int s = it % PF_STAGES, r = it / PF_STAGES;
                    if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + s * PF_STAGE_BYTES;
                    mbar_expect_tx(&full[s], PF_STAGE_BYTES);
                    tma_load_2d(st, &p.a_hi[kind], kb * PF_BK, tl.a_row, &full[s]);
                    tma_load_2d(st + PF_A_BYTES, &p.a_lo[kind], kb * PF_BK, tl.a_row, &full[s]);
                    if (MODE == 0) {
                        tma_load_2d(st + 2 * PF_A_BYTES, &p.b[kind], kb * PF_BK, brow, &full[s]);
                        tma_load_2d(st + 2 * PF_A_BYTES + PF_B_BYTES / 2, &p.b[kind], kb * PF_BK,
                                    brow + p.b_half[kind], &full[s]);
                    } else {
                        tma_load_2d(st + 2 * PF_A_BYTES, &p.b[kind], kb * PF_BK, brow, &full[s]);
                    }
                }
            }
            // the last copies have landed before the CTA can exit (already
            // true unless a wait above gave up)
            for (int i = max(0, it - PF_STAGES); i < it; i++)
                mbar_wait(&full[i % PF_STAGES], (i / PF_STAGES) & 1, p.err);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: 4 K=16 steps per stage, hi and lo against one B
            constexpr uint32_t idesc = idesc_bf16_f32(PF_BM, PF_BN);
            int it = 0, ti = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ti++) {
                const int b = ti & 1, u = ti >> 1;
                if (u > 0 && !mbar_wait(&acc_empty[b], (u - 1) & 1, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + b * PF_BN;
                const int nk = p.k_blocks[p.tiles[t].kind];
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % PF_STAGES, r = it / PF_STAGES;
                    if (!mbar_wait(&full[s], r & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t *st = smem + s * PF_STAGE_BYTES;
                    const uint64_t ah = sw128_desc(st), al = sw128_desc(st + PF_A_BYTES);
                    const uint64_t bd = sw128_desc(st + 2 * PF_A_BYTES);
#pragma unroll
                    for (int j = 0; j < PF_BK / 16; j++) {
                        umma_bf16(d, ah + 2 * j, bd + 2 * j, idesc, (kb | j) != 0);
                        umma_bf16(d, al + 2 * j, bd + 2 * j, idesc, 1u);
                    }
                    umma_commit(&empty[s]);  // frees the stage when these MMAs finish
                }
                if (ok) umma_commit(&acc_full[b]);
            }
            // every MMA has finished before tensor memory is released
            umma_commit(&drain);
            mbar_wait(&drain, 0, p.err);
        }
    } else {
        // epilogue: warp w reads tensor-memory lanes 32*(w%4) .. +31 = tile rows
        const int q = warp & 3;
        const int row = q * 32 + lane;
        int ti = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ti++) {
            const int b = ti & 1, u = ti >> 1;
            if (!mbar_wait(&acc_full[b], u & 1, p.err)) break;
            tc_fence_after();
            const PfTile tl = p.tiles[t];
            const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + b * PF_BN;
            const bool valid = row < tl.rows;
            if (MODE == 0) {
                const size_t orow = (size_t)(tl.a_row + row) * p.h_ld[tl.kind] + tl.n0;
#pragma unroll 1
                for (int c0 = 0; c0 < PF_BN / 2; c0 += 32) {
                    float g[32], v[32];
                    tmem_ld32(tb + c0, g);
                    tmem_ld32(tb + PF_BN / 2 + c0, v);
                    if (valid) {
                        uint32_t hw[16], lw[16];
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            uint16_t h0, l0, h1, l1;
                            split_bf16(swiglu(g[j], v[j]), h0, l0);
                            split_bf16(swiglu(g[j + 1], v[j + 1]), h1, l1);
                            hw[j / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                            lw[j / 2] = (uint32_t)l0 | ((uint32_t)l1 << 16);
                        }
                        uint4 *dh = reinterpret_cast<uint4 *>(p.h_hi[tl.kind] + orow + c0);
                        uint4 *dl = reinterpret_cast<uint4 *>(p.h_lo[tl.kind] + orow + c0);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            dh[j] = make_uint4(hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]);
                            dl[j] = make_uint4(lw[4 * j], lw[4 * j + 1], lw[4 * j + 2], lw[4 * j + 3]);
                        }
                    }
                }
            } else {
                int orow_i = tl.a_row + row;
                if (tl.kind == 0 && valid) orow_i = p.slot_of[orow_i];
                float *dst = p.y[tl.kind] + (size_t)orow_i * p.y_ld + tl.n0;
#pragma unroll 1
                for (int c0 = 0; c0 < PF_BN; c0 += 32) {
                    float v[32];
                    tmem_ld32(tb + c0, v);
                    if (valid) {
                        float4 *d4 = reinterpret_cast<float4 *>(dst + c0);
#pragma unroll
                        for (int j = 0; j < 8; j++) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
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
        tmem_dealloc(tmem, 2 * PF_BN);
    }
}

// ---------------------------------------------------------------------------
// Per-token RMSNorm (ds_rms_norm), split into BF16 planes, and routing:
// softmax with fast exp over the logits (given, or xn W_r^T), strict-'>'
// top-k, weights = probabilities (ds_moe_decoder.c:652-686). One warp per
// token; H a multiple of 128, E <= 256.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pf_norm_route_kernel(const float *__restrict__ x, const float *__restrict__ nw,
                                                            float eps, int M, int H, const float *logits_in, int lg_ld,
                                                            const uint16_t *__restrict__ Wr, float *logits_buf, int E,
                                                            int K, int renorm, uint16_t *xn_hi, uint16_t *xn_lo,
                                                            int *idx, float *wt) {
    const int lane = threadIdx.x & 31;
    const int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (s >= M) return;
    const float *xr = x + (size_t)s * H;
    const int nv = H / 128;  // float4 per lane
    float4 v[16];
    float ss = 0.f;
    for (int i = 0; i < nv; i++) {
        v[i] = *reinterpret_cast<const float4 *>(xr + 4 * (lane + 32 * i));
        ss = __fmaf_rn(v[i].x, v[i].x, ss);
        ss = __fmaf_rn(v[i].y, v[i].y, ss);
        ss = __fmaf_rn(v[i].z, v[i].z, ss);
        ss = __fmaf_rn(v[i].w, v[i].w, ss);
    }
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
    for (int i = 0; i < nv; i++) {
        const int c = 4 * (lane + 32 * i);
        const float4 w4 = *reinterpret_cast<const float4 *>(nw + c);
        v[i].x = __fmul_rn(__fmul_rn(v[i].x, w4.x), inv);
        v[i].y = __fmul_rn(__fmul_rn(v[i].y, w4.y), inv);
        v[i].z = __fmul_rn(__fmul_rn(v[i].z, w4.z), inv);
        v[i].w = __fmul_rn(__fmul_rn(v[i].w, w4.w), inv);
        uint16_t h[4], l[4];
        split_bf16(v[i].x, h[0], l[0]);
        split_bf16(v[i].y, h[1], l[1]);
        split_bf16(v[i].z, h[2], l[2]);
        split_bf16(v[i].w, h[3], l[3]);
        *reinterpret_cast<uint2 *>(xn_hi + (size_t)s * H + c) =
            make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
        *reinterpret_cast<uint2 *>(xn_lo + (size_t)s * H + c) =
            make_uint2((uint32_t)l[0] | ((uint32_t)l[1] << 16), (uint32_t)l[2] | ((uint32_t)l[3] << 16));
    }
    const float *lg;
    if (logits_in) {
        lg = logits_in + (size_t)s * lg_ld;
    } else {
        // router scores in F32 from the normalised row (ds_linear_nobias_bf16)
        float *out = logits_buf + (size_t)s * E;
        for (int e = 0; e < E; e++) {
            const uint16_t *wr = Wr + (size_t)e * H;
            float acc = 0.f;
            for (int i = 0; i < nv; i++) {
                const uint2 w2 = *reinterpret_cast<const uint2 *>(wr + 4 * (lane + 32 * i));
                acc = __fmaf_rn(v[i].x, __uint_as_float(w2.x << 16), acc);
                acc = __fmaf_rn(v[i].y, __uint_as_float(w2.x & 0xffff0000u), acc);
                acc = __fmaf_rn(v[i].z, __uint_as_float(w2.y << 16), acc);
                acc = __fmaf_rn(v[i].w, __uint_as_float(w2.y & 0xffff0000u), acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) out[e] = acc;
        }
        __syncwarp();
        lg = out;
    }
    route_topk_warp(lg, E, K, renorm, idx + (size_t)s * K, wt + (size_t)s * K);
}

// Segment starts of the expert-sorted rows, cursors, and the tile lists of
// both GEMM stages (shared-expert tiles first, then routed ones). One block.
__global__ void __launch_bounds__(256) pf_plan_kernel(int *counts, int E, int M_sh, int I, int S, int H, int *seg,
                                                      int *cursor, PfTile *gu_tiles, int *n_gu, PfTile *dn_tiles,
                                                      int *n_dn) {
    __shared__ int cnt[PF_MAXE], mt[PF_MAXE], seg_s[PF_MAXE], mto[PF_MAXE + 1];
    const int t = threadIdx.x;
    if (t < E) {
        cnt[t] = counts[t];
        mt[t] = (cnt[t] + PF_BM - 1) / PF_BM;
    }
    __syncthreads();
    if (t == 0) {
        int a = 0, b = 0;
        for (int e = 0; e < E; e++) {
            seg_s[e] = a;
            mto[e] = b;
            a += cnt[e];
            b += mt[e];
        }
        mto[E] = b;
    }
    __syncthreads();
    const int mts = (M_sh + PF_BM - 1) / PF_BM;
    const int gu_nt_r = I / 128, gu_nt_s = S / 128, dn_nt = H / PF_BN;
    const int sh_gu = mts * gu_nt_s, sh_dn = mts * dn_nt;
    for (int i = t; i < sh_gu; i += blockDim.x) {
        const int m = i / gu_nt_s, n = i - m * gu_nt_s;
        gu_tiles[i] = PfTile{1, 0, m * PF_BM, min(PF_BM, M_sh - m * PF_BM), n * 128};
    }
    for (int i = t; i < sh_dn; i += blockDim.x) {
        const int m = i / dn_nt, n = i - m * dn_nt;
        dn_tiles[i] = PfTile{1, 0, m * PF_BM, min(PF_BM, M_sh - m * PF_BM), n * PF_BN};
    }
    if (t < E) {
        seg[t] = seg_s[t];
        cursor[t] = 0;
        for (int m = 0; m < mt[t]; m++) {
            const int r0 = seg_s[t] + m * PF_BM, rows = min(PF_BM, cnt[t] - m * PF_BM);
            for (int n = 0; n < gu_nt_r; n++)
                gu_tiles[sh_gu + (mto[t] + m) * gu_nt_r + n] = PfTile{0, t, r0, rows, n * 128};
            for (int n = 0; n < dn_nt; n++)
                dn_tiles[sh_dn + (mto[t] + m) * dn_nt + n] = PfTile{0, t, r0, rows, n * PF_BN};
        }
        counts[t] = 0;  // ready for the next layer
    }
    if (t == 0) {
        *n_gu = sh_gu + mto[E] * gu_nt_r;
        *n_dn = sh_dn + mto[E] * dn_nt;
    }
}

// Tokens per expert over the (row, expert) pairs (block histogram first).
__global__ void __launch_bounds__(256) pf_count_kernel(int P, const int *__restrict__ pair_expert, int E, int *counts) {
    __shared__ int h[PF_MAXE];
    for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
    __syncthreads();
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P; p += gridDim.x * blockDim.x) {
        const int e = pair_expert[p];
        if ((unsigned)e < (unsigned)E) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        if (h[e]) atomicAdd(&counts[e], h[e]);
}

// Copies the split row of each (row, expert) pair to the next free slot of
// the expert's segment; slot_of[slot] = pair. pair_row == null: row = p / K.
// Source rows are ld elements apart (ld % 8 == 0). inv (optional): inv[p] =
// the slot of pair p.
__global__ void __launch_bounds__(256) pf_scatter_kernel(int P, int H, int ld, int K, const int *pair_row,
                                                         const int *pair_expert, int E, const int *seg, int *cursor,
                                                         const uint16_t *rows_hi, const uint16_t *rows_lo,
                                                         uint16_t *xg_hi, uint16_t *xg_lo, int *slot_of, int *inv) {
    const int lane = threadIdx.x & 31;
    const int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (p >= P) return;
    const int e = pair_expert[p];
    if ((unsigned)e >= (unsigned)E) return;
    const int r = pair_row ? pair_row[p] : p / K;
    int pos = 0;
    if (lane == 0) {
        pos = seg[e] + atomicAdd(&cursor[e], 1);
        slot_of[pos] = p;
        if (inv) inv[p] = pos;
    }
    pos = __shfl_sync(0xffffffffu, pos, 0);
    const uint4 *sh = reinterpret_cast<const uint4 *>(rows_hi + (size_t)r * ld);
    const uint4 *sl = reinterpret_cast<const uint4 *>(rows_lo + (size_t)r * ld);
    uint4 *dh = reinterpret_cast<uint4 *>(xg_hi + (size_t)pos * H);
    uint4 *dl = reinterpret_cast<uint4 *>(xg_lo + (size_t)pos * H);
    for (int i = lane; i < H / 8; i += 32) {
        dh[i] = sh[i];
        dl[i] = sl[i];
    }
}

// x[s] += (sum over the token's experts in ascending order of w_k * y_k) +
// shared[s]  (ds_moe_decoder.c:785-800). y_k is row s*K + k of yr, or row
// yrow[s*K + k] when given.
// One block of 128 threads per token; threads over float4 columns.
// y_alt (optional): rows [alt_lo, alt_hi) of the yrow index space are read
// from y_alt instead (row r at y_alt + (r - alt_lo) * H), so an
// expert-parallel rank reads its own experts' outputs where they were
// written, without copying them into the returned stream.
__global__ void __launch_bounds__(128) pf_combine_kernel(float *x, int M, int H, int K, const int *idx, const float *wt,
                                                         const float *yr, const int *yrow, const float *ys,
                                                         const float *y_alt, long long alt_lo, long long alt_hi) {
    const int s = blockIdx.x;
    if (s >= M) return;
    int ord[8], e[8];
    float w[8];
    const float *src[8];
    for (int k = 0; k < K; k++) {
        ord[k] = k;
        e[k] = idx[(size_t)s * K + k];
    }
    for (int a = 1; a < K; a++)  // insertion sort of the slots by expert
        for (int b = a; b > 0 && e[ord[b]] < e[ord[b - 1]]; b--) {
            int tmp = ord[b];
            ord[b] = ord[b - 1];
            ord[b - 1] = tmp;
        }
    for (int j = 0; j < K; j++) {
        const int k = ord[j];
        w[j] = wt[(size_t)s * K + k];
        const long long r = yrow ? (long long)yrow[(size_t)s * K + k] : (long long)s * K + k;
        src[j] = y_alt && r >= alt_lo && r < alt_hi ? y_alt + (size_t)(r - alt_lo) * H : yr + (size_t)r * H;
    }
    for (int c = 4 * threadIdx.x; c < H; c += 4 * blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < K; j++) {
            const float4 y = *reinterpret_cast<const float4 *>(src[j] + c);
            acc.x = __fmaf_rn(w[j], y.x, acc.x);
            acc.y = __fmaf_rn(w[j], y.y, acc.y);
            acc.z = __fmaf_rn(w[j], y.z, acc.z);
            acc.w = __fmaf_rn(w[j], y.w, acc.w);
        }
        const float4 sh = *reinterpret_cast<const float4 *>(ys + (size_t)s * H + c);
        float4 *xp = reinterpret_cast<float4 *>(x + (size_t)s * H + c);
        float4 xv = *xp;
        xv.x = __fadd_rn(xv.x, __fadd_rn(acc.x, sh.x));
        xv.y = __fadd_rn(xv.y, __fadd_rn(acc.y, sh.y));
        xv.z = __fadd_rn(xv.z, __fadd_rn(acc.z, sh.z));
        xv.w = __fadd_rn(xv.w, __fadd_rn(acc.w, sh.w));
        *xp = xv;
    }
}

}  // namespace ds

using namespace ds;

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct PfWork {
    // grown on demand; caps in bytes
    uint16_t *xn_hi = nullptr, *xn_lo = nullptr, *xg_hi = nullptr, *xg_lo = nullptr;
    uint16_t *hg_hi = nullptr, *hg_lo = nullptr, *hs_hi = nullptr, *hs_lo = nullptr;
    float *yr = nullptr, *ys = nullptr, *logits = nullptr, *wt = nullptr;
    int *idx = nullptr, *slot_of = nullptr;
    PfTile *gu_tiles = nullptr, *dn_tiles = nullptr;
    size_t c_xn_hi = 0, c_xn_lo = 0, c_xg_hi = 0, c_xg_lo = 0, c_hg_hi = 0, c_hg_lo = 0, c_hs_hi = 0, c_hs_lo = 0;
    size_t c_yr = 0, c_ys = 0, c_logits = 0, c_wt = 0, c_idx = 0, c_slot = 0, c_gu = 0, c_dn = 0;
    // dense GEMMs of the whole-decoder prefill (tile list and its count)
    PfTile *dense_tiles = nullptr;
    size_t c_dense = 0;
    int *dense_nt = nullptr;
    // fixed
    int *counts = nullptr, *seg = nullptr, *cursor = nullptr, *nt = nullptr;
    unsigned *err = nullptr;  // set by a device-side wait that gave up
};

void prefill_release(ds_cuda_ctx *c) {
    PfWork *w = (PfWork *)c->prefill;
    if (!w) return;
    void *ptrs[] = {w->xn_hi, w->xn_lo, w->xg_hi, w->xg_lo, w->hg_hi, w->hg_lo, w->hs_hi, w->hs_lo, w->yr,
                    w->ys, w->logits, w->wt, w->idx, w->slot_of, w->gu_tiles, w->dn_tiles, w->counts, w->seg,
                    w->cursor, w->nt, w->err, w->dense_tiles, w->dense_nt};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    delete w;
    c->prefill = nullptr;
}

static int pf_work(ds_cuda_ctx *c, cudaStream_t st, PfWork **out) {
    PfWork *w = (PfWork *)c->prefill;
    if (!w) {
        w = new PfWork();
        c->prefill = w;
        cudaError_t e = cudaMalloc(&w->counts, PF_MAXE * 4);
        if (e == cudaSuccess) e = cudaMalloc(&w->seg, PF_MAXE * 4);
        if (e == cudaSuccess) e = cudaMalloc(&w->cursor, PF_MAXE * 4);
        if (e == cudaSuccess) e = cudaMalloc(&w->nt, 2 * 4);
        if (e == cudaSuccess) e = cudaMalloc(&w->err, 4);
        if (e == cudaSuccess) e = cudaMalloc(&w->dense_nt, 4);
        // stream-ordered with the kernels (the context's stream does not
        // synchronise with the legacy default stream)
        if (e == cudaSuccess) e = cudaMemsetAsync(w->counts, 0, PF_MAXE * 4, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(w->err, 0, 4, st);
        if (e != cudaSuccess) {
            prefill_release(c);
            return ctx_cuda(c, e, "prefill workspace");
        }
    }
    *out = w;
    return DS_CUDA_OK;
}

#define PF_GROW(ptr, cap, bytes)                                                          \
    do {                                                                                  \
        int _rc = ctx_grow(c, (void **)&(ptr), &(cap), (bytes));                          \
        if (_rc < 0) return _rc;                                                          \
    } while (0)

static int pf_shape_ok(ds_cuda_ctx *c, const PfShape &g) {
    if (g.H % 256 || g.H > 2048 || g.I % 128 || g.I <= 0 || g.S % 128 || g.E <= 0 || g.E > PF_MAXE || g.K <= 0 ||
        g.K > 8 || g.K > g.E)
        return ctx_fail(c, DS_CUDA_EINVAL, "prefill: unsupported shape (hidden %% 256 and <= 2048, inter and shared "
                                           "inter %% 128, n_experts <= 256, top_k <= 8 required)");
    return DS_CUDA_OK;
}

static void mark(ds_cuda_ctx *c, int i, cudaStream_t st) {
    if (c->prefill_timing) cudaEventRecord(c->prefill_ev[i], st);
}

// Stage 1: RMSNorm, BF16 split planes and routing of M tokens.
static int pf_route(ds_cuda_ctx *c, const PfShape &g, const float *d_norm, const uint16_t *d_router,
                    const float *d_x, int M, const float *d_logits, uint16_t *xn_hi, uint16_t *xn_lo, int *idx,
                    float *wt, cudaStream_t st) {
    if (M <= 0) return DS_CUDA_OK;
    if (!d_logits && !d_router) return ctx_fail(c, DS_CUDA_EINVAL, "prefill: no router weights and no logits");
    PfWork *w;
    int rc = pf_work(c, st, &w);
    if (rc < 0) return rc;
    if (!d_logits) PF_GROW(w->logits, w->c_logits, (size_t)M * g.E * 4);
    mark(c, 0, st);
    pf_norm_route_kernel<<<(M + 7) / 8, 256, 0, st>>>(d_x, d_norm, g.eps, M, g.H, d_logits,
                                                      g.logits_ld ? g.logits_ld : g.E, d_router, w->logits,
                                                      g.E, g.K, c->renorm, xn_hi, xn_lo, idx, wt);
    return DS_CUDA_OK;
}

// Stage 2: the grouped GEMMs. Routed: pair p = (row pair_row[p] (or p / K),
// expert pair_expert[p]) of rows_hi/lo [n_rows x H] -> y[p] [H]. Shared:
// sh_hi/lo [n_sh x H] -> ys [n_sh x H]. Either part may be empty.
static int pf_experts(ds_cuda_ctx *c, const PfShape &g, const uint16_t *d_block, const uint16_t *d_down,
                      const uint16_t *d_sdown, const uint16_t *rows_hi, const uint16_t *rows_lo, int rows_ld,
                      const int *pair_row,
                      const int *pair_expert, int P, float *y, const uint16_t *sh_hi, const uint16_t *sh_lo, int n_sh,
                      float *ys, cudaStream_t st) {
    if (P <= 0 && n_sh <= 0) return DS_CUDA_OK;
    const int H = g.H, I = g.I, S = g.S, E = g.E;
    PfWork *w;
    int rc = pf_work(c, st, &w);
    if (rc < 0) return rc;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(pf_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
        cudaFuncSetAttribute(pf_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
        attr = true;
    }
    const size_t Pz = P > 0 ? P : 0, Sz = n_sh > 0 ? n_sh : 0;
    const size_t mt_r = Pz / PF_BM + E, mts = (Sz + PF_BM - 1) / PF_BM;
    PF_GROW(w->xg_hi, w->c_xg_hi, Pz * H * 2 + 16);
    PF_GROW(w->xg_lo, w->c_xg_lo, Pz * H * 2 + 16);
    PF_GROW(w->hg_hi, w->c_hg_hi, Pz * I * 2 + 16);
    PF_GROW(w->hg_lo, w->c_hg_lo, Pz * I * 2 + 16);
    PF_GROW(w->hs_hi, w->c_hs_hi, Sz * S * 2 + 16);
    PF_GROW(w->hs_lo, w->c_hs_lo, Sz * S * 2 + 16);
    PF_GROW(w->slot_of, w->c_slot, Pz * 4 + 16);
    PF_GROW(w->gu_tiles, w->c_gu, (mts * (S / 128) + mt_r * (I / 128)) * sizeof(PfTile));
    PF_GROW(w->dn_tiles, w->c_dn, (mts + mt_r) * (H / PF_BN) * sizeof(PfTile));
    const int grid = c->sm_count;
    mark(c, 1, st);
    if (P > 0) pf_count_kernel<<<min((P + 255) / 256, grid), 256, 0, st>>>(P, pair_expert, E, w->counts);
    pf_plan_kernel<<<1, 256, 0, st>>>(w->counts, E, n_sh > 0 ? n_sh : 0, I, S, H, w->seg, w->cursor, w->gu_tiles,
                                      w->nt, w->dn_tiles, w->nt + 1);
    mark(c, 2, st);
    if (P > 0)
        pf_scatter_kernel<<<(P + 7) / 8, 256, 0, st>>>(P, H, rows_ld, g.K, pair_row, pair_expert, E, w->seg, w->cursor,
                                                       rows_hi, rows_lo, w->xg_hi, w->xg_lo, w->slot_of, nullptr);
    // gate/up (+SwiGLU): routed A = expert-sorted rows, shared A = sh planes;
    // B = the expert block [E*2I + 2S rows x H] for both
    PfGemm gu;
    memset(&gu, 0, sizeof gu);
    const uint64_t brows = (uint64_t)E * 2 * I + 2 * (uint64_t)S;
    const uint16_t *shh = n_sh > 0 ? sh_hi : w->xg_hi, *shl = n_sh > 0 ? sh_lo : w->xg_lo;
    bool ok = tmap_bf16(&gu.a_hi[0], w->xg_hi, H, Pz, PF_BM) && tmap_bf16(&gu.a_lo[0], w->xg_lo, H, Pz, PF_BM) &&
              tmap_bf16(&gu.a_hi[1], shh, H, Sz, PF_BM) && tmap_bf16(&gu.a_lo[1], shl, H, Sz, PF_BM) &&
              tmap_bf16(&gu.b[0], d_block, H, brows, 128) && tmap_bf16(&gu.b[1], d_block, H, brows, 128);
    if (!ok) return ctx_fail(c, DS_CUDA_ECUDA, "prefill: tensor map encoding failed");
    gu.tiles = w->gu_tiles;
    gu.n_tiles = w->nt;
    gu.k_blocks[0] = gu.k_blocks[1] = H / PF_BK;
    gu.b_base[0] = 0;
    gu.b_group_rows[0] = 2 * I;
    gu.b_half[0] = I;
    gu.b_base[1] = E * 2 * I;
    gu.b_half[1] = S;
    gu.h_hi[0] = w->hg_hi;
    gu.h_lo[0] = w->hg_lo;
    gu.h_ld[0] = I;
    gu.h_hi[1] = w->hs_hi;
    gu.h_lo[1] = w->hs_lo;
    gu.h_ld[1] = S;
    gu.err = w->err;
    mark(c, 3, st);
    pf_gemm_kernel<0><<<grid, PF_THREADS, PF_SMEM, st>>>(gu);
    mark(c, 4, st);
    // down: routed A = SwiGLU rows [P x I], shared A = [n_sh x S]
    PfGemm dn;
    memset(&dn, 0, sizeof dn);
    ok = tmap_bf16(&dn.a_hi[0], w->hg_hi, I, Pz, PF_BM) && tmap_bf16(&dn.a_lo[0], w->hg_lo, I, Pz, PF_BM) &&
         tmap_bf16(&dn.a_hi[1], w->hs_hi, S, Sz, PF_BM) && tmap_bf16(&dn.a_lo[1], w->hs_lo, S, Sz, PF_BM) &&
         tmap_bf16(&dn.b[0], d_down, I, (uint64_t)E * H, PF_BN) && tmap_bf16(&dn.b[1], d_sdown, S, H, PF_BN);
    if (!ok) return ctx_fail(c, DS_CUDA_ECUDA, "prefill: tensor map encoding failed");
    dn.tiles = w->dn_tiles;
    dn.n_tiles = w->nt + 1;
    dn.k_blocks[0] = I / PF_BK;
    dn.k_blocks[1] = S / PF_BK;
    dn.b_group_rows[0] = H;
    dn.y[0] = y;
    dn.y[1] = ys;
    dn.slot_of = w->slot_of;
    dn.y_ld = H;
    dn.err = w->err;
    pf_gemm_kernel<1><<<grid, PF_THREADS, PF_SMEM, st>>>(dn);
    mark(c, 5, st);
    return DS_CUDA_OK;
}

// Stage 3: x += (sum in ascending expert order of w_k y_k) + ys.
static int pf_combine(ds_cuda_ctx *c, const PfShape &g, float *d_x, int M, const int *idx, const float *wt,
                      const float *y, const int *yrow, const float *ys, cudaStream_t st) {
    if (M <= 0) return DS_CUDA_OK;
    pf_combine_kernel<<<M, 128, 0, st>>>(d_x, M, g.H, g.K, idx, wt, y, yrow, ys, nullptr, 0, 0);
    mark(c, 6, st);
    return DS_CUDA_OK;
}

// One MoE prefill layer on device buffers. d_x [M x H] is updated in place.
int prefill_moe_enqueue(ds_cuda_ctx *c, const PfShape &g, const float *d_norm, const uint16_t *d_router,
                        const uint16_t *d_block, const uint16_t *d_down, const uint16_t *d_sdown, float *d_x, int M,
                        const float *d_logits, int *d_idx_out, float *d_w_out, cudaStream_t st) {
    if (M <= 0) return DS_CUDA_OK;
    int rc = pf_shape_ok(c, g);
    if (rc < 0) return rc;
    PfWork *w;
    rc = pf_work(c, st, &w);
    if (rc < 0) return rc;
    const size_t P = (size_t)M * g.K;
    PF_GROW(w->xn_hi, w->c_xn_hi, (size_t)M * g.H * 2);
    PF_GROW(w->xn_lo, w->c_xn_lo, (size_t)M * g.H * 2);
    PF_GROW(w->idx, w->c_idx, P * 4);
    PF_GROW(w->wt, w->c_wt, P * 4);
    PF_GROW(w->yr, w->c_yr, P * g.H * 4);
    PF_GROW(w->ys, w->c_ys, (size_t)M * g.H * 4);
    if ((rc = pf_route(c, g, d_norm, d_router, d_x, M, d_logits, w->xn_hi, w->xn_lo, w->idx, w->wt, st)) < 0) return rc;
    // pairs (token s, slot k) = index s*K + k; its expert is idx[s*K + k]
    if ((rc = pf_experts(c, g, d_block, d_down, d_sdown, w->xn_hi, w->xn_lo, g.H, nullptr, w->idx, (int)P, w->yr,
                         w->xn_hi, w->xn_lo, M, w->ys, st)) < 0)
        return rc;
    if ((rc = pf_combine(c, g, d_x, M, w->idx, w->wt, w->yr, nullptr, w->ys, st)) < 0) return rc;
    if (d_idx_out) cudaMemcpyAsync(d_idx_out, w->idx, P * 4, cudaMemcpyDeviceToDevice, st);
    if (d_w_out) cudaMemcpyAsync(d_w_out, w->wt, P * 4, cudaMemcpyDeviceToDevice, st);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return ctx_cuda(c, e, "prefill_moe launch");
    return DS_CUDA_OK;
}

// A dense split-BF16 GEMM on the same kernel, for the whole-decoder prefill:
// every tile is a "shared" (kind 1) tile over all M rows.
//   mode 1: y [M x N] (row stride y_ld) = A [M x K] . B [N x K]^T, N % 256 == 0
//   mode 0: B = [gate rows (N); up rows (N)] (N % 128 == 0); writes
//           SwiGLU(A.gate^T, A.up^T) as BF16 planes h_hi/h_lo [M x N]
// A = planes a_hi/a_lo [M x K], K % 64 == 0.
int pf_dense_gemm(ds_cuda_ctx *c, int mode, const uint16_t *a_hi, const uint16_t *a_lo, int M, int K,
                  const uint16_t *B, int N, float *y, int y_ld, uint16_t *h_hi, uint16_t *h_lo, cudaStream_t st) {
    if (M <= 0) return DS_CUDA_OK;
    if (K % PF_BK || (mode == 1 && N % PF_BN) || (mode == 0 && N % 128))
        return ctx_fail(c, DS_CUDA_EINVAL, "prefill: dense GEMM shape not tileable");
    PfWork *w;
    int rc = pf_work(c, st, &w);
    if (rc < 0) return rc;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(pf_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
        cudaFuncSetAttribute(pf_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
        attr = true;
    }
    const int mt = (M + PF_BM - 1) / PF_BM, bn = mode == 1 ? PF_BN : 128, nt = N / bn;
    std::vector<PfTile> tiles;
    tiles.reserve((size_t)mt * nt);
    // n-major within a row block: consecutive CTAs share the A tile in L2
    for (int m = 0; m < mt; m++)
        for (int n = 0; n < nt; n++) tiles.push_back(PfTile{1, 0, m * PF_BM, std::min(PF_BM, M - m * PF_BM), n * bn});
    PF_GROW(w->dense_tiles, w->c_dense, tiles.size() * sizeof(PfTile));
    const int ntiles = (int)tiles.size();
    // pageable sources: staged before the calls return; stream-ordered
    // after any earlier GEMM that read the same list
    cudaError_t e = cudaMemcpyAsync(w->dense_tiles, tiles.data(), tiles.size() * sizeof(PfTile),
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w->dense_nt, &ntiles, 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return ctx_cuda(c, e, "prefill: tile list");
    PfGemm g;
    memset(&g, 0, sizeof g);
    bool ok = tmap_bf16(&g.a_hi[1], a_hi, K, M, PF_BM) && tmap_bf16(&g.a_lo[1], a_lo, K, M, PF_BM) &&
              tmap_bf16(&g.b[1], B, K, mode == 1 ? (uint64_t)N : 2 * (uint64_t)N, mode == 1 ? PF_BN : 128);
    // kind 0 is unused: point its maps at the same tensors
    g.a_hi[0] = g.a_hi[1];
    g.a_lo[0] = g.a_lo[1];
    g.b[0] = g.b[1];
    if (!ok) return ctx_fail(c, DS_CUDA_ECUDA, "prefill: tensor map encoding failed");
    g.tiles = w->dense_tiles;
    g.n_tiles = w->dense_nt;
    g.k_blocks[0] = g.k_blocks[1] = K / PF_BK;
    g.b_half[1] = N;
    g.h_hi[1] = h_hi;
    g.h_lo[1] = h_lo;
    g.h_ld[1] = N;
    g.y[1] = y;
    g.y_ld = y_ld;
    g.err = w->err;
    const int grid = std::min(c->sm_count, ntiles);
    if (mode == 0) pf_gemm_kernel<0><<<grid, PF_THREADS, PF_SMEM, st>>>(g);
    else pf_gemm_kernel<1><<<grid, PF_THREADS, PF_SMEM, st>>>(g);
    e = cudaGetLastError();
    return e == cudaSuccess ? DS_CUDA_OK : ctx_cuda(c, e, "prefill: dense GEMM launch");
}

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
static PfShape pf_shape(const ds_cuda_decoder_config_t *cfg) {
    return PfShape{cfg->hidden, cfg->moe_inter, cfg->n_shared * cfg->moe_inter, cfg->n_experts, cfg->top_k,
                   cfg->rms_eps};
}

static int pf_layer_ptrs(ds_cuda_ctx *c, const ds_cuda_decoder_config_t *g, const ds_cuda_layer_weights_t *L,
                         bool need_router, const float **norm, const uint16_t **router, const uint16_t **block,
                         const uint16_t **down, const uint16_t **sdown) {
    const size_t H = g->hidden, I = g->moe_inter, S = (size_t)g->n_shared * g->moe_inter, E = g->n_experts;
    if (norm) *norm = (const float *)ctx_lookup(c, L->post_attn_norm, H * 4, true);
    if (router) *router = need_router ? (const uint16_t *)ctx_lookup(c, L->router, E * H * 2, true) : nullptr;
    if (block) *block = (const uint16_t *)ctx_lookup(c, L->expert_block, (E * 2 * I + 2 * S) * H * 2, true);
    if (down) *down = (const uint16_t *)ctx_lookup(c, L->down, E * H * I * 2, true);
    if (sdown) *sdown = (const uint16_t *)ctx_lookup(c, L->shared_down, H * S * 2, true);
    if ((norm && !*norm) || (router && need_router && !*router) || (block && !*block) || (down && !*down) ||
        (sdown && !*sdown))
        return ctx_fail(c, DS_CUDA_EINVAL, "prefill: a weight array is missing or could not be registered");
    return DS_CUDA_OK;
}

static int pf_check(ds_cuda_ctx *c) {
    PfWork *w = (PfWork *)c->prefill;
    if (!w) return DS_CUDA_OK;
    unsigned e = 0;
    cudaError_t ce = cudaMemcpy(&e, w->err, 4, cudaMemcpyDeviceToHost);
    if (ce != cudaSuccess) return ctx_cuda(c, ce, "prefill error flag");
    if (e) {
        cudaMemsetAsync(w->err, 0, 4, c->stream);
        return ctx_fail(c, DS_CUDA_ETIMEOUT, "prefill: a bounded device-side wait gave up");
    }
    return DS_CUDA_OK;
}

int prefill_check_flag(ds_cuda_ctx *c) { return pf_check(c); }

static cudaStream_t pf_stream(ds_cuda_ctx *c, void *s) { return s ? (cudaStream_t)s : c->stream; }

extern "C" int ds_cuda_prefill_moe_dev(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg,
                                       const ds_cuda_layer_weights_t *layer, float *d_x, int n_tokens,
                                       const float *d_logits, int *d_top_idx, float *d_top_w, void *stream) {
    if (!c || !c->ok || !cfg || !layer || (!d_x && n_tokens > 0) || n_tokens < 0) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    const float *norm;
    const uint16_t *router, *block, *down, *sdown;
    int rc = pf_layer_ptrs(c, cfg, layer, d_logits == nullptr, &norm, &router, &block, &down, &sdown);
    if (rc < 0) return rc;
    return prefill_moe_enqueue(c, pf_shape(cfg), norm, router, block, down, sdown, d_x, n_tokens, d_logits,
                               d_top_idx, d_top_w, pf_stream(c, stream));
}

extern "C" int ds_cuda_prefill_moe(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg,
                                   const ds_cuda_layer_weights_t *layer, float *x, int n_tokens, const float *logits,
                                   int *top_idx, float *top_w) {
    if (!c || !c->ok || !cfg || !layer || (!x && n_tokens > 0) || n_tokens < 0) return DS_CUDA_EINVAL;
    if (n_tokens == 0) return DS_CUDA_OK;
    cudaSetDevice(c->device);
    const size_t M = n_tokens, H = cfg->hidden, E = cfg->n_experts, K = cfg->top_k;
    float *dx = nullptr, *dl = nullptr, *dw = nullptr;
    int *di = nullptr;
    cudaStream_t st = c->stream;
    int rc = DS_CUDA_OK;
    cudaError_t e = cudaMalloc(&dx, M * H * 4);
    if (e == cudaSuccess && logits) e = cudaMalloc(&dl, M * E * 4);
    if (e == cudaSuccess) e = cudaMalloc(&di, M * K * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dw, M * K * 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dx, x, M * H * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && logits) e = cudaMemcpyAsync(dl, logits, M * E * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) rc = ctx_cuda(c, e, "prefill_moe staging");
    if (rc == DS_CUDA_OK) rc = ds_cuda_prefill_moe_dev(c, cfg, layer, dx, n_tokens, dl, di, dw, st);
    if (rc == DS_CUDA_OK) {
        e = cudaMemcpyAsync(x, dx, M * H * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess && top_idx) e = cudaMemcpyAsync(top_idx, di, M * K * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess && top_w) e = cudaMemcpyAsync(top_w, dw, M * K * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        rc = e == cudaSuccess ? pf_check(c) : ctx_cuda(c, e, "prefill_moe");
    }
    cudaFree(dx);
    cudaFree(dl);
    cudaFree(di);
    cudaFree(dw);
    return rc;
}

// The three stages on caller buffers, for expert-parallel prefill (the
// caller moves rows between devices in between).
extern "C" int ds_cuda_prefill_route_dev(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg,
                                         const ds_cuda_layer_weights_t *layer, const float *d_x, int n_tokens,
                                         const float *d_logits, uint16_t *d_xn_hi, uint16_t *d_xn_lo, int *d_top_idx,
                                         float *d_top_w, void *stream) {
    if (!c || !c->ok || !cfg || !layer || n_tokens < 0 ||
        (n_tokens > 0 && (!d_x || !d_xn_hi || !d_xn_lo || !d_top_idx || !d_top_w)))
        return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    PfShape g = pf_shape(cfg);
    int rc = pf_shape_ok(c, g);
    if (rc < 0) return rc;
    const float *norm;
    const uint16_t *router;
    rc = pf_layer_ptrs(c, cfg, layer, d_logits == nullptr, &norm, &router, nullptr, nullptr, nullptr);
    if (rc < 0) return rc;
    return pf_route(c, g, norm, router, d_x, n_tokens, d_logits, d_xn_hi, d_xn_lo, d_top_idx, d_top_w,
                    pf_stream(c, stream));
}

extern "C" int ds_cuda_prefill_experts_dev(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg,
                                           const ds_cuda_layer_weights_t *layer, const uint16_t *d_rows_hi,
                                           const uint16_t *d_rows_lo, int rows_ld, int n_rows, const int *d_pair_row,
                                           const int *d_pair_expert, int n_pairs, float *d_y,
                                           const uint16_t *d_sh_hi, const uint16_t *d_sh_lo, int n_shared_rows,
                                           float *d_ys, void *stream) {
    if (!c || !c->ok || !cfg || !layer || n_rows < 0 || n_pairs < 0 || n_shared_rows < 0 ||
        (n_pairs > 0 && (!d_rows_hi || !d_rows_lo || !d_pair_expert || !d_y)) ||
        (n_pairs > 0 && !d_pair_row && n_rows * cfg->top_k < n_pairs) || rows_ld < cfg->hidden || rows_ld % 8 ||
        (n_shared_rows > 0 && (!d_sh_hi || !d_sh_lo || !d_ys)))
        return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    PfShape g = pf_shape(cfg);
    int rc = pf_shape_ok(c, g);
    if (rc < 0) return rc;
    const uint16_t *block, *down, *sdown;
    rc = pf_layer_ptrs(c, cfg, layer, false, nullptr, nullptr, &block, &down, &sdown);
    if (rc < 0) return rc;
    return pf_experts(c, g, block, down, sdown, d_rows_hi, d_rows_lo, rows_ld, d_pair_row, d_pair_expert, n_pairs, d_y,
                      d_sh_hi, d_sh_lo, n_shared_rows, d_ys, pf_stream(c, stream));
}

extern "C" int ds_cuda_prefill_combine_dev(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg, float *d_x,
                                           int n_tokens, const int *d_top_idx, const float *d_top_w,
                                           const float *d_y, const int *d_y_row, const float *d_ys, void *stream) {
    if (!c || !c->ok || !cfg || n_tokens < 0 || (n_tokens > 0 && (!d_x || !d_top_idx || !d_top_w || !d_y || !d_ys)))
        return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    PfShape g = pf_shape(cfg);
    int rc = pf_shape_ok(c, g);
    if (rc < 0) return rc;
    return pf_combine(c, g, d_x, n_tokens, d_top_idx, d_top_w, d_y, d_y_row, d_ys, pf_stream(c, stream));
}

extern "C" int ds_cuda_prefill_check(ds_cuda_ctx_t *c) {
    if (!c || !c->ok) return DS_CUDA_EINVAL;
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return ctx_cuda(c, e, "prefill_check");
    return pf_check(c);
}

// Per-stage device times of prefill calls: enable, then read the last call's
// six stage durations (norm+route, plan, scatter, gate/up GEMM, down GEMM,
// combine) in milliseconds.
extern "C" int ds_cuda_prefill_timing(ds_cuda_ctx_t *c, int enable) {
    if (!c || !c->ok) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    if (enable && !c->prefill_ev[0])
        for (auto &e : c->prefill_ev)
            if (cudaEventCreate(&e) != cudaSuccess) return ctx_fail(c, DS_CUDA_ECUDA, "prefill_timing: events");
    c->prefill_timing = enable != 0;
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_prefill_stage_ms(ds_cuda_ctx_t *c, float *ms6) {
    if (!c || !c->ok || !ms6 || !c->prefill_ev[0]) return DS_CUDA_EINVAL;
    cudaError_t e = cudaEventSynchronize(c->prefill_ev[6]);
    for (int i = 0; i < 6 && e == cudaSuccess; i++) e = cudaEventElapsedTime(&ms6[i], c->prefill_ev[i], c->prefill_ev[i + 1]);
    if (e != cudaSuccess) return ctx_cuda(c, e, "prefill_stage_ms");
    return DS_CUDA_OK;
}

// Launchers of the grouping and combine kernels for other engines (the
// multi-stream decoder groups its token rows by expert the same way).
cudaError_t pf_count_launch(int P, const int *pair_expert, int E, int *counts, int grid, cudaStream_t st) {
    if (P > 0) pf_count_kernel<<<min((P + 255) / 256, grid), 256, 0, st>>>(P, pair_expert, E, counts);
    return cudaGetLastError();
}

cudaError_t pf_scatter_launch(int P, int H, int ld, int K, const int *pair_row, const int *pair_expert, int E,
                              const int *seg, int *cursor, const uint16_t *rows_hi, const uint16_t *rows_lo,
                              uint16_t *xg_hi, uint16_t *xg_lo, int *slot_of, int *inv, cudaStream_t st) {
    if (P > 0)
        pf_scatter_kernel<<<(P + 7) / 8, 256, 0, st>>>(P, H, ld, K, pair_row, pair_expert, E, seg, cursor, rows_hi,
                                                       rows_lo, xg_hi, xg_lo, slot_of, inv);
    return cudaGetLastError();
}

cudaError_t pf_combine_launch(float *x, int M, int H, int K, const int *idx, const float *wt, const float *y,
                              const int *yrow, const float *ys, cudaStream_t st) {
    if (M > 0) pf_combine_kernel<<<M, 128, 0, st>>>(x, M, H, K, idx, wt, y, yrow, ys, nullptr, 0, 0);
    return cudaGetLastError();
}

cudaError_t pf_combine_split_launch(float *x, int M, int H, int K, const int *idx, const float *wt, const float *y,
                                    const int *yrow, const float *ys, const float *y_alt, long long alt_lo,
                                    long long alt_hi, cudaStream_t st) {
    if (M > 0) pf_combine_kernel<<<M, 128, 0, st>>>(x, M, H, K, idx, wt, y, yrow, ys, y_alt, alt_lo, alt_hi);
    return cudaGetLastError();
}
