// kernels_moe.cu — decode-path kernels: streaming argmax LM head, MoE router
// (softmax + top-k), routed/shared expert gate_up+SwiGLU and down+combine
// (BF16 and INT8), and the per-row INT8 quantiser.
#include "kernels_moe.cuh"
#include "launch.h"

namespace ds {

// ---------------------------------------------------------------------------
// Argmax LM head: ds_argmax_matvec_bf16 (ds_kernels.c:1013-1099).
// Each warp streams two rows at a time and keeps its best (value, index);
// the grid reduces with a 64-bit atomicMax on argmax_key (value major, lower
// index wins ties), and the last CTA to finish (ticket) writes the token and
// logit and resets the slot for the next call.
// ---------------------------------------------------------------------------
template <int CPL>
__global__ void __launch_bounds__(256) argmax_bf16_kernel(const uint16_t *__restrict__ W,
                                                          const float *__restrict__ x, int rows, int n,
                                                          unsigned long long *slot, unsigned *ticket,
                                                          int *tok_out, float *val_out, const float *norm_w,
                                                          float eps) {
    pdl_wait();
    pdl_launch();
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const float inv = norm_w ? block_rms_inv(x, n, eps) : 1.f;
    XRegBF16<CPL> xr;
    xr.load_norm(x, norm_w, inv, n, lane);
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 2 * gw; r < rows; r += 2 * nw) {
        float s0, s1;
        if (r + 1 < rows) {
            row_dot2_bf16<CPL>(W + (size_t)r * n, W + (size_t)(r + 1) * n, n, xr, lane, s0, s1);
            s0 = warp_sum(s0);
            s1 = warp_sum(s1);
            if (s0 > best) { best = s0; bi = r; }
            if (s1 > best) { best = s1; bi = r + 1; }
        } else {
            s0 = warp_sum(row_dot_bf16<CPL>(W + (size_t)r * n, n, xr, lane));
            if (s0 > best) { best = s0; bi = r; }
        }
    }
    __shared__ unsigned long long cta_best;
    if (threadIdx.x == 0) cta_best = 0ull;
    __syncthreads();
    if (lane == 0 && bi != 0x7fffffff) atomicMax(&cta_best, argmax_key(best, (uint32_t)bi));
    __syncthreads();
    if (threadIdx.x == 0) {
        if (cta_best) atomicMax(slot, cta_best);
        __threadfence();
        unsigned t = atomicAdd(ticket, 1u);
        if (t == gridDim.x - 1) {
            __threadfence();
            unsigned long long k = atomicExch(slot, 0ull);
            *tok_out = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
            *val_out = f32_from_ordered((uint32_t)(k >> 32));
            *ticket = 0u;
        }
    }
}

// Router: scores = W_r x (ds_moe_router_bf16, ds_kernels.c:187-191); the
// last CTA then runs router_select (kernels_moe.cuh).

template <int CPL>
__global__ void __launch_bounds__(256) router_kernel(const uint16_t *__restrict__ Wr, const float *__restrict__ x,
                                                     int E, int n, float *scores, unsigned *ticket, int top_k,
                                                     int renorm, int *d_idx, float *d_wt, const float *norm_w,
                                                     float eps) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    // the first router row loads before the dependency wait
    Rows2<CPL> w;
    if (gw < E) w.load(Wr + (size_t)gw * n, nullptr, n, lane);
    pdl_wait();
    pdl_launch();
    const float inv = norm_w ? block_rms_inv(x, n, eps) : 1.f;
    XRegBF16<CPL> xr;
    xr.load_norm(x, norm_w, inv, n, lane);
    for (int r = gw; r < E; r += nw) {
        if (r != gw) w.load(Wr + (size_t)r * n, nullptr, n, lane);
        float s, s1;
        w.dot(xr, s, s1);
        s = warp_sum(s);
        if (lane == 0) scores[r] = s;
    }
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (threadIdx.x < 32) {
        router_select(scores, E, top_k, renorm, d_idx, d_wt);
        if (threadIdx.x == 0) *ticket = 0u;
    }
}

// Router softmax/top-k over precomputed logits (single warp).
__global__ void router_select_kernel(const float *scores, int E, int top_k, int renorm, int *d_idx, float *d_wt) {
    pdl_wait();
    pdl_launch();
    router_select(scores, E, top_k, renorm, d_idx, d_wt);
}

// ---------------------------------------------------------------------------
// Expert gate_up + SwiGLU: ds_expert_forward_fused steps 1-5
// (ds_kernels.c:322-351) for the top_k routed experts and the shared expert
// at once. Work item p is one (gate row i, up row i) pair of one expert; the
// warp writes h[p] = SwiGLU(g_i, u_i) with the optional BF16 truncations.
// ---------------------------------------------------------------------------
template <int CPL, bool I8>
__global__ void __launch_bounds__(256) moe_gate_up_kernel(MoeArgs a) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int nr = a.top_k * a.inter;
    const int ns = a.has_shared ? a.sh_inter : 0;
    const int total = nr + ns;
    const int n = a.hidden;
    const bool sim = a.simulate && !a.dense;  // the dense FFN path never truncates (ds_moe_decoder.c:75-105)
    TraceScope tr;
    if constexpr (!I8) {
        // work order: the shared expert's pairs first (their weights do not
        // depend on the routing, so they load before the dependency wait),
        // then the routed experts'. h keeps routed [0, nr), shared [nr, total).
        auto shared_rows = [&](int i, const uint16_t *&w, const uint16_t *&wu) {
            w = (const uint16_t *)a.sh_gu.w;
            wu = a.sh_up.w ? (const uint16_t *)a.sh_up.w : w + (size_t)a.sh_inter * n;
            w += (size_t)i * n;
            wu += (size_t)i * n;
        };
        // item q's two rows (and the h index it writes)
        auto item_rows = [&](int q, const uint16_t *&w, const uint16_t *&wu) {
            if (q < ns) {
                shared_rows(q, w, wu);
            } else {
                const int pr = q - ns, k = pr / a.inter, i = pr - k * a.inter;
                const uint16_t *base = (const uint16_t *)expert_mat(a, k, true).w;
                w = base + (size_t)i * n;
                wu = base + (size_t)(a.inter + i) * n;
            }
        };
        // each warp walks items gw, gw + nw, ...; the next item's rows load
        // while the current item's dots run (two row buffers; the grid is one
        // wave, so no CTA waits for a slot)
        Rows2<CPL> cur, nxt;
        if (gw < ns) {
            const uint16_t *w, *wu;
            shared_rows(gw, w, wu);
            cur.load(w, wu, n, lane);
        }
        pdl_wait();
        pdl_launch();
        tr.waited();
        const float inv = a.norm_w ? block_rms_inv(a.x, n, a.eps) : 1.f;
        XRegBF16<CPL> xr;
        xr.load_norm(a.x, a.norm_w, inv, n, lane);
        if (gw >= ns && gw < total) {
            const uint16_t *w, *wu;
            item_rows(gw, w, wu);
            cur.load(w, wu, n, lane);
        }
        for (int q = gw; q < total; q += nw) {
            const int p = q < ns ? nr + q : q - ns;
            const int qn = q + nw;
            if (qn < total) {
                const uint16_t *w, *wu;
                item_rows(qn, w, wu);
                nxt.load(w, wu, n, lane);
            }
            float g, u;
            cur.dot(xr, g, u);
            cur = nxt;
            g = warp_sum(g);
            u = warp_sum(u);
            if (lane == 0) {
                if (sim) { g = bf16_roundtrip(g); u = bf16_roundtrip(u); }
                float hv = swiglu(g, u);
                if (sim) hv = bf16_roundtrip(hv);
                a.h[p] = hv;
            }
        }
    } else {
        pdl_wait();
        pdl_launch();
        const float inv = a.norm_w ? block_rms_inv(a.x, n, a.eps) : 1.f;
        XRegI8<CPL> xr;
        xr.load_norm(a.x, a.norm_w, inv, n, lane);
        float xs = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; c++)
#pragma unroll
            for (int q = 0; q < 4; q++) xs += (xr.v[c][q].x + xr.v[c][q].y) + (xr.v[c][q].z + xr.v[c][q].w);
        xs = warp_sum(xs);
        for (int p = gw; p < total; p += nw) {
            WMat m;
            int i, half;
            if (p < nr) {
                int k = p / a.inter;
                i = p - k * a.inter;
                half = a.inter;
                m = expert_mat(a, k, true);
            } else {
                i = p - nr;
                half = a.sh_inter;
                m = a.sh_gu;
            }
            const int8_t *w = (const int8_t *)m.w;
            float g = warp_sum(row_dot_i8<CPL>(w + (size_t)i * n, n, xr, lane));
            float u = warp_sum(row_dot_i8<CPL>(w + (size_t)(i + half) * n, n, xr, lane));
            if (lane == 0) {
                g = __fmaf_rn(m.scale[i], g, __fmul_rn(m.off[i], xs));
                u = __fmaf_rn(m.scale[i + half], u, __fmul_rn(m.off[i + half], xs));
                if (a.simulate) { g = bf16_roundtrip(g); u = bf16_roundtrip(u); }
                float hv = swiglu(g, u);
                if (a.simulate) hv = bf16_roundtrip(hv);
                a.h[p] = hv;
            }
        }
    }
    tr.done(6);
}

// ---------------------------------------------------------------------------
// Expert down + combine: ds_expert_forward_fused steps 6-7, ds_expert_combine
// (ds_kernels.c:359-371) and the shared expert add (ds_vec_add,
// ds_moe_decoder.c:316). A CTA owns RB output rows; warp s < top_k computes
// routed expert s's dot, warps top_k and top_k+1 the two halves of the shared
// expert's dot. The combine runs in the reference's order:
//   out = sum_k w_k * y_k (k = 0..K-1, FMA), then + shared.
// ---------------------------------------------------------------------------
template <int CPL, bool I8, int RB>
__global__ void __launch_bounds__(256, 3) moe_down_kernel(MoeArgs a) {
    __shared__ float y[RB][8];
    const int lane = threadIdx.x & 31;
    const int slot = threadIdx.x >> 5;
    const int j0 = blockIdx.x * RB;
    const int nslots = a.top_k + (a.has_shared ? 2 : 0);
    const int nr = a.top_k * a.inter;
    TraceScope tr;
    // the shared expert's down rows do not depend on the routing: its two
    // warps load them before the dependency wait
    Rows2<CPL> pre[(RB + 1) / 2];
    const bool sh_slot = !I8 && slot >= a.top_k && slot < nslots;
    if constexpr (!I8) {
        if (sh_slot) {
            const int len = a.sh_inter >> 1, rowlen = a.sh_inter;
            const uint16_t *w = (const uint16_t *)a.sh_dn.w + (slot - a.top_k) * len;
#pragma unroll
            for (int r = 0; r < RB; r += 2) {
                int j = j0 + r;
                if (j < a.hidden)
                    pre[r / 2].load(w + (size_t)j * rowlen, j + 1 < a.hidden ? w + (size_t)(j + 1) * rowlen : nullptr,
                                    len, lane);
            }
        }
    }
    pdl_wait();
    pdl_launch();
    tr.waited();
    if (slot < nslots) {
        const float *hv;
        WMat m;
        int len, col0, rowlen;
        if (slot < a.top_k) {
            hv = a.h + slot * a.inter;
            m = expert_mat(a, slot, false);
            len = a.inter;
            col0 = 0;
            rowlen = a.inter;
        } else {
            int half = slot - a.top_k;
            len = a.sh_inter >> 1;
            hv = a.h + nr + half * len;
            m = a.sh_dn;
            col0 = half * len;
            rowlen = a.sh_inter;
        }
        if constexpr (!I8) {
            XRegBF16<CPL> hr;
            hr.load(hv, len, lane);
            const uint16_t *w = (const uint16_t *)m.w + col0;
#pragma unroll
            for (int r = 0; r < RB; r += 2) {
                int j = j0 + r;
                float s0 = 0.f, s1 = 0.f;
                if (j < a.hidden) {
                    if (!sh_slot)
                        pre[r / 2].load(w + (size_t)j * rowlen,
                                        j + 1 < a.hidden ? w + (size_t)(j + 1) * rowlen : nullptr, len, lane);
                    pre[r / 2].dot(hr, s0, s1);
                }
                s0 = warp_sum(s0);
                s1 = warp_sum(s1);
                if (lane == 0) { y[r][slot] = s0; if (r + 1 < RB) y[r + 1][slot] = s1; }
            }
        } else {
            XRegI8<CPL> hr;
            hr.load(hv, len, lane);
            float hs = 0.f;
#pragma unroll
            for (int c = 0; c < CPL; c++)
#pragma unroll
                for (int q = 0; q < 4; q++) hs += (hr.v[c][q].x + hr.v[c][q].y) + (hr.v[c][q].z + hr.v[c][q].w);
            hs = warp_sum(hs);
            const int8_t *w = (const int8_t *)m.w + col0;
#pragma unroll
            for (int r = 0; r < RB; r++) {
                int j = j0 + r;
                float s = 0.f;
                if (j < a.hidden) s = warp_sum(row_dot_i8<CPL>(w + (size_t)j * rowlen, len, hr, lane));
                if (lane == 0 && j < a.hidden) {
                    // the shared expert's two halves share one row scale/offset:
                    // scale*(d0 + d1) + off*(s0 + s1) = sum of the per-half terms
                    y[r][slot] = __fmaf_rn(m.scale[j], s, __fmul_rn(m.off[j], hs));
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < RB) {
        int j = j0 + threadIdx.x;
        if (j < a.hidden) {
            float acc = 0.f;
            for (int k = 0; k < a.top_k; k++) {
                float yk = y[threadIdx.x][k];
                if (a.simulate) yk = bf16_roundtrip(yk);
                acc = __fmaf_rn(expert_wt(a, k), yk, acc);
            }
            if (a.has_shared) {
                float sh = __fadd_rn(y[threadIdx.x][a.top_k], y[threadIdx.x][a.top_k + 1]);
                if (a.simulate) sh = bf16_roundtrip(sh);
                acc = a.top_k > 0 ? __fadd_rn(acc, sh) : sh;
            }
            if (a.out_mode == 0) a.out[j] = acc;
            else if (a.out_mode == 1) a.out[j] = __fadd_rn(a.out[j], acc);
            else a.out[j] = __fadd_rn(a.resid[j], acc);
        }
    }
    tr.done(7);
}

// ---------------------------------------------------------------------------
// Per-row asymmetric INT8 quantiser: int8_quantize_row (ds_quantize.c:29-47),
// bit-exact: scale = max((max-min)/255, 1e-10), q = clamp(roundf((w - min) *
// (1/scale)), 0, 255) - 128, offset = min. One warp per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) quantize_int8_kernel(const uint16_t *__restrict__ W, int rows, int n,
                                                            int8_t *q, float *scale, float *off) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int r = gw; r < rows; r += nw) {
        const uint16_t *row = W + (size_t)r * n;
        float mn = 1e30f, mx = -1e30f;
        for (int c = lane; c < n; c += 32) {
            float v = __uint_as_float((uint32_t)row[c] << 16);
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(DS_FULL, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(DS_FULL, mx, o));
        }
        float s = __fdiv_rn(__fsub_rn(mx, mn), 255.0f);
        if (s < 1e-10f) s = 1e-10f;
        float inv = __fdiv_rn(1.0f, s);
        if (lane == 0) { scale[r] = s; off[r] = mn; }
        for (int c = lane; c < n; c += 32) {
            float v = __uint_as_float((uint32_t)row[c] << 16);
            int qi = (int)roundf(__fmul_rn(__fsub_rn(v, mn), inv));
            qi = qi < 0 ? 0 : (qi > 255 ? 255 : qi);
            q[(size_t)r * n + c] = (int8_t)(qi - 128);
        }
    }
}

// ---------------------------------------------------------------------------
// Plain BF16 matvec y = W x (+ bias): ds_linear_nobias_bf16 / ds_linear_bf16
// at seq_len 1 (ds_kernels.c:917-943). Two rows per warp per step.
// ---------------------------------------------------------------------------
template <int CPL>
__global__ void __launch_bounds__(256) matvec_bf16_kernel(const uint16_t *__restrict__ W, const float *__restrict__ x,
                                                          const float *__restrict__ bias, float *y, int rows, int n) {
    pdl_wait();
    pdl_launch();
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    XRegBF16<CPL> xr;
    xr.load(x, n, lane);
    for (int r = 2 * gw; r < rows; r += 2 * nw) {
        float s0, s1 = 0.f;
        if (r + 1 < rows) row_dot2_bf16<CPL>(W + (size_t)r * n, W + (size_t)(r + 1) * n, n, xr, lane, s0, s1);
        else s0 = row_dot_bf16<CPL>(W + (size_t)r * n, n, xr, lane);
        s0 = warp_sum(s0);
        s1 = warp_sum(s1);
        if (lane == 0) {
            y[r] = bias ? __fadd_rn(s0, bias[r]) : s0;
            if (r + 1 < rows) y[r + 1] = bias ? __fadd_rn(s1, bias[r + 1]) : s1;
        }
    }
}

// ---------------------------------------------------------------------------
// Host launchers.
// ---------------------------------------------------------------------------
static inline int sm_count() {
    static int n = 0;
    if (!n) {
        int dev;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    }
    return n;
}

cudaError_t launch_ex(const void *func, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      void **args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, func, args);
}

#define DS_CPL_SWITCH(n, CHUNK, BODY)                 \
    do {                                              \
        int _c = ((n) / (CHUNK) + 31) / 32;           \
        if (_c <= 1) { constexpr int CPL = 1; BODY; } \
        else if (_c <= 2) { constexpr int CPL = 2; BODY; } \
        else if (_c <= 3) { constexpr int CPL = 3; BODY; } \
        else if (_c <= 4) { constexpr int CPL = 4; BODY; } \
        else if (_c <= 5) { constexpr int CPL = 5; BODY; } \
        else if (_c <= 6) { constexpr int CPL = 6; BODY; } \
        else if (_c <= 7) { constexpr int CPL = 7; BODY; } \
        else if (_c <= 8) { constexpr int CPL = 8; BODY; } \
        else return cudaErrorInvalidValue;            \
    } while (0)

cudaError_t launch_argmax_bf16(const uint16_t *W, const float *x, int rows, int n, unsigned long long *slot,
                               unsigned *ticket, int *tok, float *val, cudaStream_t st, bool pdl,
                               const float *norm_w, float eps) {
    if (n % 8 || n > 2048) return cudaErrorInvalidValue;
    // TMA-streamed variant (kernels_stream.cu): 71 us vs 84 us for the
    // register-load kernel below on the 129280 x 1280 LM head (B200)
    if (st_stages_ok(n)) return launch_argmax_tma(W, x, rows, n, slot, ticket, tok, val, st, pdl, norm_w, eps, ticket + 8);
    int warps_needed = (rows + 1) / 2;
    int grid = min((warps_needed + 7) / 8, sm_count() * 8);
    void *args[] = {&W, &x, &rows, &n, &slot, &ticket, &tok, &val, &norm_w, &eps};
    DS_CPL_SWITCH(n, 8, return launch_ex((const void *)argmax_bf16_kernel<CPL>, grid, 256, 0, st, pdl, args));
}

cudaError_t launch_router(const uint16_t *Wr, const float *x, int E, int n, float *scores, unsigned *ticket,
                          int top_k, int renorm, int *d_idx, float *d_wt, cudaStream_t st, bool pdl,
                          const float *norm_w, float eps) {
    if (n % 8 || n > 2048 || E > 256 || top_k > 8) return cudaErrorInvalidValue;
    int grid = (E + 7) / 8;
    void *args[] = {&Wr, &x, &E, &n, &scores, &ticket, &top_k, &renorm, &d_idx, &d_wt, &norm_w, &eps};
    DS_CPL_SWITCH(n, 8, return launch_ex((const void *)router_kernel<CPL>, grid, 256, 0, st, pdl, args));
}

cudaError_t launch_router_select(const float *scores, int E, int top_k, int renorm, int *d_idx, float *d_wt,
                                 cudaStream_t st, bool pdl) {
    if (E > 256 || top_k > 8) return cudaErrorInvalidValue;
    void *args[] = {&scores, &E, &top_k, &renorm, &d_idx, &d_wt};
    return launch_ex((const void *)router_select_kernel, 1, 32, 0, st, pdl, args);
}

cudaError_t launch_moe_gate_up(const MoeArgs &a, cudaStream_t st, bool pdl) {
    int chunk = a.int8 ? 16 : 8;
    if (a.hidden % chunk || a.hidden > 2048) return cudaErrorInvalidValue;
    int total = a.top_k * a.inter + (a.has_shared ? a.sh_inter : 0);
    if (total <= 0) return cudaSuccess;
    int grid = min((total + 7) / 8, sm_count() * 16);
    MoeArgs aa = a;
    void *args[] = {&aa};
    if (a.int8) {
        DS_CPL_SWITCH(a.hidden, 16, return launch_ex((const void *)moe_gate_up_kernel<CPL, true>, grid, 256, 0, st, pdl, args));
    } else {
        // BF16: one wave of CTAs (as many as fit at once), items pipelined per warp
        DS_CPL_SWITCH(a.hidden, 8, {
            static int per_sm[9] = {0};
            if (!per_sm[CPL]) {
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm[CPL], moe_gate_up_kernel<CPL, false>, 256, 0);
                if (per_sm[CPL] < 1) per_sm[CPL] = 1;
            }
            grid = min((total + 7) / 8, sm_count() * per_sm[CPL]);
            return launch_ex((const void *)moe_gate_up_kernel<CPL, false>, grid, 256, 0, st, pdl, args);
        });
    }
}

cudaError_t launch_moe_down(const MoeArgs &a, cudaStream_t st, bool pdl) {
    int chunk = a.int8 ? 16 : 8;
    int len = a.inter;
    if (a.has_shared) {
        if (a.sh_inter % (2 * chunk)) return cudaErrorInvalidValue;
        len = max(len, a.sh_inter / 2);
    }
    if ((a.top_k > 0 && a.inter % chunk) || len > 2048) return cudaErrorInvalidValue;
    if (a.top_k + (a.has_shared ? 2 : 0) > 8) return cudaErrorInvalidValue;
    constexpr int RB = 4;
    int grid = (a.hidden + RB - 1) / RB;
    MoeArgs aa = a;
    void *args[] = {&aa};
    if (a.int8) {
        DS_CPL_SWITCH(len, 16, return launch_ex((const void *)moe_down_kernel<CPL, true, RB>, grid, 256, 0, st, pdl, args));
    } else {
        DS_CPL_SWITCH(len, 8, return launch_ex((const void *)moe_down_kernel<CPL, false, RB>, grid, 256, 0, st, pdl, args));
    }
}

cudaError_t launch_matvec_bf16(const uint16_t *W, const float *x, const float *bias, float *y, int rows, int n,
                               cudaStream_t st, bool pdl) {
    if (n % 8 || n > 2048) return cudaErrorInvalidValue;
    int grid = min(((rows + 1) / 2 + 7) / 8, sm_count() * 8);
    void *args[] = {&W, &x, &bias, &y, &rows, &n};
    DS_CPL_SWITCH(n, 8, return launch_ex((const void *)matvec_bf16_kernel<CPL>, grid, 256, 0, st, pdl, args));
}

cudaError_t launch_quantize_int8(const uint16_t *W, int rows, int n, int8_t *q, float *scale, float *off,
                                 cudaStream_t st) {
    int grid = min((rows + 7) / 8, sm_count() * 16);
    quantize_int8_kernel<<<grid, 256, 0, st>>>(W, rows, n, q, scale, off);
    return cudaGetLastError();
}

}  // namespace ds

DS_TRACE_TU(moe)
