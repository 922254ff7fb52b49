// kernels_moe.cuh — batch-1 decode kernels for the MoE layer and LM head.
//
// All of these are HBM-bound matvecs: one warp streams whole weight rows with
// 16-byte non-allocating loads, keeps its slice of the activation vector in
// registers, accumulates in F32 with FMA and reduces with shuffles. Weights
// are BF16 widened exactly (u16 << 16) or per-row asymmetric INT8 dequantised
// in registers, as in the reference CPU path.
#pragma once
#include "common.cuh"

namespace ds {

// One weight matrix: BF16 rows, or INT8 rows (stored q - 128) with per-row
// F32 scale and offset (ds_quantize.h:30-37).
struct WMat {
    const void *w;
    const float *scale;
    const float *off;
};

// Arguments of the decode MoE chain for one token.
//  explicit mode  (d_idx == nullptr): gu[k], dn[k], wt[k] name the top_k experts
//  routed mode    (d_idx != nullptr): expert e = d_idx[k] is at
//                 gu_base + e*gu_stride (elements; rows for scale/off: e*2*inter)
struct MoeArgs {
    int hidden, inter, sh_inter, top_k;
    int int8, simulate, has_shared;
    int dense;               // dense FFN: sh_gu = gate [S x H], sh_up = up [S x H]; no truncation
    const float *norm_w;     // if set, x is RMS-normalised on load with these weights
    float eps;
    WMat sh_up;
    int out_mode;            // 0: out = moe; 1: out += moe; 2: out = resid + moe
    WMat gu[8], dn[8];
    float wt[8];
    WMat gu_base, dn_base;
    long long gu_stride, dn_stride;  // elements between experts
    const int *d_idx;
    const float *d_wt;
    WMat sh_gu, sh_dn;
    const float *x;          // [hidden]
    float *h;                // scratch [top_k*inter + sh_inter]
    float *out;              // [hidden]
    const float *resid;      // [hidden] for out_mode 2
};

__device__ __forceinline__ WMat expert_mat(const MoeArgs &a, int k, bool gate_up) {
    if (a.d_idx == nullptr) return gate_up ? a.gu[k] : a.dn[k];
    int e = a.d_idx[k];
    const WMat &b = gate_up ? a.gu_base : a.dn_base;
    long long st = gate_up ? a.gu_stride : a.dn_stride;
    long long rows = gate_up ? 2LL * a.inter : a.hidden;
    WMat m;
    m.w = a.int8 ? (const void *)((const int8_t *)b.w + st * e)
                 : (const void *)((const uint16_t *)b.w + st * e);
    m.scale = b.scale ? b.scale + rows * e : nullptr;
    m.off = b.off ? b.off + rows * e : nullptr;
    return m;
}
__device__ __forceinline__ float expert_wt(const MoeArgs &a, int k) {
    return a.d_idx == nullptr ? a.wt[k] : a.d_wt[k];
}

// ---------------------------------------------------------------------------
// Register-resident activation slices. Lane `l` owns chunks l, l+32, ... of
// the input; a BF16 chunk is 8 columns (16 B), an INT8 chunk is 16 columns.
// ---------------------------------------------------------------------------
// RMS inverse of src[0..n) for the whole block: 1/sqrtf(sum(x^2)/n + eps)
// (ds_rms_norm, ds_kernels.c:1387-1440). Fixed reduction order, so every CTA
// of a grid computes the identical value. All threads must call it.
__device__ __forceinline__ float block_rms_inv(const float *src, int n, float eps) {
    __shared__ float red[33];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = __fmaf_rn(src[i], src[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t = __fadd_rn(t, red[w]);
        red[32] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)n), eps)));
    }
    __syncthreads();
    float inv = red[32];
    __syncthreads();
    return inv;
}

// (x * w) * inv, the reference's operation order (ds_kernels.c:1443-1449).
__device__ __forceinline__ float4 norm4(float4 x, float4 w, float inv) {
    return make_float4(__fmul_rn(__fmul_rn(x.x, w.x), inv), __fmul_rn(__fmul_rn(x.y, w.y), inv),
                       __fmul_rn(__fmul_rn(x.z, w.z), inv), __fmul_rn(__fmul_rn(x.w, w.w), inv));
}

template <int CPL>
struct XRegBF16 {
    float4 v[CPL][2];
    // load with optional RMS normalisation (w == nullptr: plain load)
    __device__ __forceinline__ void load_norm(const float *x, const float *w, float inv, int n, int lane) {
        if (!w) { load(x, n, lane); return; }
        const int nch = n >> 3;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            int ch = lane + 32 * c;
            if (ch < nch) {
                v[c][0] = norm4(*reinterpret_cast<const float4 *>(x + 8 * ch),
                                *reinterpret_cast<const float4 *>(w + 8 * ch), inv);
                v[c][1] = norm4(*reinterpret_cast<const float4 *>(x + 8 * ch + 4),
                                *reinterpret_cast<const float4 *>(w + 8 * ch + 4), inv);
            } else {
                v[c][0] = make_float4(0.f, 0.f, 0.f, 0.f);
                v[c][1] = v[c][0];
            }
        }
    }
    __device__ __forceinline__ void load(const float *x, int n, int lane) {
        const int nch = n >> 3;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            int ch = lane + 32 * c;
            if (ch < nch) {
                v[c][0] = *reinterpret_cast<const float4 *>(x + 8 * ch);
                v[c][1] = *reinterpret_cast<const float4 *>(x + 8 * ch + 4);
            } else {
                v[c][0] = make_float4(0.f, 0.f, 0.f, 0.f);
                v[c][1] = v[c][0];
            }
        }
    }
};

// Dot of one BF16 row (n columns) with the register slice; lane partial only.
template <int CPL>
__device__ __forceinline__ float row_dot_bf16(const uint16_t *row, int n, const XRegBF16<CPL> &x, int lane) {
    const int nch = n >> 3;
    uint4 w[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        int ch = lane + 32 * c;
        w[c] = ch < nch ? ldg_stream(row + 8 * ch) : make_uint4(0, 0, 0, 0);
    }
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; c++) acc = dot8_bf16(w[c], x.v[c][0], x.v[c][1], acc);
    return acc;
}

// The lane slices of two BF16 rows held in registers, so a kernel can issue
// its weight loads before griddepcontrol.wait (weights never depend on the
// preceding kernel) and overlap them with the predecessor's tail. r1 may be
// null (one row; its dot is 0).
template <int CPL>
struct Rows2 {
    uint4 w0[CPL], w1[CPL];
    __device__ __forceinline__ void load(const uint16_t *r0, const uint16_t *r1, int n, int lane) {
        const int nch = n >> 3;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            int ch = lane + 32 * c;
            bool ok = ch < nch;
            w0[c] = ok ? ldg_stream(r0 + 8 * ch) : make_uint4(0, 0, 0, 0);
            w1[c] = ok && r1 ? ldg_stream(r1 + 8 * ch) : make_uint4(0, 0, 0, 0);
        }
    }
    __device__ __forceinline__ void dot(const XRegBF16<CPL> &x, float &s0, float &s1) const {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            a0 = dot8_bf16(w0[c], x.v[c][0], x.v[c][1], a0);
            a1 = dot8_bf16(w1[c], x.v[c][0], x.v[c][1], a1);
        }
        s0 = a0;
        s1 = a1;
    }
};

// Two rows at once (twice the bytes in flight per lane).
template <int CPL>
__device__ __forceinline__ void row_dot2_bf16(const uint16_t *r0, const uint16_t *r1, int n,
                                              const XRegBF16<CPL> &x, int lane, float &s0, float &s1) {
    const int nch = n >> 3;
    uint4 w0[CPL], w1[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        int ch = lane + 32 * c;
        bool ok = ch < nch;
        w0[c] = ok ? ldg_stream(r0 + 8 * ch) : make_uint4(0, 0, 0, 0);
        w1[c] = ok ? ldg_stream(r1 + 8 * ch) : make_uint4(0, 0, 0, 0);
    }
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        a0 = dot8_bf16(w0[c], x.v[c][0], x.v[c][1], a0);
        a1 = dot8_bf16(w1[c], x.v[c][0], x.v[c][1], a1);
    }
    s0 = a0;
    s1 = a1;
}

template <int CPL>
struct XRegI8 {
    float4 v[CPL][4];
    __device__ __forceinline__ void load_norm(const float *x, const float *w, float inv, int n, int lane) {
        if (!w) { load(x, n, lane); return; }
        const int nch = n >> 4;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            int ch = lane + 32 * c;
#pragma unroll
            for (int q = 0; q < 4; q++)
                v[c][q] = ch < nch ? norm4(*reinterpret_cast<const float4 *>(x + 16 * ch + 4 * q),
                                           *reinterpret_cast<const float4 *>(w + 16 * ch + 4 * q), inv)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    __device__ __forceinline__ void load(const float *x, int n, int lane) {
        const int nch = n >> 4;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            int ch = lane + 32 * c;
#pragma unroll
            for (int q = 0; q < 4; q++)
                v[c][q] = ch < nch ? *reinterpret_cast<const float4 *>(x + 16 * ch + 4 * q)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
};

__device__ __forceinline__ float dot4_u8(uint32_t w, const float4 &x, float acc) {
    // stored int8 q - 128 == unsigned byte (q + 128) ^ 0x80 ... the stored
    // byte s = q_u - 128 (two's complement), so q_u = s ^ 0x80.
    uint32_t u = w ^ 0x80808080u;
    acc = __fmaf_rn(ubyte_f(u, 0), x.x, acc);
    acc = __fmaf_rn(ubyte_f(u, 1), x.y, acc);
    acc = __fmaf_rn(ubyte_f(u, 2), x.z, acc);
    acc = __fmaf_rn(ubyte_f(u, 3), x.w, acc);
    return acc;
}

// Lane partial of sum_c (q_c + 128) * x_c over one INT8 row.
template <int CPL>
__device__ __forceinline__ float row_dot_i8(const int8_t *row, int n, const XRegI8<CPL> &x, int lane) {
    const int nch = n >> 4;
    uint4 w[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        int ch = lane + 32 * c;
        w[c] = ch < nch ? ldg_stream(row + 16 * ch) : make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
    }
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        acc = dot4_u8(w[c].x, x.v[c][0], acc);
        acc = dot4_u8(w[c].y, x.v[c][1], acc);
        acc = dot4_u8(w[c].z, x.v[c][2], acc);
        acc = dot4_u8(w[c].w, x.v[c][3], acc);
    }
    return acc;
}

// ---------------------------------------------------------------------------
// Router: scores = W_r x (ds_moe_router_bf16, ds_kernels.c:187-191), then the
// last CTA runs the softmax over all experts with fast exp and the k strict-'>'
// selection passes of ds_moe_decoder.c:157-183 (raw probabilities unless
// renorm).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void router_select_generic(const float *scores, int E, int top_k, int renorm, int *d_idx, float *d_wt) {
    // called by warp 0 of one CTA; any E <= 256
    __shared__ float p[256];
    const int lane = threadIdx.x & 31;
    float mx = -1e30f;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, scores[e]);
    mx = warp_max(mx);
    for (int e = lane; e < E; e += 32) p[e] = fast_expf(__fsub_rn(scores[e], mx));
    __syncwarp();
    // sum of exponentials: per-lane partials, then a fixed shuffle tree (the
    // reference sums sequentially; the difference is a few ulp of the sum)
    float part = 0.f;
    for (int e = lane; e < E; e += 32) part = __fadd_rn(part, p[e]);
    const float inv = __fdiv_rn(1.0f, warp_sum(part));
    for (int e = lane; e < E; e += 32) p[e] = __fmul_rn(p[e], inv);
    __syncwarp();
    unsigned long long taken[4] = {0, 0, 0, 0};  // E <= 256
    float wsum = 0.f;
    float wk[8];
    int ik[8];
    for (int k = 0; k < top_k; k++) {
        float bv = -1e30f;
        int bidx = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            bool t = (taken[e >> 6] >> (e & 63)) & 1ull;
            if (!t && p[e] > bv) { bv = p[e]; bidx = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(DS_FULL, bv, o);
            int oi = __shfl_xor_sync(DS_FULL, bidx, o);
            if (ov > bv || (ov == bv && oi < bidx)) { bv = ov; bidx = oi; }
        }
        taken[bidx >> 6] |= 1ull << (bidx & 63);
        wk[k] = bv;
        ik[k] = bidx;
        wsum = __fadd_rn(wsum, bv);
    }
#pragma unroll
    for (int k = 0; k < 8; k++)
        if (k < top_k && lane == k) {
            d_idx[k] = ik[k];
            d_wt[k] = renorm ? __fdiv_rn(wk[k], wsum) : wk[k];
        }
}

// The router terms of the O-projection CTAs are stored per logit, each
// logit's terms contiguous and padded to a multiple of 4 (float4 loads), and
// summed in three runs of consecutive CTAs that start at multiples of 4 (each
// run in CTA order, then (r0 + r1) + r2).
__host__ __device__ __forceinline__ int rf_pstride(int nparts) { return (nparts + 3) & ~3; }
__host__ __device__ __forceinline__ int rf_run(int nparts, int k) {
    const int r = 4 * ((nparts + 11) / 12);
    return r * k < nparts ? r * k : nparts;
}
// The sum of run `part` of logit column `col` (terms contiguous), every load
// in flight together (a run holds at most 32 terms).
__device__ __forceinline__ float rf_run_sum(const float *col, int nparts, int part) {
    const int b0 = rf_run(nparts, part), b1 = rf_run(nparts, part + 1);
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++)
        v[u] = b0 + 4 * u < b1 ? __ldcg(reinterpret_cast<const float4 *>(col + b0 + 4 * u)) : make_float4(0.f, 0.f, 0.f, 0.f);
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const float t[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (b0 + 4 * u + k < b1) acc = __fadd_rn(acc, t[k]);
    }
    return acc;
}

__device__ __forceinline__ void router_select(const float *scores, int E, int top_k, int renorm, int *d_idx, float *d_wt) {
    if (E > 64) {
        router_select_generic(scores, E, top_k, renorm, d_idx, d_wt);
        return;
    }
    // called by warp 0 of one CTA; E <= 64: lane l holds experts l and l + 32
    const int lane = threadIdx.x & 31;
    const int e0 = lane, e1 = lane + 32;
    const bool v0 = e0 < E, v1 = e1 < E;
    const float sc0 = v0 ? scores[e0] : -1e30f, sc1 = v1 ? scores[e1] : -1e30f;
    const float mx = warp_max(fmaxf(sc0, sc1));
    float p0 = v0 ? fast_expf(__fsub_rn(sc0, mx)) : 0.f;
    float p1 = v1 ? fast_expf(__fsub_rn(sc1, mx)) : 0.f;
    // sum of exponentials: per-lane partials (expert l, then l + 32), then a
    // fixed shuffle tree (the reference sums sequentially; the difference is
    // a few ulp of the sum)
    float part = 0.f;
    if (v0) part = __fadd_rn(part, p0);
    if (v1) part = __fadd_rn(part, p1);
    const float inv = __fdiv_rn(1.0f, warp_sum(part));
    p0 = __fmul_rn(p0, inv);
    p1 = __fmul_rn(p1, inv);
    // top_k selection as the reference's strict '>' scan in ascending
    // expert order picks (ds_moe_decoder.c:167-183): the largest probability
    // first, the lowest index among equals. Expert e's position is its rank:
    // the experts with a larger probability, plus those with an equal one and
    // a lower index. Each lane counts the rank of its two experts against all
    // of them (shared memory broadcasts; -1 marks a missing expert, below
    // every probability), and the first top_k write their slot.
    __shared__ float pp[64];
    __shared__ float tw[8];
    __shared__ int ti[8];
    pp[e0] = v0 ? p0 : -1.0f;
    pp[e1] = v1 ? p1 : -1.0f;
    __syncwarp();
    int r0 = 0, r1 = 0;
#pragma unroll 16
    for (int f = 0; f < 64; f++) {
        const float q = pp[f];
        r0 += (q > p0 || (q == p0 && f < e0)) ? 1 : 0;
        r1 += (q > p1 || (q == p1 && f < e1)) ? 1 : 0;
    }
    if (v0 && r0 < top_k) {
        tw[r0] = p0;
        ti[r0] = e0;
    }
    if (v1 && r1 < top_k) {
        tw[r1] = p1;
        ti[r1] = e1;
    }
    __syncwarp();
    // the selected weights' sum in selection order (for renormalisation)
    float wsum = 0.f;
    for (int k = 0; k < top_k; k++) wsum = __fadd_rn(wsum, tw[k]);
    if (lane < top_k) {
        d_idx[lane] = ti[lane];
        d_wt[lane] = renorm ? __fdiv_rn(tw[lane], wsum) : tw[lane];
    }
    __syncwarp();
}

}  // namespace ds
