// kernels_decode.cu — the rest of the batch-1 greedy decode step
// (ds_decoder_forward, ds_moe_decoder.c:911-1264): input RMSNorm + QKV +
// RoPE + KV append, decode attention, O-projection + residual, long-K matvec
// for the dense FFN down projection, and the step advance (next embedding,
// position, token log).
#include <cooperative_groups.h>
#include <cstdlib>

#include "attn_rows.cuh"
#include "kernels_decode.cuh"

namespace cg = cooperative_groups;

namespace ds {


// ---------------------------------------------------------------------------
// Input RMSNorm + QKV + RoPE + KV append (decoder_layer_forward,
// ds_moe_decoder.c:358-393). Work item t is the row pair (d, d + hd/2) of one
// head of Q, K or V, so RoPE's split-half rotation (ds_apply_rope_neox,
// ds_kernels.c:2426-2458) happens in registers:
//   out[d]      = x1 cos[d]      - x2 sin[d]
//   out[d+half] = x1 sin[d+half] + x2 cos[d+half]
// K and V are written to row `pos` of this layer's cache, layout
// [head][kv_max][head_dim], as hi/lo BF16 planes.
// ---------------------------------------------------------------------------

template <int CPL>
__global__ void __launch_bounds__(256) qkv_rope_kernel(QkvArgs a) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int n = a.hidden;
    const int half = a.head_dim >> 1;
    const int per_mat = a.n_heads * half;
    TraceScope tr;
    // task t: the rotary row pair (row0, row0 + half) of Wq, Wk or Wv
    auto task_rows = [&](int t, const uint16_t *&p0, int &m, int &h, int &d) {
        m = t / per_mat;
        int r = t - m * per_mat;
        h = r / half;
        d = r - h * half;
        const uint16_t *W = m == 0 ? a.w[0] : (m == 1 ? a.w[1] : a.w[2]);
        p0 = W + (size_t)(h * a.head_dim + d) * n;
    };
    // before the dependency wait: the first task's weights (registers), the
    // norm weight (shared memory) and, once the position is readable (every
    // layer but the first: an earlier step's advance kernel wrote it), the
    // first task's RoPE factors
    extern __shared__ float qs[];  // x [n], then the norm weight [n]
    float *xs = qs, *nws = qs + n;
    Rows2<CPL> w;
    int m0 = 0, h0 = 0, d0 = 0;
    if (gw < 3 * per_mat) {
        const uint16_t *p0;
        task_rows(gw, p0, m0, h0, d0);
        w.load(p0, p0 + (size_t)half * n, n, lane);
    }
    if (threadIdx.x == 0) {
        const size_t G = gridDim.x, b = blockIdx.x;
        for (int k = 0; k < 3; k++) {
            const size_t B = a.pf_bytes[k];
            const size_t lo = (B * b / G) & ~(size_t)15, hi = b + 1 == G ? B : (B * (b + 1) / G) & ~(size_t)15;
            if (a.pf[k] && hi > lo) prefetch_range(static_cast<const uint8_t *>(a.pf[k]) + lo, hi - lo);
        }
    }
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
        *reinterpret_cast<float4 *>(nws + i) = *reinterpret_cast<const float4 *>(a.norm_w + i);
    int pos = a.pos_ready ? __ldcg(a.d_pos) : 0;
    float rc0 = 0.f, rs0 = 0.f, rc1 = 0.f, rs1 = 0.f;
    if (a.pos_ready && lane == 0 && gw < 3 * per_mat && m0 < 2) {
        const float *cs = a.cos_t + (size_t)pos * a.head_dim, *sn = a.sin_t + (size_t)pos * a.head_dim;
        rc0 = cs[d0];
        rs0 = sn[d0];
        rc1 = cs[d0 + half];
        rs1 = sn[d0 + half];
    }
    pdl_wait();
    pdl_launch();
    tr.waited();
    if (!a.pos_ready) pos = __ldcg(a.d_pos);
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
        *reinterpret_cast<float4 *>(xs + i) = __ldcg(reinterpret_cast<const float4 *>(a.x + i));
    __syncthreads();
    const float inv = block_rms_inv(xs, n, a.eps);
    XRegBF16<CPL> xr;
    xr.load_norm(xs, nws, inv, n, lane);
    for (int t = gw; t < 3 * per_mat; t += nw) {
        const uint16_t *p0;
        int m, h, d;
        task_rows(t, p0, m, h, d);
        const int row0 = h * a.head_dim + d;
        if (t != gw) w.load(p0, p0 + (size_t)half * n, n, lane);
        float s0, s1;
        w.dot(xr, s0, s1);
        s0 = warp_sum(s0);
        s1 = warp_sum(s1);
        if (lane == 0) {
            float o0 = s0, o1 = s1;
            if (m < 2) {
                float c0 = rc0, sn0 = rs0, c1 = rc1, sn1 = rs1;
                if (!(a.pos_ready && t == gw)) {
                    const float *cs = a.cos_t + (size_t)pos * a.head_dim;
                    const float *sn = a.sin_t + (size_t)pos * a.head_dim;
                    c0 = cs[d];
                    sn0 = sn[d];
                    c1 = cs[d + half];
                    sn1 = sn[d + half];
                }
                o0 = __fsub_rn(__fmul_rn(s0, c0), __fmul_rn(s1, sn0));
                o1 = __fadd_rn(__fmul_rn(s0, sn1), __fmul_rn(s1, c1));
            }
            if (m == 0) {
                a.q_out[row0] = o0;
                a.q_out[row0 + half] = o1;
            } else {
                size_t idx = ((size_t)h * a.kv_max + pos) * a.head_dim + d;
                uint16_t *hi = m == 1 ? a.k_hi : a.v_hi;
                uint16_t *lo = m == 1 ? a.k_lo : a.v_lo;
                uint16_t h0, l0, h1, l1;
                split_bf16(o0, h0, l0);
                split_bf16(o1, h1, l1);
                hi[idx] = h0;
                lo[idx] = l0;
                hi[idx + half] = h1;
                lo[idx + half] = l1;
            }
        }
    }
    tr.done(1);
}

// ---------------------------------------------------------------------------
// Decode attention for one token, all heads (ds_causal_attention_aligned MHA
// fast path, ds_kernels.c:2181-2249 / :2124-2159).
//
// The reference runs, per head, a sequential online softmax with fast exp:
//   s_j > m : c = fexp(m - s_j); sum = sum*c + 1;  o = o*c + v_j;  m = s_j
//   else    : a = fexp(s_j - m); sum += a;          o += a*v_j
//   o *= 1/sum
// fexp(a)fexp(b) != fexp(a+b), so a plain flash-style merge would differ.
// Unrolled, key j contributes w_j v_j with
//   w_j = a_j * prod_{t>j, s_t new max} c_t,   a_j = 1 at a new max,
// and sum = sum_j w_j. This kernel evaluates exactly that: a cluster of CL
// CTAs per head splits the keys; each CTA scores its chunk (q.k * scale),
// the cluster exchanges scores through distributed shared memory, every CTA
// runs the exclusive prefix-max and the suffix product of correction factors
// over all keys, forms w_j for its chunk and accumulates w_j v_j; rank 0 sums
// the CL partial outputs (DSMEM) and scales by 1/sum.
// head_dim must be 128 (8 lanes x 16 elements per key row).
// ---------------------------------------------------------------------------

// Block-wide exclusive scan of one value per thread (blockDim == 256) with an
// associative op; reverse = scan from the last thread down. Warp 0 scans:
// lane l owns 8 consecutive logical slots, then a shuffle scan of lane totals.
template <typename Op>
__device__ __forceinline__ float block_excl_scan(float v, float ident, Op op, bool reverse, float *buf) {
    const int t = threadIdx.x;
    const int lt = reverse ? 255 - t : t;
    buf[lt] = v;
    __syncthreads();
    if (t < 32) {
        float loc[8], acc = ident;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            loc[i] = acc;
            acc = op(acc, buf[t * 8 + i]);
        }
        float inc = acc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            float y = __shfl_up_sync(DS_FULL, inc, o);
            if (t >= o) inc = op(y, inc);
        }
        float excl = __shfl_up_sync(DS_FULL, inc, 1);
        if (t == 0) excl = ident;
#pragma unroll
        for (int i = 0; i < 8; i++) buf[t * 8 + i] = op(excl, loc[i]);
    }
    __syncthreads();
    float r = buf[lt];
    __syncthreads();
    return r;
}

// Block sum of one value per thread (blockDim == 256) in a fixed order.
__device__ __forceinline__ float block_sum256(float v, float *buf) {
    buf[threadIdx.x] = v;
    __syncthreads();
    float r = 0.f;
    if (threadIdx.x < 32) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) s = __fadd_rn(s, buf[threadIdx.x * 8 + i]);
        r = warp_sum(s);
    }
    __syncthreads();
    if (threadIdx.x == 0) buf[0] = r;
    __syncthreads();
    r = buf[0];
    __syncthreads();
    return r;
}

// PRE: load the first block of KV rows before the dependency wait (for
// launches chained with programmatic dependent launch).
// SWA: V3's reference sliding window (a separate instantiation, so the
// full-causal kernels keep their registers).
template <int CL, bool PRE, bool SWA = false, int KPG = ATT_KPG>
__device__ __forceinline__ void attn_body(const AttnArgs &a) {
    __shared__ float sc_own[CL > 1 ? ATT_MAXK / CL : 1];
    __shared__ float wts[ATT_MAXK];
    __shared__ __align__(16) float corr[ATT_MAXK];  // reused as the [32][128] PV reduction buffer
    __shared__ float opart[ATT_HD];
    __shared__ float tmp[256];
    __shared__ float s_sum;
    float(*red)[ATT_HD] = reinterpret_cast<float(*)[ATT_HD]>(corr);

    TraceScope tr;
    const int crank = CL > 1 ? (int)cg::this_cluster().block_rank() : 0;
    const int h = blockIdx.x / CL;
    const int tid = threadIdx.x;
    const int g = tid >> 3, li = tid & 7;

    // The position was advanced by a kernel that completed before the
    // predecessor started its dependent part, so it (and every KV row but
    // the newest, which the predecessor writes) is readable before the
    // dependency wait: the first block of K and V rows loads here.
    const int sidx = blockIdx.y;
    const int n_all = a.d_pos[sidx] + 1;
    // V3's reference sliding window (ds_moe_decoder.c:409-436): once the
    // query is at or past the prefill length P, the keys are rows [0, P)
    // then [max(P, n - W), n); key j (0 .. n-1 below) is row j < P ? j : j + gap
    int gap = 0;
    const int swa_ref = SWA && a.swa_refs ? a.swa_refs[sidx] : a.swa_ref;
    if (SWA && a.swa_window > 0 && n_all - 1 >= swa_ref) gap = max(0, n_all - a.swa_window - swa_ref);
    const int n = n_all - gap;
    auto row = [&](int j) { return SWA ? (j < swa_ref ? j : j + gap) : j; };
    const int lo_start = a.lo_starts ? a.lo_starts[sidx] : a.lo_start;
    const int per = (n + CL - 1) / CL;
    const int j0 = min(n, crank * per), j1 = min(n, j0 + per);
    const size_t hoff = (size_t)h * a.kv_max * ATT_HD + (size_t)sidx * a.kv_stream_stride;
    const float *qsrc = a.q + (size_t)sidx * a.q_stride;
    float *out = a.out + (size_t)sidx * a.q_stride;
    const uint16_t *khi = a.k_hi + hoff, *klo = a.k_lo + hoff, *vhi = a.v_hi + hoff, *vlo = a.v_lo + hoff;
    if (tid == 0 && j1 > j0) {
        // this CTA's V rows: one range, or two around the window's gap
        const int cut = SWA && gap ? min(max(j0, swa_ref), j1) : j1;
        for (int piece = 0; piece < 2; piece++) {
            const int a0 = piece ? cut : j0, a1 = piece ? j1 : cut;
            if (a1 <= a0) continue;
            const int r0 = row(a0), r1 = row(a1 - 1) + 1;
            prefetch_range(vhi + (size_t)r0 * ATT_HD, (size_t)(r1 - r0) * ATT_HD * 2);
            const int ls = max(r0, lo_start);
            if (ls < r1) prefetch_range(vlo + (size_t)ls * ATT_HD, (size_t)(r1 - ls) * ATT_HD * 2);
        }
    }
    Row16 kraw0[KPG], vraw[KPG];
    if constexpr (PRE) {
#pragma unroll
        for (int r = 0; r < KPG; r++) {
            const int j = j0 + g + 32 * r;
            const bool old = j < j1 && j < n - 1;
            kraw0[r] = old ? load_raw16(khi + (size_t)row(j) * ATT_HD + li * 16, klo + (size_t)row(j) * ATT_HD + li * 16,
                                        row(j) >= lo_start)
                           : Row16{};
            vraw[r] = old ? load_raw16(vhi + (size_t)row(j) * ATT_HD + li * 16, vlo + (size_t)row(j) * ATT_HD + li * 16,
                                       row(j) >= lo_start)
                          : Row16{};
        }
    }
    pdl_wait();
    pdl_launch();
    tr.waited();
    if constexpr (PRE) {
#pragma unroll
        for (int r = 0; r < KPG; r++) {
            const int j = j0 + g + 32 * r;
            if (j == n - 1 && j < j1) {  // the newest row, written by the predecessor
                kraw0[r] = load_raw16(khi + (size_t)row(j) * ATT_HD + li * 16, klo + (size_t)row(j) * ATT_HD + li * 16, true);
                vraw[r] = load_raw16(vhi + (size_t)row(j) * ATT_HD + li * 16, vlo + (size_t)row(j) * ATT_HD + li * 16, true);
            }
        }
    }
    float qf[16];
    {
        const float4 *qp = reinterpret_cast<const float4 *>(qsrc + h * ATT_HD + li * 16);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float4 v = qp[i];
            qf[4 * i] = v.x; qf[4 * i + 1] = v.y; qf[4 * i + 2] = v.z; qf[4 * i + 3] = v.w;
        }
    }
    // 1. scores of this CTA's keys: 8 lanes per key, KPG keys per lane
    //    group per block (all their K loads in flight together); the first
    //    block's K and V rows were loaded above (V kept for step 5)
    for (int jb = j0, blk = 0; jb < j1; jb += 32 * KPG, blk++) {
        Row16 kraw[KPG];
#pragma unroll
        for (int r = 0; r < KPG; r++) {
            int j = jb + g + 32 * r;
            if (PRE && blk == 0) kraw[r] = kraw0[r];
            else
                kraw[r] = j < j1 ? load_raw16(khi + (size_t)row(j) * ATT_HD + li * 16, klo + (size_t)row(j) * ATT_HD + li * 16,
                                              row(j) >= lo_start)
                                 : Row16{};
        }
        if (!PRE && blk == 0) {
#pragma unroll
            for (int r = 0; r < KPG; r++) {
                int j = jb + g + 32 * r;
                vraw[r] = j < j1 ? load_raw16(vhi + (size_t)row(j) * ATT_HD + li * 16, vlo + (size_t)row(j) * ATT_HD + li * 16,
                                              row(j) >= lo_start)
                                 : Row16{};
            }
        }
#pragma unroll
        for (int r = 0; r < KPG; r++) {
            int j = jb + g + 32 * r;
            float kf[16];
            raw_to_f32(kraw[r], kf);
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) s = __fmaf_rn(qf[i], kf[i], s);
            s += __shfl_xor_sync(DS_FULL, s, 1);
            s += __shfl_xor_sync(DS_FULL, s, 2);
            s += __shfl_xor_sync(DS_FULL, s, 4);
            if (li == 0 && j < j1) {
                if (CL > 1) sc_own[j - j0] = __fmul_rn(s, a.scale);
                else wts[j] = __fmul_rn(s, a.scale);
            }
        }
    }
    // 2. gather every key's score of this head (one CTA: already in place)
    if constexpr (CL > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        for (int j = tid; j < n; j += blockDim.x) {
            int owner = j / per;
            const float *src = cluster.map_shared_rank(sc_own, owner);
            wts[j] = src[j - owner * per];
        }
    }
    __syncthreads();
    // 3. exclusive prefix max -> per-key factor a_j and correction c_j
    const int seg = (n + blockDim.x - 1) / blockDim.x;
    const int s0 = min(n, tid * seg), s1 = min(n, s0 + seg);
    float lm = -1e30f;
    for (int j = s0; j < s1; j++) lm = fmaxf(lm, wts[j]);
    float m = block_excl_scan(lm, -1e30f, [](float x, float y) { return fmaxf(x, y); }, false, tmp);
    for (int j = s0; j < s1; j++) {
        float s = wts[j];
        if (s > m) {
            corr[j] = fast_expf(__fsub_rn(m, s));
            wts[j] = 1.0f;
            m = s;
        } else {
            corr[j] = 1.0f;
            wts[j] = fast_expf(__fsub_rn(s, m));
        }
    }
    // 4. suffix product of corrections -> w_j = a_j * prod_{t>j} c_t; sum
    float lp = 1.0f;
    for (int j = s1 - 1; j >= s0; j--) lp = __fmul_rn(lp, corr[j]);
    float P = block_excl_scan(lp, 1.0f, [](float x, float y) { return __fmul_rn(x, y); }, true, tmp);
    float lsum = 0.f;
    for (int j = s1 - 1; j >= s0; j--) {
        float w = __fmul_rn(wts[j], P);
        wts[j] = w;
        P = __fmul_rn(P, corr[j]);
    }
    for (int j = s0; j < s1; j++) lsum = __fadd_rn(lsum, wts[j]);
    float S_all = block_sum256(lsum, tmp);  // includes the barrier before corr is reused
    if (tid == 0) s_sum = S_all;
    // 5. this chunk's sum_j w_j v_j
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; i++) acc[i] = 0.f;
    for (int jb = j0, blk = 0; jb < j1; jb += 32 * KPG, blk++) {
        Row16 vr[KPG];
#pragma unroll
        for (int r = 0; r < KPG; r++) {
            int j = jb + g + 32 * r;
            if (blk == 0) vr[r] = vraw[r];
            else vr[r] = j < j1 ? load_raw16(vhi + (size_t)row(j) * ATT_HD + li * 16, vlo + (size_t)row(j) * ATT_HD + li * 16,
                                             row(j) >= lo_start)
                                : Row16{};
        }
#pragma unroll
        for (int r = 0; r < KPG; r++) {
            int j = jb + g + 32 * r;
            if (j < j1) {
                float vf[16];
                raw_to_f32(vr[r], vf);
                float w = wts[j];
#pragma unroll
                for (int i = 0; i < 16; i++) acc[i] = __fmaf_rn(w, vf[i], acc[i]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 16; i++) red[g][li * 16 + i] = acc[i];
    __syncthreads();
    if (tid < ATT_HD) {
        float o = 0.f;
        for (int k = 0; k < 32; k++) o = __fadd_rn(o, red[k][tid]);
        opart[tid] = o;
    }
    if constexpr (CL > 1) cg::this_cluster().sync();
    else __syncthreads();
    // 6. rank 0 combines the cluster's partial outputs
    if (crank == 0 && tid < ATT_HD) {
        float o = 0.f;
        if constexpr (CL > 1) {
            for (int r = 0; r < CL; r++) o = __fadd_rn(o, cg::this_cluster().map_shared_rank(opart, r)[tid]);
        } else {
            o = opart[tid];
        }
        float S = s_sum;
        out[h * ATT_HD + tid] = S > 0.f ? __fmul_rn(o, __fdiv_rn(1.0f, S)) : o;
    }
    if constexpr (CL > 1) cg::this_cluster().sync();
    tr.done(2);
}

// batch 1: a cluster of ATT_CL CTAs per head splits the keys
template <bool SWA>
__global__ void __cluster_dims__(ATT_CL, 1, 1) __launch_bounds__(256) attn_decode_kernel(AttnArgs a) {
    attn_body<ATT_CL, true, SWA>(a);
}
// many streams: one CTA per (head, stream) over all of the stream's keys
// (two keys in flight per lane group: the 2-CTA-per-SM register budget holds
// without spills)
__global__ void __launch_bounds__(256, 2) attn_streams_kernel(AttnArgs a) { attn_body<1, false, false, 2>(a); }

// ---------------------------------------------------------------------------
// Generic row matvec with optional input RMSNorm, bias and residual:
//   y = [resid +] W . norm(x) [+ bias]      (n <= 2048)
// O-projection + residual: ds_linear_nobias_bf16 + ds_residual_rms_norm's add
// (ds_moe_decoder.c:447-453).
// ---------------------------------------------------------------------------

// The router terms of this CTA's 16 output rows (one pass: 2 rows per warp,
// grid x 16 == rows), then, in the last CTA, logits, softmax and top-k.
// wr16: thread e's 16 router weights of this CTA's rows (loaded before the
// dependency wait); gs: the post-attention norm weights of those rows.
__device__ void router_fold(const MvArgs &a, const float *yv, const uint4 (&wr16)[2], const float *gs) {
    const RouterFold &f = a.rf;
    __shared__ bool last;
    __shared__ float lg[256];
    __syncthreads();
    const int row0 = blockIdx.x * 16;
    const int nrow = min(16, a.rows - row0);
    const int pst = rf_pstride((int)gridDim.x);
    // thread e: sum over the 16 rows of Wr[e][r] * g[r] * y[r], rows in order
    for (int e = threadIdx.x; e <= f.E; e += blockDim.x) {
        float acc = 0.f;
        if (e < f.E) {
            const uint32_t w[8] = {wr16[0].x, wr16[0].y, wr16[0].z, wr16[0].w,
                                   wr16[1].x, wr16[1].y, wr16[1].z, wr16[1].w};
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (i < nrow)
                    acc = __fmaf_rn((i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]), __fmul_rn(gs[i], yv[i]), acc);
        } else {
            for (int i = 0; i < nrow; i++) acc = __fmaf_rn(yv[i], yv[i], acc);
        }
        f.part[(size_t)e * pst + blockIdx.x] = acc;
    }
    if (f.no_tail) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(f.ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    TraceScope tr;
    __threadfence();
    // column e summed in three runs of consecutive CTAs (rf_run_sum)
    __shared__ float ls[256][3];
    for (int t = threadIdx.x; t < 3 * (f.E + 1); t += blockDim.x) {
        const int e = t / 3, part = t - 3 * e;
        ls[e][part] = rf_run_sum(f.part + (size_t)e * pst, (int)gridDim.x, part);
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= f.E; e += blockDim.x) lg[e] = __fadd_rn(__fadd_rn(ls[e][0], ls[e][1]), ls[e][2]);
    __syncthreads();
    if (threadIdx.x < 32) {
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(lg[f.E], (float)a.rows), f.eps)));
        for (int e = threadIdx.x; e < f.E; e += 32) {
            lg[e] = __fmul_rn(lg[e], inv);
            f.scores[e] = lg[e];
        }
        __syncwarp();
        router_select(lg, f.E, f.top_k, f.renorm, f.d_idx, f.d_wt);
        if (threadIdx.x == 0) *f.ticket = 0u;
    }
    tr.done(4);
}

template <int CPL>
__global__ void __launch_bounds__(256) matvec_res_kernel(MvArgs a) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    TraceScope tr;
    // the first row pair's weights load before the dependency wait, and the
    // router's weights of this CTA's 16 rows (thread e: its 16 columns of
    // expert e) with their norm weights
    Rows2<CPL> w;
    const int r0 = 2 * gw;
    if (r0 < a.rows)
        w.load(a.W + (size_t)r0 * a.n, r0 + 1 < a.rows ? a.W + (size_t)(r0 + 1) * a.n : nullptr, a.n, lane);
    uint4 wr16[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    __shared__ float gs[16];
    if (a.rf.Wr) {
        const int rb = blockIdx.x * 16;
        if ((int)threadIdx.x < a.rf.E && rb + 16 <= a.rows) {
            const uint4 *src = reinterpret_cast<const uint4 *>(a.rf.Wr + (size_t)threadIdx.x * a.rows + rb);
            wr16[0] = ldg_stream(src);
            wr16[1] = ldg_stream(src + 1);
        } else if ((int)threadIdx.x < a.rf.E) {
            uint32_t t[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int i = 0; i < 16 && rb + i < a.rows; i++)
                t[i >> 1] |= (uint32_t)a.rf.Wr[(size_t)threadIdx.x * a.rows + rb + i] << ((i & 1) * 16);
            wr16[0] = make_uint4(t[0], t[1], t[2], t[3]);
            wr16[1] = make_uint4(t[4], t[5], t[6], t[7]);
        }
        if (threadIdx.x < 16) gs[threadIdx.x] = rb + threadIdx.x < a.rows ? a.rf.g[rb + threadIdx.x] : 0.f;
    }
    pdl_wait();
    pdl_launch();
    tr.waited();
    const float inv = a.norm_w ? block_rms_inv(a.x, a.n, a.eps) : 1.f;
    XRegBF16<CPL> xr;
    xr.load_norm(a.x, a.norm_w, inv, a.n, lane);
    __shared__ float yv[16];
    for (int r = r0; r < a.rows; r += 2 * nw) {
        if (r != r0)
            w.load(a.W + (size_t)r * a.n, r + 1 < a.rows ? a.W + (size_t)(r + 1) * a.n : nullptr, a.n, lane);
        float s0, s1;
        w.dot(xr, s0, s1);
        s0 = warp_sum(s0);
        s1 = warp_sum(s1);
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < 2; k++) {
                int rr = r + k;
                if (rr >= a.rows) break;
                float v = k ? s1 : s0;
                if (a.bias) v = __fadd_rn(v, a.bias[rr]);
                if (a.resid) v = __fadd_rn(a.resid[rr], v);
                a.y[rr] = v;
                if (r == r0) yv[2 * (threadIdx.x >> 5) + k] = v;
            }
        }
    }
    tr.done(3);
    if (a.rf.Wr) router_fold(a, yv, wr16, gs);
}

// Long-K matvec (n up to 8192, x staged in shared memory): the dense FFN down
// projection [1280 x 6848] with the residual add (ds_moe_decoder.c:101, :468).
__global__ void __launch_bounds__(128) matvec_long_kernel(MvArgs a) {
    extern __shared__ float xs[];
    TraceScope tr;
    pdl_wait();
    pdl_launch();
    tr.waited();
    for (int i = threadIdx.x; i < a.n; i += blockDim.x) xs[i] = a.x[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= a.rows) return;
    const uint16_t *wr = a.W + (size_t)row * a.n;
    const int nch = a.n >> 3;
    float acc = 0.f;
    constexpr int U = 8;
    for (int c0 = lane; c0 < nch; c0 += 32 * U) {
        uint4 w[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            int ch = c0 + 32 * u;
            w[u] = ch < nch ? ldg_stream(wr + 8 * ch) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            int ch = c0 + 32 * u;
            if (ch < nch) {
                const float4 *xp = reinterpret_cast<const float4 *>(xs + 8 * ch);
                acc = dot8_bf16(w[u], xp[0], xp[1], acc);
            }
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        float v = acc;
        if (a.bias) v = __fadd_rn(v, a.bias[row]);
        if (a.resid) v = __fadd_rn(a.resid[row], v);
        a.y[row] = v;
    }
    tr.done(5);
}

// out = RMSNorm(x; w) for one vector (ds_rms_norm, ds_kernels.c:1387-1471).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *x, const float *w, float *out, int n, float eps) {
    pdl_wait();
    pdl_launch();
    const float inv = block_rms_inv(x, n, eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], w[i]), inv);
}

// Step advance for greedy decode: next input = BF16 embedding row of the
// token just produced, widened to F32 (ds_ocr.c:2272-2279); token logged at
// its position; position advanced (ds_moe_decoder.c:997); token appended to
// the generated-token history when one is kept (ds_ocr.c:2245-2248).
__global__ void decode_advance_kernel(const uint16_t *E, int hidden, const int *d_tok, int *d_pos, int *tok_log,
                                      float *x_out, int *hist, int *hist_len, int hist_cap) {
    TraceScope tr;
    pdl_wait();
    pdl_launch();
    tr.waited();
    int tok = *d_tok;
    const int pos = *d_pos;
    // an all-NaN logit row leaves no winner (token -1): embed row 0, log -1
    const uint16_t *row = E + (size_t)(tok < 0 ? 0 : tok) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) x_out[i] = __uint_as_float((uint32_t)row[i] << 16);
    __syncthreads();
    if (threadIdx.x == 0) {
        tok_log[pos] = tok;
        *d_pos = pos + 1;
        if (hist && *hist_len < hist_cap) {
            hist[*hist_len] = tok;
            *hist_len = *hist_len + 1;
        }
    }
    tr.done(9);
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
static int sms() {
    static int n = 0;
    if (!n) {
        int dev;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    }
    return n;
}

#define DS_CPL_SWITCH2(n, CHUNK, BODY)                \
    do {                                              \
        int _c = ((n) / (CHUNK) + 31) / 32;           \
        if (_c <= 2) { constexpr int CPL = 2; BODY; } \
        else if (_c <= 4) { constexpr int CPL = 4; BODY; } \
        else if (_c <= 5) { constexpr int CPL = 5; BODY; } \
        else if (_c <= 8) { constexpr int CPL = 8; BODY; } \
        else return cudaErrorInvalidValue;            \
    } while (0)

cudaError_t launch_qkv_rope(const QkvArgs &a, cudaStream_t st, bool pdl) {
    if (a.hidden % 8 || a.hidden > 2048 || a.head_dim % 2) return cudaErrorInvalidValue;
    int tasks = 3 * a.n_heads * (a.head_dim / 2);
    int grid = min((tasks + 7) / 8, sms() * 8);
    QkvArgs aa = a;
    void *args[] = {&aa};
    const size_t smem = (size_t)a.hidden * 8;
    DS_CPL_SWITCH2(a.hidden, 8, return launch_ex((const void *)qkv_rope_kernel<CPL>, grid, 256, smem, st, pdl, args));
}

cudaError_t launch_attn_decode(const AttnArgs &a, cudaStream_t st, bool pdl, int n_streams) {
    if (a.kv_max > ATT_MAXK) return cudaErrorInvalidValue;
    AttnArgs aa = a;
    void *args[] = {&aa};
    // cluster dims are compiled into the kernel (__cluster_dims__); with the
    // sliding window, several streams run the batch-1 kernel with grid.y =
    // stream (each stream its own prefill length in swa_refs)
    if (n_streams > 1 && a.swa_window > 0)
        return launch_ex((const void *)attn_decode_kernel<true>, dim3(a.n_heads * ATT_CL, n_streams), 256, 0, st,
                         pdl, args);
    if (n_streams == 1)
        return launch_ex(a.swa_window > 0 ? (const void *)attn_decode_kernel<true> : (const void *)attn_decode_kernel<false>,
                         a.n_heads * ATT_CL, 256, 0, st, pdl, args);
    // (clusters of 2 or 4 CTAs per (head, stream) measured slower at 64 streams)
    return launch_ex((const void *)attn_streams_kernel, dim3(a.n_heads, n_streams), 256, 0, st, pdl, args);
}

cudaError_t launch_matvec_res(const MvArgs &a, cudaStream_t st, bool pdl) {
    MvArgs aa = a;
    void *args[] = {&aa};
    if (a.n % 8) return cudaErrorInvalidValue;
    if (a.n <= 2048) {
        int grid = min(((a.rows + 1) / 2 + 7) / 8, sms() * 8);
        // the router fold needs one pass: 16 output rows per CTA
        // (and its readers take the part count as (rows + 15) / 16)
        if (a.rf.Wr && (grid != (a.rows + 15) / 16 || a.rf.E > 255)) return cudaErrorInvalidValue;
        DS_CPL_SWITCH2(a.n, 8, return launch_ex((const void *)matvec_res_kernel<CPL>, grid, 256, 0, st, pdl, args));
    }
    if (a.n > 8192 || a.norm_w) return cudaErrorInvalidValue;  // x stays within the 48 KB default smem
    int grid = (a.rows + 3) / 4;
    return launch_ex((const void *)matvec_long_kernel, grid, 128, (size_t)a.n * 4, st, pdl, args);
}

cudaError_t launch_decode_advance(const uint16_t *E, int hidden, const int *d_tok, int *d_pos, int *tok_log,
                                  float *x_out, cudaStream_t st, bool pdl, int *hist, int *hist_len, int hist_cap) {
    void *args[] = {&E, &hidden, &d_tok, &d_pos, &tok_log, &x_out, &hist, &hist_len, &hist_cap};
    return launch_ex((const void *)decode_advance_kernel, 1, 256, 0, st, pdl, args);
}

}  // namespace ds

namespace ds {
cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, int n, float eps, cudaStream_t st, bool pdl) {
    void *args[] = {&x, &w, &out, &n, &eps};
    return launch_ex((const void *)rmsnorm_kernel, 1, 256, 0, st, pdl, args);
}
}  // namespace ds

DS_TRACE_TU(decode)
