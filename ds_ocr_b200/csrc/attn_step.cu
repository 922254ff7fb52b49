// attn_step.cu — batch-1 decode attention whose CTAs exchange O(cluster)
// numbers instead of every score (ds_causal_attention_aligned MHA fast path,
// ds_kernels.c:2181-2249 / :2124-2159).
//
// The reference runs, per head, a sequential online softmax with fast exp:
//   s_j > m : c = fexp(m - s_j); sum = sum*c + 1;  o = o*c + v_j;  m = s_j
//   else    : a = fexp(s_j - m); sum += a;          o += a*v_j
// Unrolled, key j contributes w_j v_j with w_j = a_j * prod_{t>j, new max} c_t
// (a_j = 1 at a new max) and sum = sum_j w_j. A cluster of CL CTAs splits a
// head's keys into CL contiguous blocks. Two facts make the exchange small:
//   * the running maximum entering block b is the max of the earlier blocks'
//     maxima, so after one exchange of block maxima each CTA applies the
//     sequential rule to its own keys with the exact arguments, giving a_j,
//     c_j and the block's correction product C_b = prod_{t in b, new max} c_t;
//   * w_j = a_j * prod_{t > j in b} c_t * prod_{b' > b} C_b', so after a
//     second exchange (the C_b) a CTA scales its partial output and its sum
//     of weights by prod_{b' > b} C_b'.
// Rank 0 then adds the partial outputs and sums and scales by 1/sum. The
// factors are the reference's; products and sums associate differently.
#include <cooperative_groups.h>

#include "attn_rows.cuh"
#include "kernels_decode.cuh"

namespace cg = cooperative_groups;

namespace ds {

template <int CL, int KPG>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(256) attn_step_kernel(AttnArgs a) {
    __shared__ float sc[ATT_MAXK / CL];  // this CTA's scores, then weights
    __shared__ float cr[ATT_MAXK / CL];  // correction factors
    __shared__ float red[32][ATT_HD];
    __shared__ float xch[4];             // block max, block correction product, sum of weights, scaled sum
    __shared__ float opart[ATT_HD];
    __shared__ float s_fac;
    TraceScope tr;
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int h = blockIdx.x / CL;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = tid >> 3, li = tid & 7;
    // the position was advanced by a kernel that completed before the
    // predecessor started its dependent part: readable before the wait
    const int n = a.d_pos[0] + 1;
    const int lo_start = a.lo_start;
    const int per = (n + CL - 1) / CL;
    const int j0 = min(n, crank * per), j1 = min(n, j0 + per);
    const int cnt = j1 - j0;
    const size_t hoff = (size_t)h * a.kv_max * ATT_HD;
    const uint16_t *khi = a.k_hi + hoff, *klo = a.k_lo + hoff, *vhi = a.v_hi + hoff, *vlo = a.v_lo + hoff;
    auto krow = [&](int j, bool lo) {
        return load_raw16(khi + (size_t)j * ATT_HD + li * 16, klo + (size_t)j * ATT_HD + li * 16, lo);
    };
    auto vrow = [&](int j, bool lo) {
        return load_raw16(vhi + (size_t)j * ATT_HD + li * 16, vlo + (size_t)j * ATT_HD + li * 16, lo);
    };
    // every row but the newest (the predecessor writes it) loads before the
    // dependency wait: the first KPG keys of each 8-lane group, K and V
    Row16 kr0[KPG], vr0[KPG];
#pragma unroll
    for (int r = 0; r < KPG; r++) {
        const int j = j0 + g + 32 * r;
        const bool old = j < j1 && j < n - 1;
        kr0[r] = old ? krow(j, j >= lo_start) : Row16{};
        vr0[r] = old ? vrow(j, j >= lo_start) : Row16{};
    }
    pdl_wait();
    pdl_launch();
    tr.waited();
#pragma unroll
    for (int r = 0; r < KPG; r++) {
        const int j = j0 + g + 32 * r;
        if (j == n - 1 && j < j1) {
            kr0[r] = krow(j, true);
            vr0[r] = vrow(j, true);
        }
    }
    float qf[16];
    {
        const float4 *qp = reinterpret_cast<const float4 *>(a.q + h * ATT_HD + li * 16);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 v = __ldcg(qp + i);
            qf[4 * i] = v.x;
            qf[4 * i + 1] = v.y;
            qf[4 * i + 2] = v.z;
            qf[4 * i + 3] = v.w;
        }
    }
    tr.mark(0);
    // 1. scores: the prefetched keys, then (long contexts) the rest
    auto score = [&](const Row16 &kr, int j) {
        float kf[16];
        raw_to_f32(kr, kf);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) s = __fmaf_rn(qf[i], kf[i], s);
        s += __shfl_xor_sync(DS_FULL, s, 1);
        s += __shfl_xor_sync(DS_FULL, s, 2);
        s += __shfl_xor_sync(DS_FULL, s, 4);
        if (li == 0 && j < j1) sc[j - j0] = __fmul_rn(s, a.scale);
    };
#pragma unroll
    for (int r = 0; r < KPG; r++) score(kr0[r], j0 + g + 32 * r);
    for (int jb = j0 + 32 * KPG; jb < j1; jb += 32) {
        const int j = jb + g;
        score(j < j1 ? krow(j, j >= lo_start) : Row16{}, j);
    }
    __syncthreads();
    tr.mark(1);
    // 2. the sequential rule over this block's keys, all 256 threads: thread
    //    t owns a contiguous segment of keys; block scans (shuffles within a
    //    warp, then the 8 warp totals) give each segment its entering
    //    maximum and the product of the later segments' corrections
    __shared__ float wtot[8];
    const int seg = (cnt + 255) / 256;
    const int s0 = min(cnt, tid * seg), s1 = min(cnt, s0 + seg);
    float lmax = -1e30f;
    for (int j = s0; j < s1; j++) lmax = fmaxf(lmax, sc[j]);
    // inclusive max scan within the warp, warp totals
    float inc = lmax;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(DS_FULL, inc, o);
        if (lane >= o) inc = fmaxf(inc, y);
    }
    if (lane == 31) wtot[warp] = inc;
    __syncthreads();
    if (tid == 0) {
        float bm = -1e30f;
        for (int w = 0; w < 8; w++) bm = fmaxf(bm, wtot[w]);
        xch[0] = bm;
    }
    cluster.sync();
    tr.mark(2);
    {
        // running max entering the block, the earlier warps, the earlier lanes
        float m = -1e30f;
        for (int b = 0; b < crank; b++) m = fmaxf(m, cluster.map_shared_rank(xch, b)[0]);
        for (int w = 0; w < warp; w++) m = fmaxf(m, wtot[w]);
        const float ex = __shfl_up_sync(DS_FULL, inc, 1);
        if (lane > 0) m = fmaxf(m, ex);
        for (int j = s0; j < s1; j++) {
            const float sj = sc[j];
            if (sj > m) {
                cr[j] = fast_expf(__fsub_rn(m, sj));
                sc[j] = 1.0f;
                m = sj;
            } else {
                cr[j] = 1.0f;
                sc[j] = fast_expf(__fsub_rn(sj, m));
            }
        }
    }
    // suffix products of the corrections: the segment, the later lanes of the
    // warp (reverse inclusive scan), the later warps
    float lp = 1.0f;
    for (int j = s1 - 1; j >= s0; j--) lp = __fmul_rn(lp, cr[j]);
    float incp = lp;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(DS_FULL, incp, o);
        if (lane + o < 32) incp = __fmul_rn(incp, y);
    }
    __syncthreads();  // wtot is reused
    if (lane == 0) wtot[warp] = incp;
    __syncthreads();
    float P = __shfl_down_sync(DS_FULL, incp, 1);
    if (lane == 31) P = 1.0f;
    for (int w = 7; w > warp; w--) P = __fmul_rn(P, wtot[w]);
    float lsum = 0.f;
    for (int j = s1 - 1; j >= s0; j--) {
        const float wj = __fmul_rn(sc[j], P);
        sc[j] = wj;
        P = __fmul_rn(P, cr[j]);
    }
    for (int j = s0; j < s1; j++) lsum = __fadd_rn(lsum, sc[j]);
    lsum = warp_sum(lsum);
    __shared__ float wsum[8];
    if (lane == 0) wsum[warp] = lsum;
    __syncthreads();
    if (tid == 0) {
        float cb = 1.0f, S = 0.f;
        for (int w = 7; w >= 0; w--) cb = __fmul_rn(cb, wtot[w]);  // every correction of the block
        for (int w = 0; w < 8; w++) S = __fadd_rn(S, wsum[w]);
        xch[1] = cb;
        xch[2] = S;
    }
    tr.mark(3);
    cluster.sync();
    tr.mark(4);
    // 3. the later blocks' factor; this block's sum_j w_j v_j
    if (tid == 0) {
        float f = 1.0f;
        for (int b = crank + 1; b < CL; b++) f = __fmul_rn(f, cluster.map_shared_rank(xch, b)[1]);
        s_fac = f;
    }
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; i++) acc[i] = 0.f;
    auto pv = [&](const Row16 &vr, int j) {
        if (j < j1) {
            float vf[16];
            raw_to_f32(vr, vf);
            const float w = sc[j - j0];
#pragma unroll
            for (int i = 0; i < 16; i++) acc[i] = __fmaf_rn(w, vf[i], acc[i]);
        }
    };
#pragma unroll
    for (int r = 0; r < KPG; r++) pv(vr0[r], j0 + g + 32 * r);
    for (int jb = j0 + 32 * KPG; jb < j1; jb += 32) {
        const int j = jb + g;
        pv(j < j1 ? vrow(j, j >= lo_start) : Row16{}, j);
    }
#pragma unroll
    for (int i = 0; i < 16; i++) red[g][li * 16 + i] = acc[i];
    __syncthreads();
    if (tid < ATT_HD) {
        float o = 0.f;
        for (int k = 0; k < 32; k++) o = __fadd_rn(o, red[k][tid]);
        opart[tid] = __fmul_rn(o, s_fac);
    }
    if (tid == 0) xch[3] = __fmul_rn(xch[2], s_fac);
    tr.mark(5);
    cluster.sync();
    tr.mark(6);
    // 4. rank 0 adds the partial outputs and sums
    if (crank == 0 && tid < ATT_HD) {
        float o = 0.f, S = 0.f;
        for (int b = 0; b < CL; b++) {
            o = __fadd_rn(o, cluster.map_shared_rank(opart, b)[tid]);
            S = __fadd_rn(S, cluster.map_shared_rank(xch, b)[3]);
        }
        a.out[h * ATT_HD + tid] = S > 0.f ? __fmul_rn(o, __fdiv_rn(1.0f, S)) : o;
    }
    tr.mark(7);
    cluster.sync();  // the other CTAs' shared memory stays alive until rank 0 has read it
    tr.done(2);
}

cudaError_t launch_attn_step(const AttnArgs &a, cudaStream_t st, bool pdl) {
    if (a.kv_max > ATT_MAXK || a.swa_window > 0 || a.q_stride != 0 || a.kv_stream_stride != 0 || a.lo_starts)
        return cudaErrorInvalidValue;
    AttnArgs aa = a;
    void *args[] = {&aa};
    return launch_ex((const void *)attn_step_kernel<ATT_CL, ATT_KPG>, a.n_heads * ATT_CL, 256, 0, st, pdl, args);
}

}  // namespace ds

DS_TRACE_TU(attn2)
