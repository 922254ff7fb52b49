// route.cuh — router softmax and top-k of one token by one warp: softmax
// with the reference's fast exp over E <= 256 scores, then k passes of a
// strict-'>' argmax that skips chosen experts (lowest index wins ties);
// weights = the probabilities, renormalised only if asked
// (ds_moe_decoder.c:157-183 and :652-686; the reference does not renorm).
#pragma once
#include "common.cuh"

namespace ds {

__device__ __forceinline__ void route_topk_warp(const float *lg, int E, int K, int renorm, int *idx_out,
                                                float *w_out) {
    const int lane = threadIdx.x & 31;
    // softmax + top-k: lane holds experts lane, lane+32, ...
    const int per = (E + 31) / 32;
    float p[8];
    float mx = -1e30f;
    for (int j = 0; j < per; j++) {
        const int e = lane + 32 * j;
        p[j] = e < E ? lg[e] : -1e30f;
        mx = fmaxf(mx, p[j]);
    }
    mx = warp_max(mx);
    float part = 0.f;
    for (int j = 0; j < per; j++) {
        const int e = lane + 32 * j;
        p[j] = e < E ? fast_expf(__fsub_rn(p[j], mx)) : 0.f;
        part = __fadd_rn(part, p[j]);
    }
    const float sinv = __fdiv_rn(1.0f, warp_sum(part));
    for (int j = 0; j < per; j++) p[j] = __fmul_rn(p[j], sinv);
    unsigned taken = 0;  // bit j: expert lane + 32j chosen
    float wk[8];
    int ik[8];
    float wsum = 0.f;
    for (int k = 0; k < K; k++) {
        float bv = -1e30f;
        int bi = 0x7fffffff;
        for (int j = 0; j < per; j++) {
            const int e = lane + 32 * j;
            if (e < E && !((taken >> j) & 1u) && p[j] > bv) {
                bv = p[j];
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        wk[k] = bv;
        ik[k] = bi;
        wsum = __fadd_rn(wsum, bv);
    }
    if (lane == 0) {
        for (int k = 0; k < K; k++) {
            idx_out[k] = ik[k];
            w_out[k] = renorm ? __fdiv_rn(wk[k], wsum) : wk[k];
        }
    }
}

}  // namespace ds
