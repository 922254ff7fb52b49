// attn_rows.cuh — KV-cache row access shared by the decode attention kernels
// (kernels_decode.cu, attn_step.cu): a key or value row is 128 head-dim
// elements, stored as a hi and a lo BF16 plane (v ~= hi + lo).
#pragma once
#include "common.cuh"

namespace ds {

constexpr int ATT_CL = 8;
constexpr int ATT_MAXK = 4096;
constexpr int ATT_HD = 128;

constexpr int ATT_KPG = 4;  // keys per 8-lane group per load batch

// 16 consecutive head-dim elements of one KV row: hi plane and (optional) lo plane.
struct Row16 {
    uint4 h0, h1, l0, l1;
};

static __device__ __forceinline__ Row16 load_raw16(const uint16_t *hi, const uint16_t *lo, bool use_lo) {
    Row16 r;
    r.h0 = ldg_stream(hi);
    r.h1 = ldg_stream(hi + 8);
    if (use_lo) {
        r.l0 = ldg_stream(lo);
        r.l1 = ldg_stream(lo + 8);
    } else {
        r.l0 = make_uint4(0, 0, 0, 0);
        r.l1 = r.l0;
    }
    return r;
}

// hi + lo widened to F32 (lo is zero for exact-BF16 rows, and x + 0 == x).
static __device__ __forceinline__ void raw_to_f32(const Row16 &r, float f[16]) {
    uint32_t hw[8] = {r.h0.x, r.h0.y, r.h0.z, r.h0.w, r.h1.x, r.h1.y, r.h1.z, r.h1.w};
    uint32_t lw[8] = {r.l0.x, r.l0.y, r.l0.z, r.l0.w, r.l1.x, r.l1.y, r.l1.z, r.l1.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        f[2 * i] = __fadd_rn(bf16_lo(hw[i]), bf16_lo(lw[i]));
        f[2 * i + 1] = __fadd_rn(bf16_hi(hw[i]), bf16_hi(lw[i]));
    }
}

}  // namespace ds
