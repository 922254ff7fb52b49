// attn_prefill_tc.cu — the prefill's causal attention (ds_causal_attention,
// ds_kernels.c:2061-2114 via ds_decoder_prefill) on the tensor cores.
//
// The reference runs, per head and query, a sequential online softmax with
// fast exp over the keys in order:
//   s_j > m : c = fexp(m - s_j); sum = sum*c + 1;  o = o*c + v_j;  m = s_j
//   else    : a = fexp(s_j - m); sum += a;          o += a*v_j
// A CTA takes 128 queries of one head and walks the keys in blocks of 64.
// Per block b, with the running maximum carried per query:
//   S_b = Q K_b^T on the tensor cores (tcgen05, accumulator in tensor
//        memory). Q and K are split into BF16 planes (v = hi + lo; the cache
//        already stores K that way) and S = Qh Kh + Qh Kl + Ql Kh: ~2^-16
//        relative, in F32;
//   the query's two threads (one per 32-key half) read its row of S and
//        apply the sequential rule to their keys with exact arguments (the
//        second half starts from max(m, max of the first half), which is
//        exactly the reference's running maximum there): a_j, c_j, the
//        block's weights w_j = a_j * prod_{t > j in the block} c_t and
//        correction C_b = prod_t c_t (the product runs from the last key
//        down, the first half continuing the second half's product);
//   O <- O * C_b (in tensor memory; skipped when every C_b of a warp is 1)
//        and O += W_b V_b on the tensor cores, W split into BF16 planes the
//        same way (Wh Vh + Wh Vl + Wl Vh), sum <- sum * C_b + sum_j w_j.
// The factors are the reference's; products and sums associate in blocks
// (the CUDA-core kernel in prefill_full.cu does the same block recurrence).
//
// Roles: 256 row threads (8 warps; warps w and w + 4 share tensor-memory
// lanes 32 (w % 4) .. +31, i.e. query rows, and take the two key halves)
// and one issuing thread (TMA loads, MMAs). Shared memory: Q planes
// (64 KB), two stages of K planes and V planes (32 KB + 32 KB each), the W
// planes (32 KB). Tensor memory: two S buffers (64 columns each) so S_{b+1}
// is computed while the rows work on S_b, and O (128 columns). K and W are
// K-major operands; V is loaded as stored ([key][dim]) and taken by the MMA
// as an MN-major B operand. All operand tiles use the 128-byte swizzle
// (16-byte chunk c of a 128-byte row r at chunk c ^ (r % 8), 8-row atoms of
// 1024 B), the layout TMA writes with SWIZZLE_128B.
#include "kernels_decode.cuh"
#include "tmap.h"
#include "umma.cuh"

namespace ds {


constexpr int PT_Q = 128;                   // queries per CTA
constexpr int PT_K = 64;                    // keys per block
constexpr int PT_HD = 128;                  // head dim
constexpr int PT_QTILE = 128 * 128;         // swizzled 128-row x 64-column BF16 tile (16 KB)
constexpr int PT_KTILE = 64 * 128;          // swizzled 64-row x 64-column BF16 tile (8 KB)
constexpr int PT_QPLANES = 4 * PT_QTILE;    // Q hi, Q lo: two 64-column tiles each
constexpr int PT_KV = 4 * PT_KTILE;         // one stage of K (or V) hi and lo planes
constexpr int PT_WPLANES = 2 * PT_QTILE;    // W hi, W lo: 128 queries x 64 keys
constexpr int PT_SMEM = PT_QPLANES + 4 * PT_KV + PT_WPLANES + 1024;
constexpr int PT_ROWS = 256;                // 8 row warps
constexpr int PT_THREADS = PT_ROWS + 32;    // + the issuing warp

struct AttnTcArgs {
    CUtensorMap k_hi, k_lo, v_hi, v_lo;     // the layer's planes as [heads * kv_max] x 128, 64-row boxes
    const float *q;                         // [T x q_stride], head h at column h * 128
    int kv_max, p0, T, q_stride;
    float scale;
    float *out;                             // [T x q_stride]
    unsigned *err;
};

// Shared-memory descriptor of an MN-major BF16 operand in the 128-byte
// swizzle: 64 MN-elements (128 B) per row, one row per K index, 8-row atoms
// of 1024 B (stride byte offset) and 64-element MN blocks `lbo` bytes apart
// (leading byte offset), version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_mn_desc(const void *smem_tile, uint32_t lbo) {
    const uint64_t start = (smem_u32(smem_tile) >> 4) & 0x3fffu;
    return start | ((uint64_t)(lbo >> 4) << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// 32 consecutive F32 columns of this thread's tensor-memory lane, stored.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
        "tcgen05.wait::st.sync.aligned;"
        :: "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
           "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
           "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
           "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
           "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
           "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
           "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
           "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
           "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
           "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
           "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// Barrier of the two warps that share query rows (ids 1..4, 64 threads),
// returning whether any of them passed `bad`.
__device__ __forceinline__ bool pair_sync_or(int id, bool bad) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"((uint32_t)bad), "r"(id) : "memory");
    return r != 0;
}
__device__ __forceinline__ void pair_sync(int id) { asm volatile("bar.sync %0, 64;" :: "r"(id) : "memory"); }

__device__ __forceinline__ bool err_set(const unsigned *err) {
    return *reinterpret_cast<const volatile unsigned *>(err) != 0u;
}

__global__ void __launch_bounds__(PT_THREADS, 1) attn_prefill_tc_kernel(const __grid_constant__ AttnTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *qpl = smem;                                   // Q hi (2 tiles), Q lo (2 tiles)
    uint8_t *kst = smem + PT_QPLANES;                      // K stages: hi (2 tiles), lo (2 tiles)
    uint8_t *vst = kst + 2 * PT_KV;                        // V stages: hi (2 tiles), lo (2 tiles)
    uint8_t *wpl = vst + 2 * PT_KV;                        // W hi, W lo
    __shared__ uint64_t kfull[2], vfull[2], sfull[2], sfree[2], wfull, pvdone;
    __shared__ uint32_t tmem_base;
    __shared__ float2 xch[PT_Q];                           // per query: the two halves' exchange
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int h = blockIdx.x;
    const int q0 = (gridDim.y - 1 - blockIdx.y) * PT_Q;    // the longest query blocks launch first
    const int qend = min(a.T, q0 + PT_Q);                  // queries q0 .. qend-1 (relative to p0)
    const int nb = (a.p0 + qend - 1) / PT_K + 1;           // key blocks up to the last query's position
    if (tid == 0) {
        for (int s = 0; s < 2; s++) {
            mbar_init(&kfull[s], 1);
            mbar_init(&vfull[s], 1);
            mbar_init(&sfull[s], 1);
            mbar_init(&sfree[s], PT_ROWS / 32);
        }
        mbar_init(&wfull, PT_ROWS / 32);
        mbar_init(&pvdone, 1);
        mbar_fence_init();
    }
    if (warp == 8) tmem_alloc(&tmem_base, 256);
    if (warp < 8) {
        // Q: thread (row i, half hf) splits head dims 64 hf .. +63 of query
        // q0 + i into tile hf of the two planes (zeros for rows past T)
        const int i = tid & 127, hf = tid >> 7;
        const bool qvalid = q0 + i < a.T;
        const float *qr = a.q + (size_t)(q0 + i) * a.q_stride + h * PT_HD + hf * 64;
#pragma unroll 4
        for (int c = 0; c < 8; c++) {
            float f[8];
            if (qvalid) {
                const float4 u0 = __ldcg(reinterpret_cast<const float4 *>(qr + 8 * c));
                const float4 u1 = __ldcg(reinterpret_cast<const float4 *>(qr + 8 * c + 4));
                f[0] = u0.x; f[1] = u0.y; f[2] = u0.z; f[3] = u0.w;
                f[4] = u1.x; f[5] = u1.y; f[6] = u1.z; f[7] = u1.w;
            } else {
#pragma unroll
                for (int k = 0; k < 8; k++) f[k] = 0.f;
            }
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                uint16_t h0, l0, h1, l1;
                split_bf16(f[2 * k], h0, l0);
                split_bf16(f[2 * k + 1], h1, l1);
                hw[k] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                lw[k] = (uint32_t)l0 | ((uint32_t)l1 << 16);
            }
            const uint32_t o = hf * PT_QTILE + (i >> 3) * 1024 + (i & 7) * 128 + ((c ^ (i & 7)) << 4);
            *reinterpret_cast<uint4 *>(qpl + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(qpl + 2 * PT_QTILE + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        fence_proxy_async();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;  // columns 0..63, 64..127: the S buffers; 128..255: O
    constexpr uint32_t idesc_s = idesc_bf16_f32(PT_Q, PT_K);
    constexpr uint32_t idesc_pv = idesc_bf16_f32(PT_Q, PT_HD) | (1u << 16);  // B (V) MN-major

    if (warp == 8) {
        if (lane == 0) {
            const int y0 = h * a.kv_max;
            auto load_k = [&](int b) {
                uint8_t *d = kst + (b & 1) * PT_KV;
                mbar_expect_tx(&kfull[b & 1], PT_KV);
                tma_load_2d(d, &a.k_hi, 0, y0 + b * PT_K, &kfull[b & 1]);
                tma_load_2d(d + PT_KTILE, &a.k_hi, 64, y0 + b * PT_K, &kfull[b & 1]);
                tma_load_2d(d + 2 * PT_KTILE, &a.k_lo, 0, y0 + b * PT_K, &kfull[b & 1]);
                tma_load_2d(d + 3 * PT_KTILE, &a.k_lo, 64, y0 + b * PT_K, &kfull[b & 1]);
            };
            auto load_v = [&](int b) {
                uint8_t *d = vst + (b & 1) * PT_KV;
                mbar_expect_tx(&vfull[b & 1], PT_KV);
                tma_load_2d(d, &a.v_hi, 0, y0 + b * PT_K, &vfull[b & 1]);
                tma_load_2d(d + PT_KTILE, &a.v_hi, 64, y0 + b * PT_K, &vfull[b & 1]);
                tma_load_2d(d + 2 * PT_KTILE, &a.v_lo, 0, y0 + b * PT_K, &vfull[b & 1]);
                tma_load_2d(d + 3 * PT_KTILE, &a.v_lo, 64, y0 + b * PT_K, &vfull[b & 1]);
            };
            // O += W V for block c (W written by the rows, V in stage c & 1)
            auto pv = [&](int c) {
                const uint8_t *v = vst + (c & 1) * PT_KV;
                const uint64_t dwh = sw128_desc(wpl), dwl = sw128_desc(wpl + PT_QTILE);
                const uint64_t dvh = sw128_mn_desc(v, PT_KTILE), dvl = sw128_mn_desc(v + 2 * PT_KTILE, PT_KTILE);
#pragma unroll
                for (int j = 0; j < PT_K / 16; j++) {
                    umma_bf16(tmem + 128, dwh + 2 * j, dvh + 128 * j, idesc_pv, (c | j) != 0);
                    umma_bf16(tmem + 128, dwh + 2 * j, dvl + 128 * j, idesc_pv, 1u);
                    umma_bf16(tmem + 128, dwl + 2 * j, dvh + 128 * j, idesc_pv, 1u);
                }
                umma_commit(&pvdone);
            };
            bool ok = !err_set(a.err);
            if (ok) {
                load_k(0);
                load_v(0);
                if (nb > 1) {
                    load_k(1);
                    load_v(1);
                }
            }
            for (int b = 0; b < nb && ok; b++) {
                const int s = b & 1;
                ok = mbar_wait(&kfull[s], (b >> 1) & 1, a.err);
                if (ok && b >= 2) ok = mbar_wait(&sfree[s], ((b - 2) >> 1) & 1, a.err);
                if (!ok) break;
                tc_fence_after();
                const uint8_t *k = kst + s * PT_KV;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const uint64_t dqh = sw128_desc(qpl + c * PT_QTILE), dql = sw128_desc(qpl + (2 + c) * PT_QTILE);
                    const uint64_t dkh = sw128_desc(k + c * PT_KTILE), dkl = sw128_desc(k + (2 + c) * PT_KTILE);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        umma_bf16(tmem + s * PT_K, dqh + 2 * j, dkh + 2 * j, idesc_s, (c | j) != 0);
                        umma_bf16(tmem + s * PT_K, dqh + 2 * j, dkl + 2 * j, idesc_s, 1u);
                        umma_bf16(tmem + s * PT_K, dql + 2 * j, dkh + 2 * j, idesc_s, 1u);
                    }
                }
                umma_commit(&sfull[s]);
                if (b >= 1) {
                    // K stage (b+1)&1 held block b-1, whose S is done: refill it now
                    if (b + 1 < nb) {
                        ok = mbar_wait(&sfull[s ^ 1], ((b - 1) >> 1) & 1, a.err);
                        if (ok) load_k(b + 1);
                    }
                    if (ok) ok = mbar_wait(&wfull, (b - 1) & 1, a.err);
                    if (!ok) break;
                    tc_fence_after();
                    ok = mbar_wait(&vfull[s ^ 1], ((b - 1) >> 1) & 1, a.err);
                    if (!ok) break;
                    pv(b - 1);
                    // V stage (b+1)&1 is free once that PV is done
                    if (b + 1 < nb) {
                        ok = mbar_wait(&pvdone, (b - 1) & 1, a.err);
                        if (ok) load_v(b + 1);
                    }
                }
                if (ok && err_set(a.err)) ok = false;
            }
            if (ok) {
                ok = mbar_wait(&wfull, (nb - 1) & 1, a.err);
                if (ok) ok = mbar_wait(&vfull[(nb - 1) & 1], ((nb - 1) >> 1) & 1, a.err);
                if (ok) {
                    tc_fence_after();
                    pv(nb - 1);
                    mbar_wait(&pvdone, (nb - 1) & 1, a.err);
                }
            }
        }
        __syncwarp();
        __syncthreads();  // the row threads have read O
        tc_fence_after();
        tmem_dealloc(tmem, 256);
        return;
    }

    // ---- row threads: (query q0 + i, key half hf) ----
    const int i = tid & 127, hf = tid >> 7, pid = 1 + (warp & 3);
    const bool qvalid = q0 + i < a.T;
    const int qpos = a.p0 + q0 + i;
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's lanes
    float m = -1e30f, L = 0.f;
    bool bad = false;
    for (int b = 0; b < nb; b++) {
        const int s = b & 1;
        bad |= !mbar_wait(&sfull[s], (b >> 1) & 1, a.err);
        tc_fence_after();
        float sv[32], so[32];
        tmem_ld32(tl + s * PT_K + hf * 32, sv);
        tmem_ld32(tl + s * PT_K + (hf ^ 1) * 32, so);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[s]);
        const int kb = b * PT_K;
        const int nv = qvalid ? max(0, min(32, qpos - (kb + hf * 32) + 1)) : 0;
        const int nvo = qvalid ? max(0, min(32, qpos - (kb + (hf ^ 1) * 32) + 1)) : 0;
        // the other half's maximum: the second half starts from the running
        // maximum after the first
        float mo = -1e30f;
#pragma unroll
        for (int j = 0; j < 32; j++)
            if (j < nvo) mo = fmaxf(mo, __fmul_rn(so[j], a.scale));
        if (hf) m = fmaxf(m, mo);
        // The sequential rule: a_j in place; at a new maximum, c_j in place
        // and the key's bit set. The running maximum before each key is a one-operation chain; the
        // rest is independent per key. At a new maximum (d = s_j - m > 0) the
        // reference's c_j = fexp(m - s_j) = fexp(-d), else a_j = fexp(d): the
        // argument is -|d| either way (round-to-nearest is sign-symmetric).
        uint32_t nm = 0;
        float pm[32];
#pragma unroll
        for (int j = 0; j < 32; j++) {
            sv[j] = __fmul_rn(sv[j], a.scale);
            pm[j] = m;
            if (j < nv) m = fmaxf(m, sv[j]);
        }
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const float d = __fsub_rn(sv[j], pm[j]);
            if (j < nv) nm |= (d > 0.f ? 1u : 0u) << j;
            sv[j] = j < nv ? fast_expf(-fabsf(d)) : 0.f;
        }
        if (!hf) m = fmaxf(m, mo);  // the running maximum at the block's end
        // w_j = a_j * prod_{t > j} c_t (a_j = 1 at a new maximum), from the
        // block's last key down: the second half first, the first half
        // continuing its product; C = the whole product
        auto backward = [&](float P) {
#pragma unroll
            for (int j = 31; j >= 0; j--) {
                const bool isn = (nm >> j) & 1u;
                const float wj = isn ? P : __fmul_rn(sv[j], P);
                if (isn) P = __fmul_rn(P, sv[j]);
                sv[j] = wj;
            }
            return P;
        };
        float ls = 0.f, C;
        if (hf) {
            const float P1 = backward(1.0f);
#pragma unroll
            for (int j = 0; j < 32; j++) ls = __fadd_rn(ls, sv[j]);
            xch[i] = make_float2(P1, ls);
        }
        if (pair_sync_or(pid, bad)) {
            bad = true;
            break;
        }
        if (!hf) {
            const float2 x = xch[i];
            C = backward(x.x);
#pragma unroll
            for (int j = 0; j < 32; j++) ls = __fadd_rn(ls, sv[j]);
            L = __fadd_rn(__fmul_rn(L, C), __fadd_rn(ls, x.y));
            xch[i].x = C;
        }
        pair_sync(pid);
        if (hf) C = xch[i].x;
        // W and O are free once the previous block's W V is done
        if (b > 0) bad |= !mbar_wait(&pvdone, (b - 1) & 1, a.err);
        tc_fence_after();
        // O <- O * C on this half's 64 columns (a warp whose rows all have
        // C = 1 leaves O as it is)
        if (b > 0 && __any_sync(0xffffffffu, C != 1.0f)) {
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                float t[32];
                const uint32_t ta = tl + 128 + hf * 64 + 32 * c;
                tmem_ld32(ta, t);
#pragma unroll
                for (int k = 0; k < 32; k++) t[k] = __fmul_rn(t[k], C);
                tmem_st32(ta, t);
            }
        }
        // this half's 32 weights into the W planes (keys 32 hf .. +31 of row i)
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                uint16_t h0, l0, h1, l1;
                split_bf16(sv[8 * c + 2 * k], h0, l0);
                split_bf16(sv[8 * c + 2 * k + 1], h1, l1);
                hw[k] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                lw[k] = (uint32_t)l0 | ((uint32_t)l1 << 16);
            }
            const uint32_t o = (i >> 3) * 1024 + (i & 7) * 128 + ((((hf * 4 + c) ^ (i & 7))) << 4);
            *reinterpret_cast<uint4 *>(wpl + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(wpl + PT_QTILE + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfull);
    }
    // O / sum into the output row (1 / sum from the first half's thread)
    if (!hf) xch[i].y = L > 0.f ? __fdiv_rn(1.0f, L) : 0.f;
    pair_sync(pid);
    const float inv = xch[i].y;
    if (!bad) bad = !mbar_wait(&pvdone, (nb - 1) & 1, a.err);
    bad = __any_sync(0xffffffffu, bad);
    tc_fence_after();
    if (!bad) {
        float *orow = a.out + (size_t)(q0 + i) * a.q_stride + h * PT_HD + hf * 64;
#pragma unroll 1
        for (int c = 0; c < 2; c++) {
            float t[32];
            tmem_ld32(tl + 128 + hf * 64 + 32 * c, t);
            if (qvalid)
#pragma unroll
                for (int k = 0; k < 32; k += 4)
                    *reinterpret_cast<float4 *>(orow + 32 * c + k) =
                        make_float4(__fmul_rn(t[k], inv), __fmul_rn(t[k + 1], inv), __fmul_rn(t[k + 2], inv),
                                    __fmul_rn(t[k + 3], inv));
        }
    }
    tc_fence_before();
    __syncthreads();  // O read: the issuing warp may release tensor memory
}

bool attn_prefill_tc_ok(int head_dim, int kv_max, int n_heads) {
    return head_dim == PT_HD && kv_max >= 1 && n_heads >= 1;
}

cudaError_t launch_attn_prefill_tc(const float *q, const uint16_t *k_hi, const uint16_t *k_lo,
                                   const uint16_t *v_hi, const uint16_t *v_lo, int kv_max, int n_heads, int p0, int T,
                                   int q_stride, float scale, float *out, unsigned *err, cudaStream_t st) {
    AttnTcArgs a = {};
    const uint64_t rows = (uint64_t)n_heads * kv_max;
    if (!tmap_bf16(&a.k_hi, k_hi, PT_HD, rows, PT_K) || !tmap_bf16(&a.k_lo, k_lo, PT_HD, rows, PT_K) ||
        !tmap_bf16(&a.v_hi, v_hi, PT_HD, rows, PT_K) || !tmap_bf16(&a.v_lo, v_lo, PT_HD, rows, PT_K))
        return cudaErrorInvalidValue;
    a.q = q;
    a.kv_max = kv_max;
    a.p0 = p0;
    a.T = T;
    a.q_stride = q_stride;
    a.scale = scale;
    a.out = out;
    a.err = err;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             PT_SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    attn_prefill_tc_kernel<<<dim3(n_heads, (T + PT_Q - 1) / PT_Q), PT_THREADS, PT_SMEM, st>>>(a);
    return cudaGetLastError();
}

}  // namespace ds
