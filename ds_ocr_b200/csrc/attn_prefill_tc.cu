// attn_prefill_tc.cu — the prefill's causal attention (ds_causal_attention,
// ds_kernels.c:2061-2114 via ds_decoder_prefill) on the tensor cores.
//
// The reference runs, per head and query, a sequential online softmax with
// fast exp over the keys in order:
//   s_j > m : c = fexp(m - s_j); sum = sum*c + 1;  o = o*c + v_j;  m = s_j
//   else    : a = fexp(s_j - m); sum += a;          o += a*v_j
// A CTA takes 128 queries of one head and walks the keys in blocks of 128.
// Per block b, with the running maximum carried per query:
//   S_b = Q K_b^T on the tensor cores (tcgen05, accumulator in tensor
//        memory). Q and K are split into BF16 planes (v = hi + lo; the cache
//        already stores K that way) and S = Qh Kh + Qh Kl + Ql Kh: ~2^-16
//        relative, in F32;
//   each query's thread reads its row of S and applies the sequential rule
//        to its keys with exact arguments: a_j, c_j, the block's weights
//        w_j = a_j * prod_{t > j in the block} c_t and correction
//        C_b = prod_t c_t;
//   O <- O * C_b (in tensor memory) and O += W_b V_b on the tensor cores, W
//        split into BF16 planes the same way (W Vh + W Vl with W = Wh + Wl,
//        dropping Wl Vl), sum <- sum * C_b + sum_j w_j.
// The factors are the reference's; products and sums associate in blocks
// (the CUDA-core kernel in prefill_full.cu does the same block recurrence).
//
// Roles: 128 row threads (4 warps; thread i owns query row i = tensor-memory
// lane i) and one issuing thread (TMA loads of the K planes, the MMAs).
// Shared memory: Q planes (64 KB), K planes reused as the W planes once S
// is computed (64 KB), V^T planes (64 KB; the row threads transpose V into
// the K-major layout the MMA's B operand takes). Operand tiles use the
// 128-byte-swizzled K-major layout of pf_gemm_kernel (prefill.cu): 128 rows
// of 64 BF16 (128 B), 16-byte chunk c of row r stored at chunk c ^ (r % 8),
// 8-row atoms of 1024 B.
#include "kernels_decode.cuh"
#include "tmap.h"
#include "umma.cuh"

namespace ds {

constexpr int PT_Q = 128;                  // queries per CTA
constexpr int PT_K = 128;                  // keys per block
constexpr int PT_HD = 128;                 // head dim
constexpr int PT_CHUNK = 128 * 128;        // one swizzled 128-row x 64-column BF16 tile (16 KB)
constexpr int PT_PLANE = 2 * PT_CHUNK;     // 128 x 128 BF16 (two 64-column tiles)
constexpr int PT_SMEM = 6 * PT_PLANE + 1024;
constexpr int PT_THREADS = 160;            // 4 row warps + the issuing warp

struct AttnTcArgs {
    CUtensorMap k_hi, k_lo;                // the layer's K planes as [heads * kv_max] x 128
    const float *q;                        // [T x q_stride], head h at column h * 128
    const uint16_t *v_hi, *v_lo;           // [head][kv_max][128]
    int kv_max, p0, T, q_stride;
    float scale;
    float *out;                            // [T x q_stride]
    unsigned *err;
};

// Byte offset of element (r, c) (r < 128, c < 128) in a plane stored as two
// swizzled 64-column tiles.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    const int t = c >> 6, cc = c & 63;
    return (uint32_t)(t * PT_CHUNK + (r >> 3) * 1024 + (r & 7) * 128 + ((((cc >> 3) ^ (r & 7))) << 4) + (cc & 7) * 2);
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

// Named barrier over the row threads and the issuing thread's warp.
__device__ __forceinline__ void pt_bar() { asm volatile("bar.sync 1, %0;" :: "r"(PT_THREADS) : "memory"); }


__global__ void __launch_bounds__(PT_THREADS, 1) attn_prefill_tc_kernel(const __grid_constant__ AttnTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *qh = smem, *ql = smem + PT_PLANE;            // Q planes
    uint8_t *kh = smem + 2 * PT_PLANE, *kl = kh + PT_PLANE;  // K planes, then the W planes
    uint8_t *vh = smem + 4 * PT_PLANE, *vl = vh + PT_PLANE;  // V^T planes
    __shared__ uint64_t kfull, sdone, pvdone;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int h = blockIdx.x, q0 = blockIdx.y * PT_Q;
    const int qend = min(a.T, q0 + PT_Q);                   // queries q0 .. qend-1 (relative to p0)
    const int qlast = a.p0 + qend - 1;                      // last key position any of them attends
    const int nb = qlast / PT_K + 1;
    if (tid == 0) {
        mbar_init(&kfull, 1);
        mbar_init(&sdone, 1);
        mbar_init(&pvdone, 1);
        mbar_fence_init();
    }
    if (warp == 4) tmem_alloc(&tmem_base, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;  // columns 0..127: S; 128..255: O
    constexpr uint32_t idesc = idesc_bf16_f32(PT_Q, PT_K);

    if (warp == 4) {
        // the issuing warp: lane 0 loads the K planes and issues the MMAs;
        // the whole warp joins the named barriers
        for (int b = 0; b < nb; b++) {
            if (lane == 0) {
                if (b > 0) mbar_wait(&pvdone, (b - 1) & 1, a.err);  // W and V^T of block b-1 consumed
                mbar_expect_tx(&kfull, 4 * PT_CHUNK);
                const int y = h * a.kv_max + b * PT_K;
                tma_load_2d(kh, &a.k_hi, 0, y, &kfull);
                tma_load_2d(kh + PT_CHUNK, &a.k_hi, 64, y, &kfull);
                tma_load_2d(kl, &a.k_lo, 0, y, &kfull);
                tma_load_2d(kl + PT_CHUNK, &a.k_lo, 64, y, &kfull);
            }
            pt_bar();  // the row threads have written V^T (and Q)
            if (lane == 0) {
                mbar_wait(&kfull, b & 1, a.err);
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const uint64_t dqh = sw128_desc(qh + c * PT_CHUNK), dql = sw128_desc(ql + c * PT_CHUNK);
                    const uint64_t dkh = sw128_desc(kh + c * PT_CHUNK), dkl = sw128_desc(kl + c * PT_CHUNK);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        umma_bf16(tmem, dqh + 2 * j, dkh + 2 * j, idesc, (c | j) != 0);
                        umma_bf16(tmem, dqh + 2 * j, dkl + 2 * j, idesc, 1u);
                        umma_bf16(tmem, dql + 2 * j, dkh + 2 * j, idesc, 1u);
                    }
                }
                umma_commit(&sdone);
            }
            pt_bar();  // the row threads have written W and rescaled O
            if (lane == 0) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const uint64_t dwh = sw128_desc(kh + c * PT_CHUNK), dwl = sw128_desc(kl + c * PT_CHUNK);
                    const uint64_t dvh = sw128_desc(vh + c * PT_CHUNK), dvl = sw128_desc(vl + c * PT_CHUNK);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        umma_bf16(tmem + PT_K, dwh + 2 * j, dvh + 2 * j, idesc, (b | c | j) != 0);
                        umma_bf16(tmem + PT_K, dwh + 2 * j, dvl + 2 * j, idesc, 1u);
                        umma_bf16(tmem + PT_K, dwl + 2 * j, dvh + 2 * j, idesc, 1u);
                    }
                }
                umma_commit(&pvdone);
            }
        }
        pt_bar();  // the row threads have read O
        tc_fence_after();
        tmem_dealloc(tmem, 256);
        return;
    }

    // ---- row threads: thread i owns query q0 + i (tensor-memory lane i) ----
    const int i = tid;
    const bool qvalid = q0 + i < a.T;
    const int qpos = a.p0 + q0 + i;
    const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's lanes
    // Q row into the two swizzled planes (zeros for rows past T)
    {
        const float *qr = a.q + (size_t)(q0 + i) * a.q_stride + h * PT_HD;
#pragma unroll 4
        for (int c = 0; c < PT_HD / 8; c++) {
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
            const uint32_t o = sw_off(i, 8 * c);
            *reinterpret_cast<uint4 *>(qh + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(ql + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
    }
    float m = -1e30f, L = 0.f;
    const size_t vbase = (size_t)h * a.kv_max * PT_HD;
    for (int b = 0; b < nb; b++) {
        if (b > 0) mbar_wait(&pvdone, (b - 1) & 1, a.err);  // V^T and O of block b-1 consumed
        // V^T: this thread's key row kb0 + i into column i of the planes
        {
            const int key = b * PT_K + i;
            const bool kv = key < a.kv_max;
            const uint16_t *rh = a.v_hi + vbase + (size_t)key * PT_HD, *rl = a.v_lo + vbase + (size_t)key * PT_HD;
#pragma unroll 2
            for (int c = 0; c < PT_HD / 8; c++) {
                const uint4 uh = kv ? ldg_stream(rh + 8 * c) : make_uint4(0, 0, 0, 0);
                const uint4 ul = kv ? ldg_stream(rl + 8 * c) : make_uint4(0, 0, 0, 0);
                const uint32_t wh[4] = {uh.x, uh.y, uh.z, uh.w}, wl[4] = {ul.x, ul.y, ul.z, ul.w};
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int d = 8 * c + k;
                    const uint32_t o = sw_off(d, i);
                    *reinterpret_cast<uint16_t *>(vh + o) = (uint16_t)(wh[k >> 1] >> ((k & 1) * 16));
                    *reinterpret_cast<uint16_t *>(vl + o) = (uint16_t)(wl[k >> 1] >> ((k & 1) * 16));
                }
            }
        }
        fence_proxy_async();
        pt_bar();  // V^T (and Q) written
        mbar_wait(&sdone, b & 1, a.err);
        tc_fence_after();
        // this query's scores of the block
        float sv[PT_K];
#pragma unroll
        for (int c = 0; c < PT_K / 32; c++) {
            float t[32];
            tmem_ld32(tl + 32 * c, t);
#pragma unroll
            for (int k = 0; k < 32; k++) sv[32 * c + k] = t[k];
        }
        const int nv = qvalid ? max(0, min(PT_K, qpos - b * PT_K + 1)) : 0;
        // the sequential rule: a_j in place; at a new maximum, c_j in place
        // and the key's bit set
        uint32_t nm[PT_K / 32] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < PT_K; j++) {
            if (j < nv) {
                const float sj = __fmul_rn(sv[j], a.scale);
                if (sj > m) {
                    sv[j] = fast_expf(__fsub_rn(m, sj));
                    nm[j >> 5] |= 1u << (j & 31);
                    m = sj;
                } else {
                    sv[j] = fast_expf(__fsub_rn(sj, m));
                }
            } else {
                sv[j] = 0.f;
            }
        }
        // w_j = a_j * prod_{t > j} c_t (a_j = 1 at a new maximum); C = prod c
        float P = 1.0f;
#pragma unroll
        for (int j = PT_K - 1; j >= 0; j--) {
            const bool isn = (nm[j >> 5] >> (j & 31)) & 1u;
            const float wj = isn ? P : __fmul_rn(sv[j], P);
            if (isn) P = __fmul_rn(P, sv[j]);
            sv[j] = wj;
        }
        float ls = 0.f;
#pragma unroll
        for (int j = 0; j < PT_K; j++) ls = __fadd_rn(ls, sv[j]);
        L = __fadd_rn(__fmul_rn(L, P), ls);
        // O <- O * C (the block's correction), before this block's W V is added
        if (b > 0) {
#pragma unroll 1
            for (int c = 0; c < PT_HD / 32; c++) {
                float t[32];
                tmem_ld32(tl + PT_K + 32 * c, t);
#pragma unroll
                for (int k = 0; k < 32; k++) t[k] = __fmul_rn(t[k], P);
                tmem_st32(tl + PT_K + 32 * c, t);
            }
        }
        // W's row into the two planes (over the K planes: S is computed)
#pragma unroll
        for (int c = 0; c < PT_K / 8; c++) {
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                uint16_t h0, l0, h1, l1;
                split_bf16(sv[8 * c + 2 * k], h0, l0);
                split_bf16(sv[8 * c + 2 * k + 1], h1, l1);
                hw[k] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                lw[k] = (uint32_t)l0 | ((uint32_t)l1 << 16);
            }
            const uint32_t o = sw_off(i, 8 * c);
            *reinterpret_cast<uint4 *>(kh + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(kl + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        fence_proxy_async();
        tc_fence_before();
        pt_bar();  // W written, O rescaled
    }
    // O / sum into the output row
    mbar_wait(&pvdone, (nb - 1) & 1, a.err);
    tc_fence_after();
    float *orow = a.out + (size_t)(q0 + i) * a.q_stride + h * PT_HD;
    const float inv = L > 0.f ? __fdiv_rn(1.0f, L) : 0.f;
#pragma unroll 1
    for (int c = 0; c < PT_HD / 32; c++) {
        float t[32];
        tmem_ld32(tl + PT_K + 32 * c, t);
        if (qvalid)
#pragma unroll
            for (int k = 0; k < 32; k += 4)
                *reinterpret_cast<float4 *>(orow + 32 * c + k) =
                    make_float4(__fmul_rn(t[k], inv), __fmul_rn(t[k + 1], inv), __fmul_rn(t[k + 2], inv),
                                __fmul_rn(t[k + 3], inv));
    }
    tc_fence_before();
    pt_bar();  // O read: the issuing warp may release tensor memory
}

bool attn_prefill_tc_ok(int head_dim, int kv_max, int n_heads) {
    return head_dim == PT_HD && kv_max >= 1 && n_heads >= 1;
}

cudaError_t launch_attn_prefill_tc(const float *q, const uint16_t *k_hi, const uint16_t *k_lo,
                                   const uint16_t *v_hi, const uint16_t *v_lo, int kv_max, int n_heads, int p0, int T,
                                   int q_stride, float scale, float *out, unsigned *err, cudaStream_t st) {
    AttnTcArgs a = {};
    if (!tmap_bf16(&a.k_hi, k_hi, PT_HD, (uint64_t)n_heads * kv_max, PT_K) ||
        !tmap_bf16(&a.k_lo, k_lo, PT_HD, (uint64_t)n_heads * kv_max, PT_K))
        return cudaErrorInvalidValue;
    a.q = q;
    a.v_hi = v_hi;
    a.v_lo = v_lo;
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
