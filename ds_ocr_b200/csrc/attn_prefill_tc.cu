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
//   the query's four threads (one per 16-key quarter) read its row of S
//        and apply the sequential rule to their keys with exact arguments
//        (a quarter starts from max(m, maxima of the earlier quarters),
//        which is exactly the reference's running maximum there): a_j, c_j,
//        the quarter's weights w_j = a_j * prod_{t > j in the quarter} c_t
//        and product P_q; the later quarters' products then scale each
//        quarter's weights, and C_b = P_3 P_2 P_1 P_0;
//   O <- O * C_b (in tensor memory; skipped when every C_b of a warp is 1)
//        and O += W_b V_b on the tensor cores, W split into BF16 planes the
//        same way (Wh Vh + Wh Vl + Wl Vh), sum <- sum * C_b + sum_j w_j.
// The factors are the reference's; products and sums associate in blocks
// (the CUDA-core kernel in prefill_full.cu does the same block recurrence).
//
// Roles: 512 row threads (16 warps; warps w, w + 4, w + 8, w + 12 share
// tensor-memory lanes 32 (w % 4) .. +31, i.e. query rows, and take the four
// 16-key quarters of each block) and one issuing thread (TMA loads, MMAs).
// The A operands of both products live in tensor memory, so the MMAs read
// only their B operand from shared memory (which bounds them): tensor memory
// holds two S buffers (64 columns each, so S_{b+1} is computed while the
// rows work on S_b), O (128), the Q planes (2 x 64, written once) and the W
// planes (2 x 32, written per block), BF16 pairs packed per 32-bit column.
// Shared memory holds three stages each of the K and V planes (32 KB a
// stage), refilled as soon as the block two behind is consumed. K is the
// K-major B operand of S; V is loaded as stored ([key][dim]) and taken as an
// MN-major B operand. Both use the 128-byte swizzle TMA writes with
// SWIZZLE_128B (16-byte chunk c of a 128-byte row r at chunk c ^ (r % 8),
// 8-row atoms of 1024 B).
#include "kernels_decode.cuh"
#include "tmap.h"
#include "umma.cuh"

namespace ds {


constexpr int PT_Q = 128;                   // queries per CTA
constexpr int PT_K = 64;                    // keys per block
constexpr int PT_HD = 128;                  // head dim
constexpr int PT_KTILE = 64 * 128;          // swizzled 64-row x 64-column BF16 tile (8 KB)
constexpr int PT_KV = 4 * PT_KTILE;         // one stage of K (or V) hi and lo planes
constexpr int PT_NS = 3;                    // stages of K and of V
constexpr int PT_SMEM = 2 * PT_NS * PT_KV + 1024;
constexpr int PT_ROWS = 512;                // 16 row warps: 4 threads per query
constexpr int PT_THREADS = PT_ROWS + 64;    // + the two issuing warps
// tensor-memory columns
constexpr uint32_t PT_TS = 0;               // S buffers: 0..63, 64..127
constexpr uint32_t PT_TO = 128;             // O: 128 columns
constexpr uint32_t PT_TQ = 256;             // Q hi: 64 columns of BF16 pairs; Q lo: the next 64
constexpr uint32_t PT_TW = 384;             // two W buffers of 64: hi (32 columns of pairs), lo (32)
constexpr uint32_t PT_TCOLS = 512;

// Optional per-block timestamps of the longest CTA (head 0, last query
// block), compiled in with -DPT_TRACE: the issuing threads' and a row
// thread's progress through each key block, read back from pt_trace.
#ifdef PT_TRACE
__device__ unsigned long long pt_trace[12][64];
#define PT_MARK(k, b) do { if (blockIdx.x == 0 && blockIdx.y == 0 && (b) < 64) pt_trace[k][b] = ds_gtime(); } while (0)
#else
#define PT_MARK(k, b) do { } while (0)
#endif

struct AttnTcArgs {
    CUtensorMap k_hi, k_lo, v_hi, v_lo;     // the layer's planes as [heads * kv_max] x 128, 64-row boxes
    const float *q;                         // [T x q_stride], head h at column h * 128
    int kv_max, p0, T, q_stride;
    float scale;
    float *out;                             // [T x q_stride]
    unsigned *err;
};

// 16 / 8 / 32 consecutive 32-bit columns of this thread's tensor-memory lane,
// stored (then waited for).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n\t"
        "tcgen05.wait::st.sync.aligned;"
        :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, "
        "%9, %10, %11, %12, %13, %14, %15, %16};\n\t"
        "tcgen05.wait::st.sync.aligned;"
        :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
           "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
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

// split_bf16 of two values at once (v ~= hi + lo, each a BF16 rounded to
// nearest even), packed low value first: cvt.rn.bf16x2 rounds exactly as
// bf16_rne_bits for finite inputs.
__device__ __forceinline__ void split2_bf16(float v0, float v1, uint32_t &hi, uint32_t &lo) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(v1), "f"(v0));
    const float r0 = __fsub_rn(v0, __uint_as_float(hi << 16));
    const float r1 = __fsub_rn(v1, __uint_as_float(hi & 0xffff0000u));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r1), "f"(r0));
}

// tcgen05.mma (kind::f16, one CTA) with A in tensor memory (128 lanes = M
// rows, K = 16 BF16 as 8 columns of pairs) and B a shared-memory descriptor
// given as its low word (start address and leading byte offset) and high
// word; ACC = 0 overwrites D.
template <int ACC>
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a_tmem, uint32_t blo, uint32_t bhi, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .b64 bd;\n\t.reg .pred p;\n\t"
        "mov.b64 bd, {%2, %3};\n\tsetp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, p;\n\t}"
        :: "r"(d), "r"(a_tmem), "r"(blo), "r"(bhi), "r"(idesc), "n"(ACC) : "memory");
}
// High word of both B descriptors: stride byte offset 1024 B (8-row atoms),
// version 1, 128-byte swizzle.
constexpr uint32_t PT_DHI = 64u | (1u << 14) | (2u << 29);
// Low word of a K-major tile's descriptor (leading byte offset field 1), or
// of an MN-major one with 64-element blocks `lbo` bytes apart.
__device__ __forceinline__ uint32_t dlo_k(const void *p) { return ((smem_u32(p) >> 4) & 0x3fffu) | (1u << 16); }
__device__ __forceinline__ uint32_t dlo_mn(const void *p, uint32_t lbo) {
    return ((smem_u32(p) >> 4) & 0x3fffu) | ((lbo >> 4) << 16);
}

// Barrier of the four warps that share query rows (ids 1..4, 128 threads),
// returning whether any of them passed `bad`.
__device__ __forceinline__ bool group_sync_or(int id, bool bad) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"((uint32_t)bad), "r"(id) : "memory");
    return r != 0;
}
__device__ __forceinline__ void group_sync(int id) { asm volatile("bar.sync %0, 128;" :: "r"(id) : "memory"); }

__device__ __forceinline__ bool err_set(const unsigned *err) {
    return *reinterpret_cast<const volatile unsigned *>(err) != 0u;
}

__global__ void __launch_bounds__(PT_THREADS, 1) attn_prefill_tc_kernel(const __grid_constant__ AttnTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *kst = smem;                                   // K stages: hi (2 tiles), lo (2 tiles)
    uint8_t *vst = smem + PT_NS * PT_KV;                   // V stages: the same
    __shared__ uint64_t kfull[PT_NS], vfull[PT_NS], sfull[2], sfree[2], qfull, wfull[2], pvdone[2];
    __shared__ uint32_t tmem_base;
    __shared__ float xmax[4][PT_Q];                        // per key quarter and query: its maximum
    __shared__ float2 xprod[4][PT_Q];                      // ... its product of c_j and sum of weights
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int h = blockIdx.x;
    const int q0 = (gridDim.y - 1 - blockIdx.y) * PT_Q;    // the longest query blocks launch first
    const int qend = min(a.T, q0 + PT_Q);                  // queries q0 .. qend-1 (relative to p0)
    const int nb = (a.p0 + qend - 1) / PT_K + 1;           // key blocks up to the last query's position
    if (tid == PT_ROWS) {
        for (int s = 0; s < PT_NS; s++) {
            mbar_init(&kfull[s], 1);
            mbar_init(&vfull[s], 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&sfull[s], 1);
            mbar_init(&sfree[s], PT_ROWS / 32);
        }
        mbar_init(&qfull, PT_ROWS / 32);
        mbar_init(&wfull[0], PT_ROWS / 32);
        mbar_init(&wfull[1], PT_ROWS / 32);
        mbar_init(&pvdone[0], 1);
        mbar_init(&pvdone[1], 1);
        mbar_fence_init();
    }
    if (warp == PT_ROWS / 32) tmem_alloc(&tmem_base, PT_TCOLS);
    // row thread (query q0 + i, quarter qt): head dims 32 qt .. +31 of its
    // query split into BF16 pairs (zeros for rows past T)
    const int i = tid & 127, qt = (tid >> 7) & 3;
    const bool qvalid = warp < PT_ROWS / 32 && q0 + i < a.T;
    uint32_t qh[16], ql[16];
    {
        const float *qr = a.q + (size_t)(q0 + i) * a.q_stride + h * PT_HD + qt * 32;
#pragma unroll
        for (int c = 0; c < 8; c++) {
            float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
            if (qvalid) u = __ldcg(reinterpret_cast<const float4 *>(qr + 4 * c));
            split2_bf16(u.x, u.y, qh[2 * c], ql[2 * c]);
            split2_bf16(u.z, u.w, qh[2 * c + 1], ql[2 * c + 1]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    constexpr uint32_t idesc_s = idesc_bf16_f32(PT_Q, PT_K);
    constexpr uint32_t idesc_pv = idesc_bf16_f32(PT_Q, PT_HD) | (1u << 16);  // B (V) MN-major

    if (warp >= PT_ROWS / 32) {
        // two issuing threads on different SM sub-partitions: warp 16 issues
        // S and refills K, warp 17 issues W V and refills V
        if (lane == 0) {
            const bool is_s = warp == PT_ROWS / 32;
            const int y0 = h * a.kv_max;
            auto load = [&](uint8_t *dst, uint64_t *bar, const CUtensorMap *hi, const CUtensorMap *lo, int b) {
                mbar_expect_tx(bar, PT_KV);
                tma_load_2d(dst, hi, 0, y0 + b * PT_K, bar);
                tma_load_2d(dst + PT_KTILE, hi, 64, y0 + b * PT_K, bar);
                tma_load_2d(dst + 2 * PT_KTILE, lo, 0, y0 + b * PT_K, bar);
                tma_load_2d(dst + 3 * PT_KTILE, lo, 64, y0 + b * PT_K, bar);
            };
            bool ok = !err_set(a.err);
            if (is_s) {
                auto load_k = [&](int b) { load(kst + (b % PT_NS) * PT_KV, &kfull[b % PT_NS], &a.k_hi, &a.k_lo, b); };
                const uint32_t k_lo = dlo_k(kst);
                if (ok)
                    for (int b = 0; b < PT_NS && b < nb; b++) load_k(b);
                if (ok) ok = mbar_wait(&qfull, 0, a.err);  // the Q planes are in tensor memory
                for (int b = 0; b < nb && ok; b++) {
                    const int s = b & 1;
                    ok = mbar_wait(&kfull[b % PT_NS], (b / PT_NS) & 1, a.err);
                    if (ok && b >= 2) ok = mbar_wait(&sfree[s], ((b - 2) >> 1) & 1, a.err);
                    if (!ok) break;
                    PT_MARK(0, b);
                    tc_fence_after();
                    // S(b) = Q K_b^T (three split products) into S buffer s
                    const uint32_t d = tmem + PT_TS + s * PT_K, kb = k_lo + (b % PT_NS) * (PT_KV >> 4);
#pragma unroll
                    for (int c = 0; c < 2; c++) {
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const uint32_t qa = tmem + PT_TQ + 8 * (4 * c + j), qb = qa + 64;
                            const uint32_t kh = kb + c * (PT_KTILE >> 4) + 2 * j, kl = kh + ((2 * PT_KTILE) >> 4);
                            if (c == 0 && j == 0)
                                umma_ts<0>(d, qa, kh, PT_DHI, idesc_s);
                            else
                                umma_ts<1>(d, qa, kh, PT_DHI, idesc_s);
                            umma_ts<1>(d, qa, kl, PT_DHI, idesc_s);
                            umma_ts<1>(d, qb, kh, PT_DHI, idesc_s);
                        }
                    }
                    umma_commit(&sfull[s]);
                    PT_MARK(1, b);
                    // K stage of block b-1 is free once its S is done (its
                    // barrier's next phase is S(b+1), not yet issued)
                    if (b >= 1 && b + 2 < nb) {
                        ok = mbar_wait(&sfull[s ^ 1], ((b - 1) >> 1) & 1, a.err);
                        if (ok) load_k(b + 2);
                    }
                }
            } else {
                auto load_v = [&](int b) { load(vst + (b % PT_NS) * PT_KV, &vfull[b % PT_NS], &a.v_hi, &a.v_lo, b); };
                const uint32_t v_lo = dlo_mn(vst, PT_KTILE);
                if (ok)
                    for (int b = 0; b < PT_NS && b < nb; b++) load_v(b);
                for (int c = 0; c < nb && ok; c++) {
                    ok = mbar_wait(&vfull[c % PT_NS], (c / PT_NS) & 1, a.err);
                    // the previous W V done (before this commit, so the parity
                    // is unambiguous): its V stage takes block c + 2
                    if (ok && c >= 1) ok = mbar_wait(&pvdone[(c - 1) & 1], ((c - 1) >> 1) & 1, a.err);
                    if (ok) ok = mbar_wait(&wfull[c & 1], (c >> 1) & 1, a.err);
                    if (!ok) break;
                    PT_MARK(2, c);
                    tc_fence_after();
                    // O += W V of block c: A = the W planes in tensor memory
                    const uint32_t d = tmem + PT_TO, vb = v_lo + (c % PT_NS) * (PT_KV >> 4);
#pragma unroll
                    for (int j = 0; j < PT_K / 16; j++) {
                        const uint32_t wh = tmem + PT_TW + (c & 1) * 64 + 8 * j, wl = wh + 32;
                        const uint32_t vh = vb + 128 * j, vl = vh + ((2 * PT_KTILE) >> 4);
                        if (c == 0 && j == 0)
                            umma_ts<0>(d, wh, vh, PT_DHI, idesc_pv);
                        else
                            umma_ts<1>(d, wh, vh, PT_DHI, idesc_pv);
                        umma_ts<1>(d, wh, vl, PT_DHI, idesc_pv);
                        umma_ts<1>(d, wl, vh, PT_DHI, idesc_pv);
                    }
                    umma_commit(&pvdone[c & 1]);
                    PT_MARK(3, c);
                    if (c >= 1 && c + 2 < nb) load_v(c + 2);
                }
                if (ok) mbar_wait(&pvdone[(nb - 1) & 1], ((nb - 1) >> 1) & 1, a.err);
            }
        }
        __syncwarp();
        __syncthreads();  // the row threads have read O
        tc_fence_after();
        if (warp == PT_ROWS / 32) tmem_dealloc(tmem, PT_TCOLS);
        return;
    }

    // ---- row threads: (query q0 + i, key quarter qt of each block) ----
    const int gid = 1 + (warp & 3);
    const int qpos = a.p0 + q0 + i;
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's lanes
    tmem_st16(tl + PT_TQ + 16 * qt, qh);
    tmem_st16(tl + PT_TQ + 64 + 16 * qt, ql);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&qfull);
    // O is accumulated as O / R, R the product of the block corrections
    // since the last renormalisation (so W_b / R_b is added and O needs no
    // per-block rescale); R is folded back into O only when it gets small
    float m = -1e30f, L = 0.f, R = 1.0f;
    bool bad = false;
    for (int b = 0; b < nb; b++) {
        const int s = b & 1;
        bad |= !mbar_wait(&sfull[s], (b >> 1) & 1, a.err);
        if (tid == 0) PT_MARK(5, b);
        tc_fence_after();
        float sv[16];
        tmem_ld16(tl + PT_TS + s * PT_K + qt * 16, sv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[s]);
        const int nv = qvalid ? max(0, min(16, qpos - (b * PT_K + qt * 16) + 1)) : 0;
        // blocks below the diagonal have every key valid in every row of the
        // warp: no masking there
        const bool full = __all_sync(0xffffffffu, nv == 16);
        // this quarter's maximum, shared with the row's other three threads
        float t[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            sv[j] = __fmul_rn(sv[j], a.scale);
            t[j] = (full || j < nv) ? sv[j] : -1e30f;
        }
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
            for (int j = 0; j < w; j++) t[j] = fmaxf(t[j], t[j + w]);
        xmax[qt][i] = t[0];
        if (group_sync_or(gid, bad)) {
            bad = true;
            break;
        }
        // the running maximum before this quarter (exactly the reference's
        // there) and at the block's end
        float mend = m;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float x = xmax[q][i];
            if (q < qt) m = fmaxf(m, x);
            mend = fmaxf(mend, x);
        }
        // The sequential rule: a_j in place, or c_j at a new maximum. The
        // running maximum before each key is a one-operation chain; the rest
        // is independent per key. At a new maximum (d = s_j - m > 0) the
        // reference's c_j = fexp(m - s_j) = fexp(-d), else a_j = fexp(d): the
        // argument is -|d| either way (round-to-nearest is sign-symmetric).
        // The quarter has a new maximum iff its running maximum moves.
        const float m0 = m;
        float pm[16], raw[16];
        if (full) {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                pm[j] = m;
                m = fmaxf(m, sv[j]);
            }
#pragma unroll
            for (int j = 0; j < 16; j++) {
                raw[j] = sv[j];
                sv[j] = fast_expf_nonpos(-fabsf(__fsub_rn(sv[j], pm[j])));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                pm[j] = m;
                if (j < nv) m = fmaxf(m, sv[j]);
            }
#pragma unroll
            for (int j = 0; j < 16; j++) {
                raw[j] = j < nv ? sv[j] : -1e30f;  // masked keys are never a new maximum
                sv[j] = j < nv ? fast_expf_nonpos(-fabsf(__fsub_rn(sv[j], pm[j]))) : 0.f;
            }
        }
        const bool anynew = __any_sync(0xffffffffu, m > m0);
        m = mend;
        // w_j = a_j * prod_{t > j in the quarter} c_t (a_j = 1 at a new
        // maximum), from the quarter's last key down; P = the whole product
        float P = 1.0f;
        if (anynew) {
#pragma unroll
            for (int j = 15; j >= 0; j--) {
                const bool isn = raw[j] > pm[j];
                const float wj = isn ? P : __fmul_rn(sv[j], P);
                if (isn) P = __fmul_rn(P, sv[j]);
                sv[j] = wj;
            }
        }
        float ls = 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) ls = __fadd_rn(ls, sv[j]);
        xprod[qt][i] = make_float2(P, ls);
        group_sync(gid);
        // the product of the later quarters (this quarter's weights take
        // it), the block's correction C and its weight sum, in the same
        // order in all four threads
        float Cr = 1.0f, lsb = 0.f, Sq = 1.0f;
#pragma unroll
        for (int q = 3; q >= 0; q--) {
            const float2 x = xprod[q][i];
            if (q == qt) Sq = Cr;
            lsb = __fadd_rn(lsb, __fmul_rn(x.y, Cr));
            Cr = __fmul_rn(Cr, x.x);
        }
        const float C = Cr;
        L = __fadd_rn(__fmul_rn(L, C), lsb);
        if (__any_sync(0xffffffffu, Sq != 1.0f))
#pragma unroll
            for (int j = 0; j < 16; j++) sv[j] = __fmul_rn(sv[j], Sq);
        // W buffer b & 1 is free once the W V of block b-2 is done
        if (b >= 2) bad |= !mbar_wait(&pvdone[(b - 2) & 1], ((b - 2) >> 1) & 1, a.err);
        float Rn = __fmul_rn(R, C);
        const bool renorm = Rn < 0x1p-60f;  // also C = 0: O * 0 as the reference
        if (__any_sync(0xffffffffu, renorm)) {
            // O (as O / R) <- O * C, i.e. times Rn, once the previous block's
            // W V is in; then R = 1 for these rows
            if (b >= 1) bad |= !mbar_wait(&pvdone[(b - 1) & 1], ((b - 1) >> 1) & 1, a.err);
            tc_fence_after();
            if (b >= 1) {
                const float f = renorm ? Rn : 1.0f;
                float o[32];
                const uint32_t ta = tl + PT_TO + qt * 32;
                tmem_ld32(ta, o);
#pragma unroll
                for (int k = 0; k < 32; k++) o[k] = __fmul_rn(o[k], f);
                tmem_st32(ta, o);
            }
            if (renorm) Rn = 1.0f;
        }
        R = Rn;
        if (__any_sync(0xffffffffu, Rn != 1.0f)) {
            const float ir = __fdiv_rn(1.0f, Rn);
#pragma unroll
            for (int j = 0; j < 16; j++) sv[j] = __fmul_rn(sv[j], ir);
        }
        uint32_t wh[8], wl[8];
#pragma unroll
        for (int k = 0; k < 8; k++) split2_bf16(sv[2 * k], sv[2 * k + 1], wh[k], wl[k]);
        if (tid == 0) PT_MARK(6, b);
        tc_fence_after();
        // this quarter's 16 weights (keys 16 qt .. +15 of row i) into W buffer b & 1
        const uint32_t tw = tl + PT_TW + (b & 1) * 64 + 8 * qt;
        tmem_st8(tw, wh);
        tmem_st8(tw + 32, wl);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfull[b & 1]);
        if (tid == 0) PT_MARK(7, b);
    }
    // O = (O / R) * R / sum into this quarter's 32 output columns
    const float f = L > 0.f ? __fdiv_rn(R, L) : 0.f;
    if (!bad && nb >= 2) bad = !mbar_wait(&pvdone[(nb - 2) & 1], ((nb - 2) >> 1) & 1, a.err);
    if (!bad) bad = !mbar_wait(&pvdone[(nb - 1) & 1], ((nb - 1) >> 1) & 1, a.err);
    bad = __any_sync(0xffffffffu, bad);
    tc_fence_after();
    if (!bad) {
        float o[32];
        tmem_ld32(tl + PT_TO + qt * 32, o);
        if (qvalid) {
            float *orow = a.out + (size_t)(q0 + i) * a.q_stride + h * PT_HD + qt * 32;
#pragma unroll
            for (int k = 0; k < 32; k += 4)
                *reinterpret_cast<float4 *>(orow + k) =
                    make_float4(__fmul_rn(o[k], f), __fmul_rn(o[k + 1], f), __fmul_rn(o[k + 2], f),
                                __fmul_rn(o[k + 3], f));
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
