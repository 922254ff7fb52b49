// prefill_full.cu — the per-token kernels of the whole-decoder prefill
// (ds_decoder_prefill, ds_moe_decoder.c:480-905); the GEMMs run on the
// tensor-core prefill kernel (prefill.cu), the MoE block on the MoE prefill;
// decoder.cu strings them together.
#include "kernels_decode.cuh"

namespace ds {

// Row r of x [M x H] (optionally RMS-normalised with weight nw, as
// ds_rms_norm) as BF16 planes hi/lo [M x H]. One block of 256 per row.
__global__ void __launch_bounds__(256) pd_split_kernel(const float *__restrict__ x, int H, const float *__restrict__ nw,
                                                       float eps, uint16_t *hi, uint16_t *lo) {
    __shared__ float part[8];
    const size_t r = blockIdx.x;
    const float *xr = x + r * H;
    float inv = 1.f;
    if (nw) {
        float ss = 0.f;
        for (int c = threadIdx.x * 4; c < H; c += 1024) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c);
            ss = __fmaf_rn(v.x, v.x, ss);
            ss = __fmaf_rn(v.y, v.y, ss);
            ss = __fmaf_rn(v.z, v.z, ss);
            ss = __fmaf_rn(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        ss = 0.f;
        for (int w = 0; w < 8; w++) ss = __fadd_rn(ss, part[w]);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
    }
    for (int c = threadIdx.x * 4; c < H; c += 1024) {
        float4 v = *reinterpret_cast<const float4 *>(xr + c);
        if (nw) {
            const float4 g = *reinterpret_cast<const float4 *>(nw + c);
            v.x = __fmul_rn(__fmul_rn(v.x, g.x), inv);
            v.y = __fmul_rn(__fmul_rn(v.y, g.y), inv);
            v.z = __fmul_rn(__fmul_rn(v.z, g.z), inv);
            v.w = __fmul_rn(__fmul_rn(v.w, g.w), inv);
        }
        uint16_t h[4], l[4];
        split_bf16(v.x, h[0], l[0]);
        split_bf16(v.y, h[1], l[1]);
        split_bf16(v.z, h[2], l[2]);
        split_bf16(v.w, h[3], l[3]);
        *reinterpret_cast<uint2 *>(hi + r * H + c) =
            make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
        *reinterpret_cast<uint2 *>(lo + r * H + c) =
            make_uint2((uint32_t)l[0] | ((uint32_t)l[1] << 16), (uint32_t)l[2] | ((uint32_t)l[3] << 16));
    }
}

// RoPE (ds_apply_rope_neox, ds_kernels.c:2426-2458) on the Q and K columns of
// qkv [T x 3QD] at positions p0 + t, Q to q [T x QD]; K and V rows written to
// the layer's cache planes at row p0 + t (layout [head][kv_max][hd]). One
// thread per (token, matrix, head, d < hd/2) rotary pair.
__global__ void pd_rope_kv_kernel(const float *__restrict__ qkv, int T, int NH, int HD, int p0,
                                  const float *__restrict__ cos_t, const float *__restrict__ sin_t, float *q,
                                  uint16_t *k_hi, uint16_t *k_lo, uint16_t *v_hi, uint16_t *v_lo, int kv_max) {
    const int half = HD / 2, QD = NH * HD;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long per_tok = 3LL * NH * half;
    if (i >= per_tok * T) return;
    const int t = (int)(i / per_tok);
    int r = (int)(i - (long long)t * per_tok);
    const int m = r / (NH * half);
    r -= m * NH * half;
    const int h = r / half, d = r - h * half;
    const float *row = qkv + (size_t)t * 3 * QD + (size_t)m * QD + h * HD;
    const float x1 = row[d], x2 = row[d + half];
    const int pos = p0 + t;
    float o0 = x1, o1 = x2;
    if (m < 2) {
        const float *cs = cos_t + (size_t)pos * HD, *sn = sin_t + (size_t)pos * HD;
        o0 = __fsub_rn(__fmul_rn(x1, cs[d]), __fmul_rn(x2, sn[d]));
        o1 = __fadd_rn(__fmul_rn(x1, sn[d + half]), __fmul_rn(x2, cs[d + half]));
    }
    if (m == 0) {
        q[(size_t)t * QD + h * HD + d] = o0;
        q[(size_t)t * QD + h * HD + d + half] = o1;
        return;
    }
    const size_t idx = ((size_t)h * kv_max + pos) * HD + d;
    uint16_t *hp = m == 1 ? k_hi : v_hi, *lp = m == 1 ? k_lo : v_lo;
    uint16_t a, b;
    split_bf16(o0, a, b);
    hp[idx] = a;
    lp[idx] = b;
    split_bf16(o1, a, b);
    hp[idx + half] = a;
    lp[idx + half] = b;
}

// The same with four consecutive rotary pairs per thread (hd/2 % 4 == 0):
// float4 loads of the row and of the tables, 8-byte plane stores, the same
// arithmetic per element.
__device__ __forceinline__ uint2 pack4_bf16(uint16_t a, uint16_t b, uint16_t c, uint16_t d) {
    return make_uint2((uint32_t)a | ((uint32_t)b << 16), (uint32_t)c | ((uint32_t)d << 16));
}
__global__ void pd_rope_kv4_kernel(const float *__restrict__ qkv, int T, int NH, int HD, int p0,
                                   const float *__restrict__ cos_t, const float *__restrict__ sin_t, float *q,
                                   uint16_t *k_hi, uint16_t *k_lo, uint16_t *v_hi, uint16_t *v_lo, int kv_max) {
    const int half = HD / 2, QD = NH * HD, g4 = half / 4;
    const unsigned per_tok = 3u * NH * g4;
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= per_tok * (unsigned)T) return;
    const int t = (int)(i / per_tok);
    int r = (int)(i - (unsigned)t * per_tok);
    const int m = r / (NH * g4);
    r -= m * NH * g4;
    const int h = r / g4, d = 4 * (r - h * g4);
    const float *row = qkv + (size_t)t * 3 * QD + (size_t)m * QD + h * HD;
    const float4 x1 = *reinterpret_cast<const float4 *>(row + d), x2 = *reinterpret_cast<const float4 *>(row + d + half);
    const int pos = p0 + t;
    float a0[4] = {x1.x, x1.y, x1.z, x1.w}, a1[4] = {x2.x, x2.y, x2.z, x2.w};
    if (m < 2) {
        const float *cs = cos_t + (size_t)pos * HD, *sn = sin_t + (size_t)pos * HD;
        const float4 c0 = *reinterpret_cast<const float4 *>(cs + d), s0 = *reinterpret_cast<const float4 *>(sn + d);
        const float4 c1 = *reinterpret_cast<const float4 *>(cs + d + half);
        const float4 s1 = *reinterpret_cast<const float4 *>(sn + d + half);
        const float cc0[4] = {c0.x, c0.y, c0.z, c0.w}, ss0[4] = {s0.x, s0.y, s0.z, s0.w};
        const float cc1[4] = {c1.x, c1.y, c1.z, c1.w}, ss1[4] = {s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float u = a0[k], v = a1[k];
            a0[k] = __fsub_rn(__fmul_rn(u, cc0[k]), __fmul_rn(v, ss0[k]));
            a1[k] = __fadd_rn(__fmul_rn(u, ss1[k]), __fmul_rn(v, cc1[k]));
        }
    }
    if (m == 0) {
        float *qr = q + (size_t)t * QD + h * HD;
        *reinterpret_cast<float4 *>(qr + d) = make_float4(a0[0], a0[1], a0[2], a0[3]);
        *reinterpret_cast<float4 *>(qr + d + half) = make_float4(a1[0], a1[1], a1[2], a1[3]);
        return;
    }
    const size_t idx = ((size_t)h * kv_max + pos) * HD + d;
    uint16_t *hp = m == 1 ? k_hi : v_hi, *lp = m == 1 ? k_lo : v_lo;
    uint16_t hh[8], ll[8];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        split_bf16(a0[k], hh[k], ll[k]);
        split_bf16(a1[k], hh[4 + k], ll[4 + k]);
    }
    *reinterpret_cast<uint2 *>(hp + idx) = pack4_bf16(hh[0], hh[1], hh[2], hh[3]);
    *reinterpret_cast<uint2 *>(lp + idx) = pack4_bf16(ll[0], ll[1], ll[2], ll[3]);
    *reinterpret_cast<uint2 *>(hp + idx + half) = pack4_bf16(hh[4], hh[5], hh[6], hh[7]);
    *reinterpret_cast<uint2 *>(lp + idx + half) = pack4_bf16(ll[4], ll[5], ll[6], ll[7]);
}

// x += y over n floats (n % 4 == 0): the residual adds (ds_vec_add).
__global__ void pd_add_kernel(float *x, const float *__restrict__ y, size_t n4) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    float4 a = reinterpret_cast<float4 *>(x)[i];
    const float4 b = reinterpret_cast<const float4 *>(y)[i];
    a.x = __fadd_rn(a.x, b.x);
    a.y = __fadd_rn(a.y, b.y);
    a.z = __fadd_rn(a.z, b.z);
    a.w = __fadd_rn(a.w, b.w);
    reinterpret_cast<float4 *>(x)[i] = a;
}

// After the prefill: the first token's embedding becomes the next decode
// input, the token is logged against the last prefill position (as a decode
// step logs its token against its input position) and appended to the
// history (the generation loop records it, ds_ocr.c:2245-2248), and the
// position is p0 + T.
__global__ void pd_finish_kernel(const uint16_t *E, int H, const int *tok, float *x_out, int *pos, int p_next,
                                 int *tok_log, int *hist, int *hist_len, int hist_cap) {
    int t = *tok;
    const uint16_t *row = E + (size_t)(t < 0 ? 0 : t) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) x_out[i] = __uint_as_float((uint32_t)row[i] << 16);
    if (threadIdx.x == 0) {
        *pos = p_next;
        tok_log[p_next - 1] = t;
        if (hist && *hist_len < hist_cap) {
            hist[*hist_len] = t;
            *hist_len = *hist_len + 1;
        }
    }
}

cudaError_t launch_pd_split(const float *x, int M, int H, const float *nw, float eps, uint16_t *hi, uint16_t *lo,
                            cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    pd_split_kernel<<<M, 256, 0, st>>>(x, H, nw, eps, hi, lo);
    return cudaGetLastError();
}

cudaError_t launch_pd_rope_kv(const float *qkv, int T, int NH, int HD, int p0, const float *cos_t, const float *sin_t,
                              float *q, uint16_t *k_hi, uint16_t *k_lo, uint16_t *v_hi, uint16_t *v_lo, int kv_max,
                              cudaStream_t st) {
    if ((HD / 2) % 4 == 0 && (long long)3 * NH * (HD / 8) * T < (1LL << 31)) {
        const unsigned n4 = 3u * NH * (HD / 8) * (unsigned)T;
        pd_rope_kv4_kernel<<<(n4 + 255) / 256, 256, 0, st>>>(qkv, T, NH, HD, p0, cos_t, sin_t, q, k_hi, k_lo, v_hi,
                                                              v_lo, kv_max);
        return cudaGetLastError();
    }
    const long long n = 3LL * NH * (HD / 2) * T;
    pd_rope_kv_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(qkv, T, NH, HD, p0, cos_t, sin_t, q, k_hi, k_lo,
                                                                  v_hi, v_lo, kv_max);
    return cudaGetLastError();
}

cudaError_t launch_pd_add(float *x, const float *y, size_t n, cudaStream_t st) {
    const size_t n4 = n / 4;
    pd_add_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(x, y, n4);
    return cudaGetLastError();
}

cudaError_t launch_pd_finish(const uint16_t *E, int H, const int *tok, float *x_out, int *pos, int p_next,
                             int *tok_log, int *hist, int *hist_len, int hist_cap, cudaStream_t st) {
    pd_finish_kernel<<<1, 256, 0, st>>>(E, H, tok, x_out, pos, p_next, tok_log, hist, hist_len, hist_cap);
    return cudaGetLastError();
}

}  // namespace ds

namespace ds {

// ---------------------------------------------------------------------------
// Prefill attention (ds_causal_attention_heads_aligned, ds_kernels.c:
// 2061-2114): query t attends keys 0 .. p0 + t with the decode rule (the
// sequential softmax with fast exp). Unrolled, key j contributes
// w_j v_j with w_j = a_j * prod_{t > j} c_t (a_j = fexp(s_j - m) or 1 at a new
// maximum, c_t = fexp(m - s_t) at a new maximum t, else 1, m the running
// maximum before the key). A CTA takes PA_QB queries of one head and walks
// the keys in blocks of PA_KC, in order, keeping per query the running
// maximum m, the running sum L and the output O (registers); per block:
//   1. the block's K rows, widened to F32, are staged transposed (Kt[d][j])
//      next to the transposed queries (Qt[d][q]), and the scores come from
//      8 x 8 register tiles with float4 loads along both tile edges;
//      they are stored key-major (St[j][q]);
//   2. two threads per query scan the block's scores against m: a_j and
//      c_j exactly as the sequential loop evaluates them, the block's
//      correction product C and local weights w_j = a_j * prod_{t>j in
//      block} c_t;
//   3. the V rows are staged (V[j][d]) over the K tile and
//      O = O * C + sum_j w_j v_j, L = L * C + sum_j w_j (8 x 8 tiles).
// That is the sequential recurrence applied a block at a time: the same
// factors, only the order of the F32 products differs. Query blocks are
// launched longest first.
// ---------------------------------------------------------------------------
constexpr int PA_QB = 128;   // queries per CTA
constexpr int PA_KC = 128;   // keys per block
constexpr int PA_HD = 128;
constexpr int PA_LD = 132;   // padded F32 row of every shared tile
constexpr int PA_TILE = PA_HD * PA_LD;  // floats per 128-row tile
constexpr int PA_SMEM = (3 * PA_TILE + 9 * PA_QB) * 4;

struct PrefillAttnArgs {
    const float *q;  // [T x q_stride], head h at column h*128
    const uint16_t *k_hi, *k_lo, *v_hi, *v_lo;  // layer planes [head][kv_max][128]
    int kv_max, p0, T, lo_start, q_stride;
    float scale;
    float *out;  // [T x q_stride]
};

// Rows c0 .. c0+rows-1 of a plane pair widened to F32: row-major buf[j][d]
// (transposed = false) or buf[d][j] (transposed = true).
// Transposed: consecutive threads take consecutive rows (conflict-free
// column writes); row-major: consecutive threads take one row's 16-byte
// pieces (coalesced reads, conflict-free float4 writes).
template <bool TRANSPOSED>
__device__ __forceinline__ void pa_stage(float *buf, const uint16_t *hi, const uint16_t *lo, int c0, int rows,
                                         int lo_start) {
    for (int u = threadIdx.x; u < rows * 16; u += blockDim.x) {
        const int r = TRANSPOSED ? u % rows : u >> 4, c = TRANSPOSED ? (u / rows) * 8 : (u & 15) * 8;
        const int j = c0 + r;
        const uint4 h = ldg_stream(hi + (size_t)j * PA_HD + c);
        uint4 l = make_uint4(0, 0, 0, 0);
        if (j >= lo_start) l = ldg_stream(lo + (size_t)j * PA_HD + c);
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
        float f[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            f[2 * i] = __fadd_rn(bf16_lo(hw[i]), bf16_lo(lw[i]));
            f[2 * i + 1] = __fadd_rn(bf16_hi(hw[i]), bf16_hi(lw[i]));
        }
        if (TRANSPOSED) {
#pragma unroll
            for (int i = 0; i < 8; i++) buf[(c + i) * PA_LD + r] = f[i];
        } else {
            float4 *d = reinterpret_cast<float4 *>(buf + r * PA_LD + c);
            d[0] = make_float4(f[0], f[1], f[2], f[3]);
            d[1] = make_float4(f[4], f[5], f[6], f[7]);
        }
    }
}

// 8 floats: p[0..3] and p[gap..gap+3].
__device__ __forceinline__ void pa_load8(const float *p, float v[8], int gap = 4) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = *reinterpret_cast<const float4 *>(p + gap);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__global__ void __launch_bounds__(256, 1) attn_prefill_kernel(PrefillAttnArgs a) {
    extern __shared__ __align__(16) float pa_smem[];
    float *qt = pa_smem;                  // [128 d][PA_LD] queries, transposed
    float *kv = qt + PA_TILE;             // [128 d][PA_LD] keys transposed, then [128 j][PA_LD] values
    float *st = kv + PA_TILE;             // [128 j][PA_LD] scores, then weights
    float *m_run = st + PA_TILE;          // [PA_QB] running maximum
    float *l_run = m_run + PA_QB;         // [PA_QB] running sum
    float *cq = l_run + PA_QB;            // [PA_QB] this block's correction product
    float *hm = cq + PA_QB;               // [2][PA_QB] half-block maxima
    float *hp = hm + 2 * PA_QB;           // [2][PA_QB] half-block correction products
    float *hs = hp + 2 * PA_QB;           // [2][PA_QB] half-block weight sums
    const int h = blockIdx.x;
    const int qb0 = (gridDim.y - 1 - blockIdx.y) * PA_QB;  // longest query blocks first
    const int tid = threadIdx.x;
    const int nq = min(PA_QB, a.T - qb0);
    const int n_end = a.p0 + qb0 + nq;  // keys of the block's last query
    const size_t hoff = (size_t)h * a.kv_max * PA_HD;
    const uint16_t *khi = a.k_hi + hoff, *klo = a.k_lo + hoff, *vhi = a.v_hi + hoff, *vlo = a.v_lo + hoff;
    for (int u = tid; u < PA_QB * PA_HD; u += 256) {
        const int i = u / PA_HD, d = u - i * PA_HD;
        qt[d * PA_LD + i] = i < nq ? a.q[(size_t)(qb0 + i) * a.q_stride + h * PA_HD + d] : 0.f;
    }
    if (tid < PA_QB) {
        m_run[tid] = -1e30f;  // the sequential loop's initial maximum
        l_run[tid] = 0.f;
    }
    // 8 x 8 tiles: queries 8tq .. 8tq+7; keys (phase 1) or dims (phase 3)
    // 4tk .. 4tk+3 and 64+4tk .. 64+4tk+3, so a warp's float4 loads are contiguous
    const int tq = tid >> 4, tk = tid & 15;
    auto col = [&](int j) { return j < 4 ? 4 * tk + j : 60 + 4 * tk + j; };
    const int sq = tid & 127, half = tid >> 7;  // scan: query sq, keys 64*half .. +63
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int d = 0; d < 8; d++) acc[i][d] = 0.f;
    for (int c0 = 0; c0 < n_end; c0 += PA_KC) {
        const int rows = min(PA_KC, n_end - c0);
        __syncthreads();
        pa_stage<true>(kv, khi, klo, c0, rows, a.lo_start);
        __syncthreads();
        // 1. scores S[q][j] = q . k_j * scale, stored St[j][q]
        {
            float s[8][8];
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) s[i][j] = 0.f;
#pragma unroll 2
            for (int d = 0; d < PA_HD; d++) {
                float qv[8], kv8[8];
                pa_load8(qt + d * PA_LD + 8 * tq, qv);
                pa_load8(kv + d * PA_LD + 4 * tk, kv8, 64);
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) s[i][j] = __fmaf_rn(qv[i], kv8[j], s[i][j]);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 *o = reinterpret_cast<float4 *>(st + col(j) * PA_LD + 8 * tq);
                o[0] = make_float4(__fmul_rn(s[0][j], a.scale), __fmul_rn(s[1][j], a.scale),
                                   __fmul_rn(s[2][j], a.scale), __fmul_rn(s[3][j], a.scale));
                o[1] = make_float4(__fmul_rn(s[4][j], a.scale), __fmul_rn(s[5][j], a.scale),
                                   __fmul_rn(s[6][j], a.scale), __fmul_rn(s[7][j], a.scale));
            }
        }
        __syncthreads();
        // the V rows replace the K tile (the scores are all in St)
        pa_stage<false>(kv, vhi, vlo, c0, rows, a.lo_start);
        // 2. the rule's factors: two threads per query, 64 keys each
        const int n_q = a.p0 + qb0 + sq + 1;            // keys of query sq
        const int kb0 = 64 * half;                      // this thread's first key of the block
        const int kend = min(min(64, rows - kb0), n_q - c0 - kb0);  // its valid keys (may be <= 0)
        float lm = -1e30f;
        for (int k = 0; k < kend; k++) lm = fmaxf(lm, st[(kb0 + k) * PA_LD + sq]);
        hm[half * PA_QB + sq] = lm;
        __syncthreads();
        const float m_in = m_run[sq];
        float m = half == 0 ? m_in : fmaxf(m_in, hm[sq]);
        float lp = 1.f;
        for (int k = 0; k < 64; k++) {
            float *p = st + (kb0 + k) * PA_LD + sq;
            if (k >= kend) {
                *p = 0.f;  // beyond the query's keys: a = 0, c = 1
                continue;
            }
            const float s = *p;
            if (s > m) {
                const float cj = fast_expf(__fsub_rn(m, s));
                *p = cj == 0.f ? -0.f : -cj;  // sign set: a new maximum (a_j = 1)
                lp = __fmul_rn(lp, cj);
                m = s;
            } else {
                *p = fast_expf(__fsub_rn(s, m));
            }
        }
        hp[half * PA_QB + sq] = lp;
        __syncthreads();
        float P = half == 0 ? hp[PA_QB + sq] : 1.f;  // corrections of the later half
        float lsum = 0.f;
        for (int k = 63; k >= 0; k--) {
            float *p = st + (kb0 + k) * PA_LD + sq;
            const float v = *p;
            const bool nm = signbit(v);
            const float w = nm ? P : __fmul_rn(v, P);
            if (nm) P = __fmul_rn(P, -v);
            *p = w;
            lsum = __fadd_rn(lsum, w);
        }
        hs[half * PA_QB + sq] = lsum;
        __syncthreads();
        if (half == 0) {
            const float C = __fmul_rn(hp[sq], hp[PA_QB + sq]);
            cq[sq] = C;
            l_run[sq] = __fadd_rn(__fmul_rn(l_run[sq], C), __fadd_rn(hs[sq], hs[PA_QB + sq]));
            m_run[sq] = fmaxf(m_in, fmaxf(hm[sq], hm[PA_QB + sq]));
        }
        __syncthreads();
        // 3. O = O * C + W V over this block's keys (queries 8tq.., dims col(0..7))
        {
            float C8[8];
            pa_load8(cq + 8 * tq, C8);
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int d = 0; d < 8; d++) acc[i][d] = __fmul_rn(acc[i][d], C8[i]);
#pragma unroll 2
            for (int j = 0; j < rows; j++) {
                float w8[8], v8[8];
                pa_load8(st + j * PA_LD + 8 * tq, w8);
                pa_load8(kv + j * PA_LD + 4 * tk, v8, 64);
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int d = 0; d < 8; d++) acc[i][d] = __fmaf_rn(w8[i], v8[d], acc[i][d]);
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int qi = 8 * tq + i;
        if (qi >= nq) continue;
        const float L = l_run[qi];
        const float inv = __fdiv_rn(1.0f, L);
        float o[8];
#pragma unroll
        for (int d = 0; d < 8; d++) o[d] = L > 0.f ? __fmul_rn(acc[i][d], inv) : acc[i][d];
        float *dst = a.out + (size_t)(qb0 + qi) * a.q_stride + h * PA_HD + 4 * tk;
        *reinterpret_cast<float4 *>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<float4 *>(dst + 64) = make_float4(o[4], o[5], o[6], o[7]);
    }
}

// The same attention with 32 queries per CTA (4 x 2 score tiles, 8 threads
// per query in the scan), for prefills short enough that 128-query blocks
// would leave SMs idle.
constexpr int PS_QB = 32;     // queries per CTA
constexpr int PS_KC = 64;     // keys per block
constexpr int PS_LD = 132;    // padded F32 row
constexpr int PS_HD = 128;
constexpr int PS_SLD = 68;    // score row stride
constexpr int PS_SMEM = (2 * PS_KC * PS_LD + PS_QB * PS_LD + PS_QB * PS_SLD + 3 * PS_QB) * 4;



__global__ void __launch_bounds__(256, 2) attn_prefill_small_kernel(PrefillAttnArgs a) {
    extern __shared__ __align__(16) float ps_smem[];
    float *kb = ps_smem;                  // [PS_KC][PS_LD]
    float *vb = kb + PS_KC * PS_LD;       // [PS_KC][PS_LD]
    float *qs = vb + PS_KC * PS_LD;       // [PS_QB][PS_LD]
    float *sw = qs + PS_QB * PS_LD;       // [PS_QB][PS_SLD] scores, then weights
    float *m_run = sw + PS_QB * PS_SLD;   // [PS_QB] running maximum
    float *l_run = m_run + PS_QB;         // [PS_QB] running sum
    float *cq = l_run + PS_QB;            // [PS_QB] this block's correction product
    const int h = blockIdx.x, qb0 = blockIdx.y * PS_QB, tid = threadIdx.x;
    const int nq = min(PS_QB, a.T - qb0);
    const int n_end = a.p0 + qb0 + nq;  // keys of the block's last query
    const size_t hoff = (size_t)h * a.kv_max * PS_HD;
    const uint16_t *khi = a.k_hi + hoff, *klo = a.k_lo + hoff, *vhi = a.v_hi + hoff, *vlo = a.v_lo + hoff;
    for (int u = tid; u < PS_QB * PS_HD; u += 256) {
        const int i = u / PS_HD, d = u - i * PS_HD;
        qs[i * PS_LD + d] = i < nq ? a.q[(size_t)(qb0 + i) * a.q_stride + h * PS_HD + d] : 0.f;
    }
    if (tid < PS_QB) {
        m_run[tid] = -1e30f;  // the sequential loop's initial maximum
        l_run[tid] = 0.f;
    }
    // score tile: 2 queries x 4 keys (key kg + 16 r); scan: 8 keys of one
    // query; output tile: 4 queries x 4 dims
    const int kg = tid & 15, qp = tid >> 4;
    const int sq = tid >> 3, sg = tid & 7;
    const int dq = tid & 31, qg = tid >> 5;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int d = 0; d < 4; d++) acc[i][d] = 0.f;
    for (int c0 = 0; c0 < n_end; c0 += PS_KC) {
        const int rows = min(PS_KC, n_end - c0);
        __syncthreads();
        pa_stage<false>(kb, khi, klo, c0, rows, a.lo_start);
        pa_stage<false>(vb, vhi, vlo, c0, rows, a.lo_start);
        __syncthreads();
        // 1. scores
        {
            float s[2][4];
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int r = 0; r < 4; r++) s[i][r] = 0.f;
            const float4 *q0 = reinterpret_cast<const float4 *>(qs + (2 * qp) * PS_LD);
            const float4 *q1 = reinterpret_cast<const float4 *>(qs + (2 * qp + 1) * PS_LD);
#pragma unroll 4
            for (int c = 0; c < PS_HD / 4; c++) {
                const float4 a0 = q0[c], a1 = q1[c];
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    const float4 k4 = reinterpret_cast<const float4 *>(kb + (kg + 16 * r) * PS_LD)[c];
                    s[0][r] = __fmaf_rn(a0.x, k4.x, s[0][r]);
                    s[0][r] = __fmaf_rn(a0.y, k4.y, s[0][r]);
                    s[0][r] = __fmaf_rn(a0.z, k4.z, s[0][r]);
                    s[0][r] = __fmaf_rn(a0.w, k4.w, s[0][r]);
                    s[1][r] = __fmaf_rn(a1.x, k4.x, s[1][r]);
                    s[1][r] = __fmaf_rn(a1.y, k4.y, s[1][r]);
                    s[1][r] = __fmaf_rn(a1.z, k4.z, s[1][r]);
                    s[1][r] = __fmaf_rn(a1.w, k4.w, s[1][r]);
                }
            }
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int r = 0; r < 4; r++) sw[(2 * qp + i) * PS_SLD + kg + 16 * r] = __fmul_rn(s[i][r], a.scale);
        }
        __syncthreads();
        // 2. the rule's factors for this block, 8 threads per query
        {
            const int n_q = a.p0 + qb0 + sq + 1;  // keys of query sq
            float *row = sw + sq * PS_SLD;
            const float m_in = m_run[sq];
            const int j0 = sg * 8;
            float sv[8];
            float lm = -1e30f;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const bool ok = c0 + j0 + k < n_q && j0 + k < rows;
                sv[k] = ok ? row[j0 + k] : -INFINITY;
                if (ok) lm = fmaxf(lm, sv[k]);
            }
            // exclusive prefix maximum over the 8 lanes of this query
            float inc = lm;
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                const float y = __shfl_up_sync(DS_FULL, inc, o, 8);
                if (sg >= o) inc = fmaxf(inc, y);
            }
            float m = __shfl_up_sync(DS_FULL, inc, 1, 8);
            m = fmaxf(m_in, sg == 0 ? -1e30f : m);
            float av[8], cv[8];
            float lp = 1.f;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                if (sv[k] == -INFINITY) {  // beyond the query's keys
                    av[k] = 0.f;
                    cv[k] = 1.f;
                } else if (sv[k] > m) {
                    cv[k] = fast_expf(__fsub_rn(m, sv[k]));
                    av[k] = 1.f;
                    m = sv[k];
                } else {
                    cv[k] = 1.f;
                    av[k] = fast_expf(__fsub_rn(sv[k], m));
                }
                lp = __fmul_rn(lp, cv[k]);
            }
            // exclusive suffix product over the 8 lanes, then the weights
            float sinc = lp;
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                const float y = __shfl_down_sync(DS_FULL, sinc, o, 8);
                if (sg + o < 8) sinc = __fmul_rn(sinc, y);
            }
            float P = __shfl_down_sync(DS_FULL, sinc, 1, 8);
            if (sg == 7) P = 1.f;
            float lsum = 0.f;
#pragma unroll
            for (int k = 7; k >= 0; k--) {
                const float w = __fmul_rn(av[k], P);
                P = __fmul_rn(P, cv[k]);
                row[j0 + k] = w;
                lsum = __fadd_rn(lsum, w);
            }
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) lsum = __fadd_rn(lsum, __shfl_xor_sync(DS_FULL, lsum, o, 8));
            const float C = __shfl_sync(DS_FULL, sinc, 0, 8);  // product over the whole block
            float mb = lm;
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(DS_FULL, mb, o, 8));
            __syncwarp();
            if (sg == 0) {
                cq[sq] = C;
                l_run[sq] = __fadd_rn(__fmul_rn(l_run[sq], C), lsum);
                m_run[sq] = fmaxf(m_in, mb);
            }
        }
        __syncthreads();
        // 3. O = O * C + W V
        {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float C = cq[4 * qg + i];
#pragma unroll
                for (int d = 0; d < 4; d++) acc[i][d] = __fmul_rn(acc[i][d], C);
            }
            for (int j = 0; j < rows; j++) {
                const float4 v4 = reinterpret_cast<const float4 *>(vb + j * PS_LD)[dq];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float w = sw[(4 * qg + i) * PS_SLD + j];
                    acc[i][0] = __fmaf_rn(w, v4.x, acc[i][0]);
                    acc[i][1] = __fmaf_rn(w, v4.y, acc[i][1]);
                    acc[i][2] = __fmaf_rn(w, v4.z, acc[i][2]);
                    acc[i][3] = __fmaf_rn(w, v4.w, acc[i][3]);
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int qi = 4 * qg + i;
        if (qi >= nq) continue;
        const float L = l_run[qi];
        const float inv = __fdiv_rn(1.0f, L);
        float4 o;
        o.x = L > 0.f ? __fmul_rn(acc[i][0], inv) : acc[i][0];
        o.y = L > 0.f ? __fmul_rn(acc[i][1], inv) : acc[i][1];
        o.z = L > 0.f ? __fmul_rn(acc[i][2], inv) : acc[i][2];
        o.w = L > 0.f ? __fmul_rn(acc[i][3], inv) : acc[i][3];
        *reinterpret_cast<float4 *>(a.out + (size_t)(qb0 + qi) * a.q_stride + h * PS_HD + 4 * dq) = o;
    }
}

cudaError_t launch_attn_prefill(const float *q, const uint16_t *k_hi, const uint16_t *k_lo, const uint16_t *v_hi,
                                const uint16_t *v_lo, int kv_max, int n_heads, int p0, int T, int lo_start,
                                int q_stride, float scale, float *out, cudaStream_t st) {
    PrefillAttnArgs a{q, k_hi, k_lo, v_hi, v_lo, kv_max, p0, T, lo_start, q_stride, scale, out};
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PA_SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             PS_SMEM);
        if (e != cudaSuccess) return e;
    }
    if (n_heads * ((T + PA_QB - 1) / PA_QB) < sms)
        attn_prefill_small_kernel<<<dim3(n_heads, (T + PS_QB - 1) / PS_QB), 256, PS_SMEM, st>>>(a);
    else
        attn_prefill_kernel<<<dim3(n_heads, (T + PA_QB - 1) / PA_QB), 256, PA_SMEM, st>>>(a);
    return cudaGetLastError();
}

}  // namespace ds
