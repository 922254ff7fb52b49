// prefill_full.cu — the per-token kernels of the whole-decoder prefill
// (ds_decoder_prefill, ds_moe_decoder.c:480-905); the GEMMs run on the
// tensor-core prefill kernel (prefill.cu), the attention on the exact
// decode attention with one query per token (kernels_decode.cu), the MoE
// block on the MoE prefill; decoder.cu strings them together.
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

// Per-query positions p0 + t and lo-plane starts for the attention.
__global__ void pd_positions_kernel(int *pos, int *lo_starts, int T, int p0, int lo_start) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    pos[t] = p0 + t;
    lo_starts[t] = lo_start;
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

cudaError_t launch_pd_positions(int *pos, int *lo_starts, int T, int p0, int lo_start, cudaStream_t st) {
    pd_positions_kernel<<<(T + 255) / 256, 256, 0, st>>>(pos, lo_starts, T, p0, lo_start);
    return cudaGetLastError();
}

cudaError_t launch_pd_finish(const uint16_t *E, int H, const int *tok, float *x_out, int *pos, int p_next,
                             int *tok_log, int *hist, int *hist_len, int hist_cap, cudaStream_t st) {
    pd_finish_kernel<<<1, 256, 0, st>>>(E, H, tok, x_out, pos, p_next, tok_log, hist, hist_len, hist_cap);
    return cudaGetLastError();
}

}  // namespace ds
