// select.cu — LM-head token selection with the sampling settings of
// ds_decoder_forward (ds_moe_decoder.c:1021-1263): repetition penalty,
// n-gram blocking and temperature sampling, on the device, as kernels of
// the batch-1 decode step.
//
//   fast path (temperature <= 0, :1033-1099), after the streaming argmax:
//     select_dots_kernel   one warp per history entry (and one for the
//                          argmax winner): the row dots W[t] . x_final
//     select_fast_kernel   one CTA: the winner's value penalised once if it
//                          is in the history; every history token other than
//                          the winner penalised and taken on a strict '>'
//                          (the earliest occurrence of the maximum); then
//                          whether the winner completes a seen n-gram, which
//                          sends the step to the full path
//   full path (:1101-1263), skipped by an early exit unless needed:
//     select_logits_kernel every logit (HBM-bound matvec over the vocab)
//     select_full_kernel   one CTA: the penalty once per history
//                          OCCURRENCE, banned tokens set to -1e30, strict
//                          '>' argmax; temperature > 0: softmax with expf
//                          and a double sum, sampled with the next caller-
//                          supplied uniform by a cumulative F32 sum
// The fast path re-scores history tokens only, as the reference does: a
// penalised winner keeps the token when a token outside the history would
// now score higher.
#include "kernels_decode.cuh"

namespace ds {

__device__ __forceinline__ float sel_penalise(float v, float rp) {
    return v > 0.f ? __fdiv_rn(v, rp) : __fmul_rn(v, rp);
}

// W[row] . x for one warp (hidden a multiple of 256).
__device__ __forceinline__ float sel_row_dot(const uint16_t *W, const float *x, int H, int row, int lane) {
    const uint16_t *w = W + (size_t)row * H;
    float s = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
        const uint4 u = ldg_stream(w + c);
        const float4 x0 = *reinterpret_cast<const float4 *>(x + c);
        const float4 x1 = *reinterpret_cast<const float4 *>(x + c + 4);
        s = __fmaf_rn(bf16_lo(u.x), x0.x, s);
        s = __fmaf_rn(bf16_hi(u.x), x0.y, s);
        s = __fmaf_rn(bf16_lo(u.y), x0.z, s);
        s = __fmaf_rn(bf16_hi(u.y), x0.w, s);
        s = __fmaf_rn(bf16_lo(u.z), x1.x, s);
        s = __fmaf_rn(bf16_hi(u.z), x1.y, s);
        s = __fmaf_rn(bf16_lo(u.w), x1.z, s);
        s = __fmaf_rn(bf16_hi(u.w), x1.w, s);
    }
    return warp_sum(s);
}

// The arguments of stream blockIdx.y (the same pointers for one stream).
__device__ __forceinline__ SelectArgs sel_stream(const SelectArgs &a0) {
    SelectArgs a = a0;
    const int s = blockIdx.y;
    if (s) {
        a.x += (size_t)s * a.x_ld;
        a.hist += (size_t)s * a.cap;
        a.hist_len += s;
        a.hval += (size_t)s * a.cap;
        a.bval += s;
        a.logits += (size_t)s * a.V;
        a.tok += s;
        a.val += s;
        a.full += s;
        if (a.unif) a.unif += (size_t)s * a.unif_ld;
        if (a.unif_pos) a.unif_pos += s;
    }
    return a;
}

// Warp i < len: hval[i] = W[hist[i]] . x (0 for an out-of-range token);
// warp i == cap: bval = W[*tok] . x (the argmax winner's value recomputed,
// as the reference does with ds_bf16_dot_row).
__global__ void __launch_bounds__(256) select_dots_kernel(SelectArgs a0) {
    const SelectArgs a = sel_stream(a0);
    const int lane = threadIdx.x & 31;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int len = *a.hist_len;
    if (i == a.cap) {
        const int t = *a.tok;
        const float v = (t >= 0 && t < a.V) ? sel_row_dot(a.W, a.x, a.H, t, lane) : -1e30f;
        if (lane == 0) *a.bval = v;
        return;
    }
    if (i >= len || i >= a.cap) return;
    const int t = a.hist[i];
    const float v = (t >= 0 && t < a.V) ? sel_row_dot(a.W, a.x, a.H, t, lane) : 0.f;
    if (lane == 0) a.hval[i] = v;
}

// Block-wide arg-max of (value, -index): the largest value, the smallest
// index among equals. 1024 threads.
__device__ __forceinline__ void sel_block_argmax(float &v, int &i, float *sv, int *si) {
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(DS_FULL, v, o);
        const int oi = __shfl_xor_sync(DS_FULL, i, o);
        if (ov > v || (ov == v && oi < i)) {
            v = ov;
            i = oi;
        }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) {
        sv[w] = v;
        si[w] = i;
    }
    __syncthreads();
    if (w == 0) {
        v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
        i = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(DS_FULL, v, o);
            const int oi = __shfl_xor_sync(DS_FULL, i, o);
            if (ov > v || (ov == v && oi < i)) {
                v = ov;
                i = oi;
            }
        }
        if (lane == 0) {
            sv[0] = v;
            si[0] = i;
        }
    }
    __syncthreads();
    v = sv[0];
    i = si[0];
    __syncthreads();
}

// True when token tok would complete an n-gram of the history: some
// earlier window hist[i .. i+p-1] equals the last p tokens and is followed
// by tok (p = ngram - 1). Block-wide (every thread gets the answer).
__device__ __forceinline__ bool sel_banned(const int *hist, int len, int ngram, int tok) {
    bool hit = false;
    if (ngram > 0 && len >= ngram - 1) {
        const int p = ngram - 1;
        for (int i = threadIdx.x; i <= len - p - 1; i += blockDim.x) {
            if (hist[i + p] != tok) continue;
            bool m = true;
            for (int j = 0; j < p && m; j++) m = hist[i + j] == hist[len - p + j];
            hit = hit || m;
        }
    }
    return __syncthreads_or(hit) != 0;
}

__global__ void __launch_bounds__(1024) select_fast_kernel(SelectArgs a0) {
    const SelectArgs a = sel_stream(a0);
    __shared__ float sv[32];
    __shared__ int si[32];
    if (a.temperature > 0.f) {  // temperature sampling always takes the full path
        if (threadIdx.x == 0) *a.full = 1;
        return;
    }
    const int len = *a.hist_len;
    int best = *a.tok;
    // the recomputed row dot with a penalty; the argmax kernel's value without
    float bv = a.rp > 1.f ? *a.bval : *a.val;
    if (a.rp > 1.f && len > 0) {
        bool in = false;
        for (int i = threadIdx.x; i < len; i += blockDim.x) in = in || a.hist[i] == best;
        if (__syncthreads_or(in)) bv = sel_penalise(bv, a.rp);
        float v = -INFINITY;
        int at = 0x7fffffff;
        for (int i = threadIdx.x; i < len; i += blockDim.x) {
            const int t = a.hist[i];
            if (t < 0 || t >= a.V || t == best) continue;
            const float pv = sel_penalise(a.hval[i], a.rp);
            if (pv > v) {  // ascending i per thread: the first of equals stays
                v = pv;
                at = i;
            }
        }
        sel_block_argmax(v, at, sv, si);
        if (at != 0x7fffffff && v > bv) {
            bv = v;
            best = a.hist[at];
        }
    }
    const bool banned = sel_banned(a.hist, len, a.ngram, best);
    if (threadIdx.x == 0) {
        *a.tok = best;
        *a.val = bv;
        *a.full = banned ? 1 : 0;
    }
}

// Every logit, when the full path runs. Grid-stride over rows, one warp
// per row; every CTA returns at once when the flag is clear.
__global__ void __launch_bounds__(256) select_logits_kernel(SelectArgs a) {
    if (!*a.full) return;
    const int lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < a.V; r += nw) {
        const float v = sel_row_dot(a.W, a.x, a.H, r, lane);
        if (lane == 0) a.logits[r] = v;
    }
}

// Every logit of every stream whose full path runs, several streams at
// once: one warp per four LM-head rows keeps them in registers (each lane
// the same 8-element chunks that sel_row_dot gives it, so each logit is the
// same sum in the same order) and dots them with each flagged stream's x,
// each x load serving the four rows; the head streams from HBM once per
// step instead of once per stream.
constexpr int SEL_RW = 4;  // LM-head rows per warp

template <int CH>
__global__ void __launch_bounds__(256) select_logits_streams_kernel(SelectArgs a) {
    const int lane = threadIdx.x & 31;
    const int S = a.n_streams;
    bool any = false;
    for (int s = 0; s < S; s++) any = any || a.full[s];
    if (!any) return;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const int n_grp = (a.V + SEL_RW - 1) / SEL_RW;
    for (int grp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; grp < n_grp; grp += nw) {
        const int r0 = grp * SEL_RW;
        uint4 u[SEL_RW][CH];
#pragma unroll
        for (int q = 0; q < SEL_RW; q++) {
            const int r = min(r0 + q, a.V - 1);  // a short last group repeats the last row
            const uint16_t *w = a.W + (size_t)r * a.H;
#pragma unroll
            for (int k = 0; k < CH; k++) u[q][k] = ldg_stream(w + lane * 8 + k * 256);
        }
        for (int s = 0; s < S; s++) {
            if (!a.full[s]) continue;
            const float *x = a.x + (size_t)s * a.x_ld;
            float acc[SEL_RW];
#pragma unroll
            for (int q = 0; q < SEL_RW; q++) acc[q] = 0.f;
#pragma unroll
            for (int k = 0; k < CH; k++) {
                const int c = lane * 8 + k * 256;
                const float4 x0 = *reinterpret_cast<const float4 *>(x + c);
                const float4 x1 = *reinterpret_cast<const float4 *>(x + c + 4);
#pragma unroll
                for (int q = 0; q < SEL_RW; q++) {
                    acc[q] = __fmaf_rn(bf16_lo(u[q][k].x), x0.x, acc[q]);
                    acc[q] = __fmaf_rn(bf16_hi(u[q][k].x), x0.y, acc[q]);
                    acc[q] = __fmaf_rn(bf16_lo(u[q][k].y), x0.z, acc[q]);
                    acc[q] = __fmaf_rn(bf16_hi(u[q][k].y), x0.w, acc[q]);
                    acc[q] = __fmaf_rn(bf16_lo(u[q][k].z), x1.x, acc[q]);
                    acc[q] = __fmaf_rn(bf16_hi(u[q][k].z), x1.y, acc[q]);
                    acc[q] = __fmaf_rn(bf16_lo(u[q][k].w), x1.z, acc[q]);
                    acc[q] = __fmaf_rn(bf16_hi(u[q][k].w), x1.w, acc[q]);
                }
            }
#pragma unroll
            for (int q = 0; q < SEL_RW; q++) {
                const float v = warp_sum(acc[q]);
                if (lane == 0 && r0 + q < a.V) a.logits[(size_t)s * a.V + r0 + q] = v;
            }
        }
    }
}

__global__ void __launch_bounds__(1024) select_full_kernel(SelectArgs a0) {
    const SelectArgs a = sel_stream(a0);
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ double sd[32];
    __shared__ float sf[32];
    if (!*a.full) return;
    const int len = *a.hist_len;
    const int tid = threadIdx.x, nt = blockDim.x;
    float *lg = a.logits;
    // 1. the penalty once per history occurrence: the first occurrence of
    //    each token applies all of that token's divisions in turn
    if (a.rp > 1.f) {
        for (int i = tid; i < len; i += nt) {
            const int t = a.hist[i];
            if (t < 0 || t >= a.V) continue;
            bool first = true;
            for (int j = 0; j < i && first; j++) first = a.hist[j] != t;
            if (!first) continue;
            int k = 1;
            for (int j = i + 1; j < len; j++) k += a.hist[j] == t;
            float v = lg[t];
            for (int q = 0; q < k; q++) v = sel_penalise(v, a.rp);
            lg[t] = v;
        }
    }
    __syncthreads();
    // 2. tokens that would complete a seen n-gram
    if (a.ngram > 0 && len >= a.ngram - 1) {
        const int p = a.ngram - 1;
        for (int i = tid; i <= len - p - 1; i += nt) {
            bool m = true;
            for (int j = 0; j < p && m; j++) m = a.hist[i + j] == a.hist[len - p + j];
            const int t = a.hist[i + p];
            if (m && t >= 0 && t < a.V) lg[t] = -1e30f;
        }
    }
    __syncthreads();
    // 3. strict '>' argmax: the largest logit, the lowest index among equals
    float v = -INFINITY;
    int at = 0x7fffffff;
    for (int i = tid; i < a.V; i += nt) {
        const float x = lg[i];
        if (x > v) {
            v = x;
            at = i;
        }
    }
    sel_block_argmax(v, at, sv, si);
    int tok = at == 0x7fffffff ? 0 : at;
    const float best = v;
    // 4. temperature sampling: exponentials and their double sum in a
    //    coalesced pass; then the cumulative F32 sum over contiguous
    //    per-warp segments, each walked 32 elements at a time with a warp
    //    scan, to the first element where it reaches r
    if (a.temperature > 0.f) {
        double ds = 0.0;
        for (int i = tid; i < a.V; i += nt) {
            const float e = expf(__fdiv_rn(__fsub_rn(lg[i], best), a.temperature));
            lg[i] = e;
            ds += (double)e;
        }
        for (int o = 16; o > 0; o >>= 1) ds += __shfl_xor_sync(DS_FULL, ds, o);
        const int w = tid >> 5, lane = tid & 31, nwarp = nt >> 5;
        if (lane == 0) sd[w] = ds;
        __syncthreads();
        double tot = 0.0;
        for (int q = 0; q < nwarp; q++) tot += sd[q];
        const float inv = (float)(1.0 / tot);
        const int seg = ((a.V + nwarp - 1) / nwarp + 31) & ~31;
        const int s0 = min(a.V, w * seg), s1 = min(a.V, s0 + seg);
        float fs = 0.f;
        for (int i = s0 + lane; i < s1; i += 32) fs = __fadd_rn(fs, __fmul_rn(lg[i], inv));
        for (int o = 16; o > 0; o >>= 1) fs = __fadd_rn(fs, __shfl_xor_sync(DS_FULL, fs, o));
        if (lane == 0) sf[w] = fs;
        __syncthreads();
        float carry = 0.f;  // exclusive prefix of the segment sums, in warp order
        for (int q = 0; q < w; q++) carry = __fadd_rn(carry, sf[q]);
        const float r = a.unif[*a.unif_pos];
        int hit = 0x7fffffff;
        for (int base = s0; base < s1; base += 32) {
            const int i = base + lane;
            float x = i < s1 ? __fmul_rn(lg[i], inv) : 0.f;
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(DS_FULL, x, o);
                if (lane >= o) x = __fadd_rn(x, y);
            }
            const float cum = __fadd_rn(carry, x);
            const unsigned b = __ballot_sync(DS_FULL, i < s1 && cum >= r);
            if (b) {
                hit = base + __ffs(b) - 1;
                break;
            }
            carry = __fadd_rn(carry, __shfl_sync(DS_FULL, x, 31));
        }
        __syncthreads();
        if (lane == 0) si[w] = hit;
        __syncthreads();
        int h = 0x7fffffff;
        for (int q = 0; q < nwarp; q++) h = min(h, si[q]);
        tok = h == 0x7fffffff ? a.V - 1 : h;
        __syncthreads();
        if (tid == 0) *a.unif_pos = *a.unif_pos + 1;
    }
    if (tid == 0) {
        *a.tok = tok;
        *a.val = best;
    }
}

static int sel_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    }
    return n;
}

cudaError_t launch_select(const SelectArgs &a, cudaStream_t st) {
    const int S = a.n_streams > 1 ? a.n_streams : 1;
    if (a.H % 256 || a.H > 2048 || a.cap <= 0 || !a.hist || !a.hist_len || !a.tok || !a.val || !a.full ||
        !a.logits || (S > 1 && a.x_ld < a.H))
        return cudaErrorInvalidValue;
    SelectArgs aa = a;
    void *args[] = {&aa};
    cudaError_t e = cudaSuccess;
    if (a.temperature <= 0.f && a.rp > 1.f) {  // the history dots feed the penalty only
        const int warps = a.cap + 1;
        e = launch_ex((const void *)select_dots_kernel, dim3((warps + 7) / 8, S), 256, 0, st, false, args);
        if (e != cudaSuccess) return e;
    }
    e = launch_ex((const void *)select_fast_kernel, dim3(1, S), 1024, 0, st, false, args);
    if (e != cudaSuccess) return e;
    if (S == 1) {
        e = launch_ex((const void *)select_logits_kernel, sel_sms() * 8, 256, 0, st, false, args);
    } else {
        const void *k = nullptr;
        switch (a.H / 256) {
            case 1: k = (const void *)select_logits_streams_kernel<1>; break;
            case 2: k = (const void *)select_logits_streams_kernel<2>; break;
            case 3: k = (const void *)select_logits_streams_kernel<3>; break;
            case 4: k = (const void *)select_logits_streams_kernel<4>; break;
            case 5: k = (const void *)select_logits_streams_kernel<5>; break;
            case 6: k = (const void *)select_logits_streams_kernel<6>; break;
            case 7: k = (const void *)select_logits_streams_kernel<7>; break;
            default: k = (const void *)select_logits_streams_kernel<8>; break;
        }
        e = launch_ex(k, sel_sms() * 8, 256, 0, st, false, args);
    }
    if (e != cudaSuccess) return e;
    return launch_ex((const void *)select_full_kernel, dim3(1, S), 1024, 0, st, false, args);
}

}  // namespace ds
