// ep.cu — device-side bookkeeping of expert-parallel prefill: which split
// rows go to which rank (dispatch), which (row, expert) pairs a rank received,
// and where each returned expert output lands (the combine index).
//
// Ranks own contiguous expert blocks of experts_per_rank experts. A token is
// sent once to every rank owning one of its top-k experts, in the order
// (destination rank ascending, token ascending); with the row go the k expert
// ids served there (-1 for the others) and, in the last meta slot, the
// offset of the row's first pair within its destination's pairs. Expert outputs come back one row per
// (token, k) pair in the order (rank ascending, token ascending, k
// ascending); inv[s*K + k] is that pair's row in the returned stream, so the
// combine reads them without a scatter.
//
// These are planning kernels over a few thousand tokens: the dispatch plan
// gives each CTA 256 tokens (each CTA reads all top-k ids for its offsets),
// the pair list one thread per received row.
#include "ctx.h"

namespace ds {

constexpr int EP_META = 8;  // int32 slots after the two BF16 planes of a payload row

// Exclusive block scan of NV ints per thread at once (one pair of
// barriers for all of them); tot[v] gets the block total of value v.
template <int NV>
__device__ __forceinline__ void ep_scan_multi(int (&v)[NV], int (&excl)[NV], int (&tot)[NV]) {
    __shared__ int wt[NV][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    int inc[NV];
#pragma unroll
    for (int q = 0; q < NV; q++) {
        int x = v[q];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        inc[q] = x;
        if (lane == 31) wt[q][warp] = x;
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int q = 0; q < NV; q++) {
            int t = lane < nwarp ? wt[q][lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, t, o);
                if (lane >= o) t += y;
            }
            wt[q][lane] = t;  // inclusive over warps
        }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < NV; q++) {
        excl[q] = (warp ? wt[q][warp - 1] : 0) + inc[q] - v[q];
        tot[q] = wt[q][nwarp - 1];
    }
}

// Rows (a 0/1 flag) and pairs token s sends to each of the eight possible
// destinations: v[q] and v[8 + q].
__device__ __forceinline__ void ep_token_counts(const int *__restrict__ idx, int s, int K, int e_per, int (&v)[16]) {
    unsigned mask = 0;
#pragma unroll
    for (int q = 0; q < 16; q++) v[q] = 0;
    for (int k = 0; k < K; k++) {
        const int g = idx[s * K + k] / e_per;
        mask |= 1u << g;
#pragma unroll
        for (int q = 0; q < 8; q++) v[8 + q] += g == q;
    }
#pragma unroll
    for (int q = 0; q < 8; q++) v[q] = (mask >> q) & 1u;
}

constexpr int EP_PLAN_TOK = 256;  // tokens (threads) per CTA of the dispatch plan

// Plans the dispatch of n tokens and writes each sent row's meta into the
// payload (row pitch `ld` int16 elements; the meta sits at int16 offset
// 2*H). counts[0..G) = rows per destination, counts[G..2G) = pairs per
// destination. send_tok[i] = token of send row i. Each CTA owns 256 tokens
// (one per thread): it first reads every token's top-k ids (a few tens of
// KB, from L2) for the per-destination totals and the counts of the tokens
// before its own, then one block scan places its rows.
__global__ void __launch_bounds__(EP_PLAN_TOK) ep_dispatch_plan_kernel(int n, int K, int G, int e_per,
                                                                       const int *__restrict__ idx, int H, int ld,
                                                                       uint16_t *payload, int *send_tok, int *counts,
                                                                       int *inv) {
    __shared__ int s_before[16], s_total[16];
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < 16) {
        s_before[tid] = 0;
        s_total[tid] = 0;
    }
    __syncthreads();
    const int blk0 = blockIdx.x * EP_PLAN_TOK;
    int before[16], total[16];
#pragma unroll
    for (int q = 0; q < 16; q++) before[q] = total[q] = 0;
    for (int s = tid; s < n; s += EP_PLAN_TOK) {
        int v[16];
        ep_token_counts(idx, s, K, e_per, v);
        const bool b = s < blk0;
#pragma unroll
        for (int q = 0; q < 16; q++) {
            total[q] += v[q];
            before[q] += b ? v[q] : 0;
        }
    }
#pragma unroll
    for (int q = 0; q < 16; q++) {
        int t = total[q], b = before[q];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            t += __shfl_xor_sync(0xffffffffu, t, o);
            b += __shfl_xor_sync(0xffffffffu, b, o);
        }
        if (lane == 0) {
            if (t) atomicAdd(&s_total[q], t);
            if (b) atomicAdd(&s_before[q], b);
        }
    }
    __syncthreads();
    const int s = blk0 + tid;
    int v[16], ex[16], bt[16];
    if (s < n) ep_token_counts(idx, s, K, e_per, v);
    else
#pragma unroll
        for (int q = 0; q < 16; q++) v[q] = 0;
    ep_scan_multi<16>(v, ex, bt);
    if (s < n) {
        int row_base = 0, pair_base = 0;
#pragma unroll
        for (int q = 0; q < 8; q++) {
            if (q < G && v[q]) {
                const int row = row_base + s_before[q] + ex[q];
                const int p_in = s_before[8 + q] + ex[8 + q];  // within the destination's pairs
                send_tok[row] = s;
                int *meta = reinterpret_cast<int *>(payload + (size_t)row * ld + 2 * H);
                int j = 0;
                for (int k = 0; k < K; k++) {
                    const int e = idx[s * K + k];
                    const bool mine = e / e_per == q;
                    meta[k] = mine ? e : -1;
                    if (mine) inv[s * K + k] = pair_base + p_in + j++;
                }
                for (int k = K; k < EP_META - 1; k++) meta[k] = -1;
                // the row's first pair within its destination's pairs: the
                // receiver places its pairs without a scan
                meta[EP_META - 1] = p_in;
            }
            row_base += q < G ? s_total[q] : 0;
            pair_base += q < G ? s_total[8 + q] : 0;
        }
    }
    if (blockIdx.x == 0 && tid < G) {
        counts[tid] = s_total[tid];
        counts[G + tid] = s_total[8 + tid];
    }
}

// Copies each send row's two BF16 planes into the payload (one warp per row).
__global__ void __launch_bounds__(256) ep_pack_rows_kernel(int rows, int H, int ld, const int *__restrict__ send_tok,
                                                           const uint16_t *__restrict__ xn_hi,
                                                           const uint16_t *__restrict__ xn_lo, uint16_t *payload,
                                                           const int *counts, int G) {
    const int lane = threadIdx.x & 31;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int total = 0;
    for (int g = 0; g < G; g++) total += counts[g];
    if (i >= rows || i >= total) return;
    const int s = send_tok[i];
    const uint4 *sh = reinterpret_cast<const uint4 *>(xn_hi + (size_t)s * H);
    const uint4 *sl = reinterpret_cast<const uint4 *>(xn_lo + (size_t)s * H);
    uint4 *d = reinterpret_cast<uint4 *>(payload + (size_t)i * ld);
    for (int j = lane; j < H / 8; j += 32) {
        d[j] = sh[j];
        d[H / 8 + j] = sl[j];
    }
}

struct EpCounts {
    int c[8];
};

// Compact (row, expert) pairs of R received payload rows, row-major; out[g]
// = pairs whose row came from rank g (rows arrive grouped by source rank,
// recv.c[g] rows each), out[G] = total. One thread per row over many CTAs:
// each row carries the offset of its first pair within its source's section
// (meta slot EP_META - 1, written by the dispatch), and a section's pair
// count is its last row's offset plus that row's pairs.
__device__ __forceinline__ int ep_row_pairs(const int *meta, int K) {
    int c = 0;
    for (int k = 0; k < K; k++) c += meta[k] >= 0;
    return c;
}

__global__ void __launch_bounds__(256) ep_pairs_kernel(int R, int K, int G, EpCounts recv,
                                                       const uint16_t *__restrict__ payload, int H, int ld,
                                                       int *pair_row, int *pair_expert, int *out) {
    __shared__ int base[9];
    if (threadIdx.x == 0) {
        int b = 0, r_end = 0;
        for (int g = 0; g < G; g++) {
            base[g] = b;
            r_end += recv.c[g];
            if (recv.c[g] > 0) {
                const int *m = reinterpret_cast<const int *>(payload + (size_t)(r_end - 1) * ld + 2 * H);
                b += m[EP_META - 1] + ep_row_pairs(m, K);
            }
        }
        base[G] = b;
        if (blockIdx.x == 0) {
            for (int g = 0; g < G; g++) out[g] = base[g + 1] - base[g];
            out[G] = b;
        }
    }
    __syncthreads();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    int g = 0, acc = recv.c[0];
    while (g + 1 < G && r >= acc) acc += recv.c[++g];
    const int *meta = reinterpret_cast<const int *>(payload + (size_t)r * ld + 2 * H);
    int j = base[g] + meta[EP_META - 1];
    for (int k = 0; k < K; k++) {
        const int e = meta[k];
        if (e >= 0) {
            pair_row[j] = r;
            pair_expert[j] = e;
            j++;
        }
    }
}

}  // namespace ds

using namespace ds;

extern "C" int ds_cuda_ep_dispatch_dev(ds_cuda_ctx_t *c, int n_tokens, int top_k, int n_ranks,
                                       int experts_per_rank, const int *d_top_idx, const uint16_t *d_xn_hi,
                                       const uint16_t *d_xn_lo, int hidden, uint16_t *d_payload, int *d_send_tok,
                                       int *d_counts, int *d_inv, void *stream) {
    if (!c || !c->ok || n_tokens < 0 || top_k <= 0 || top_k > EP_META - 1 || n_ranks <= 0 || n_ranks > 8 ||
        experts_per_rank <= 0 || hidden % 8 ||
        (n_tokens > 0 && (!d_top_idx || !d_xn_hi || !d_xn_lo || !d_payload || !d_send_tok || !d_inv)) || !d_counts)
        return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    const int ld = 2 * hidden + 2 * EP_META;
    ep_dispatch_plan_kernel<<<n_tokens > 0 ? (n_tokens + EP_PLAN_TOK - 1) / EP_PLAN_TOK : 1, EP_PLAN_TOK, 0, st>>>(
        n_tokens, top_k, n_ranks, experts_per_rank, d_top_idx, hidden, ld, d_payload, d_send_tok, d_counts, d_inv);
    // rows <= n * min(top_k, n_ranks)
    const int max_rows = n_tokens * (top_k < n_ranks ? top_k : n_ranks);
    if (max_rows > 0)
        ep_pack_rows_kernel<<<(max_rows + 7) / 8, 256, 0, st>>>(max_rows, hidden, ld, d_send_tok, d_xn_hi, d_xn_lo,
                                                               d_payload, d_counts, n_ranks);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DS_CUDA_OK : ctx_cuda(c, e, "ep_dispatch");
}

extern "C" int ds_cuda_ep_pairs_dev(ds_cuda_ctx_t *c, int n_rows, int top_k, int n_ranks, const int *recv_counts,
                                    const uint16_t *d_payload, int hidden, int *d_pair_row, int *d_pair_expert,
                                    int *d_counts, void *stream) {
    if (!c || !c->ok || n_rows < 0 || top_k <= 0 || top_k > EP_META - 1 || n_ranks <= 0 || n_ranks > 8 ||
        !recv_counts || !d_counts || (n_rows > 0 && (!d_payload || !d_pair_row || !d_pair_expert)))
        return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    EpCounts rc = {};
    int sum = 0;
    for (int g = 0; g < n_ranks; g++) {
        rc.c[g] = recv_counts[g];
        sum += recv_counts[g];
    }
    if (sum != n_rows) return ctx_fail(c, DS_CUDA_EINVAL, "ep_pairs: receive counts do not add up to n_rows");
    ep_pairs_kernel<<<n_rows > 0 ? (n_rows + 255) / 256 : 1, 256, 0, st>>>(
        n_rows, top_k, n_ranks, rc, d_payload, hidden, 2 * hidden + 2 * EP_META, d_pair_row, d_pair_expert, d_counts);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DS_CUDA_OK : ctx_cuda(c, e, "ep_pairs");
}
