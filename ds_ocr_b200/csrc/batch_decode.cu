// batch_decode.cu — greedy decode of up to 64 independent streams at once
// (config 3 at 64 streams): every decode step of ds_decoder_forward
// (ds_moe_decoder.c:911-1264) for all streams in lockstep, each stream with
// its own KV cache and position.
//
// Batch-1 decode is a chain of matvecs; with S streams every weight row
// meets S token rows, so the linear layers become tensor-core GEMMs with the
// weights as the A operand (csrc/skinny.cu): QKV, O-proj + residual, the
// router, the dense FFN, and the MoE experts grouped by expert (the S x 6
// (token, expert) pairs are counted and sorted by expert, each active
// expert's weights stream once per step against its <= 64 token rows, and
// the shared expert runs on all rows). Attention stays per stream and per
// head (attn_decode_kernel with a stream grid dimension), and the LM head is
// the tensor-core batched argmax (csrc/lmhead_tc.cu). Activations enter each
// GEMM as two BF16 planes (hi, lo), so the products are F32-class.
#include <cmath>
#include <algorithm>
#include <cstring>
#include <vector>

#include "ctx.h"
#include "kernels_decode.cuh"
#include "route.cuh"
#include "skinny.cuh"
#include "tmap.h"

using namespace ds;

cudaError_t sk_gemm_launch(int mode, const SkGemm &g, int grid, cudaStream_t st);
cudaError_t sk_split_launch(const float *x, int n, int K, int x_ld, const float *w, float eps, uint16_t *planes,
                            int lo_off, float *normed, cudaStream_t st, const float *ws, int max_split, int nsplit,
                            const float *resid, float *x_out);
cudaError_t pf_count_launch(int P, const int *pair_expert, int E, int *counts, int grid, cudaStream_t st);
cudaError_t pf_scatter_launch(int P, int H, int ld, int K, const int *pair_row, const int *pair_expert, int E,
                              const int *seg, int *cursor, const uint16_t *rows_hi, const uint16_t *rows_lo,
                              uint16_t *xg_hi, uint16_t *xg_lo, int *slot_of, int *inv, cudaStream_t st);
cudaError_t pf_combine_launch(float *x, int M, int H, int K, const int *idx, const float *wt, const float *y,
                              const int *yrow, const float *ys, cudaStream_t st);

namespace ds {

// RoPE of q and k and the KV append for every stream at its own position
// (the element math of qkv_rope_kernel), reading the QKV GEMM's split-K
// parts. One thread per (stream, matrix, head, rotary pair).
__global__ void bd_rope_kv_kernel(const float *__restrict__ ws, int max_split, int nsplit, int S, int NH, int HD,
                                  const int *pos, const float *cos_t, const float *sin_t, float *q_out,
                                  uint16_t *k_hi, uint16_t *k_lo, uint16_t *v_hi, uint16_t *v_lo, int kv_max,
                                  long long kv_stream_stride) {
    const int half = HD / 2, QD = NH * HD;
    const int per_s = 3 * NH * half;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= S * per_s) return;
    const int s = t / per_s, r = t - s * per_s;
    const int m = r / (NH * half), r2 = r - m * NH * half, h = r2 / half, d = r2 - h * half;
    const int row0 = h * HD + d;
    // the QKV GEMM's split-K parts, feature m*QD + row
    const float s0 = sk_part_sum(ws, max_split, nsplit, s, m * QD + row0);
    const float s1 = sk_part_sum(ws, max_split, nsplit, s, m * QD + row0 + half);
    const int p = pos[s];
    float o0 = s0, o1 = s1;
    if (m < 2) {
        const float *cs = cos_t + (size_t)p * HD;
        const float *sn = sin_t + (size_t)p * HD;
        o0 = __fsub_rn(__fmul_rn(s0, cs[d]), __fmul_rn(s1, sn[d]));
        o1 = __fadd_rn(__fmul_rn(s0, sn[d + half]), __fmul_rn(s1, cs[d + half]));
    }
    if (m == 0) {
        q_out[(size_t)s * QD + row0] = o0;
        q_out[(size_t)s * QD + row0 + half] = o1;
    } else {
        const size_t idx = (size_t)s * kv_stream_stride + ((size_t)h * kv_max + p) * HD + d;
        uint16_t *hi = m == 1 ? k_hi : v_hi;
        uint16_t *lo = m == 1 ? k_lo : v_lo;
        uint16_t h0, l0, h1, l1;
        split_bf16(o0, h0, l0);
        split_bf16(o1, h1, l1);
        hi[idx] = h0;
        lo[idx] = l0;
        hi[idx + half] = h1;
        lo[idx + half] = l1;
    }
}

// Router logits from the router GEMM's split-K parts, then softmax + top-k
// of every stream's token (one warp each).
__global__ void bd_route_kernel(const float *ws, int max_split, int nsplit, float *logits, int S, int E, int K,
                                int renorm, int *idx, float *wt) {
    const int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (s >= S) return;
    for (int e = lane; e < E; e += 32) logits[(size_t)s * E + e] = sk_part_sum(ws, max_split, nsplit, s, e);
    __syncwarp();
    route_topk_warp(logits + (size_t)s * E, E, K, renorm, idx + (size_t)s * K, wt + (size_t)s * K);
}

// Expert segments of the sorted pair rows and the MoE tile lists: per active
// expert I/64 gate/up tiles and H/128 down tiles, then the shared expert's.
__global__ void __launch_bounds__(256) bd_plan_kernel(int *counts, int E, int S, int I, int Sh, int H, int *seg,
                                                      int *cursor, SkTile *gu, SkTile *dn, int *nt) {
    __shared__ int cnt[256], seg_s[256], act[257];
    const int t = threadIdx.x;
    if (t < E) cnt[t] = counts[t];
    __syncthreads();
    if (t == 0) {
        int a = 0, n = 0;
        for (int e = 0; e < E; e++) {
            seg_s[e] = a;
            act[e] = n;
            a += cnt[e];
            n += cnt[e] > 0;
        }
        act[E] = n;
    }
    __syncthreads();
    const int gpe = I / 64, dpe = H / 128, n_act = act[E];
    if (t < E) {
        seg[t] = seg_s[t];
        cursor[t] = 0;
        if (cnt[t] > 0) {
            for (int i = 0; i < gpe; i++)
                gu[act[t] * gpe + i] =
                    SkTile{0, t * 2 * I + i * 64, t * 2 * I + I + i * 64, 0, 0, seg_s[t], cnt[t], i * 64, H / 64};
            for (int j = 0; j < dpe; j++)
                dn[act[t] * dpe + j] = SkTile{0, t * H + j * 128, 0, 0, 0, seg_s[t], cnt[t], j * 128, I / 64};
        }
        counts[t] = 0;  // ready for the next layer
    }
    const int sg = Sh / 64;
    for (int i = t; i < sg; i += blockDim.x)
        gu[n_act * gpe + i] = SkTile{0, E * 2 * I + i * 64, E * 2 * I + Sh + i * 64, 0, 1, 0, S, i * 64, H / 64};
    for (int j = t; j < dpe; j += blockDim.x)
        dn[n_act * dpe + j] = SkTile{1, j * 128, 0, 0, 1, 0, S, j * 128, Sh / 64};
    if (t == 0) {
        nt[0] = n_act * gpe + sg;
        nt[1] = n_act * dpe + dpe;
    }
}

// Next step's input: the embedding row (tied LM head) of each stream's
// token; the token is logged at the stream's position, which advances.
__global__ void bd_advance_kernel(const uint16_t *E, int H, const int *tok, int V, int *pos, int *tok_log,
                                  int kv_max, float *x, int *hist, int *hist_len, int hist_cap) {
    const int s = blockIdx.x;
    int t = tok[s];
    if (t < 0 || t >= V) t = 0;  // no winner (all-NaN logits): embed row 0
    const uint16_t *row = E + (size_t)t * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) x[(size_t)s * H + i] = __uint_as_float((uint32_t)row[i] << 16);
    __syncthreads();
    if (threadIdx.x == 0) {
        const int p = pos[s];
        if (p < kv_max) tok_log[(size_t)s * kv_max + p] = t;
        pos[s] = p + 1;
        // the stream's generated-token history takes the selected token
        // (-1 when no logit won), as the batch-1 advance does
        const int n = hist_len[s];
        if (n < hist_cap) {
            hist[(size_t)s * hist_cap + n] = tok[s];
            hist_len[s] = n + 1;
        }
    }
}

}  // namespace ds

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct BdLayer {
    bool dense;
    const float *in_norm, *post_norm;
    SkGemm qkv, oproj, router, gu, dn;  // dense: gu = dense gate/up, dn = dense down
    float *x_in, *x_mid, *x_out;        // residual buffers of this layer
    // the input row is still split-K parts of the previous layer's dense
    // down projection: x_in = in_resid + parts
    bool in_parts;
    const float *in_resid;
};

struct BatchModel {
    ds_cuda_ctx *owner = nullptr;
    ds_cuda_decoder_config_t cfg;
    int S = 0, PbMax = 0;
    std::vector<BdLayer> layers;
    const float *final_norm = nullptr;
    const uint16_t *lm_head = nullptr;
    std::vector<void *> allocs;
    // activations
    float *xa = nullptr, *xb = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *logits = nullptr, *wt = nullptr;
    float *yp = nullptr, *ys = nullptr, *xfinal = nullptr, *val = nullptr;
    uint16_t *p0 = nullptr, *p1 = nullptr, *p2 = nullptr, *pp = nullptr, *hp = nullptr, *hs = nullptr, *hd = nullptr;
    int *idx = nullptr, *counts = nullptr, *seg = nullptr, *cursor = nullptr, *slot_of = nullptr, *inv = nullptr;
    int *nt = nullptr, *tok = nullptr, *pos = nullptr, *tok_log = nullptr, *lo_starts = nullptr;
    SkTile *tiles = nullptr;  // static lists, then the MoE gate/up and down lists
    float *ws = nullptr;      // split-K partial sums
    int sp_qkv = 1, sp_o = 1, sp_r = 1, sp_dd = 1;
    bool out_parts = false;   // the last layer's output is split-K parts
    const float *out_resid = nullptr;
    SkTile *moe_gu = nullptr, *moe_dn = nullptr;
    uint16_t *kv = nullptr;
    float *cos_t = nullptr, *sin_t = nullptr;
    unsigned *err = nullptr;
    // LM-head selection settings (select.cu), shared by the streams; each
    // stream keeps its own history, uniforms and selection scratch
    float rp = 1.f, temperature = 0.f;
    int ngram = 0;
    int hist_cap = 0;
    int *hist = nullptr, *hist_len = nullptr, *sel_full = nullptr, *unif_pos = nullptr;
    float *hval = nullptr, *bval = nullptr, *sel_logits = nullptr, *unif = nullptr;
    int unif_n = 0;     // uniforms supplied per stream
    int unif_used = 0;  // sampled steps launched since the uniforms were set
    // V3's reference sliding window (0: off) and each stream's prefill length
    int swa_window = 0;
    int *swa_refs = nullptr;
    bool sampling() const { return rp > 1.f || ngram > 0 || temperature > 0.f; }
    std::vector<int> host_lo;   // per layer and stream
    std::vector<int> host_pos;  // per stream: the position the next token is written at
    cudaGraphExec_t graph = nullptr;

    size_t plane_elems() const { return (size_t)cfg.n_layers * cfg.n_heads * cfg.kv_max * cfg.head_dim; }
    long long stream_stride() const { return 4 * (long long)plane_elems(); }
    uint16_t *plane(int p, int l) const {
        return kv + p * plane_elems() + (size_t)l * cfg.n_heads * cfg.kv_max * cfg.head_dim;
    }
};

static std::map<int, BatchModel *> g_bmodels;
static int g_next_bm = 1;

static void bm_free(BatchModel *m) {
    if (m->graph) cudaGraphExecDestroy(m->graph);
    for (void *p : m->allocs) cudaFree(p);
    delete m;
}

template <typename T>
static int bm_alloc(ds_cuda_ctx *c, BatchModel *m, T **p, size_t elems) {
    void *d = nullptr;
    if (cudaMalloc(&d, elems * sizeof(T) + 16) != cudaSuccess) {
        cudaGetLastError();
        return ctx_fail(c, DS_CUDA_ENOMEM, "batch decoder: cudaMalloc(%zu) failed", elems * sizeof(T));
    }
    cudaMemset(d, 0, elems * sizeof(T) + 16);
    m->allocs.push_back(d);
    *p = (T *)d;
    return DS_CUDA_OK;
}

#define BK(expr)                  \
    do {                          \
        int _rc = (expr);         \
        if (_rc < 0) return _rc;  \
    } while (0)
#define BKL(expr, what)                                         \
    do {                                                        \
        cudaError_t _e = (expr);                                \
        if (_e != cudaSuccess) return ctx_cuda(c, _e, what);    \
    } while (0)

static int bm_tiles(ds_cuda_ctx *c, SkTile *dst, const std::vector<SkTile> &v) {
    if (v.empty()) return DS_CUDA_OK;
    if (cudaMemcpy(dst, v.data(), v.size() * sizeof(SkTile), cudaMemcpyHostToDevice) != cudaSuccess)
        return ctx_fail(c, DS_CUDA_ECUDA, "batch decoder: tile upload");
    return DS_CUDA_OK;
}

static int enqueue_step(ds_cuda_ctx *c, BatchModel *m, cudaStream_t st) {
    const auto &g = m->cfg;
    const int S = m->S, H = g.hidden, NH = g.n_heads, HD = g.head_dim, QD = NH * HD, E = g.n_experts, K = g.top_k;
    const int I = g.moe_inter, Sh = g.n_shared * g.moe_inter;
    const int grid = c->sm_count;
    for (int l = 0; l < g.n_layers; l++) {
        BdLayer &L = m->layers[l];
        BKL(sk_split_launch(L.x_in, S, H, H, L.in_norm, g.rms_eps, m->p0, 64, nullptr, st,
                            L.in_parts ? m->ws : nullptr, SK_MAX_SPLIT, m->sp_dd, L.in_resid, L.x_in),
            "bd norm");
        BKL(sk_gemm_launch(0, L.qkv, grid, st), "bd qkv");
        const int nthr = S * 3 * NH * (HD / 2);
        bd_rope_kv_kernel<<<(nthr + 255) / 256, 256, 0, st>>>(m->ws, SK_MAX_SPLIT, m->sp_qkv, S, NH, HD, m->pos,
                                                              m->cos_t, m->sin_t, m->q,
                                                              m->plane(0, l), m->plane(1, l), m->plane(2, l),
                                                              m->plane(3, l), g.kv_max, m->stream_stride());
        AttnArgs aa = {};
        aa.q = m->q;
        aa.k_hi = m->plane(0, l);
        aa.k_lo = m->plane(1, l);
        aa.v_hi = m->plane(2, l);
        aa.v_lo = m->plane(3, l);
        aa.kv_max = g.kv_max;
        aa.n_heads = NH;
        aa.d_pos = m->pos;
        aa.scale = 1.0f / sqrtf((float)HD);
        aa.out = m->att;
        aa.kv_stream_stride = m->stream_stride();
        aa.q_stride = QD;
        aa.lo_starts = m->lo_starts + (size_t)l * S;
        aa.swa_window = m->swa_window;
        aa.swa_refs = m->swa_refs;
        BKL(launch_attn_decode(aa, st, false, S), "bd attention");
        BKL(sk_split_launch(m->att, S, QD, QD, nullptr, 0.f, m->p1, 64, nullptr, st, nullptr, 0, 0, nullptr, nullptr),
            "bd split attn");
        BKL(sk_gemm_launch(0, L.oproj, grid, st), "bd o-proj");
        // x_mid = x_in + O-proj (its split-K parts), then the post-norm planes
        BKL(sk_split_launch(L.x_mid, S, H, H, L.post_norm, g.rms_eps, m->p2, 64, nullptr, st, m->ws, SK_MAX_SPLIT,
                            m->sp_o, L.x_in, L.x_mid),
            "bd post norm");
        if (L.dense) {
            BKL(sk_gemm_launch(1, L.gu, grid, st), "bd dense gate/up");
            BKL(sk_gemm_launch(0, L.dn, grid, st), "bd dense down");
        } else {
            const int P = S * K;
            BKL(sk_gemm_launch(0, L.router, grid, st), "bd router");
            bd_route_kernel<<<(S + 7) / 8, 256, 0, st>>>(m->ws, SK_MAX_SPLIT, m->sp_r, m->logits, S, E, K, c->renorm,
                                                         m->idx, m->wt);
            BKL(pf_count_launch(P, m->idx, E, m->counts, grid, st), "bd count");
            bd_plan_kernel<<<1, 256, 0, st>>>(m->counts, E, S, I, Sh, H, m->seg, m->cursor, m->moe_gu, m->moe_dn,
                                              m->nt);
            BKL(pf_scatter_launch(P, H, H, K, nullptr, m->idx, E, m->seg, m->cursor, m->p2, m->p2 + (size_t)64 * H,
                                  m->pp, m->pp + (size_t)m->PbMax * H, m->slot_of, m->inv, st),
                "bd scatter");
            BKL(sk_gemm_launch(1, L.gu, grid, st), "bd moe gate/up");
            BKL(sk_gemm_launch(0, L.dn, grid, st), "bd moe down");
            BKL(pf_combine_launch(L.x_mid, S, H, K, m->idx, m->wt, m->yp, m->inv, m->ys, st), "bd combine");
        }
    }
    float *x_last = m->layers.back().x_out;
    BKL(sk_split_launch(x_last, S, H, H, m->final_norm, g.rms_eps, m->p0, 64, m->xfinal, st,
                        m->out_parts ? m->ws : nullptr, SK_MAX_SPLIT, m->sp_dd, m->out_resid, x_last),
        "bd final norm");
    int rc = lmhead_tc_enqueue(c, m->xfinal, m->lm_head, H, g.vocab, S, m->tok, m->val, st);
    if (rc < 0) return rc;
    if (m->sampling()) {
        // the reference's selection rules per stream on the argmax winner
        // (ds_moe_decoder.c:1021-1263); the full-logits path runs for the
        // streams that need it
        SelectArgs sa = {};
        sa.W = m->lm_head;
        sa.x = m->xfinal;
        sa.H = H;
        sa.V = g.vocab;
        sa.hist = m->hist;
        sa.hist_len = m->hist_len;
        sa.cap = m->hist_cap;
        sa.hval = m->hval;
        sa.bval = m->bval;
        sa.logits = m->sel_logits;
        sa.tok = m->tok;
        sa.val = m->val;
        sa.full = m->sel_full;
        sa.rp = m->rp;
        sa.ngram = m->ngram;
        sa.temperature = m->temperature;
        sa.unif = m->unif;
        sa.unif_pos = m->unif_pos;
        sa.n_streams = S;
        sa.x_ld = H;
        sa.unif_ld = m->hist_cap;
        BKL(launch_select(sa, st), "bd token selection");
    }
    bd_advance_kernel<<<S, 256, 0, st>>>(m->lm_head, H, m->tok, g.vocab, m->pos, m->tok_log, g.kv_max,
                                         m->layers[0].x_in, m->hist, m->hist_len, m->hist_cap);
    BKL(cudaGetLastError(), "bd advance");
    return DS_CUDA_OK;
}

#define LOOKB(ptr, bytes) ctx_lookup(c, (ptr), (bytes), true)

extern "C" int ds_cuda_batch_decoder_create(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg,
                                            const ds_cuda_layer_weights_t *lw, const float *final_norm,
                                            const uint16_t *lm_head, int n_streams) {
    if (!c || !c->ok || !cfg || !lw || !final_norm || !lm_head) return DS_CUDA_EINVAL;
    const auto &g = *cfg;
    const int H = g.hidden, NH = g.n_heads, HD = g.head_dim, QD = NH * HD, E = g.n_experts, K = g.top_k;
    const int I = g.moe_inter, Sh = g.n_shared * g.moe_inter, D = g.dense_inter, S = n_streams;
    if (S < 1 || S > SK_TOK || HD != 128 || H % 128 || QD % 128 || H > 2048 || I % 64 || Sh % 64 || Sh <= 0 ||
        D % 64 || E > 256 || K > 8 || K > E || g.kv_max <= 0 || g.kv_max > 4096 || g.use_int8 || g.vocab <= 0)
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_create: unsupported configuration");
    cudaSetDevice(c->device);
    BatchModel *m = new BatchModel();
    m->owner = c;
    m->cfg = g;
    m->S = S;
    m->PbMax = S * K + 64;
    int rc = DS_CUDA_OK;
#define BA(p, n)                                          \
    do {                                                  \
        if (rc == DS_CUDA_OK) rc = bm_alloc(c, m, &(p), (n)); \
    } while (0)
    // selection state: history and uniforms hold kv_max + 512 entries per
    // stream (as the batch-1 decoder's); logits for the full path
    m->hist_cap = g.kv_max + 512;
    BA(m->hist, (size_t)S * m->hist_cap);
    BA(m->hval, (size_t)S * m->hist_cap);
    BA(m->unif, (size_t)S * m->hist_cap);
    BA(m->hist_len, (size_t)S);
    BA(m->unif_pos, (size_t)S);
    BA(m->sel_full, (size_t)S);
    BA(m->bval, (size_t)S);
    BA(m->swa_refs, (size_t)S);
    BA(m->sel_logits, (size_t)S * g.vocab);
    BA(m->xa, (size_t)S * H);
    BA(m->xb, (size_t)S * H);
    BA(m->qkv, (size_t)S * 3 * QD);
    BA(m->q, (size_t)S * QD);
    BA(m->att, (size_t)S * QD);
    BA(m->logits, (size_t)S * E);
    BA(m->wt, (size_t)S * K);
    BA(m->yp, (size_t)m->PbMax * H);
    BA(m->ys, (size_t)S * H);
    BA(m->xfinal, (size_t)S * H);
    BA(m->val, (size_t)S);
    BA(m->p0, (size_t)128 * H);
    BA(m->p1, (size_t)128 * QD);
    BA(m->p2, (size_t)128 * H);
    BA(m->pp, (size_t)2 * m->PbMax * H);
    BA(m->hp, (size_t)2 * m->PbMax * I);
    BA(m->hs, (size_t)128 * Sh);
    BA(m->hd, (size_t)128 * D);
    BA(m->idx, (size_t)S * K);
    BA(m->counts, 256);
    BA(m->seg, 256);
    BA(m->cursor, 256);
    BA(m->slot_of, (size_t)m->PbMax);
    BA(m->inv, (size_t)S * K);
    BA(m->nt, 16);
    BA(m->tok, (size_t)S);
    BA(m->pos, (size_t)S);
    BA(m->tok_log, (size_t)S * g.kv_max);
    BA(m->lo_starts, (size_t)g.n_layers * S);
    BA(m->err, 4);
    BA(m->kv, (size_t)S * 4 * m->plane_elems());
    BA(m->cos_t, (size_t)g.kv_max * HD);
    BA(m->sin_t, (size_t)g.kv_max * HD);
    // static tile lists (per layer shape, shared by all layers) + MoE lists
    // split K where a layer has too few 128-row output tiles to fill the
    // SMs (QKV, O-proj, router, dense down); the parts meet in `ws`
    const int sp_qkv = 5, sp_o = 10, sp_r = 20, sp_dd = 15;
    m->sp_qkv = sp_qkv;
    m->sp_o = sp_o;
    m->sp_r = sp_r;
    m->sp_dd = sp_dd;
    const int n_qkv = (3 * QD / 128) * sp_qkv, n_o = (H / 128) * sp_o, n_r = ((E + 127) / 128) * sp_r;
    const int n_dgu = D / 64, n_ddn = (H / 128) * sp_dd;
    const int n_moe_gu = E * (I / 64) + Sh / 64, n_moe_dn = E * (H / 128) + H / 128;
    const int n_static = n_qkv + n_o + n_r + n_dgu + n_ddn;
    BA(m->tiles, (size_t)n_static + n_moe_gu + n_moe_dn);
    BA(m->ws, (size_t)std::max(3 * QD / 128, H / 128) * SK_MAX_SPLIT * 128 * SK_TOK);
#undef BA
    if (rc < 0) {
        bm_free(m);
        return rc;
    }
    SkTile *t_qkv = m->tiles, *t_o = t_qkv + n_qkv, *t_r = t_o + n_o, *t_dgu = t_r + n_r, *t_ddn = t_dgu + n_dgu;
    m->moe_gu = t_ddn + n_ddn;
    m->moe_dn = m->moe_gu + n_moe_gu;
    // counts of the static lists live in nt[2..6]
    std::vector<SkTile> v;
    for (int mtx = 0; mtx < 3; mtx++)
        for (int t = 0; t < QD / 128; t++)
            sk_push_split(v, SkTile{mtx, t * 128, 0, 0, 0, 0, S, mtx * QD + t * 128, H / 64}, sp_qkv,
                          mtx * (QD / 128) + t);
    rc = bm_tiles(c, t_qkv, v);
    v.clear();
    for (int t = 0; t < H / 128; t++) sk_push_split(v, SkTile{0, t * 128, 0, 0, 0, 0, S, t * 128, QD / 64}, sp_o, t);
    if (rc == DS_CUDA_OK) rc = bm_tiles(c, t_o, v);
    v.clear();
    for (int t = 0; t < (E + 127) / 128; t++)
        sk_push_split(v, SkTile{0, t * 128, 0, 0, 0, 0, S, t * 128, H / 64}, sp_r, t);
    if (rc == DS_CUDA_OK) rc = bm_tiles(c, t_r, v);
    v.clear();
    for (int t = 0; t < n_dgu; t++) v.push_back(SkTile{0, t * 64, t * 64, 1, 0, 0, S, t * 64, H / 64});
    if (rc == DS_CUDA_OK) rc = bm_tiles(c, t_dgu, v);
    v.clear();
    for (int t = 0; t < H / 128; t++) sk_push_split(v, SkTile{0, t * 128, 0, 0, 0, 0, S, t * 128, D / 64}, sp_dd, t);
    if (rc == DS_CUDA_OK) rc = bm_tiles(c, t_ddn, v);
    int counts_h[7] = {0, 0, n_qkv, n_o, n_r, n_dgu, n_ddn};
    if (rc == DS_CUDA_OK && cudaMemcpy(m->nt, counts_h, sizeof counts_h, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = ctx_fail(c, DS_CUDA_ECUDA, "batch decoder: counts upload");
    // RoPE table, as ds_compute_rope_neox (ds_kernels.c:2399-2424) in host float math
    if (rc == DS_CUDA_OK) {
        std::vector<float> cs((size_t)g.kv_max * HD), sn(cs.size());
        const int half = HD / 2;
        for (int s = 0; s < g.kv_max; s++) {
            const float p = (float)s;
            for (int d = 0; d < half; d++) {
                const float freq = 1.0f / powf(g.rope_theta, (float)(2 * d) / (float)HD);
                const float ang = p * freq, cv = cosf(ang), sv = sinf(ang);
                cs[(size_t)s * HD + d] = cs[(size_t)s * HD + d + half] = cv;
                sn[(size_t)s * HD + d] = sn[(size_t)s * HD + d + half] = sv;
            }
        }
        cudaMemcpy(m->cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(m->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
        m->host_lo.assign((size_t)g.n_layers * S, 0);
        m->host_pos.assign(S, 0);
    }
    if (rc == DS_CUDA_OK) {
        m->final_norm = (const float *)LOOKB(final_norm, (size_t)H * 4);
        m->lm_head = (const uint16_t *)LOOKB(lm_head, (size_t)g.vocab * H * 2);
        if (!m->final_norm || !m->lm_head) rc = ctx_fail(c, DS_CUDA_ENOTREG, "batch_decoder_create: head weights");
    }
    // per layer: weights, tensor maps and the residual buffers
    float *cur = m->xa;
    bool pending = false;            // cur is (pending_resid + split-K parts)
    const float *pending_resid = nullptr;
    for (int l = 0; l < g.n_layers && rc == DS_CUDA_OK; l++) {
        const ds_cuda_layer_weights_t &w = lw[l];
        BdLayer L;
        memset(&L, 0, sizeof L);
        L.dense = l < g.first_dense;
        const uint16_t *wq = (const uint16_t *)LOOKB(w.wq, (size_t)QD * H * 2);
        const uint16_t *wk = (const uint16_t *)LOOKB(w.wk, (size_t)QD * H * 2);
        const uint16_t *wv = (const uint16_t *)LOOKB(w.wv, (size_t)QD * H * 2);
        const uint16_t *wo = (const uint16_t *)LOOKB(w.wo, (size_t)H * QD * 2);
        L.in_norm = (const float *)LOOKB(w.input_norm, (size_t)H * 4);
        L.post_norm = (const float *)LOOKB(w.post_attn_norm, (size_t)H * 4);
        bool ok = wq && wk && wv && wo && L.in_norm && L.post_norm;
        float *other = cur == m->xa ? m->xb : m->xa;
        L.x_in = cur;
        L.x_mid = other;
        L.in_parts = pending;
        L.in_resid = pending_resid;
        pending = false;
        // QKV: three weight maps into one [S x 3QD] output
        ok = ok && tmap_bf16(&L.qkv.a[0], wq, H, QD, 64) && tmap_bf16(&L.qkv.a[1], wk, H, QD, 64) &&
             tmap_bf16(&L.qkv.a[2], wv, H, QD, 64) && tmap_bf16(&L.qkv.b[0], m->p0, H, 128, 64);
        L.qkv.lo_off[0] = 64;
        L.qkv.tiles = t_qkv;
        L.qkv.n_tiles = m->nt + 2;
        for (int i = 0; i < 3; i++) {
            L.qkv.out[i] = m->qkv;
            L.qkv.out_ld[i] = 3 * QD;
            L.qkv.out_n[i] = 3 * QD;
        }
        L.qkv.err = m->err;
        // O-proj + residual
        ok = ok && tmap_bf16(&L.oproj.a[0], wo, QD, H, 64) && tmap_bf16(&L.oproj.b[0], m->p1, QD, 128, 64);
        L.oproj.lo_off[0] = 64;
        L.oproj.tiles = t_o;
        L.oproj.n_tiles = m->nt + 3;
        L.oproj.out[0] = other;
        L.oproj.resid[0] = cur;
        L.oproj.out_ld[0] = H;
        L.oproj.out_n[0] = H;
        L.oproj.err = m->err;
        if (L.dense) {
            const uint16_t *dg = (const uint16_t *)LOOKB(w.dense_gate, (size_t)D * H * 2);
            const uint16_t *du = (const uint16_t *)LOOKB(w.dense_up, (size_t)D * H * 2);
            const uint16_t *dd = (const uint16_t *)LOOKB(w.dense_down, (size_t)H * D * 2);
            ok = ok && dg && du && dd && tmap_bf16(&L.gu.a[0], dg, H, D, 64) && tmap_bf16(&L.gu.a[1], du, H, D, 64) &&
                 tmap_bf16(&L.gu.b[0], m->p2, H, 128, 64) && tmap_bf16(&L.dn.a[0], dd, D, H, 64) &&
                 tmap_bf16(&L.dn.b[0], m->hd, D, 128, 64);
            L.gu.lo_off[0] = 64;
            L.gu.tiles = t_dgu;
            L.gu.n_tiles = m->nt + 5;
            L.gu.h_hi[0] = m->hd;
            L.gu.h_lo[0] = m->hd + (size_t)64 * D;
            L.gu.h_ld[0] = D;
            L.gu.err = m->err;
            L.dn.lo_off[0] = 64;
            L.dn.tiles = t_ddn;
            L.dn.n_tiles = m->nt + 6;
            // x_out = x_mid + down(...): the down GEMM leaves split-K parts,
            // the next reader assembles them into cur
            L.dn.out_ld[0] = H;
            L.dn.out_n[0] = H;
            L.dn.err = m->err;
            L.x_out = cur;
            pending = true;
            pending_resid = other;
        } else {
            const uint16_t *rt = (const uint16_t *)LOOKB(w.router, (size_t)E * H * 2);
            const uint16_t *blk = (const uint16_t *)LOOKB(w.expert_block, ((size_t)E * 2 * I + 2 * (size_t)Sh) * H * 2);
            const uint16_t *dw = (const uint16_t *)LOOKB(w.down, (size_t)E * H * I * 2);
            const uint16_t *sd = (const uint16_t *)LOOKB(w.shared_down, (size_t)H * Sh * 2);
            ok = ok && rt && blk && dw && sd;
            ok = ok && tmap_bf16(&L.router.a[0], rt, H, E, 64) && tmap_bf16(&L.router.b[0], m->p2, H, 128, 64);
            L.router.lo_off[0] = 64;
            L.router.tiles = t_r;
            L.router.n_tiles = m->nt + 4;
            L.router.out[0] = m->logits;
            L.router.out_ld[0] = E;
            L.router.out_n[0] = E;
            L.router.err = m->err;
            ok = ok && tmap_bf16(&L.gu.a[0], blk, H, (uint64_t)E * 2 * I + 2 * Sh, 64) &&
                 tmap_bf16(&L.gu.b[0], m->pp, H, 2 * (uint64_t)m->PbMax, 64) &&
                 tmap_bf16(&L.gu.b[1], m->p2, H, 128, 64);
            L.gu.lo_off[0] = m->PbMax;
            L.gu.lo_off[1] = 64;
            L.gu.tiles = m->moe_gu;
            L.gu.n_tiles = m->nt + 0;
            L.gu.h_hi[0] = m->hp;
            L.gu.h_lo[0] = m->hp + (size_t)m->PbMax * I;
            L.gu.h_ld[0] = I;
            L.gu.h_hi[1] = m->hs;
            L.gu.h_lo[1] = m->hs + (size_t)64 * Sh;
            L.gu.h_ld[1] = Sh;
            L.gu.err = m->err;
            ok = ok && tmap_bf16(&L.dn.a[0], dw, I, (uint64_t)E * H, 64) && tmap_bf16(&L.dn.a[1], sd, Sh, H, 64) &&
                 tmap_bf16(&L.dn.b[0], m->hp, I, 2 * (uint64_t)m->PbMax, 64) &&
                 tmap_bf16(&L.dn.b[1], m->hs, Sh, 128, 64);
            L.dn.lo_off[0] = m->PbMax;
            L.dn.lo_off[1] = 64;
            L.dn.tiles = m->moe_dn;
            L.dn.n_tiles = m->nt + 1;
            L.dn.out[0] = m->yp;
            L.dn.out[1] = m->ys;
            L.dn.out_ld[0] = L.dn.out_ld[1] = H;
            L.dn.out_n[0] = L.dn.out_n[1] = H;
            L.dn.err = m->err;
            L.x_out = other;  // the combine adds into x_mid in place
            cur = other;
        }
        for (SkGemm *gp : {&L.qkv, &L.oproj, &L.router, &L.gu, &L.dn}) {
            gp->ws = m->ws;
            gp->max_split = SK_MAX_SPLIT;
        }
        if (!ok) rc = ctx_fail(c, DS_CUDA_ENOTREG, "batch_decoder_create: layer %d weights or tensor maps", l);
        m->layers.push_back(L);
    }
    m->out_parts = pending;
    m->out_resid = pending_resid;
    if (rc < 0) {
        bm_free(m);
        return rc;
    }
    const int id = g_next_bm++;
    g_bmodels[id] = m;
    return id;
}

static BatchModel *bm_get(ds_cuda_ctx *c, int id) {
    auto it = g_bmodels.find(id);
    return it == g_bmodels.end() || it->second->owner != c ? nullptr : it->second;
}

extern "C" int ds_cuda_batch_decoder_destroy(ds_cuda_ctx_t *c, int id) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    g_bmodels.erase(id);
    bm_free(m);
    return DS_CUDA_OK;
}

static uint16_t bm_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

extern "C" int ds_cuda_batch_decoder_load_kv(ds_cuda_ctx_t *c, int id, int stream, int layer, int pos0, int n,
                                             const float *k, const float *v) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || !k || !v || stream < 0 || stream >= m->S || layer < 0 || layer >= m->cfg.n_layers || pos0 < 0 ||
        n <= 0 || pos0 + n > m->cfg.kv_max)
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_load_kv: bad argument");
    cudaSetDevice(c->device);
    const int NH = m->cfg.n_heads, HD = m->cfg.head_dim;
    std::vector<uint16_t> hi((size_t)n * HD), lo((size_t)n * HD);
    bool exact = true;
    for (int which = 0; which < 2; which++) {
        const float *src = which == 0 ? k : v;
        for (int h = 0; h < NH; h++) {
            for (int i = 0; i < n; i++)
                for (int d = 0; d < HD; d++) {
                    const float f = src[(size_t)i * NH * HD + (size_t)h * HD + d];
                    const uint16_t a = bm_bf16(f);
                    uint32_t au = (uint32_t)a << 16;
                    float af;
                    memcpy(&af, &au, 4);
                    const uint16_t b = bm_bf16(f - af);
                    hi[(size_t)i * HD + d] = a;
                    lo[(size_t)i * HD + d] = b;
                    if (b) exact = false;
                }
            const size_t off = (size_t)stream * m->stream_stride() + ((size_t)h * m->cfg.kv_max + pos0) * HD;
            BKL(cudaMemcpy(m->plane(which * 2, layer) + off, hi.data(), hi.size() * 2, cudaMemcpyHostToDevice),
                "batch kv copy");
            BKL(cudaMemcpy(m->plane(which * 2 + 1, layer) + off, lo.data(), lo.size() * 2, cudaMemcpyHostToDevice),
                "batch kv copy");
        }
    }
    int &ls = m->host_lo[(size_t)layer * m->S + stream];
    if (exact && pos0 <= ls) ls = std::max(ls, pos0 + n);
    if (!exact && pos0 < ls) ls = pos0;
    BKL(cudaMemcpy(m->lo_starts + (size_t)layer * m->S + stream, &ls, 4, cudaMemcpyHostToDevice), "lo start");
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_batch_decoder_set_len(ds_cuda_ctx_t *c, int id, int stream, int len) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || stream < 0 || stream >= m->S || len < 0 || len >= m->cfg.kv_max)
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_set_len: bad argument");
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (int l = 0; l < m->cfg.n_layers; l++) {
        int &ls = m->host_lo[(size_t)l * m->S + stream];
        if (ls > len) {
            ls = len;
            cudaMemcpy(m->lo_starts + (size_t)l * m->S + stream, &ls, 4, cudaMemcpyHostToDevice);
        }
    }
    BKL(cudaMemcpy(m->pos + stream, &len, 4, cudaMemcpyHostToDevice), "batch set_len");
    m->host_pos[stream] = len;
    return DS_CUDA_OK;
}

// Every stream must have room for n more tokens (a step writes KV at pos).
static int bm_room(ds_cuda_ctx *c, BatchModel *m, int n) {
    for (int p : m->host_pos)
        if (p + n > m->cfg.kv_max) return ctx_fail(c, DS_CUDA_ESTATE, "batch decoder: KV cache full");
    return DS_CUDA_OK;
}
static void bm_advance(BatchModel *m, int n) {
    for (int &p : m->host_pos) p += n;
}

static int bm_check(ds_cuda_ctx *c, BatchModel *m) {
    unsigned e = 0;
    BKL(cudaMemcpy(&e, m->err, 4, cudaMemcpyDeviceToHost), "batch error flag");
    if (e) {
        cudaMemset(m->err, 0, 4);
        return ctx_fail(c, DS_CUDA_ETIMEOUT, "batch decoder: a bounded device-side wait gave up");
    }
    return DS_CUDA_OK;
}

// Temperature sampling takes one uniform per stream per step.
static int bm_uniforms(ds_cuda_ctx *c, BatchModel *m, int n) {
    if (m->temperature <= 0.f) return DS_CUDA_OK;
    if (m->unif_used + n > m->unif_n)
        return ctx_fail(c, DS_CUDA_ESTATE, "batch decoder: %d uniforms left for %d temperature-sampled steps",
                        m->unif_n - m->unif_used, n);
    return DS_CUDA_OK;
}
static void bm_used(BatchModel *m, int n) {
    if (m->temperature > 0.f) m->unif_used += n;
}

// The step graph bakes in the settings: drop it when they change.
static void bm_drop_graph(ds_cuda_ctx *c, BatchModel *m) {
    cudaStreamSynchronize(c->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
}

extern "C" int ds_cuda_batch_decoder_set_sampling(ds_cuda_ctx_t *c, int id, float repeat_penalty,
                                                  int no_repeat_ngram_size, float temperature) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || !(repeat_penalty > 0.f) || no_repeat_ngram_size < 0 || !(temperature >= 0.f))
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_set_sampling: bad argument");
    const bool on = repeat_penalty > 1.f || no_repeat_ngram_size > 0 || temperature > 0.f;
    if (on && m->cfg.hidden % 256)
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_set_sampling: hidden must be a multiple of 256");
    cudaSetDevice(c->device);
    bm_drop_graph(c, m);
    m->rp = repeat_penalty;
    m->ngram = no_repeat_ngram_size;
    m->temperature = temperature;
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_batch_decoder_set_history(ds_cuda_ctx_t *c, int id, int stream, const int *tokens, int n) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || stream < 0 || stream >= m->S || n < 0 || n > m->hist_cap || (n > 0 && !tokens))
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_set_history: bad argument");
    cudaSetDevice(c->device);
    BKL(cudaStreamSynchronize(c->stream), "batch set history");
    if (n)
        BKL(cudaMemcpy(m->hist + (size_t)stream * m->hist_cap, tokens, (size_t)n * 4, cudaMemcpyHostToDevice),
            "batch history copy");
    BKL(cudaMemcpy(m->hist_len + stream, &n, 4, cudaMemcpyHostToDevice), "batch history length");
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_batch_decoder_get_history(ds_cuda_ctx_t *c, int id, int stream, int *tokens, int cap) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || stream < 0 || stream >= m->S || cap < 0 || (cap > 0 && !tokens))
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_get_history: bad argument");
    cudaSetDevice(c->device);
    BKL(cudaStreamSynchronize(c->stream), "batch get history");
    int n = 0;
    BKL(cudaMemcpy(&n, m->hist_len + stream, 4, cudaMemcpyDeviceToHost), "batch history length");
    const int k = std::min(n, cap);
    if (k > 0)
        BKL(cudaMemcpy(tokens, m->hist + (size_t)stream * m->hist_cap, (size_t)k * 4, cudaMemcpyDeviceToHost),
            "batch history copy");
    return n;
}

// Uniforms for temperature sampling: u is [S x n], row s the uniforms
// stream s consumes in order, one per sampled step. Every stream restarts
// from its first uniform.
extern "C" int ds_cuda_batch_decoder_set_uniforms(ds_cuda_ctx_t *c, int id, const float *u, int n) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || n < 0 || n > m->hist_cap || (n > 0 && !u))
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_set_uniforms: bad argument (at most %d per stream)",
                        m ? m->hist_cap : 0);
    cudaSetDevice(c->device);
    BKL(cudaStreamSynchronize(c->stream), "batch set uniforms");
    if (n)
        BKL(cudaMemcpy2D(m->unif, (size_t)m->hist_cap * 4, u, (size_t)n * 4, (size_t)n * 4, m->S,
                         cudaMemcpyHostToDevice),
            "batch uniform copy");
    BKL(cudaMemset(m->unif_pos, 0, (size_t)m->S * 4), "batch uniform positions");
    m->unif_n = n;
    m->unif_used = 0;
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_batch_decoder_set_window(ds_cuda_ctx_t *c, int id, int sliding_window_size,
                                                const int *prefill_token_counts) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || sliding_window_size < 0 || (sliding_window_size > 0 && !prefill_token_counts))
        return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_set_window: bad argument");
    std::vector<int> refs(m->S, 0);
    for (int s = 0; s < m->S && sliding_window_size > 0; s++) {
        refs[s] = prefill_token_counts[s];
        if (refs[s] < 0) return ctx_fail(c, DS_CUDA_EINVAL, "batch_decoder_set_window: negative prefill count");
    }
    cudaSetDevice(c->device);
    bm_drop_graph(c, m);
    BKL(cudaMemcpy(m->swa_refs, refs.data(), (size_t)m->S * 4, cudaMemcpyHostToDevice), "batch window");
    m->swa_window = sliding_window_size;
    return DS_CUDA_OK;
}

// One step for all streams: embeds [S x H] (NULL: the embeddings of the
// previous tokens); tokens [S] out; final_x [S x H] optional.
extern "C" int ds_cuda_batch_decoder_forward(ds_cuda_ctx_t *c, int id, const float *embeds, int *tokens,
                                             float *final_x) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || !tokens) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    cudaStream_t st = c->stream;
    const size_t SH = (size_t)m->S * m->cfg.hidden;
    BK(bm_room(c, m, 1));
    BK(bm_uniforms(c, m, 1));
    if (embeds) BKL(cudaMemcpyAsync(m->layers[0].x_in, embeds, SH * 4, cudaMemcpyHostToDevice, st), "embeds");
    BK(enqueue_step(c, m, st));
    BKL(cudaMemcpyAsync(tokens, m->tok, (size_t)m->S * 4, cudaMemcpyDeviceToHost, st), "tokens");
    if (final_x) BKL(cudaMemcpyAsync(final_x, m->xfinal, SH * 4, cudaMemcpyDeviceToHost, st), "final x");
    BKL(cudaStreamSynchronize(st), "batch forward");
    bm_advance(m, 1);
    bm_used(m, 1);
    return bm_check(c, m);
}

// n_steps steps on the device (one CUDA graph per step, captured on first
// use), each stream's token feeding its next step. Enqueue only.
extern "C" int ds_cuda_batch_decoder_generate_dev(ds_cuda_ctx_t *c, int id, int n_steps, void *stream) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || n_steps < 0) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    if (n_steps == 0) return DS_CUDA_OK;
    BK(bm_room(c, m, n_steps));
    BK(bm_uniforms(c, m, n_steps));
    bm_advance(m, n_steps);
    bm_used(m, n_steps);
    if (!m->graph) {
        // the first step runs uncaptured (scratch allocation), then capture
        BK(enqueue_step(c, m, st));
        n_steps--;
        cudaGraph_t gr = nullptr;
        BKL(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "batch capture");
        int rc = enqueue_step(c, m, st);
        cudaError_t e = cudaStreamEndCapture(st, &gr);
        if (rc < 0) {
            if (gr) cudaGraphDestroy(gr);
            return rc;
        }
        if (e == cudaSuccess) e = cudaGraphInstantiate(&m->graph, gr, 0);
        if (gr) cudaGraphDestroy(gr);
        if (e != cudaSuccess) return ctx_cuda(c, e, "batch graph");
    }
    for (int i = 0; i < n_steps; i++) BKL(cudaGraphLaunch(m->graph, st), "batch graph launch");
    return DS_CUDA_OK;
}

// tokens [n_steps x S]: the greedy tokens of every stream per step.
extern "C" int ds_cuda_batch_decoder_generate(ds_cuda_ctx_t *c, int id, const float *first_embeds, int n_steps,
                                              int *tokens) {
    BatchModel *m = bm_get(c, id);
    if (!c || !m || !tokens || n_steps <= 0) return DS_CUDA_EINVAL;
    for (int i = 0; i < n_steps; i++) {
        int rc = ds_cuda_batch_decoder_forward(c, id, i == 0 ? first_embeds : nullptr, tokens + (size_t)i * m->S,
                                               nullptr);
        if (rc < 0) return rc;
    }
    return DS_CUDA_OK;
}

void ctx_release_batch_models(ds_cuda_ctx *c) {
    for (auto it = g_bmodels.begin(); it != g_bmodels.end();) {
        if (it->second->owner == c) {
            bm_free(it->second);
            it = g_bmodels.erase(it);
        } else {
            ++it;
        }
    }
}
