// decoder.cu — batch-1 greedy decode of the DeepSeek3B-MoE decoder on one
// GPU: weights and KV cache resident in HBM, one decode step = one CUDA graph
// of kernels chained with programmatic dependent launch (each kernel's
// prologue overlaps its predecessor's tail), replayed once per token.
#include <cmath>
#include <cstring>
#include <vector>

#include "ctx.h"
#include "kernels_decode.cuh"
#include "mega.h"
#include "moe_step.h"
#include "prefill.h"

using namespace ds;

struct DecLayer {
    const uint16_t *wq, *wk, *wv, *wo;
    const float *in_norm, *post_norm;
    bool dense;
    const uint16_t *dgate, *dup, *ddown;
    const uint16_t *router, *block, *down, *sdown;
    WMat gu, dn, sgu, sdn;  // INT8
};

struct DecoderModel {
    ds_cuda_decoder_config_t cfg;
    std::vector<DecLayer> layers;
    const float *final_norm = nullptr;
    const uint16_t *lm_head = nullptr;
    const uint16_t *embed = nullptr;  // token embedding table (the LM head unless set)
    // device state
    float *xa = nullptr, *xb = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr, *xfinal = nullptr;
    float *scores = nullptr, *wt = nullptr, *val = nullptr;
    float *rpart = nullptr;  // router terms of the O-proj CTAs (router folded into the O-proj)
    int *idx = nullptr, *pos = nullptr, *tok = nullptr, *tok_log = nullptr;
    unsigned *tickets = nullptr;  // [0] LM head, [1] router, [8] LM-head wait error, [9] MoE-step wait error
    unsigned long long *slot = nullptr;
    unsigned long long *step_bar = nullptr;  // grid-barrier counters of the MoE-step and dense-step kernels
    unsigned long long *step_done = nullptr; // completion counters of the MoE-step kernel (top_k + 1)
    bool fused_moe = false;                  // MoE layers run as one kernel (moe_step.cu)
    uint16_t *kv = nullptr;  // 4 planes: k_hi, k_lo, v_hi, v_lo, each [L][heads][kv_max][hd]
    float *cos_t = nullptr, *sin_t = nullptr;
    std::vector<int> lo_start;  // per layer: rows below are exact BF16
    int host_len = 0;
    cudaGraphExec_t graph = nullptr, graph_final = nullptr;
    // persistent-kernel engine (mega.cu)
    bool mega = false;
    bool mega_dirty = true;     // parameter block must be re-uploaded
    bool xa_staged = false;     // the host staged the next step's input embedding in xa
    int mega_grid = 0;
    MegaParams *mega_dp = nullptr;
    MegaLayer *mega_dl = nullptr;
    float *att_sc = nullptr, *att_part = nullptr, *att_sum = nullptr;
    unsigned *bar = nullptr;
    long long *trace = nullptr;
    bool pdl = true;
    int launches = 0;
    // LM-head selection with sampling settings (select.cu); history of the
    // generated tokens, kept in every mode
    float rp = 1.f, temperature = 0.f;
    int ngram = 0;
    int hist_cap = 0;
    int *hist = nullptr, *hist_len = nullptr, *sel_full = nullptr, *unif_pos = nullptr;
    float *hval = nullptr, *bval = nullptr, *logits = nullptr, *unif = nullptr;
    int unif_n = 0;       // uniforms supplied
    int unif_used = 0;    // uniforms consumed by launched steps (host count)
    bool sampling() const { return rp > 1.f || ngram > 0 || temperature > 0.f; }
    // V3's reference sliding-window attention: window, prefill length
    int swa_window = 0, swa_ref = 0;
    // whole-decoder prefill: fused [wq; wk; wv] per layer and the dense
    // layers' gate/up and down with the width padded to a multiple of 128
    // (built on first use), and a workspace for pf_cap tokens
    std::vector<uint16_t *> pf_wqkv, pf_dgu, pf_ddown, pf_router;  // router: zero-padded to 256 rows
    int pf_dpad = 0;
    int pf_cap = 0;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_att = nullptr, *pf_y = nullptr;
    float *pf_lg = nullptr;  // router logits [tokens x 256]
    uint16_t *pf_ahi = nullptr, *pf_alo = nullptr, *pf_hhi = nullptr, *pf_hlo = nullptr;
    std::vector<void *> allocs;

    size_t plane_elems() const {
        return (size_t)cfg.n_layers * cfg.n_heads * cfg.kv_max * cfg.head_dim;
    }
    uint16_t *plane(int p, int l) const {
        return kv + p * plane_elems() + (size_t)l * cfg.n_heads * cfg.kv_max * cfg.head_dim;
    }
};

static void drop_graphs(DecoderModel *m) {
    m->mega_dirty = true;
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->graph_final) cudaGraphExecDestroy(m->graph_final);
    m->graph = m->graph_final = nullptr;
}

static void free_model(DecoderModel *m) {
    drop_graphs(m);
    for (auto *v : {&m->pf_wqkv, &m->pf_dgu, &m->pf_ddown, &m->pf_router})
        for (uint16_t *p : *v) cudaFree(p);
    void *ws[] = {m->pf_x, m->pf_qkv, m->pf_q, m->pf_att, m->pf_y, m->pf_ahi, m->pf_alo, m->pf_hhi, m->pf_hlo,
                  m->pf_lg};
    for (void *p : ws) cudaFree(p);
    for (void *p : m->allocs) cudaFree(p);
    delete m;
}

void ctx_release_models(ds_cuda_ctx *c) {
    for (auto &kv : c->models) free_model(kv.second);
    c->models.clear();
}

static DecoderModel *get_model(ds_cuda_ctx *c, int id) {
    auto it = c->models.find(id);
    return it == c->models.end() ? nullptr : it->second;
}

template <typename T>
static int dalloc(ds_cuda_ctx *c, DecoderModel *m, T **p, size_t elems) {
    void *d = nullptr;
    if (cudaMalloc(&d, elems * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return ctx_fail(c, DS_CUDA_ENOMEM, "decoder: cudaMalloc(%zu) failed", elems * sizeof(T));
    }
    cudaMemset(d, 0, elems * sizeof(T));
    m->allocs.push_back(d);
    *p = (T *)d;
    return DS_CUDA_OK;
}

#define CK(expr)                 \
    do {                         \
        int _rc = (expr);        \
        if (_rc < 0) return _rc; \
    } while (0)
#define CKL(expr, what)                                             \
    do {                                                            \
        cudaError_t _e = (expr);                                    \
        if (_e != cudaSuccess) return ctx_cuda(c, _e, what);        \
    } while (0)

// All kernels of one decode step, in dependency order.
static int enqueue_step(ds_cuda_ctx *c, DecoderModel *m, cudaStream_t st, bool with_final) {
    const auto &g = m->cfg;
    const int H = g.hidden, NH = g.n_heads, HD = g.head_dim;
    const bool pdl = m->pdl;
    int launches = 0;
    for (int l = 0; l < g.n_layers; l++) {
        const DecLayer &L = m->layers[l];
        QkvArgs qa = {};
        qa.x = m->xa;
        qa.norm_w = L.in_norm;
        qa.eps = g.rms_eps;
        qa.hidden = H;
        qa.w[0] = L.wq;
        qa.w[1] = L.wk;
        qa.w[2] = L.wv;
        qa.cos_t = m->cos_t;
        qa.sin_t = m->sin_t;
        qa.d_pos = m->pos;
        qa.q_out = m->q;
        qa.k_hi = m->plane(0, l);
        qa.k_lo = m->plane(1, l);
        qa.v_hi = m->plane(2, l);
        qa.v_lo = m->plane(3, l);
        qa.kv_max = g.kv_max;
        qa.n_heads = NH;
        qa.head_dim = HD;
        qa.pos_ready = l > 0 ? 1 : 0;  // layer 0 follows the step-advance kernel that writes it
        if (L.dense && m->fused_moe) {
            // the dense FFN's weights into L2 while QKV, attention and the
            // O-projection (latency-bound) leave the HBM idle
            qa.pf[0] = L.dgate;
            qa.pf[1] = L.dup;
            qa.pf[2] = L.ddown;
            qa.pf_bytes[0] = qa.pf_bytes[1] = qa.pf_bytes[2] = (size_t)g.dense_inter * H * 2;
        }
        CKL(launch_qkv_rope(qa, st, pdl), "qkv launch");
        AttnArgs aa = {};
        aa.q = m->q;
        aa.k_hi = qa.k_hi;
        aa.k_lo = qa.k_lo;
        aa.v_hi = qa.v_hi;
        aa.v_lo = qa.v_lo;
        aa.kv_max = g.kv_max;
        aa.n_heads = NH;
        aa.d_pos = m->pos;
        aa.lo_start = m->lo_start[l];
        aa.scale = 1.0f / sqrtf((float)HD);
        aa.out = m->attn;
        aa.swa_window = m->swa_window;
        aa.swa_ref = m->swa_ref;
        if (m->fused_moe && aa.swa_window <= 0) CKL(launch_attn_step(aa, st, pdl), "attention launch");
        else CKL(launch_attn_decode(aa, st, pdl), "attention launch");
        MvArgs oa = {};
        oa.W = L.wo;
        oa.x = m->attn;
        oa.resid = m->xa;
        oa.y = m->xb;
        oa.rows = H;
        oa.n = NH * HD;
        // MoE layers: the router rides in the O-proj (its logits are linear in
        // the O-proj output; the last CTA applies the RMS scale and the top-k)
        const bool fold = !L.dense && g.use_int8 == 0 && H % 16 == 0 && g.n_experts <= 255;
        const bool fused = fold && m->fused_moe;
        if (fold) {
            oa.rf.Wr = L.router;
            oa.rf.g = L.post_norm;
            oa.rf.eps = g.rms_eps;
            oa.rf.E = g.n_experts;
            oa.rf.top_k = g.top_k;
            oa.rf.renorm = c->renorm;
            oa.rf.part = m->rpart;
            oa.rf.ticket = m->tickets + 1;
            oa.rf.scores = m->scores;
            oa.rf.d_idx = m->idx;
            oa.rf.d_wt = m->wt;
            oa.rf.no_tail = fused ? 1 : 0;  // the MoE-step kernel reduces the parts itself
        }
        CKL(launch_matvec_res(oa, st, pdl), "o-proj launch");
        launches += 3;
        if (fused) {
            MoeStepArgs ms = {};
            ms.H = H;
            ms.I = g.moe_inter;
            ms.S = g.n_shared * g.moe_inter;
            ms.E = g.n_experts;
            ms.K = g.top_k;
            ms.simulate = c->simulate;
            ms.renorm = c->renorm;
            ms.eps = g.rms_eps;
            ms.x = m->xb;
            ms.norm_w = L.post_norm;
            ms.rpart = m->rpart;
            ms.nparts = (H + 15) / 16;
            ms.block = L.block;
            ms.down = L.down;
            ms.sdown = L.sdown;
            ms.h = m->h;
            ms.out = m->xa;
            ms.d_idx = m->idx;
            ms.d_wt = m->wt;
            ms.scores = m->scores;
            ms.bar = m->step_bar;
            ms.done = m->step_done;
            ms.err = m->tickets + 9;
            if (l + 1 < g.n_layers) {
                const DecLayer &N = m->layers[l + 1];
                ms.pf[0] = N.wq;
                ms.pf[1] = N.wk;
                ms.pf[2] = N.wv;
                ms.pf_bytes = (size_t)NH * HD * H * 2;
            }
            CKL(launch_moe_step(ms, c->sm_count, st, pdl), "moe step launch");
            launches += 1;
            continue;
        }
        if (L.dense && m->fused_moe && dense_step_supported(H, g.dense_inter, c->sm_count)) {
            DenseStepArgs ds = {};
            ds.H = H;
            ds.D = g.dense_inter;
            ds.eps = g.rms_eps;
            ds.x = m->xb;
            ds.norm_w = L.post_norm;
            ds.gate = L.dgate;
            ds.up = L.dup;
            ds.down = L.ddown;
            ds.h = m->h;
            ds.out = m->xa;
            ds.bar = m->step_bar + 1;
            ds.err = m->tickets + 9;
            if (l + 1 < g.n_layers) {
                const DecLayer &N = m->layers[l + 1];
                ds.pf[0] = N.wq;
                ds.pf[1] = N.wk;
                ds.pf[2] = N.wv;
                ds.pf_bytes = (size_t)NH * HD * H * 2;
            }
            CKL(launch_dense_step(ds, c->sm_count, st, pdl), "dense step launch");
            launches += 1;
        } else if (L.dense) {
            MoeArgs da = {};
            da.hidden = H;
            da.sh_inter = g.dense_inter;
            da.has_shared = 1;
            da.dense = 1;
            da.norm_w = L.post_norm;
            da.eps = g.rms_eps;
            da.sh_gu.w = L.dgate;
            da.sh_up.w = L.dup;
            da.x = m->xb;
            da.h = m->h;
            CKL(launch_moe_gate_up(da, st, pdl), "dense gate_up launch");
            MvArgs dd = {};
            dd.W = L.ddown;
            dd.x = m->h;
            dd.resid = m->xb;
            dd.y = m->xa;
            dd.rows = H;
            dd.n = g.dense_inter;
            CKL(launch_matvec_res(dd, st, pdl), "dense down launch");
            launches += 2;
        } else {
            MoeArgs a = {};
            a.hidden = H;
            a.inter = g.moe_inter;
            a.sh_inter = g.n_shared * g.moe_inter;
            a.top_k = g.top_k;
            a.simulate = c->simulate;
            a.has_shared = a.sh_inter > 0;
            a.norm_w = L.post_norm;
            a.eps = g.rms_eps;
            a.int8 = g.use_int8;
            size_t fused = (size_t)2 * g.moe_inter * H;
            if (g.use_int8) {
                a.gu_base = L.gu;
                a.dn_base = L.dn;
                a.sh_gu = L.sgu;
                a.sh_dn = L.sdn;
            } else {
                a.gu_base.w = L.block;
                a.dn_base.w = L.down;
                a.sh_gu.w = L.block + (size_t)g.n_experts * fused;
                a.sh_dn.w = L.sdown;
            }
            a.gu_stride = (long long)fused;
            a.dn_stride = (long long)H * g.moe_inter;
            a.x = m->xb;
            a.h = m->h;
            a.out = m->xa;
            a.resid = m->xb;
            a.out_mode = 2;
            if (!fold) {
                CKL(launch_router(L.router, m->xb, g.n_experts, H, m->scores, m->tickets + 1, g.top_k, c->renorm,
                                  m->idx, m->wt, st, pdl, L.post_norm, g.rms_eps),
                    "router launch");
                launches += 1;
            }
            a.d_idx = m->idx;
            a.d_wt = m->wt;
            CKL(launch_moe_gate_up(a, st, pdl), "moe gate_up launch");
            CKL(launch_moe_down(a, st, pdl), "moe down launch");
            launches += 2;
        }
    }
    if (with_final) {
        // the final RMS-normed hidden state, for callers that ask for it
        // (the LM-head kernel normalises on load and does not store it)
        CKL(launch_rmsnorm(m->xa, m->final_norm, m->xfinal, H, g.rms_eps, st, pdl), "final norm launch");
        launches += 1;
    }
    if (m->sampling()) {
        if (!with_final) {
            CKL(launch_rmsnorm(m->xa, m->final_norm, m->xfinal, H, g.rms_eps, st, pdl), "final norm launch");
            launches += 1;
        }
        if (m->temperature <= 0.f) {
            CKL(launch_argmax_bf16(m->lm_head, m->xa, g.vocab, H, m->slot, m->tickets + 0, m->tok, m->val, st, pdl,
                                   m->final_norm, g.rms_eps),
                "lm head launch");
            launches += m->rp > 1.f ? 2 : 1;  // the argmax (and the history dots for the penalty)
        }
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
        sa.logits = m->logits;
        sa.tok = m->tok;
        sa.val = m->val;
        sa.full = m->sel_full;
        sa.rp = m->rp;
        sa.ngram = m->ngram;
        sa.temperature = m->temperature;
        sa.unif = m->unif;
        sa.unif_pos = m->unif_pos;
        CKL(launch_select(sa, st), "token selection launch");
        launches += 3;
    } else {
        CKL(launch_argmax_bf16(m->lm_head, m->xa, g.vocab, H, m->slot, m->tickets + 0, m->tok, m->val, st, pdl,
                               m->final_norm, g.rms_eps),
            "lm head launch");
        launches += 1;
    }
    CKL(launch_decode_advance(m->embed, H, m->tok, m->pos, m->tok_log, m->xa, st, pdl, m->hist, m->hist_len,
                              m->hist_cap),
        "advance launch");
    launches += 1;
    m->launches = launches;
    return DS_CUDA_OK;
}

static int capture(ds_cuda_ctx *c, DecoderModel *m, bool with_final, cudaGraphExec_t *out) {
    cudaStream_t st = c->stream;
    for (int attempt = 0; attempt < 2; attempt++) {
        cudaGraph_t graph = nullptr;
        CKL(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture");
        int rc = enqueue_step(c, m, st, with_final);
        cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc < 0) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (e == cudaSuccess) e = cudaGraphInstantiate(out, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (e == cudaSuccess) return DS_CUDA_OK;
        cudaGetLastError();
        if (!m->pdl) return ctx_cuda(c, e, "graph capture");
        m->pdl = false;  // retry without programmatic edges
    }
    return ctx_fail(c, DS_CUDA_ECUDA, "graph capture failed");
}

static int ensure_graph(ds_cuda_ctx *c, DecoderModel *m, bool with_final) {
    cudaGraphExec_t *g = with_final ? &m->graph_final : &m->graph;
    if (*g) return DS_CUDA_OK;
    return capture(c, m, with_final, g);
}

// ---------------------------------------------------------------------------
// Persistent-kernel engine: parameter block upload and launch
// ---------------------------------------------------------------------------
static MegaParams mega_params(ds_cuda_ctx *c, DecoderModel *m) {
    const auto &g = m->cfg;
    MegaParams p = {};
    p.H = g.hidden;
    p.NH = g.n_heads;
    p.HD = g.head_dim;
    p.D = g.dense_inter;
    p.I = g.moe_inter;
    p.E = g.n_experts;
    p.S = g.n_shared * g.moe_inter;
    p.K = g.top_k;
    p.V = g.vocab;
    p.L = g.n_layers;
    p.kv_max = g.kv_max;
    p.eps = g.rms_eps;
    p.scale = 1.0f / sqrtf((float)g.head_dim);
    p.simulate = c->simulate;
    p.renorm = c->renorm;
    p.layers = m->mega_dl;
    p.final_norm = m->final_norm;
    p.lm_head = m->lm_head;
    p.embed = m->embed;
    p.cos_t = m->cos_t;
    p.sin_t = m->sin_t;
    p.xa = m->xa;
    p.xb = m->xb;
    p.q = m->q;
    p.att_sc = m->att_sc;
    p.att_part = m->att_part;
    p.att_sum = m->att_sum;
    p.h = m->h;
    p.rscore = m->scores;
    p.slot = m->slot;
    p.bar = m->bar;
    p.pos = m->pos;
    p.tok = m->tok;
    p.tok_log = m->tok_log;
    p.val = m->val;
    return p;
}

// Enqueues n_steps greedy steps as one persistent-kernel launch.
static int mega_run(ds_cuda_ctx *c, DecoderModel *m, int n_steps, bool first_from_token, float *final_x,
                    cudaStream_t st) {
    if (m->mega_dirty) {
        std::vector<MegaLayer> hl(m->cfg.n_layers);
        for (int l = 0; l < m->cfg.n_layers; l++) {
            const DecLayer &L = m->layers[l];
            MegaLayer &d = hl[l];
            d.wq = L.wq;
            d.wk = L.wk;
            d.wv = L.wv;
            d.wo = L.wo;
            d.in_norm = L.in_norm;
            d.post_norm = L.post_norm;
            d.dense = L.dense;
            d.dgate = L.dgate;
            d.dup = L.dup;
            d.ddown = L.ddown;
            d.router = L.router;
            d.block = L.block;
            d.down = L.down;
            d.sdown = L.sdown;
            d.k_hi = m->plane(0, l);
            d.k_lo = m->plane(1, l);
            d.v_hi = m->plane(2, l);
            d.v_lo = m->plane(3, l);
            d.lo_start = m->lo_start[l];
        }
        CKL(cudaMemcpyAsync(m->mega_dl, hl.data(), hl.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice, st),
            "mega layers upload");
        CKL(cudaStreamSynchronize(st), "mega layers upload");
        m->mega_dirty = false;
    }
    // the per-launch fields travel in a fresh parameter block each launch
    // (stream-ordered copy from pinned staging)
    MegaParams p = mega_params(c, m);
    p.n_steps = n_steps;
    p.first_from_token = first_from_token ? 1 : 0;
    p.final_x = final_x;
    // phase timing trace for performance work (DS_CUDA_MEGA_TRACE=<file>)
    static const char *trace_file = getenv("DS_CUDA_MEGA_TRACE");
    if (trace_file) {
        if (!m->trace) CK(dalloc(c, m, &m->trace, (size_t)2 * 4096 * 5));
        CKL(cudaMemsetAsync(m->trace, 0, (size_t)2 * 4096 * 5 * 8, st), "trace reset");
        p.trace = m->trace;
        p.trace_cap = 4096;
    }
    CK(ctx_pinned(c, sizeof(MegaParams) + 64));
    CKL(cudaStreamSynchronize(st), "mega params staging");  // the staging buffer may be in use
    memcpy(c->pin, &p, sizeof p);
    CKL(cudaMemcpyAsync(m->mega_dp, c->pin, sizeof p, cudaMemcpyHostToDevice, st), "mega params upload");
    CKL(cudaMemsetAsync(m->slot, 0, 2 * sizeof(unsigned long long), st), "slot reset");
    CKL(cudaMemsetAsync(m->bar, 0, 3 * sizeof(unsigned), st), "barrier reset");
    CKL(launch_mega(m->mega_dp, m->mega_grid, st), "persistent decode launch");
    return DS_CUDA_OK;
}

static int mega_check(ds_cuda_ctx *c, DecoderModel *m) {
    unsigned e = 0;
    CKL(cudaMemcpy(&e, m->bar + 2, sizeof e, cudaMemcpyDeviceToHost), "error flag read");
    static const char *trace_file = getenv("DS_CUDA_MEGA_TRACE");
    if (trace_file && m->trace) {
        std::vector<long long> t((size_t)2 * 4096 * 5);
        cudaMemcpy(t.data(), m->trace, t.size() * 8, cudaMemcpyDeviceToHost);
        if (FILE *f = fopen(trace_file, "w")) {
            for (int s = 0; s < 2; s++)
                for (int i = 0; i < 4096; i++) {
                    const long long *r = &t[((size_t)s * 4096 + i) * 5];
                    if (!r[4]) continue;
                    fprintf(f, "%d,%d,%lld,%lld,%lld,%lld,%lld\n", s, i, r[0], r[1], r[2], r[3], r[4]);
                }
            fclose(f);
        }
    }
    if (e) return ctx_fail(c, DS_CUDA_ETIMEOUT, "persistent decode: a bounded device-side wait gave up");
    return DS_CUDA_OK;
}

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
#define LOOK(ptr, bytes) ctx_lookup(c, (ptr), (bytes), true)

extern "C" int ds_cuda_decoder_create(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg,
                                      const ds_cuda_layer_weights_t *lw, const float *final_norm,
                                      const uint16_t *lm_head) {
    if (!c || !cfg || !lw || !final_norm || !lm_head) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_create: null argument");
    const auto &g = *cfg;
    if (g.head_dim != 128 || g.hidden % 16 || g.hidden > 2048 || g.n_heads * g.head_dim > 2048 ||
        g.kv_max <= 0 || g.kv_max > 4096 || g.n_layers <= 0 || g.moe_inter % 16 || g.top_k > 6 ||
        g.n_experts > 256 || g.dense_inter % 8 || g.dense_inter > 8192 || g.vocab <= 0)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_create: unsupported configuration");
    cudaSetDevice(c->device);
    DecoderModel *m = new DecoderModel();
    m->cfg = g;
    const size_t H = g.hidden, QD = (size_t)g.n_heads * g.head_dim, I = g.moe_inter, S = (size_t)g.n_shared * I;
    const size_t E = g.n_experts;
    int rc = DS_CUDA_OK;
    for (int l = 0; l < g.n_layers && rc == DS_CUDA_OK; l++) {
        const ds_cuda_layer_weights_t &w = lw[l];
        DecLayer L = {};
        L.wq = (const uint16_t *)LOOK(w.wq, QD * H * 2);
        L.wk = (const uint16_t *)LOOK(w.wk, QD * H * 2);
        L.wv = (const uint16_t *)LOOK(w.wv, QD * H * 2);
        L.wo = (const uint16_t *)LOOK(w.wo, H * QD * 2);
        L.in_norm = (const float *)LOOK(w.input_norm, H * 4);
        L.post_norm = (const float *)LOOK(w.post_attn_norm, H * 4);
        L.dense = l < g.first_dense;
        bool ok = L.wq && L.wk && L.wv && L.wo && L.in_norm && L.post_norm;
        if (L.dense) {
            size_t D = g.dense_inter;
            L.dgate = (const uint16_t *)LOOK(w.dense_gate, D * H * 2);
            L.dup = (const uint16_t *)LOOK(w.dense_up, D * H * 2);
            L.ddown = (const uint16_t *)LOOK(w.dense_down, H * D * 2);
            ok = ok && L.dgate && L.dup && L.ddown;
        } else {
            L.router = (const uint16_t *)LOOK(w.router, E * H * 2);
            ok = ok && L.router;
            if (g.use_int8) {
                L.gu = WMat{LOOK(w.gu_q, E * 2 * I * H), (const float *)LOOK(w.gu_scale, E * 2 * I * 4),
                            (const float *)LOOK(w.gu_off, E * 2 * I * 4)};
                L.dn = WMat{LOOK(w.dn_q, E * H * I), (const float *)LOOK(w.dn_scale, E * H * 4),
                            (const float *)LOOK(w.dn_off, E * H * 4)};
                L.sgu = WMat{LOOK(w.sgu_q, 2 * S * H), (const float *)LOOK(w.sgu_scale, 2 * S * 4),
                             (const float *)LOOK(w.sgu_off, 2 * S * 4)};
                L.sdn = WMat{LOOK(w.sdn_q, H * S), (const float *)LOOK(w.sdn_scale, H * 4),
                             (const float *)LOOK(w.sdn_off, H * 4)};
                ok = ok && L.gu.w && L.gu.scale && L.gu.off && L.dn.w && L.dn.scale && L.dn.off && L.sgu.w &&
                     L.sgu.scale && L.sgu.off && L.sdn.w && L.sdn.scale && L.sdn.off;
            } else {
                L.block = (const uint16_t *)LOOK(w.expert_block, (E * 2 * I * H + 2 * S * H) * 2);
                L.down = (const uint16_t *)LOOK(w.down, E * H * I * 2);
                L.sdown = (const uint16_t *)LOOK(w.shared_down, H * S * 2);
                ok = ok && L.block && L.down && L.sdown;
            }
        }
        if (!ok) rc = ctx_fail(c, DS_CUDA_ENOTREG, "decoder_create: layer %d weights missing or not registrable", l);
        m->layers.push_back(L);
    }
    if (rc == DS_CUDA_OK) {
        m->final_norm = (const float *)LOOK(final_norm, H * 4);
        m->lm_head = (const uint16_t *)LOOK(lm_head, (size_t)g.vocab * H * 2);
        if (!m->final_norm || !m->lm_head) rc = ctx_fail(c, DS_CUDA_ENOTREG, "decoder_create: head weights");
        m->embed = m->lm_head;
    }
    size_t hcap = std::max((size_t)g.top_k * I + S, (size_t)g.dense_inter);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->xa, H);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->xb, H);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->xfinal, H);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->q, QD);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->attn, QD);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->h, hcap);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->scores, 256);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->rpart, (size_t)rf_pstride((H + 15) / 16) * (g.n_experts + 1));
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->wt, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->val, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->idx, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->pos, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->tok, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->tok_log, (size_t)g.kv_max + 16);
    // the generated-token history holds as many tokens as the reference's
    // (max_seq + 512, ds_ocr.c:894)
    m->hist_cap = g.kv_max + 512;
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->hist, (size_t)m->hist_cap);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->hval, (size_t)m->hist_cap);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->unif, (size_t)m->hist_cap);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->hist_len, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->sel_full, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->unif_pos, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->bval, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->logits, (size_t)g.vocab);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->tickets, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->slot, 16);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->step_bar, 2);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->step_done, 16);
    if (rc == DS_CUDA_OK) {
        // the MoE block as one kernel where its shapes allow (BF16 experts);
        // DS_CUDA_DECODE_PER_PHASE=1 keeps the per-phase kernels (same numerics)
        const char *pp = getenv("DS_CUDA_DECODE_PER_PHASE");
        m->fused_moe = !(pp && pp[0] == '1') && !g.use_int8 && g.engine == 0 &&
                       moe_step_supported(g.hidden, g.moe_inter, g.n_shared * g.moe_inter, g.n_experts, g.top_k,
                                          c->sm_count);
    }
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->kv, 4 * m->plane_elems());
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->cos_t, (size_t)g.kv_max * g.head_dim);
    if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->sin_t, (size_t)g.kv_max * g.head_dim);
    if (rc == DS_CUDA_OK) {
        // RoPE cos/sin cache exactly as ds_compute_rope_neox (ds_kernels.c:2399-2424)
        // over positions 0..kv_max-1 (ds_ocr.c:934-941), in host float math.
        std::vector<float> cs((size_t)g.kv_max * g.head_dim), sn(cs.size());
        int half = g.head_dim / 2;
        for (int s = 0; s < g.kv_max; s++) {
            float p = (float)s;
            for (int d = 0; d < half; d++) {
                float freq = 1.0f / powf(g.rope_theta, (float)(2 * d) / (float)g.head_dim);
                float ang = p * freq;
                float cv = cosf(ang), sv = sinf(ang);
                cs[(size_t)s * g.head_dim + d] = cv;
                cs[(size_t)s * g.head_dim + d + half] = cv;
                sn[(size_t)s * g.head_dim + d] = sv;
                sn[(size_t)s * g.head_dim + d + half] = sv;
            }
        }
        cudaMemcpy(m->cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(m->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
        m->lo_start.assign(g.n_layers, 0);
    }
    if (rc == DS_CUDA_OK && g.engine == 1) {
        // the persistent kernel is specialised for hidden = heads*head_dim =
        // 1280 (5 x 256-column register slices) and BF16 experts
        int G = mega_grid(c->device);
        int S = g.n_shared * g.moe_inter;
        // one gate/up pair plus the CTA's router rows must fit one 46 KB region
        bool fits = G >= g.n_heads && 4 * g.hidden + ((g.n_experts + G - 1) / G) * 2 * g.hidden <= 46 * 1024 &&
                    2 * g.dense_inter <= 46 * 1024 && 2 * (g.top_k * g.moe_inter + S) <= 46 * 1024;
        if (g.use_int8 || g.hidden != 1280 || g.n_heads * g.head_dim != 1280 || g.top_k > 8 ||
            g.top_k * g.moe_inter + S > 8192 || g.dense_inter > 8192 || !fits) {
            rc = ctx_fail(c, DS_CUDA_EINVAL, "decoder_create: configuration not supported by the persistent engine "
                                             "(use engine = 0)");
        } else {
            m->mega = true;
            m->mega_grid = G;
            rc = dalloc(c, m, &m->att_sc, (size_t)g.n_heads * g.kv_max);
            if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->att_part, (size_t)g.n_heads * G * g.head_dim);
            if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->att_sum, 64);
            if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->bar, 16);
            if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->mega_dl, (size_t)g.n_layers);
            if (rc == DS_CUDA_OK) rc = dalloc(c, m, &m->mega_dp, 1);
        }
    }
    if (rc != DS_CUDA_OK) {
        free_model(m);
        return rc;
    }
    int id = c->next_model++;
    c->models[id] = m;
    return id;
}

extern "C" int ds_cuda_decoder_destroy(ds_cuda_ctx_t *c, int id) {
    if (!c) return DS_CUDA_EINVAL;
    DecoderModel *m = get_model(c, id);
    if (!m) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_destroy: unknown model %d", id);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    c->models.erase(id);
    free_model(m);
    return DS_CUDA_OK;
}

static inline uint16_t f2bf_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

extern "C" int ds_cuda_decoder_load_kv(ds_cuda_ctx_t *c, int id, int layer, int pos0, int n, const float *k,
                                       const float *v) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || !k || !v || layer < 0 || layer >= m->cfg.n_layers || pos0 < 0 || n <= 0 || pos0 + n > m->cfg.kv_max)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_load_kv: bad argument");
    cudaSetDevice(c->device);
    const int NH = m->cfg.n_heads, HD = m->cfg.head_dim;
    std::vector<uint16_t> hi((size_t)n * HD), lo((size_t)n * HD);
    bool exact = true;
    for (int which = 0; which < 2; which++) {
        const float *src = which == 0 ? k : v;
        for (int h = 0; h < NH; h++) {
            for (int i = 0; i < n; i++)
                for (int d = 0; d < HD; d++) {
                    float f = src[(size_t)i * NH * HD + (size_t)h * HD + d];
                    uint16_t a = f2bf_rne(f);
                    uint32_t au = (uint32_t)a << 16;
                    float af;
                    memcpy(&af, &au, 4);
                    uint16_t b = f2bf_rne(f - af);
                    hi[(size_t)i * HD + d] = a;
                    lo[(size_t)i * HD + d] = b;
                    if (b != 0) exact = false;
                }
            size_t off = ((size_t)h * m->cfg.kv_max + pos0) * HD;
            CKL(cudaMemcpy(m->plane(which * 2, layer) + off, hi.data(), hi.size() * 2, cudaMemcpyHostToDevice), "kv copy");
            CKL(cudaMemcpy(m->plane(which * 2 + 1, layer) + off, lo.data(), lo.size() * 2, cudaMemcpyHostToDevice), "kv copy");
        }
    }
    // the lo plane may be skipped below lo_start only while every row there is exact
    int &ls = m->lo_start[layer];
    int new_ls = ls;
    if (exact && pos0 <= ls) new_ls = std::max(ls, pos0 + n);
    if (!exact && pos0 < ls) new_ls = pos0;
    if (new_ls != ls) {
        ls = new_ls;
        drop_graphs(m);  // lo_start is baked into the captured graph
    }
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_decoder_set_len(ds_cuda_ctx_t *c, int id, int len) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || len < 0 || len >= m->cfg.kv_max) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_len: bad argument");
    cudaSetDevice(c->device);
    // rows at or beyond len will be rewritten by decode steps with F32 values
    for (int l = 0; l < m->cfg.n_layers; l++)
        if (m->lo_start[l] > len) {
            m->lo_start[l] = len;
            drop_graphs(m);
        }
    CKL(cudaMemcpyAsync(m->pos, &len, sizeof(int), cudaMemcpyHostToDevice, c->stream), "set len");
    CKL(cudaStreamSynchronize(c->stream), "set len");
    m->host_len = len;
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_decoder_get_len(ds_cuda_ctx_t *c, int id) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_get_len: unknown model");
    return m->host_len;
}

extern "C" int ds_cuda_decoder_forward(ds_cuda_ctx_t *c, int id, const float *embed, float *final_x, float *logit) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || !embed) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_forward: bad argument");
    if (m->host_len + 1 > m->cfg.kv_max) return ctx_fail(c, DS_CUDA_ESTATE, "decoder_forward: KV cache full");
    if (m->temperature > 0.f && m->unif_used + 1 > m->unif_n)
        return ctx_fail(c, DS_CUDA_ESTATE, "decoder_forward: no uniform left for temperature sampling");
    cudaSetDevice(c->device);
    const int H = m->cfg.hidden;
    if (!m->mega) CK(ensure_graph(c, m, final_x != nullptr));
    CK(ctx_pinned(c, (size_t)H * 8 + 64 + sizeof(MegaParams)));
    memcpy(c->pin, embed, (size_t)H * 4);
    CKL(cudaMemcpyAsync(m->xa, c->pin, (size_t)H * 4, cudaMemcpyHostToDevice, c->stream), "embed copy");
    if (m->mega) {
        CK(mega_run(c, m, 1, false, final_x ? m->xfinal : nullptr, c->stream));
    } else {
        CKL(cudaGraphLaunch(final_x ? m->graph_final : m->graph, c->stream), "graph launch");
    }
    char *pb = (char *)c->pin;
    CKL(cudaMemcpyAsync(pb, m->tok, 4, cudaMemcpyDeviceToHost, c->stream), "token copy");
    CKL(cudaMemcpyAsync(pb + 4, m->val, 4, cudaMemcpyDeviceToHost, c->stream), "logit copy");
    CKL(cudaMemcpyAsync(pb + 8, m->tickets + 8, 8, cudaMemcpyDeviceToHost, c->stream), "error flags copy");
    if (final_x) CKL(cudaMemcpyAsync(pb + 64, m->xfinal, (size_t)H * 4, cudaMemcpyDeviceToHost, c->stream), "x copy");
    CKL(cudaStreamSynchronize(c->stream), "decoder_forward");
    if (m->mega) CK(mega_check(c, m));
    unsigned flags[2];
    memcpy(flags, pb + 8, 8);
    if (flags[0] | flags[1]) return ctx_fail(c, DS_CUDA_ETIMEOUT, "decoder_forward: a bounded device-side wait gave up");
    int tok;
    memcpy(&tok, pb, 4);
    if (logit) memcpy(logit, pb + 4, 4);
    if (final_x) memcpy(final_x, pb + 64, (size_t)H * 4);
    m->host_len++;
    if (m->temperature > 0.f) m->unif_used++;
    return tok;
}

extern "C" int ds_cuda_decoder_generate_dev(ds_cuda_ctx_t *c, int id, int n_steps, void *stream) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || n_steps < 0) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_generate_dev: bad argument");
    if (m->host_len + n_steps > m->cfg.kv_max) return ctx_fail(c, DS_CUDA_ESTATE, "decoder_generate: KV cache full");
    if (m->temperature > 0.f && m->unif_used + n_steps > m->unif_n)
        return ctx_fail(c, DS_CUDA_ESTATE, "decoder_generate: %d uniforms left for %d temperature-sampled steps",
                        m->unif_n - m->unif_used, n_steps);
    cudaSetDevice(c->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    if (n_steps == 0) return DS_CUDA_OK;
    if (m->mega) {
        // step 0 consumes the embedding of the last token the model produced
        // (or the one ds_cuda_decoder_generate staged in xa)
        CK(mega_run(c, m, n_steps, !m->xa_staged, nullptr, st));
        m->xa_staged = false;
    } else {
        CK(ensure_graph(c, m, false));
        for (int s = 0; s < n_steps; s++) CKL(cudaGraphLaunch(m->graph, st), "graph launch");
    }
    m->host_len += n_steps;
    if (m->temperature > 0.f) m->unif_used += n_steps;
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_decoder_generate(ds_cuda_ctx_t *c, int id, const float *first_embed, int n_steps,
                                        int *tokens) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || n_steps <= 0 || !tokens) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_generate: bad argument");
    cudaSetDevice(c->device);
    const int H = m->cfg.hidden;
    int start = m->host_len;
    if (first_embed) {
        CK(ctx_pinned(c, (size_t)H * 4));
        memcpy(c->pin, first_embed, (size_t)H * 4);
        CKL(cudaMemcpyAsync(m->xa, c->pin, (size_t)H * 4, cudaMemcpyHostToDevice, c->stream), "embed copy");
        m->xa_staged = true;
    }
    CK(ds_cuda_decoder_generate_dev(c, id, n_steps, nullptr));
    CKL(cudaMemcpyAsync(tokens, m->tok_log + start, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, c->stream),
        "token copy");
    CKL(cudaStreamSynchronize(c->stream), "decoder_generate");
    if (m->mega) CK(mega_check(c, m));
    unsigned flags[2];
    CKL(cudaMemcpy(flags, m->tickets + 8, 8, cudaMemcpyDeviceToHost), "error flags read");
    if (flags[0] | flags[1]) return ctx_fail(c, DS_CUDA_ETIMEOUT, "decoder_generate: a bounded device-side wait gave up");
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_decoder_launches_per_step(ds_cuda_ctx_t *c, int id) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m) return ctx_fail(c, DS_CUDA_EINVAL, "unknown model");
    if (m->mega) return 0;  // the persistent engine: one launch per generate call, whatever n_steps
    if (!m->launches) CK(ensure_graph(c, m, false));
    return m->launches;
}

// Sampling settings of the LM head (the reference's ctx->repeat_penalty,
// no_repeat_ngram_size and temperature, ds_ocr.h; read by ds_decoder_forward,
// ds_moe_decoder.c:1021-1263). Graph engine only.
extern "C" int ds_cuda_decoder_set_sampling(ds_cuda_ctx_t *c, int id, float repeat_penalty, int no_repeat_ngram_size,
                                            float temperature) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || !(repeat_penalty > 0.f) || no_repeat_ngram_size < 0 || !(temperature >= 0.f))
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_sampling: bad argument");
    const bool on = repeat_penalty > 1.f || no_repeat_ngram_size > 0 || temperature > 0.f;
    if (m->mega && on)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_sampling: the persistent engine decodes greedily only");
    if (m->cfg.hidden % 256) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_sampling: hidden must be a multiple of 256");
    cudaSetDevice(c->device);
    CKL(cudaStreamSynchronize(c->stream), "set sampling");
    m->rp = repeat_penalty;
    m->ngram = no_repeat_ngram_size;
    m->temperature = temperature;
    drop_graphs(m);
    return DS_CUDA_OK;
}

// Replaces the generated-token history (the reference's ctx->token_history;
// its generation loop appends every produced token, ds_ocr.c:2245-2248, and
// so does each decode step here).
extern "C" int ds_cuda_decoder_set_history(ds_cuda_ctx_t *c, int id, const int *tokens, int n) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || n < 0 || n > m->hist_cap || (n > 0 && !tokens))
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_history: bad argument");
    cudaSetDevice(c->device);
    CKL(cudaStreamSynchronize(c->stream), "set history");
    if (n) CKL(cudaMemcpy(m->hist, tokens, (size_t)n * 4, cudaMemcpyHostToDevice), "history copy");
    CKL(cudaMemcpy(m->hist_len, &n, 4, cudaMemcpyHostToDevice), "history length");
    return DS_CUDA_OK;
}

// Copies up to cap history tokens out; returns the history length.
extern "C" int ds_cuda_decoder_get_history(ds_cuda_ctx_t *c, int id, int *tokens, int cap) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || cap < 0 || (cap > 0 && !tokens)) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_get_history: bad argument");
    cudaSetDevice(c->device);
    CKL(cudaStreamSynchronize(c->stream), "get history");
    int n = 0;
    CKL(cudaMemcpy(&n, m->hist_len, 4, cudaMemcpyDeviceToHost), "history length");
    const int k = n < cap ? n : cap;
    if (k > 0) CKL(cudaMemcpy(tokens, m->hist, (size_t)k * 4, cudaMemcpyDeviceToHost), "history copy");
    return n;
}

// Uniforms in [0, 1] for temperature sampling, one consumed per sampled step
// in order (the reference draws (float)rand() / RAND_MAX each step,
// ds_moe_decoder.c:1251). Replaces any unconsumed ones.
extern "C" int ds_cuda_decoder_set_uniforms(ds_cuda_ctx_t *c, int id, const float *u, int n) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || n < 0 || n > m->hist_cap || (n > 0 && !u))
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_uniforms: bad argument (at most %d)", m ? m->hist_cap : 0);
    cudaSetDevice(c->device);
    CKL(cudaStreamSynchronize(c->stream), "set uniforms");
    if (n) CKL(cudaMemcpy(m->unif, u, (size_t)n * 4, cudaMemcpyHostToDevice), "uniform copy");
    const int zero = 0;
    CKL(cudaMemcpy(m->unif_pos, &zero, 4, cudaMemcpyHostToDevice), "uniform position");
    m->unif_n = n;
    m->unif_used = 0;
    return DS_CUDA_OK;
}

// V3's reference sliding-window decode attention (R-SWA): the reference's
// cfg->sliding_window_size and ctx->prefill_token_count (ds_ocr.h), read by
// decoder_layer_forward (ds_moe_decoder.c:409-436). 0 disables. Graph
// engine only.
extern "C" int ds_cuda_decoder_set_window(ds_cuda_ctx_t *c, int id, int sliding_window_size,
                                          int prefill_token_count) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || sliding_window_size < 0 || prefill_token_count < 0)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_window: bad argument");
    if (m->mega && sliding_window_size > 0)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_window: the persistent engine attends causally only");
    cudaSetDevice(c->device);
    CKL(cudaStreamSynchronize(c->stream), "set window");
    m->swa_window = sliding_window_size;
    m->swa_ref = prefill_token_count;
    drop_graphs(m);
    return DS_CUDA_OK;
}

// The token embedding table the step advance reads the next input from
// (the reference's tok_embeddings_bf16, ds_ocr.c:2272-2279); by default the
// LM head (tied embeddings). Host pointer to [vocab x hidden] BF16.
extern "C" int ds_cuda_decoder_set_embeddings(ds_cuda_ctx_t *c, int id, const uint16_t *embed_tokens) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || !embed_tokens) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_set_embeddings: bad argument");
    cudaSetDevice(c->device);
    const void *d = ctx_lookup(c, embed_tokens, (size_t)m->cfg.vocab * m->cfg.hidden * 2, true);
    if (!d) return ctx_fail(c, DS_CUDA_ENOTREG, "decoder_set_embeddings: table not registrable");
    CKL(cudaStreamSynchronize(c->stream), "set embeddings");
    m->embed = (const uint16_t *)d;
    drop_graphs(m);
    return DS_CUDA_OK;
}

// ---------------------------------------------------------------------------
// Whole-decoder prefill (ds_decoder_prefill, ds_moe_decoder.c:480-905): T
// input embeddings at positions len .. len+T-1 through every layer, their
// K/V rows written to this model's cache, and the first generated token
// (LM-head argmax of the last row's final RMSNorm). Per layer: input
// RMSNorm split into BF16 planes; the QKV projection as one tensor-core GEMM
// against [wq; wk; wv]; RoPE and the cache writes; the exact decode
// attention over keys 0 .. len+t for every query (blocks of queries per
// CTA); the O-projection
// GEMM and residual; then the MoE prefill block, or for a dense layer the
// gate/up GEMM with SwiGLU in its epilogue and the down GEMM, and residual.
// ---------------------------------------------------------------------------
static int pf_weights(ds_cuda_ctx *c, DecoderModel *m) {
    if (!m->pf_wqkv.empty()) return DS_CUDA_OK;
    const auto &g = m->cfg;
    const size_t H = g.hidden, QD = (size_t)g.n_heads * g.head_dim, D = g.dense_inter;
    m->pf_dpad = (int)((D + 127) / 128 * 128);
    const size_t Dp = m->pf_dpad;
    cudaStream_t st = c->stream;
    for (int l = 0; l < g.n_layers; l++) {
        const DecLayer &L = m->layers[l];
        uint16_t *w = nullptr;
        CKL(cudaMalloc(&w, 3 * QD * H * 2), "prefill qkv weights");
        m->pf_wqkv.push_back(w);
        CKL(cudaMemcpyAsync(w, L.wq, QD * H * 2, cudaMemcpyDeviceToDevice, st), "qkv copy");
        CKL(cudaMemcpyAsync(w + QD * H, L.wk, QD * H * 2, cudaMemcpyDeviceToDevice, st), "qkv copy");
        CKL(cudaMemcpyAsync(w + 2 * QD * H, L.wv, QD * H * 2, cudaMemcpyDeviceToDevice, st), "qkv copy");
        uint16_t *gu = nullptr, *dn = nullptr;
        if (L.dense) {
            CKL(cudaMalloc(&gu, 2 * Dp * H * 2), "prefill dense weights");
            CKL(cudaMalloc(&dn, H * Dp * 2), "prefill dense weights");
            CKL(cudaMemsetAsync(gu, 0, 2 * Dp * H * 2, st), "dense pad");
            CKL(cudaMemsetAsync(dn, 0, H * Dp * 2, st), "dense pad");
            CKL(cudaMemcpyAsync(gu, L.dgate, D * H * 2, cudaMemcpyDeviceToDevice, st), "dense copy");
            CKL(cudaMemcpyAsync(gu + Dp * H, L.dup, D * H * 2, cudaMemcpyDeviceToDevice, st), "dense copy");
            CKL(cudaMemcpy2DAsync(dn, Dp * 2, L.ddown, D * 2, D * 2, H, cudaMemcpyDeviceToDevice, st), "dense copy");
        }
        m->pf_dgu.push_back(gu);
        m->pf_ddown.push_back(dn);
        uint16_t *rt = nullptr;
        if (!L.dense && g.n_experts <= 256) {
            // the router as a GEMM B operand: E rows, zero rows up to 256
            CKL(cudaMalloc(&rt, (size_t)256 * H * 2), "prefill router weights");
            CKL(cudaMemsetAsync(rt, 0, (size_t)256 * H * 2, st), "router pad");
            CKL(cudaMemcpyAsync(rt, L.router, (size_t)g.n_experts * H * 2, cudaMemcpyDeviceToDevice, st),
                "router copy");
        }
        m->pf_router.push_back(rt);
    }
    // the copies ran on the context's stream; a prefill may run on another
    CKL(cudaStreamSynchronize(st), "prefill weights");
    return DS_CUDA_OK;
}

static int pf_workspace(ds_cuda_ctx *c, DecoderModel *m, int T) {
    if (T <= m->pf_cap) return DS_CUDA_OK;
    void *old[] = {m->pf_x, m->pf_qkv, m->pf_q, m->pf_att, m->pf_y, m->pf_ahi, m->pf_alo, m->pf_hhi, m->pf_hlo,
                   m->pf_lg};
    // an earlier prefill may still be using the old buffers, on any stream
    CKL(cudaDeviceSynchronize(), "prefill workspace");
    for (void *p : old) cudaFree(p);
    const auto &g = m->cfg;
    const size_t n = (size_t)T, H = g.hidden, QD = (size_t)g.n_heads * g.head_dim, Dp = m->pf_dpad;
    const size_t A = std::max(H, QD);
    cudaError_t e = cudaMalloc(&m->pf_x, n * H * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_qkv, n * 3 * QD * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_q, n * QD * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_att, n * QD * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_y, n * H * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_ahi, n * A * 2);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_alo, n * A * 2);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_hhi, n * std::max<size_t>(Dp, 1) * 2);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_hlo, n * std::max<size_t>(Dp, 1) * 2);
    if (e == cudaSuccess) e = cudaMalloc(&m->pf_lg, n * 256 * 4);
    if (e != cudaSuccess) {
        cudaGetLastError();
        m->pf_cap = 0;
        return ctx_fail(c, DS_CUDA_ENOMEM, "decoder_prefill: workspace for %d tokens", T);
    }
    m->pf_cap = T;
    return DS_CUDA_OK;
}

// d_embeds: the input rows in device memory, or null when the caller has
// already placed them in the workspace's x (pf_workspace first).
static int prefill_enqueue(ds_cuda_ctx *c, DecoderModel *m, const float *d_embeds, int T, cudaStream_t st) {
    const auto &g = m->cfg;
    const int H = g.hidden, NH = g.n_heads, HD = g.head_dim, QD = NH * HD;
    if (c->simulate)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_prefill: the BF16-truncation numerics mode is decode-only");
    if (H % 256 || QD % 256 || g.moe_inter % 128 || (g.n_shared * g.moe_inter) % 128)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_prefill: unsupported shape");
    for (const DecLayer &L : m->layers)
        if (!L.dense && (!L.block || !L.down || !L.router || (g.n_shared && !L.sdown)))
            return ctx_fail(c, DS_CUDA_EINVAL, "decoder_prefill: needs the BF16 expert weights (INT8-only model)");
    CK(pf_weights(c, m));
    CK(pf_workspace(c, m, T));
    const int p0 = m->host_len;
    const PfShape shape{H, g.moe_inter, g.n_shared * g.moe_inter, g.n_experts, g.top_k, g.rms_eps};
    if (d_embeds)
        CKL(cudaMemcpyAsync(m->pf_x, d_embeds, (size_t)T * H * 4, cudaMemcpyDeviceToDevice, st), "prefill input");
    bool lo_changed = false;
    for (int l = 0; l < g.n_layers; l++) {
        const DecLayer &L = m->layers[l];
        CKL(launch_pd_split(m->pf_x, T, H, L.in_norm, g.rms_eps, m->pf_ahi, m->pf_alo, st), "prefill norm");
        CK(pf_dense_gemm(c, 1, m->pf_ahi, m->pf_alo, T, H, m->pf_wqkv[l], 3 * QD, m->pf_qkv, 3 * QD, nullptr, nullptr,
                         st));
        CKL(launch_pd_rope_kv(m->pf_qkv, T, NH, HD, p0, m->cos_t, m->sin_t, m->pf_q, m->plane(0, l), m->plane(1, l),
                              m->plane(2, l), m->plane(3, l), g.kv_max, st),
            "prefill rope");
        // the new rows carry lo planes: lo starts at p0 at the latest
        if (m->lo_start[l] > p0) {
            m->lo_start[l] = p0;
            lo_changed = true;
        }
        // tensor cores (split-BF16 Q K^T and W V, the sequential rule on each
        // query's row of the score tile); DS_CUDA_PREFILL_ATTN_CUDA_CORES=1
        // keeps the CUDA-core kernel (same block recurrence) for comparison
        static const char *cc = getenv("DS_CUDA_PREFILL_ATTN_CUDA_CORES");
        if (!(cc && cc[0] == '1') && attn_prefill_tc_ok(HD, g.kv_max, NH))
            CKL(launch_attn_prefill_tc(m->pf_q, m->plane(0, l), m->plane(1, l), m->plane(2, l), m->plane(3, l),
                                       g.kv_max, NH, p0, T, QD, 1.0f / sqrtf((float)HD), m->pf_att, m->tickets + 10,
                                       st),
                "prefill attention");
        else
            CKL(launch_attn_prefill(m->pf_q, m->plane(0, l), m->plane(1, l), m->plane(2, l), m->plane(3, l),
                                    g.kv_max, NH, p0, T, m->lo_start[l], QD, 1.0f / sqrtf((float)HD), m->pf_att, st),
                "prefill attention");
        CKL(launch_pd_split(m->pf_att, T, QD, nullptr, 0.f, m->pf_ahi, m->pf_alo, st), "prefill split");
        CK(pf_dense_gemm(c, 1, m->pf_ahi, m->pf_alo, T, QD, L.wo, H, m->pf_y, H, nullptr, nullptr, st));
        CKL(launch_pd_add(m->pf_x, m->pf_y, (size_t)T * H, st), "prefill residual");
        if (L.dense) {
            const int Dp = m->pf_dpad;
            CKL(launch_pd_split(m->pf_x, T, H, L.post_norm, g.rms_eps, m->pf_ahi, m->pf_alo, st), "prefill norm");
            CK(pf_dense_gemm(c, 0, m->pf_ahi, m->pf_alo, T, H, m->pf_dgu[l], Dp, nullptr, 0, m->pf_hhi, m->pf_hlo,
                             st));
            CK(pf_dense_gemm(c, 1, m->pf_hhi, m->pf_hlo, T, Dp, m->pf_ddown[l], H, m->pf_y, H, nullptr, nullptr, st));
            CKL(launch_pd_add(m->pf_x, m->pf_y, (size_t)T * H, st), "prefill residual");
        } else {
            // router logits for every token as one GEMM on the normed rows
            // (the MoE block normalises again for its own planes)
            const float *lg = nullptr;
            PfShape sh = shape;
            if (m->pf_router[l]) {
                CKL(launch_pd_split(m->pf_x, T, H, L.post_norm, g.rms_eps, m->pf_ahi, m->pf_alo, st), "router norm");
                CK(pf_dense_gemm(c, 1, m->pf_ahi, m->pf_alo, T, H, m->pf_router[l], 256, m->pf_lg, 256, nullptr,
                                 nullptr, st));
                lg = m->pf_lg;
                sh.logits_ld = 256;
            }
            CK(prefill_moe_enqueue(c, sh, L.post_norm, L.router, L.block, L.down, L.sdown, m->pf_x, T, lg, nullptr,
                                   nullptr, st));
        }
    }
    if (lo_changed) drop_graphs(m);  // the decode graph bakes lo_start in
    const float *last = m->pf_x + (size_t)(T - 1) * H;
    CKL(launch_argmax_bf16(m->lm_head, last, g.vocab, H, m->slot, m->tickets + 0, m->tok, m->val, st, false,
                           m->final_norm, g.rms_eps),
        "prefill lm head");
    CKL(launch_rmsnorm(last, m->final_norm, m->xfinal, H, g.rms_eps, st, false), "prefill final norm");
    CKL(launch_pd_finish(m->embed, H, m->tok, m->xa, m->pos, p0 + T, m->tok_log, m->hist, m->hist_len,
                         m->hist_cap, st),
        "prefill finish");
    m->host_len = p0 + T;
    m->xa_staged = true;
    return DS_CUDA_OK;
}

// d_embeds [n_tokens x hidden] F32 in device memory; enqueued on `stream`
// (NULL: the context's); the first token stays on the device (read it with
// ds_cuda_decoder_generate or the next forward's history).
extern "C" int ds_cuda_decoder_prefill_dev(ds_cuda_ctx_t *c, int id, const float *d_embeds, int n_tokens,
                                           void *stream) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || !d_embeds || n_tokens <= 0) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_prefill: bad argument");
    if (m->host_len + n_tokens > m->cfg.kv_max) return ctx_fail(c, DS_CUDA_ESTATE, "decoder_prefill: KV cache full");
    cudaSetDevice(c->device);
    return prefill_enqueue(c, m, d_embeds, n_tokens, stream ? (cudaStream_t)stream : c->stream);
}

// Host embeddings [n_tokens x hidden]; returns the first generated token;
// final_x (optional) the last row's final RMS-normed state, logit its LM-head
// logit. The next forward/generate continues from position len + n_tokens
// with the first token's embedding already staged.
extern "C" int ds_cuda_decoder_prefill(ds_cuda_ctx_t *c, int id, const float *embeds, int n_tokens, float *final_x,
                                       float *logit) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || !embeds || n_tokens <= 0) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_prefill: bad argument");
    if (m->host_len + n_tokens > m->cfg.kv_max) return ctx_fail(c, DS_CUDA_ESTATE, "decoder_prefill: KV cache full");
    cudaSetDevice(c->device);
    const size_t H = m->cfg.hidden, bytes = (size_t)n_tokens * H * 4;
    // the rows go through the context's pinned buffer straight into the
    // workspace's x (one DMA, no device allocation per call)
    CK(pf_weights(c, m));
    CK(pf_workspace(c, m, n_tokens));
    CK(ctx_pinned(c, bytes));
    CKL(cudaStreamSynchronize(c->stream), "prefill staging");  // the pinned buffer is free
    memcpy(c->pin, embeds, bytes);
    int rc = ctx_cuda(c, cudaMemcpyAsync(m->pf_x, c->pin, bytes, cudaMemcpyHostToDevice, c->stream), "prefill input");
    if (rc == DS_CUDA_OK) rc = prefill_enqueue(c, m, nullptr, n_tokens, c->stream);
    int tok = 0;
    float val = 0.f;
    if (rc == DS_CUDA_OK) rc = ctx_cuda(c, cudaMemcpyAsync(&tok, m->tok, 4, cudaMemcpyDeviceToHost, c->stream), "token");
    if (rc == DS_CUDA_OK) rc = ctx_cuda(c, cudaMemcpyAsync(&val, m->val, 4, cudaMemcpyDeviceToHost, c->stream), "logit");
    if (rc == DS_CUDA_OK && final_x)
        rc = ctx_cuda(c, cudaMemcpyAsync(final_x, m->xfinal, H * 4, cudaMemcpyDeviceToHost, c->stream), "final x");
    if (rc == DS_CUDA_OK) rc = ctx_cuda(c, cudaStreamSynchronize(c->stream), "decoder_prefill");
    if (rc == DS_CUDA_OK) {
        unsigned flag = 0;
        cudaMemcpy(&flag, m->tickets + 10, sizeof flag, cudaMemcpyDeviceToHost);
        if (flag) rc = ctx_fail(c, DS_CUDA_ETIMEOUT, "decoder_prefill: a bounded device-side wait gave up");
    }
    if (rc == DS_CUDA_OK) rc = prefill_check_flag(c);
    if (rc < 0) return rc;
    if (logit) *logit = val;
    return tok;
}

// The cache rows [pos0, pos0+n) of one layer as F32 [n x heads*head_dim]
// (hi + lo planes), the layout ds_cuda_decoder_load_kv takes.
extern "C" int ds_cuda_decoder_get_kv(ds_cuda_ctx_t *c, int id, int layer, int pos0, int n, float *k, float *v) {
    DecoderModel *m = c ? get_model(c, id) : nullptr;
    if (!m || layer < 0 || layer >= m->cfg.n_layers || pos0 < 0 || n <= 0 || pos0 + n > m->cfg.kv_max || !k || !v)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_get_kv: bad argument");
    cudaSetDevice(c->device);
    CKL(cudaStreamSynchronize(c->stream), "get kv");
    const int NH = m->cfg.n_heads, HD = m->cfg.head_dim, QD = NH * HD;
    std::vector<uint16_t> hi((size_t)n * HD), lo((size_t)n * HD);
    for (int which = 0; which < 2; which++) {
        float *out = which ? v : k;
        for (int h = 0; h < NH; h++) {
            const size_t off = ((size_t)h * m->cfg.kv_max + pos0) * HD;
            CKL(cudaMemcpy(hi.data(), m->plane(2 * which, layer) + off, hi.size() * 2, cudaMemcpyDeviceToHost), "kv");
            CKL(cudaMemcpy(lo.data(), m->plane(2 * which + 1, layer) + off, lo.size() * 2, cudaMemcpyDeviceToHost),
                "kv");
            for (int i = 0; i < n; i++)
                for (int d = 0; d < HD; d++) {
                    const uint32_t a = (uint32_t)hi[(size_t)i * HD + d] << 16, b = (uint32_t)lo[(size_t)i * HD + d] << 16;
                    float fa, fb;
                    memcpy(&fa, &a, 4);
                    memcpy(&fb, &b, 4);
                    out[(size_t)i * QD + h * HD + d] = fa + fb;
                }
        }
    }
    return DS_CUDA_OK;
}
