// ep_nccl.cu — the expert-parallel prefill MoE layer behind the C ABI:
// ds_cuda_ep_unique_id / ds_cuda_ep_init / ds_cuda_ep_free and
// ds_cuda_prefill_moe_ep. A C host that replaces the reference's prefill MoE
// block (ds_moe_decoder.c:630-809) runs it on G GPUs, one process per GPU,
// with no Python: the library moves the token rows between the ranks with
// NCCL point-to-point transfers (an all-to-all(v) per direction).
//
// Per layer, on each rank (this rank's tokens x [n x H], experts split into
// contiguous blocks of E/G, shared expert replicated):
//   route     RMSNorm into two BF16 planes, softmax/top-k (local);
//   dispatch  plan + pack one payload row per (token, owning rank);
//             row counts exchanged, then the payload all-to-all on a
//             communication stream while the compute stream runs the shared
//             expert on the local rows (overlap);
//   experts   the grouped tensor-core GEMMs over the received (row, expert)
//             pairs;
//   return    the outputs travel back in request order (all-to-all);
//   combine   x += sum_k w_k y_k in ascending expert order, plus shared: the
//             single-GPU arithmetic, so results are bit-identical to it.
// The counts are needed on the host to size the transfers: each rank
// announces to every peer the rows it sends and the pairs it asks of it, so
// the layer synchronises the compute stream once (after dispatch). Each
// rank's own rows and outputs are device-to-device copies; NCCL carries only
// what crosses to another GPU.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or $DS_CUDA_NCCL_LIB),
// so the library itself has no link-time dependency on it; only the entry
// points of this file need it. Types and enum values used here are the
// public, stable ones of nccl.h (ncclUniqueId is 128 bytes; ncclInt8 = 0,
// ncclInt32 = 2; ncclSuccess = 0).
#include <dlfcn.h>

#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "ctx.h"

cudaError_t pf_combine_split_launch(float *x, int M, int H, int K, const int *idx, const float *wt, const float *y,
                                    const int *yrow, const float *ys, const float *y_alt, long long alt_lo,
                                    long long alt_hi, cudaStream_t st);

namespace {

struct NcclUid {
    char internal[128];
};
typedef void *NcclComm;
typedef int (*nccl_get_uid_t)(NcclUid *);
typedef int (*nccl_init_rank_t)(NcclComm *, int, NcclUid, int);
typedef int (*nccl_destroy_t)(NcclComm);
typedef int (*nccl_group_t)();
typedef int (*nccl_send_t)(const void *, size_t, int, int, NcclComm, cudaStream_t);
typedef int (*nccl_recv_t)(void *, size_t, int, int, NcclComm, cudaStream_t);
typedef const char *(*nccl_err_t)(int);
constexpr int NCCL_INT8 = 0;

struct Nccl {
    void *h = nullptr;
    nccl_get_uid_t get_uid = nullptr;
    nccl_init_rank_t init_rank = nullptr;
    nccl_destroy_t destroy = nullptr;
    nccl_group_t group_start = nullptr, group_end = nullptr;
    nccl_send_t send = nullptr;
    nccl_recv_t recv = nullptr;
    nccl_err_t err = nullptr;
};

// Loads NCCL once per process; null (and *why set) if it is not available.
const Nccl *nccl_load(std::string *why) {
    static Nccl n;
    static bool tried = false;
    static std::string fail;
    if (!tried) {
        tried = true;
        const char *env = getenv("DS_CUDA_NCCL_LIB");
        const char *names[] = {env, "libnccl.so.2", "libnccl.so"};
        for (const char *nm : names) {
            if (!nm || !*nm) continue;
            n.h = dlopen(nm, RTLD_NOW | RTLD_GLOBAL);
            if (n.h) break;
        }
        if (!n.h) {
            fail = "NCCL library not found (set DS_CUDA_NCCL_LIB)";
        } else {
            n.get_uid = (nccl_get_uid_t)dlsym(n.h, "ncclGetUniqueId");
            n.init_rank = (nccl_init_rank_t)dlsym(n.h, "ncclCommInitRank");
            n.destroy = (nccl_destroy_t)dlsym(n.h, "ncclCommDestroy");
            n.group_start = (nccl_group_t)dlsym(n.h, "ncclGroupStart");
            n.group_end = (nccl_group_t)dlsym(n.h, "ncclGroupEnd");
            n.send = (nccl_send_t)dlsym(n.h, "ncclSend");
            n.recv = (nccl_recv_t)dlsym(n.h, "ncclRecv");
            n.err = (nccl_err_t)dlsym(n.h, "ncclGetErrorString");
            if (!n.get_uid || !n.init_rank || !n.destroy || !n.group_start || !n.group_end || !n.send || !n.recv)
                fail = "NCCL library lacks a required symbol";
        }
    }
    if (!fail.empty()) {
        if (why) *why = fail;
        return nullptr;
    }
    return &n;
}

// Per-context expert-parallel state: the communicator, a communication
// stream, and device buffers grown on demand.
struct EpState {
    const Nccl *nc = nullptr;
    NcclComm comm = nullptr;
    int rank = 0, world = 1;
    cudaStream_t cs = nullptr;                 // payload all-to-all
    cudaEvent_t ev_packed = nullptr, ev_recv = nullptr, ev_counts = nullptr;
    struct Buf {
        void *p = nullptr;
        size_t cap = 0;
    };
    Buf hi, lo, idx, w, payload, send_tok, counts, inv, cnt_pack, cnt_recv, rpayload, pair_row, pair_expert, pcounts,
        y, ys, yback;
    int *h_counts = nullptr;                   // pinned: [2G] dispatch counts, [2G] received (rows, pairs) per peer
};

}  // namespace

static EpState *ep_of(ds_cuda_ctx *c) { return static_cast<EpState *>(c->ep); }

static int ep_grow(ds_cuda_ctx *c, EpState::Buf &b, size_t bytes) {
    bytes = bytes ? bytes : 16;
    if (b.cap >= bytes) return DS_CUDA_OK;
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.cap = 0;
    if (cudaMalloc(&b.p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return ctx_fail(c, DS_CUDA_ENOMEM, "prefill_moe_ep: cudaMalloc(%zu) failed", bytes);
    }
    b.cap = bytes;
    return DS_CUDA_OK;
}

static int nccl_check(ds_cuda_ctx *c, const EpState *s, int r, const char *what) {
    if (r == 0) return DS_CUDA_OK;
    return ctx_fail(c, DS_CUDA_ECUDA, "%s: NCCL error %d (%s)", what, r, s && s->nc && s->nc->err ? s->nc->err(r) : "");
}

// Releases the expert-parallel state of a context (its communicator,
// stream, events and buffers); called by ds_cuda_free.
void ep_release(ds_cuda_ctx *c) {
    EpState *s = ep_of(c);
    if (!s) return;
    if (s->cs) cudaStreamSynchronize(s->cs);
    if (s->comm && s->nc) s->nc->destroy(s->comm);
    EpState::Buf *bufs[] = {&s->hi, &s->lo, &s->idx, &s->w, &s->payload, &s->send_tok, &s->counts, &s->inv,
                            &s->cnt_recv, &s->rpayload, &s->pair_row, &s->pair_expert, &s->pcounts, &s->y,
                            &s->ys, &s->yback};
    for (auto *b : bufs)
        if (b->p) cudaFree(b->p);
    if (s->h_counts) cudaFreeHost(s->h_counts);
    if (s->ev_packed) cudaEventDestroy(s->ev_packed);
    if (s->ev_recv) cudaEventDestroy(s->ev_recv);
    if (s->ev_counts) cudaEventDestroy(s->ev_counts);
    if (s->cs) cudaStreamDestroy(s->cs);
    delete s;
    c->ep = nullptr;
}

extern "C" int ds_cuda_ep_unique_id(ds_cuda_ctx_t *c, void *id_out) {
    if (!c || !c->ok || !id_out) return DS_CUDA_EINVAL;
    std::string why;
    const Nccl *nc = nccl_load(&why);
    if (!nc) return ctx_fail(c, DS_CUDA_EINVAL, "ep_unique_id: %s", why.c_str());
    NcclUid u;
    int r = nc->get_uid(&u);
    if (r) return ctx_fail(c, DS_CUDA_ECUDA, "ep_unique_id: NCCL error %d", r);
    memcpy(id_out, &u, sizeof u);
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_ep_init(ds_cuda_ctx_t *c, int rank, int world, const void *id) {
    if (!c || !c->ok || !id || world < 1 || world > 8 || rank < 0 || rank >= world)
        return ctx_fail(c, DS_CUDA_EINVAL, "ep_init: bad argument (rank %d of %d, 1 <= world <= 8)", rank, world);
    if (c->ep) return ctx_fail(c, DS_CUDA_ESTATE, "ep_init: already initialised (ds_cuda_ep_free first)");
    std::string why;
    const Nccl *nc = nccl_load(&why);
    if (!nc) return ctx_fail(c, DS_CUDA_EINVAL, "ep_init: %s", why.c_str());
    cudaSetDevice(c->device);
    EpState *s = new EpState;
    s->nc = nc;
    s->rank = rank;
    s->world = world;
    c->ep = s;
    NcclUid u;
    memcpy(&u, id, sizeof u);
    int r = nc->init_rank(&s->comm, world, u, rank);
    if (r) {
        s->comm = nullptr;
        ep_release(c);
        return ctx_fail(c, DS_CUDA_ECUDA, "ep_init: ncclCommInitRank error %d (%s)", r, nc->err ? nc->err(r) : "");
    }
    if (cudaStreamCreateWithFlags(&s->cs, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->ev_packed, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->ev_recv, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->ev_counts, cudaEventDisableTiming) != cudaSuccess ||
        cudaMallocHost((void **)&s->h_counts, 64 * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        ep_release(c);
        return ctx_fail(c, DS_CUDA_ENOMEM, "ep_init: stream/event/pinned allocation failed");
    }
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_ep_free(ds_cuda_ctx_t *c) {
    if (!c) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    ep_release(c);
    return DS_CUDA_OK;
}

// all-to-all(v) of byte rows on `st`: row counts per peer (host), rows are
// `row_b` bytes, laid out rank after rank on both sides. This rank's own
// section is a stream-ordered device-to-device copy; NCCL moves only the
// sections of the other ranks (its point-to-point kernels copy to self at a
// fraction of the HBM rate, and at one rank every row is a self row).
static int ep_a2a(ds_cuda_ctx *c, EpState *s, const void *send, const int *send_rows, void *recv, const int *recv_rows,
                  size_t row_b, cudaStream_t st, const char *what, bool copy_self = true) {
    const Nccl *nc = s->nc;
    size_t so = 0, ro = 0;
    for (int p = 0; p < s->world; p++) {
        if (p == s->rank) {
            if (send_rows[p] != recv_rows[p])
                return ctx_fail(c, DS_CUDA_ESTATE, "%s: %d rows sent to self, %d expected", what, send_rows[p],
                                recv_rows[p]);
            if (send_rows[p] > 0 && copy_self) {
                cudaError_t e = cudaMemcpyAsync(static_cast<char *>(recv) + ro * row_b,
                                                static_cast<const char *>(send) + so * row_b,
                                                (size_t)send_rows[p] * row_b, cudaMemcpyDeviceToDevice, st);
                if (e != cudaSuccess) return ctx_cuda(c, e, what);
            }
        }
        so += send_rows[p];
        ro += recv_rows[p];
    }
    if (s->world == 1) return DS_CUDA_OK;
    int r = nc->group_start();
    so = 0;
    ro = 0;
    for (int p = 0; p < s->world && r == 0; p++) {
        if (p != s->rank && send_rows[p] > 0)
            r = nc->send(static_cast<const char *>(send) + so * row_b, (size_t)send_rows[p] * row_b, NCCL_INT8, p,
                         s->comm, st);
        if (r == 0 && p != s->rank && recv_rows[p] > 0)
            r = nc->recv(static_cast<char *>(recv) + ro * row_b, (size_t)recv_rows[p] * row_b, NCCL_INT8, p, s->comm,
                         st);
        so += send_rows[p];
        ro += recv_rows[p];
    }
    int r2 = nc->group_end();
    return nccl_check(c, s, r ? r : r2, what);
}

#define EPK(expr)                    \
    do {                             \
        int _rc = (expr);            \
        if (_rc < 0) return _rc;     \
    } while (0)
#define EPC(expr, what)                                           \
    do {                                                          \
        cudaError_t _e = (expr);                                  \
        if (_e != cudaSuccess) return ctx_cuda(c, _e, what);      \
    } while (0)

extern "C" int ds_cuda_prefill_moe_ep(ds_cuda_ctx_t *c, const ds_cuda_decoder_config_t *cfg,
                                      const ds_cuda_layer_weights_t *layer, float *d_x, int n_tokens,
                                      const float *d_logits, int *d_top_idx, float *d_top_w, void *stream) {
    if (!c || !c->ok || !cfg || !layer || n_tokens < 0 || (n_tokens > 0 && !d_x))
        return DS_CUDA_EINVAL;
    EpState *s = ep_of(c);
    if (!s) return ctx_fail(c, DS_CUDA_ESTATE, "prefill_moe_ep: ds_cuda_ep_init has not been called");
    const int G = s->world, H = cfg->hidden, K = cfg->top_k, E = cfg->n_experts;
    if (E % G) return ctx_fail(c, DS_CUDA_EINVAL, "prefill_moe_ep: %d experts do not split over %d ranks", E, G);
    cudaSetDevice(c->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    const size_t n = (size_t)n_tokens, ld = (size_t)2 * H + 16, row_b = ld * 2;
    const size_t cap_rows = n * (size_t)(K < G ? K : G);
    EPK(ep_grow(c, s->hi, n * H * 2));
    EPK(ep_grow(c, s->lo, n * H * 2));
    EPK(ep_grow(c, s->idx, n * K * 4));
    EPK(ep_grow(c, s->w, n * K * 4));
    EPK(ep_grow(c, s->payload, cap_rows * row_b));
    EPK(ep_grow(c, s->send_tok, cap_rows * 4));
    EPK(ep_grow(c, s->counts, 2 * G * 4));
    EPK(ep_grow(c, s->cnt_pack, 2 * G * 4));
    EPK(ep_grow(c, s->cnt_recv, 2 * G * 4));
    EPK(ep_grow(c, s->inv, n * K * 4));
    EPK(ep_grow(c, s->ys, n * H * 4));
    uint16_t *hi = (uint16_t *)s->hi.p, *lo = (uint16_t *)s->lo.p;
    int *idx = (int *)s->idx.p;
    float *w = (float *)s->w.p;
    // 1. route; 2. dispatch plan + pack
    EPK(ds_cuda_prefill_route_dev(c, cfg, layer, d_x, n_tokens, d_logits, hi, lo, idx, w, st));
    EPK(ds_cuda_ep_dispatch_dev(c, n_tokens, K, G, E / G, idx, hi, lo, H, (uint16_t *)s->payload.p,
                                (int *)s->send_tok.p, (int *)s->counts.p, (int *)s->inv.p, st));
    EPC(cudaEventRecord(s->ev_packed, st), "event");
    // (rows, pairs) to every peer as one 8-byte record: the rows it will
    // receive and the (row, expert) pairs it will compute for this rank, so
    // one host synchronisation sizes every transfer of the layer
    int *cnt = (int *)s->counts.p, *pack = (int *)s->cnt_pack.p;
    EPC(cudaMemcpy2DAsync(pack, 8, cnt, 4, 4, G, cudaMemcpyDeviceToDevice, st), "counts pack");
    EPC(cudaMemcpy2DAsync(pack + 1, 8, cnt + G, 4, 4, G, cudaMemcpyDeviceToDevice, st), "counts pack");
    std::vector<int> ones(G, 1);
    EPK(ep_a2a(c, s, pack, ones.data(), s->cnt_recv.p, ones.data(), 8, st, "prefill_moe_ep counts"));
    int *hc = s->h_counts;
    EPC(cudaMemcpyAsync(hc, cnt, 2 * G * 4, cudaMemcpyDeviceToHost, st), "counts copy");
    EPC(cudaMemcpyAsync(hc + 2 * G, s->cnt_recv.p, 2 * G * 4, cudaMemcpyDeviceToHost, st), "counts copy");
    EPC(cudaEventRecord(s->ev_counts, st), "event");
    // 3a. the shared expert on the local rows, queued before the host waits
    //     for the counts so the GPU has work meanwhile
    if (n_tokens > 0)
        EPK(ds_cuda_prefill_experts_dev(c, cfg, layer, nullptr, nullptr, H, 0, nullptr, nullptr, 0, nullptr, hi, lo,
                                        n_tokens, (float *)s->ys.p, st));
    EPC(cudaEventSynchronize(s->ev_counts), "prefill_moe_ep dispatch counts");
    std::vector<int> send_rows(hc, hc + G), back_recv(hc + G, hc + 2 * G), recv_rows(G), back_send(G);
    size_t R = 0, P = 0, Bk = 0, self_y0 = 0, self_b0 = 0;
    for (int p = 0; p < G; p++) {
        recv_rows[p] = hc[2 * G + 2 * p];
        back_send[p] = hc[2 * G + 2 * p + 1];
        if (p < s->rank) {
            self_y0 += back_send[p];
            self_b0 += back_recv[p];
        }
        R += recv_rows[p];
        P += back_send[p];
        Bk += back_recv[p];
    }
    EPK(ep_grow(c, s->rpayload, R * row_b));
    EPK(ep_grow(c, s->pair_row, R * K * 4));
    EPK(ep_grow(c, s->pair_expert, R * K * 4));
    EPK(ep_grow(c, s->pcounts, (G + 1) * 4));
    EPK(ep_grow(c, s->y, P * H * 4));
    EPK(ep_grow(c, s->yback, Bk * H * 4));
    // 3b. payload all-to-all on the communication stream (after the pack,
    //     beside the shared expert)
    EPC(cudaStreamWaitEvent(s->cs, s->ev_packed, 0), "event wait");
    EPK(ep_a2a(c, s, s->payload.p, send_rows.data(), s->rpayload.p, recv_rows.data(), row_b, s->cs,
               "prefill_moe_ep dispatch all-to-all"));
    EPC(cudaEventRecord(s->ev_recv, s->cs), "event");
    EPC(cudaStreamWaitEvent(st, s->ev_recv, 0), "event wait");
    // 4. the received (row, expert) pairs (their count per source rank is
    //    the back_send the peers announced), the routed experts
    EPK(ds_cuda_ep_pairs_dev(c, (int)R, K, G, recv_rows.data(), (const uint16_t *)s->rpayload.p, H,
                             (int *)s->pair_row.p, (int *)s->pair_expert.p, (int *)s->pcounts.p, st));
    const uint16_t *rp = (const uint16_t *)s->rpayload.p;
    if (P > 0)
        EPK(ds_cuda_prefill_experts_dev(c, cfg, layer, rp, rp + H, (int)ld, (int)R, (const int *)s->pair_row.p,
                                        (const int *)s->pair_expert.p, (int)P, (float *)s->y.p, nullptr, nullptr, 0,
                                        nullptr, st));
    // 5. outputs back in request order; 6. combine
    //    (this rank's own outputs stay in y: the combine reads that
    //    section of the returned stream from there)
    EPK(ep_a2a(c, s, s->y.p, back_send.data(), s->yback.p, back_recv.data(), (size_t)H * 4, st,
               "prefill_moe_ep return all-to-all", false));
    if (n_tokens > 0)
        EPC(pf_combine_split_launch(d_x, n_tokens, H, K, idx, w, (const float *)s->yback.p, (const int *)s->inv.p,
                                    (const float *)s->ys.p, (const float *)s->y.p + self_y0 * H, (long long)self_b0,
                                    (long long)(self_b0 + back_recv[s->rank]), st),
            "prefill_moe_ep combine");
    if (c->prefill_timing) EPC(cudaEventRecord(c->prefill_ev[6], st), "stage event");  // the combine's stage end
    if (d_top_idx) EPC(cudaMemcpyAsync(d_top_idx, idx, n * K * 4, cudaMemcpyDeviceToDevice, st), "idx copy");
    if (d_top_w) EPC(cudaMemcpyAsync(d_top_w, w, n * K * 4, cudaMemcpyDeviceToDevice, st), "w copy");
    return DS_CUDA_OK;
}
