// api.cu — the C ABI declared in include/ds_cuda.h: context, weight
// registration keyed by host pointer, and the host-pointer / device-pointer
// entry points of the decode MoE layer, LM head, matvec and INT8 quantiser.
#include <sys/mman.h>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "ds_cuda.h"
#include "launch.h"
#include "ctx.h"

using namespace ds;

// ---------------------------------------------------------------------------
// Context helpers
// ---------------------------------------------------------------------------
int ctx_fail(ds_cuda_ctx *c, int code, const char *fmt, ...) {
    if (c) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        c->err = buf;
    }
    return code;
}

int ctx_cuda(ds_cuda_ctx *c, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return DS_CUDA_OK;
    return ctx_fail(c, e == cudaErrorInvalidValue ? DS_CUDA_EINVAL : DS_CUDA_ECUDA, "%s: %s", what,
                    cudaGetErrorString(e));
}

int ctx_grow(ds_cuda_ctx *c, void **p, size_t *cap, size_t need) {
    if (*cap >= need) return DS_CUDA_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    size_t n = need < 4096 ? 4096 : need;
    if (cudaMalloc(p, n) != cudaSuccess) {
        cudaGetLastError();
        return ctx_fail(c, DS_CUDA_ENOMEM, "cudaMalloc(%zu) failed", n);
    }
    *cap = n;
    return DS_CUDA_OK;
}

int ctx_pinned(ds_cuda_ctx *c, size_t need) {
    if (c->pin_cap >= need) return DS_CUDA_OK;
    if (c->pin) cudaFreeHost(c->pin);
    c->pin = nullptr;
    c->pin_cap = 0;
    size_t n = need < 65536 ? 65536 : need;
    if (cudaMallocHost(&c->pin, n) != cudaSuccess) {
        cudaGetLastError();
        return ctx_fail(c, DS_CUDA_ENOMEM, "cudaMallocHost(%zu) failed", n);
    }
    c->pin_cap = n;
    return DS_CUDA_OK;
}

// Device address of [p, p+bytes) inside a registration; optionally register
// the range on first use (the Metal context wraps unknown buffers the same
// way, ds_metal.m:56-68).
const void *ctx_lookup(ds_cuda_ctx *c, const void *p, size_t bytes, bool auto_register) {
    if (!p) return nullptr;
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    auto it = c->regs.upper_bound(a);
    if (it != c->regs.begin()) {
        --it;
        const Reg &r = it->second;
        if (a >= r.host && a + bytes <= r.host + r.bytes) return (const char *)r.dev + (a - r.host);
    }
    if (!auto_register) return nullptr;
    if (ctx_register(c, p, bytes) != DS_CUDA_OK) return nullptr;
    return ctx_lookup(c, p, bytes, false);
}

int ctx_register(ds_cuda_ctx *c, const void *p, size_t bytes) {
    if (!p || bytes == 0) return ctx_fail(c, DS_CUDA_EINVAL, "register: null pointer or zero size");
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    auto it = c->regs.find(a);
    if (it != c->regs.end()) {
        if (it->second.bytes >= bytes) return DS_CUDA_OK;
        cudaFree(it->second.dev);
        c->reg_bytes -= it->second.bytes;
        c->regs.erase(it);
    }
    void *d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) {
        cudaGetLastError();
        return ctx_fail(c, DS_CUDA_ENOMEM, "register: cudaMalloc(%zu) failed", bytes);
    }
    cudaError_t e = cudaMemcpy(d, p, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return ctx_cuda(c, e, "register: copy to device");
    }
    c->regs[a] = Reg{a, bytes, d};
    c->reg_bytes += bytes;
    return DS_CUDA_OK;
}

void *ctx_adopt(ds_cuda_ctx *c, void *dev, size_t bytes) {
    if (!dev || !bytes) return nullptr;
    void *key = mmap(nullptr, bytes, PROT_NONE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
    if (key == MAP_FAILED) return nullptr;
    c->key_ranges.emplace_back(key, bytes);
    const uintptr_t a = reinterpret_cast<uintptr_t>(key);
    c->regs[a] = Reg{a, bytes, dev};
    c->reg_bytes += bytes;
    return key;
}

static int h2d(ds_cuda_ctx *c, void *d, const void *h, size_t bytes) {
    return ctx_cuda(c, cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, c->stream), "copy to device");
}
static int d2h_sync(ds_cuda_ctx *c, void *h, const void *d, size_t bytes) {
    int rc = ctx_cuda(c, cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, c->stream), "copy to host");
    if (rc) return rc;
    return ctx_cuda(c, cudaStreamSynchronize(c->stream), "synchronize");
}

#define CK(expr)                  \
    do {                          \
        int _rc = (expr);         \
        if (_rc < 0) return _rc;  \
    } while (0)

static cudaStream_t pick_stream(ds_cuda_ctx *c, void *s) { return s ? (cudaStream_t)s : c->stream; }

// ---------------------------------------------------------------------------
// Lifecycle
// ---------------------------------------------------------------------------
extern "C" ds_cuda_ctx_t *ds_cuda_init(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) return nullptr;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) return nullptr;
    ds_cuda_ctx *c = new ds_cuda_ctx();
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return nullptr;
    }
    // fixed small scratch: tickets, argmax slots, top-k results
    bool ok = cudaMalloc(&c->d_tickets, 64 * sizeof(unsigned)) == cudaSuccess &&
              cudaMalloc(&c->d_slots, 512 * sizeof(unsigned long long)) == cudaSuccess &&
              cudaMalloc(&c->d_tok, 512 * sizeof(int)) == cudaSuccess &&
              cudaMalloc(&c->d_val, 512 * sizeof(float)) == cudaSuccess &&
              cudaMalloc(&c->d_scores, 256 * sizeof(float)) == cudaSuccess &&
              cudaMalloc(&c->d_idx, 64 * sizeof(int)) == cudaSuccess &&
              cudaMalloc(&c->d_wt, 64 * sizeof(float)) == cudaSuccess;
    if (ok) {
        ok = cudaMemset(c->d_tickets, 0, 64 * sizeof(unsigned)) == cudaSuccess &&
             cudaMemset(c->d_slots, 0, 512 * sizeof(unsigned long long)) == cudaSuccess;
    }
    if (!ok) {
        ds_cuda_free(c);
        return nullptr;
    }
    c->ok = true;
    return c;
}

extern "C" void ds_cuda_free(ds_cuda_ctx_t *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    ctx_release_models(c);
    ctx_release_batch_models(c);
    prefill_release(c);
    ep_release(c);
    for (auto &e : c->prefill_ev)
        if (e) cudaEventDestroy(e);
    for (auto &kv : c->regs) cudaFree(kv.second.dev);
    for (auto &r : c->key_ranges) munmap(r.first, r.second);
    void *bufs[] = {c->d_tickets, c->d_slots, c->d_tok, c->d_val, c->d_scores, c->d_idx, c->d_wt,
                    c->d_x, c->d_out, c->d_h, c->d_tmp, c->d_lt_planes, c->d_lt_err, c->d_sk_scratch};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (c->pin) cudaFreeHost(c->pin);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" int ds_cuda_is_available(const ds_cuda_ctx_t *c) { return c && c->ok ? 1 : 0; }

extern "C" const char *ds_cuda_last_error(const ds_cuda_ctx_t *c) {
    return c ? c->err.c_str() : "no context (ds_cuda_init returned NULL: no usable sm_100 device)";
}

extern "C" void *ds_cuda_stream(ds_cuda_ctx_t *c) { return c ? (void *)c->stream : nullptr; }

extern "C" int ds_cuda_synchronize(ds_cuda_ctx_t *c) {
    if (!c) return DS_CUDA_EINVAL;
    return ctx_cuda(c, cudaStreamSynchronize(c->stream), "synchronize");
}

extern "C" int ds_cuda_set_numerics(ds_cuda_ctx_t *c, int simulate_bf16, int renorm_topk) {
    if (!c) return DS_CUDA_EINVAL;
    c->simulate = simulate_bf16 ? 1 : 0;
    c->renorm = renorm_topk ? 1 : 0;
    return DS_CUDA_OK;
}

// ---------------------------------------------------------------------------
// Registration
// ---------------------------------------------------------------------------
extern "C" int ds_cuda_register_bf16(ds_cuda_ctx_t *c, const uint16_t *data, size_t n) {
    if (!c) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    return ctx_register(c, data, n * sizeof(uint16_t));
}
extern "C" int ds_cuda_register_f32(ds_cuda_ctx_t *c, const float *data, size_t n) {
    if (!c) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    return ctx_register(c, data, n * sizeof(float));
}
extern "C" int ds_cuda_register_expert_block(ds_cuda_ctx_t *c, const void *block, size_t bytes) {
    if (!c) return DS_CUDA_EINVAL;
    cudaSetDevice(c->device);
    return ctx_register(c, block, bytes);
}
extern "C" int ds_cuda_register_int8_block(ds_cuda_ctx_t *c, const ds_cuda_int8_block_t *b) {
    if (!c || !b || !b->qweight || !b->scale || !b->offset || b->out_dim <= 0 || b->in_dim <= 0)
        return ctx_fail(c, DS_CUDA_EINVAL, "register_int8_block: incomplete block");
    cudaSetDevice(c->device);
    CK(ctx_register(c, b->qweight, (size_t)b->out_dim * b->in_dim));
    CK(ctx_register(c, b->scale, (size_t)b->out_dim * sizeof(float)));
    return ctx_register(c, b->offset, (size_t)b->out_dim * sizeof(float));
}
extern "C" int ds_cuda_unregister(ds_cuda_ctx_t *c, const void *p) {
    if (!c || !p) return DS_CUDA_EINVAL;
    auto it = c->regs.find(reinterpret_cast<uintptr_t>(p));
    if (it == c->regs.end()) return ctx_fail(c, DS_CUDA_ENOTREG, "unregister: %p is not a registration base", p);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    cudaFree(it->second.dev);
    c->reg_bytes -= it->second.bytes;
    c->regs.erase(it);
    return DS_CUDA_OK;
}

extern "C" const void *ds_cuda_device_ptr(ds_cuda_ctx_t *c, const void *p) {
    return c ? ctx_lookup(c, p, 1, false) : nullptr;
}
extern "C" size_t ds_cuda_registered_bytes(const ds_cuda_ctx_t *c) { return c ? c->reg_bytes : 0; }

// ---------------------------------------------------------------------------
// MoE experts (Metal-shaped calls)
// ---------------------------------------------------------------------------
static bool moe_shape_ok(int hidden, int inter, int top_k, bool shared, int chunk) {
    if (hidden <= 0 || hidden % chunk || hidden > 2048) return false;
    if (top_k < 0 || top_k + (shared ? 2 : 0) > 8) return false;
    if (top_k > 0 && (inter <= 0 || inter % chunk || inter > 2048)) return false;
    return true;
}

// Stage x (and optionally the current output) into device scratch.
static int stage_vec(ds_cuda_ctx *c, float **d, size_t *cap, const float *h, int n) {
    CK(ctx_grow(c, (void **)d, cap, (size_t)n * sizeof(float)));
    CK(ctx_pinned(c, (size_t)n * sizeof(float)));
    memcpy(c->pin, h, (size_t)n * sizeof(float));
    return h2d(c, *d, c->pin, (size_t)n * sizeof(float));
}
static int fetch_vec(ds_cuda_ctx *c, float *h, const float *d, int n) {
    CK(ctx_pinned(c, (size_t)n * sizeof(float)));
    CK(d2h_sync(c, c->pin, d, (size_t)n * sizeof(float)));
    memcpy(h, c->pin, (size_t)n * sizeof(float));
    return DS_CUDA_OK;
}

static int run_moe(ds_cuda_ctx *c, MoeArgs &a, cudaStream_t st) {
    CK(ctx_cuda(c, launch_moe_gate_up(a, st, false), "moe gate_up launch"));
    return ctx_cuda(c, launch_moe_down(a, st, false), "moe down launch");
}

static int ensure_h(ds_cuda_ctx *c, int elems) {
    return ctx_grow(c, (void **)&c->d_h, &c->h_cap, (size_t)elems * sizeof(float));
}

extern "C" int ds_cuda_moe_experts(ds_cuda_ctx_t *c, const float *x, const uint16_t **gu, const uint16_t **dn,
                                   const float *w, int top_k, int hidden, int inter, float *output) {
    if (!c || !x || !output || (top_k > 0 && (!gu || !dn || !w)))
        return ctx_fail(c, DS_CUDA_EINVAL, "moe_experts: null argument");
    if (!moe_shape_ok(hidden, inter, top_k, false, 8))
        return ctx_fail(c, DS_CUDA_EINVAL, "moe_experts: unsupported shape hidden=%d inter=%d top_k=%d", hidden,
                        inter, top_k);
    cudaSetDevice(c->device);
    MoeArgs a = {};
    a.hidden = hidden;
    a.inter = inter;
    a.top_k = top_k;
    a.simulate = c->simulate;
    for (int k = 0; k < top_k; k++) {
        a.gu[k].w = ctx_lookup(c, gu[k], (size_t)2 * inter * hidden * 2, true);
        a.dn[k].w = ctx_lookup(c, dn[k], (size_t)hidden * inter * 2, true);
        if (!a.gu[k].w || !a.dn[k].w) return ctx_fail(c, DS_CUDA_ENOTREG, "moe_experts: weight registration failed");
        a.wt[k] = w[k];
    }
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, hidden));
    CK(ctx_grow(c, (void **)&c->d_out, &c->out_cap, (size_t)hidden * sizeof(float)));
    CK(ensure_h(c, top_k * inter));
    a.x = c->d_x;
    a.h = c->d_h;
    a.out = c->d_out;
    a.out_mode = 0;
    CK(run_moe(c, a, c->stream));
    return fetch_vec(c, output, c->d_out, hidden);
}

extern "C" int ds_cuda_shared_experts(ds_cuda_ctx_t *c, const float *x, const uint16_t *gu, const uint16_t *dn,
                                      int hidden, int shared_inter, float *output) {
    if (!c || !x || !gu || !dn || !output) return ctx_fail(c, DS_CUDA_EINVAL, "shared_experts: null argument");
    if (!moe_shape_ok(hidden, 16, 0, true, 8) || shared_inter <= 0 || shared_inter % 16 || shared_inter > 4096)
        return ctx_fail(c, DS_CUDA_EINVAL, "shared_experts: unsupported shape");
    cudaSetDevice(c->device);
    MoeArgs a = {};
    a.hidden = hidden;
    a.sh_inter = shared_inter;
    a.has_shared = 1;
    a.simulate = c->simulate;
    a.sh_gu.w = ctx_lookup(c, gu, (size_t)2 * shared_inter * hidden * 2, true);
    a.sh_dn.w = ctx_lookup(c, dn, (size_t)hidden * shared_inter * 2, true);
    if (!a.sh_gu.w || !a.sh_dn.w) return ctx_fail(c, DS_CUDA_ENOTREG, "shared_experts: weight registration failed");
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, hidden));
    CK(stage_vec(c, &c->d_out, &c->out_cap, output, hidden));
    CK(ensure_h(c, shared_inter));
    a.x = c->d_x;
    a.h = c->d_h;
    a.out = c->d_out;
    a.out_mode = 1;
    CK(run_moe(c, a, c->stream));
    return fetch_vec(c, output, c->d_out, hidden);
}

extern "C" int ds_cuda_expert_forward_fused(ds_cuda_ctx_t *c, float *out, const float *x, const uint16_t *gu,
                                            const uint16_t *dn, int hidden, int inter) {
    float one = 1.0f;
    const uint16_t *g[1] = {gu}, *d[1] = {dn};
    if (!c) return DS_CUDA_EINVAL;
    // out = 1.0 * expert(x): the combine FMA with weight 1 is exact.
    return ds_cuda_moe_experts(c, x, g, d, &one, 1, hidden, inter, out);
}

extern "C" int ds_cuda_expert_forward_fused_int4(ds_cuda_ctx_t *c, float *out, const float *x,
                                                 const ds_cuda_int8_block_t *gub, const ds_cuda_int8_block_t *dnb,
                                                 int hidden, int inter) {
    if (!c || !out || !x || !gub || !dnb) return ctx_fail(c, DS_CUDA_EINVAL, "expert_forward_fused_int4: null argument");
    if (gub->out_dim != 2 * inter || gub->in_dim != hidden || dnb->out_dim != hidden || dnb->in_dim != inter)
        return ctx_fail(c, DS_CUDA_EINVAL, "expert_forward_fused_int4: block shapes do not match hidden/inter");
    if (!moe_shape_ok(hidden, inter, 1, false, 16))
        return ctx_fail(c, DS_CUDA_EINVAL, "expert_forward_fused_int4: unsupported shape");
    cudaSetDevice(c->device);
    CK(ds_cuda_register_int8_block(c, gub));
    CK(ds_cuda_register_int8_block(c, dnb));
    MoeArgs a = {};
    a.hidden = hidden;
    a.inter = inter;
    a.top_k = 1;
    a.int8 = 1;
    a.simulate = c->simulate;
    a.gu[0] = WMat{ctx_lookup(c, gub->qweight, 1, false), (const float *)ctx_lookup(c, gub->scale, 4, false),
                   (const float *)ctx_lookup(c, gub->offset, 4, false)};
    a.dn[0] = WMat{ctx_lookup(c, dnb->qweight, 1, false), (const float *)ctx_lookup(c, dnb->scale, 4, false),
                   (const float *)ctx_lookup(c, dnb->offset, 4, false)};
    a.wt[0] = 1.0f;
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, hidden));
    CK(ctx_grow(c, (void **)&c->d_out, &c->out_cap, (size_t)hidden * sizeof(float)));
    CK(ensure_h(c, inter));
    a.x = c->d_x;
    a.h = c->d_h;
    a.out = c->d_out;
    CK(run_moe(c, a, c->stream));
    return fetch_vec(c, out, c->d_out, hidden);
}

// ---------------------------------------------------------------------------
// Whole MoE layer (router -> top-k -> experts -> combine -> shared)
// ---------------------------------------------------------------------------
int moe_layer_enqueue(ds_cuda_ctx *c, MoeArgs &a, const uint16_t *d_router, int n_experts, int *d_idx,
                      float *d_wt, cudaStream_t st, bool pdl) {
    CK(ctx_cuda(c,
                launch_router(d_router, a.x, n_experts, a.hidden, c->d_scores, c->d_tickets + 1, a.top_k, c->renorm,
                              d_idx, d_wt, st, pdl),
                "router launch"));
    a.d_idx = d_idx;
    a.d_wt = d_wt;
    CK(ctx_cuda(c, launch_moe_gate_up(a, st, pdl), "moe gate_up launch"));
    return ctx_cuda(c, launch_moe_down(a, st, pdl), "moe down launch");
}

static int layer_checks(ds_cuda_ctx *c, int hidden, int inter, int shared_inter, int n_experts, int top_k, int chunk) {
    if (!moe_shape_ok(hidden, inter, top_k, shared_inter > 0, chunk) || n_experts <= 0 || n_experts > 256 ||
        top_k > n_experts || (shared_inter > 0 && (shared_inter % (2 * chunk) || shared_inter > 4096)))
        return ctx_fail(c, DS_CUDA_EINVAL, "moe_layer: unsupported shape hidden=%d inter=%d shared=%d E=%d k=%d",
                        hidden, inter, shared_inter, n_experts, top_k);
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_moe_layer_dev(ds_cuda_ctx_t *c, const float *d_x, float *d_out, const uint16_t *d_router,
                                     const uint16_t *d_block, const uint16_t *d_down, const uint16_t *d_sdown,
                                     int hidden, int inter, int shared_inter, int n_experts, int top_k,
                                     int *d_top_idx, float *d_top_w, void *stream) {
    if (!c || !d_x || !d_out || !d_router || !d_block || !d_down) return ctx_fail(c, DS_CUDA_EINVAL, "moe_layer_dev: null argument");
    CK(layer_checks(c, hidden, inter, shared_inter, n_experts, top_k, 8));
    cudaSetDevice(c->device);
    MoeArgs a = {};
    a.hidden = hidden;
    a.inter = inter;
    a.sh_inter = shared_inter;
    a.top_k = top_k;
    a.simulate = c->simulate;
    a.has_shared = shared_inter > 0 && d_sdown;
    size_t fused = (size_t)2 * inter * hidden;
    a.gu_base.w = d_block;
    a.gu_stride = (long long)fused;
    a.dn_base.w = d_down;
    a.dn_stride = (long long)hidden * inter;
    a.sh_gu.w = d_block + (size_t)n_experts * fused;
    a.sh_dn.w = d_sdown;
    a.x = d_x;
    a.out = d_out;
    CK(ensure_h(c, top_k * inter + shared_inter));
    a.h = c->d_h;
    return moe_layer_enqueue(c, a, d_router, n_experts, d_top_idx ? d_top_idx : c->d_idx,
                             d_top_w ? d_top_w : c->d_wt, pick_stream(c, stream), false);
}

extern "C" int ds_cuda_moe_layer(ds_cuda_ctx_t *c, const float *x, float *out, const uint16_t *router,
                                 const uint16_t *block, const uint16_t *down, const uint16_t *sdown, int hidden,
                                 int inter, int shared_inter, int n_experts, int top_k, int *top_idx, float *top_w) {
    if (!c || !x || !out || !router || !block || !down) return ctx_fail(c, DS_CUDA_EINVAL, "moe_layer: null argument");
    CK(layer_checks(c, hidden, inter, shared_inter, n_experts, top_k, 8));
    cudaSetDevice(c->device);
    size_t fused = (size_t)2 * inter * hidden;
    const uint16_t *dr = (const uint16_t *)ctx_lookup(c, router, (size_t)n_experts * hidden * 2, true);
    const uint16_t *db =
        (const uint16_t *)ctx_lookup(c, block, ((size_t)n_experts * fused + (size_t)2 * shared_inter * hidden) * 2, true);
    const uint16_t *dd = (const uint16_t *)ctx_lookup(c, down, (size_t)n_experts * hidden * inter * 2, true);
    const uint16_t *ds_ = shared_inter > 0 && sdown
                              ? (const uint16_t *)ctx_lookup(c, sdown, (size_t)hidden * shared_inter * 2, true)
                              : nullptr;
    if (!dr || !db || !dd || (shared_inter > 0 && sdown && !ds_))
        return ctx_fail(c, DS_CUDA_ENOTREG, "moe_layer: weight registration failed");
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, hidden));
    CK(ctx_grow(c, (void **)&c->d_out, &c->out_cap, (size_t)hidden * sizeof(float)));
    CK(ds_cuda_moe_layer_dev(c, c->d_x, c->d_out, dr, db, dd, ds_, hidden, inter, shared_inter, n_experts, top_k,
                             c->d_idx, c->d_wt, nullptr));
    CK(fetch_vec(c, out, c->d_out, hidden));
    if (top_idx) CK(d2h_sync(c, top_idx, c->d_idx, (size_t)top_k * sizeof(int)));
    if (top_w) CK(d2h_sync(c, top_w, c->d_wt, (size_t)top_k * sizeof(float)));
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_moe_layer_int8(ds_cuda_ctx_t *c, const float *x, float *out, const uint16_t *router,
                                      const int8_t *gu_q, const float *gu_s, const float *gu_o, const int8_t *dn_q,
                                      const float *dn_s, const float *dn_o, const int8_t *sgu_q, const float *sgu_s,
                                      const float *sgu_o, const int8_t *sdn_q, const float *sdn_s, const float *sdn_o,
                                      int hidden, int inter, int shared_inter, int n_experts, int top_k, int *top_idx,
                                      float *top_w) {
    if (!c || !x || !out || !router || !gu_q || !gu_s || !gu_o || !dn_q || !dn_s || !dn_o)
        return ctx_fail(c, DS_CUDA_EINVAL, "moe_layer_int8: null argument");
    bool shared = shared_inter > 0 && sgu_q && sdn_q;
    CK(layer_checks(c, hidden, inter, shared ? shared_inter : 0, n_experts, top_k, 16));
    cudaSetDevice(c->device);
    size_t E = (size_t)n_experts, H = hidden, I = inter, S = shared_inter;
    MoeArgs a = {};
    a.hidden = hidden;
    a.inter = inter;
    a.sh_inter = shared ? shared_inter : 0;
    a.top_k = top_k;
    a.int8 = 1;
    a.simulate = c->simulate;
    a.has_shared = shared;
    const uint16_t *dr = (const uint16_t *)ctx_lookup(c, router, E * H * 2, true);
    a.gu_base = WMat{ctx_lookup(c, gu_q, E * 2 * I * H, true), (const float *)ctx_lookup(c, gu_s, E * 2 * I * 4, true),
                     (const float *)ctx_lookup(c, gu_o, E * 2 * I * 4, true)};
    a.dn_base = WMat{ctx_lookup(c, dn_q, E * H * I, true), (const float *)ctx_lookup(c, dn_s, E * H * 4, true),
                     (const float *)ctx_lookup(c, dn_o, E * H * 4, true)};
    a.gu_stride = (long long)(2 * I * H);
    a.dn_stride = (long long)(H * I);
    if (shared) {
        a.sh_gu = WMat{ctx_lookup(c, sgu_q, 2 * S * H, true), (const float *)ctx_lookup(c, sgu_s, 2 * S * 4, true),
                       (const float *)ctx_lookup(c, sgu_o, 2 * S * 4, true)};
        a.sh_dn = WMat{ctx_lookup(c, sdn_q, H * S, true), (const float *)ctx_lookup(c, sdn_s, H * 4, true),
                       (const float *)ctx_lookup(c, sdn_o, H * 4, true)};
    }
    if (!dr || !a.gu_base.w || !a.gu_base.scale || !a.gu_base.off || !a.dn_base.w || !a.dn_base.scale ||
        !a.dn_base.off || (shared && (!a.sh_gu.w || !a.sh_gu.scale || !a.sh_gu.off || !a.sh_dn.w || !a.sh_dn.scale ||
                                      !a.sh_dn.off)))
        return ctx_fail(c, DS_CUDA_ENOTREG, "moe_layer_int8: weight registration failed");
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, hidden));
    CK(ctx_grow(c, (void **)&c->d_out, &c->out_cap, (size_t)hidden * sizeof(float)));
    CK(ensure_h(c, top_k * inter + a.sh_inter));
    a.x = c->d_x;
    a.out = c->d_out;
    a.h = c->d_h;
    CK(moe_layer_enqueue(c, a, dr, n_experts, c->d_idx, c->d_wt, c->stream, false));
    CK(fetch_vec(c, out, c->d_out, hidden));
    if (top_idx) CK(d2h_sync(c, top_idx, c->d_idx, (size_t)top_k * sizeof(int)));
    if (top_w) CK(d2h_sync(c, top_w, c->d_wt, (size_t)top_k * sizeof(float)));
    return DS_CUDA_OK;
}

// Device-pointer form of ds_cuda_moe_layer_int8 (every pointer device
// memory, enqueued on `stream`, nothing copied to or from the host).
extern "C" int ds_cuda_moe_layer_int8_dev(ds_cuda_ctx_t *c, const float *d_x, float *d_out, const uint16_t *d_router,
                                          const int8_t *gu_q, const float *gu_s, const float *gu_o,
                                          const int8_t *dn_q, const float *dn_s, const float *dn_o,
                                          const int8_t *sgu_q, const float *sgu_s, const float *sgu_o,
                                          const int8_t *sdn_q, const float *sdn_s, const float *sdn_o, int hidden,
                                          int inter, int shared_inter, int n_experts, int top_k, int *d_top_idx,
                                          float *d_top_w, void *stream) {
    if (!c || !d_x || !d_out || !d_router || !gu_q || !gu_s || !gu_o || !dn_q || !dn_s || !dn_o)
        return ctx_fail(c, DS_CUDA_EINVAL, "moe_layer_int8_dev: null argument");
    bool shared = shared_inter > 0 && sgu_q && sgu_s && sgu_o && sdn_q && sdn_s && sdn_o;
    CK(layer_checks(c, hidden, inter, shared ? shared_inter : 0, n_experts, top_k, 16));
    cudaSetDevice(c->device);
    size_t H = hidden, I = inter;
    MoeArgs a = {};
    a.hidden = hidden;
    a.inter = inter;
    a.sh_inter = shared ? shared_inter : 0;
    a.top_k = top_k;
    a.int8 = 1;
    a.simulate = c->simulate;
    a.has_shared = shared;
    a.gu_base = WMat{gu_q, gu_s, gu_o};
    a.dn_base = WMat{dn_q, dn_s, dn_o};
    a.gu_stride = (long long)(2 * I * H);
    a.dn_stride = (long long)(H * I);
    if (shared) {
        a.sh_gu = WMat{sgu_q, sgu_s, sgu_o};
        a.sh_dn = WMat{sdn_q, sdn_s, sdn_o};
    }
    a.x = d_x;
    a.out = d_out;
    CK(ensure_h(c, top_k * inter + a.sh_inter));
    a.h = c->d_h;
    return moe_layer_enqueue(c, a, d_router, n_experts, d_top_idx ? d_top_idx : c->d_idx,
                             d_top_w ? d_top_w : c->d_wt, pick_stream(c, stream), false);
}

// ---------------------------------------------------------------------------
// LM head argmax and matvec
// ---------------------------------------------------------------------------
extern "C" int ds_cuda_argmax_matvec_bf16_dev(ds_cuda_ctx_t *c, const float *d_x, const uint16_t *d_W, int in_dim,
                                              int out_dim, int *d_token, float *d_logit, void *stream) {
    if (!c || !d_x || !d_W || !d_token || out_dim <= 0) return ctx_fail(c, DS_CUDA_EINVAL, "argmax_dev: bad argument");
    if (in_dim <= 0 || in_dim % 8 || in_dim > 2048) return ctx_fail(c, DS_CUDA_EINVAL, "argmax_dev: in_dim %d unsupported", in_dim);
    cudaSetDevice(c->device);
    return ctx_cuda(c,
                    launch_argmax_bf16(d_W, d_x, out_dim, in_dim, c->d_slots, c->d_tickets + 0, d_token,
                                       d_logit ? d_logit : c->d_val, pick_stream(c, stream), false),
                    "argmax launch");
}

extern "C" int ds_cuda_argmax_matvec_bf16(ds_cuda_ctx_t *c, const float *x, const uint16_t *W, int in_dim,
                                          int out_dim, float *logit) {
    if (!c || !x || !W) return ctx_fail(c, DS_CUDA_EINVAL, "argmax: null argument");
    cudaSetDevice(c->device);
    const uint16_t *dW = (const uint16_t *)ctx_lookup(c, W, (size_t)out_dim * in_dim * 2, true);
    if (!dW) return ctx_fail(c, DS_CUDA_ENOTREG, "argmax: weight registration failed");
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, in_dim));
    CK(ds_cuda_argmax_matvec_bf16_dev(c, c->d_x, dW, in_dim, out_dim, c->d_tok, c->d_val, nullptr));
    int tok;
    float val;
    CK(d2h_sync(c, &tok, c->d_tok, sizeof(int)));
    CK(d2h_sync(c, &val, c->d_val, sizeof(float)));
    if (logit) *logit = val;
    return tok;
}

extern "C" int ds_cuda_lm_head_argmax(ds_cuda_ctx_t *c, const float *x, const uint16_t *W, int hidden, int vocab) {
    return ds_cuda_argmax_matvec_bf16(c, x, W, hidden, vocab, nullptr);
}

extern "C" int ds_cuda_argmax_matvec_bf16_batch(ds_cuda_ctx_t *c, const float *x, const uint16_t *W, int in_dim,
                                                int out_dim, int batch, int *tokens, float *logits) {
    if (!c || !x || !W || !tokens || batch <= 0 || batch > 512)
        return ctx_fail(c, DS_CUDA_EINVAL, "argmax_batch: bad argument");
    cudaSetDevice(c->device);
    const uint16_t *dW = (const uint16_t *)ctx_lookup(c, W, (size_t)out_dim * in_dim * 2, true);
    if (!dW) return ctx_fail(c, DS_CUDA_ENOTREG, "argmax_batch: weight registration failed");
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, in_dim * batch));
    CK(batch_argmax_enqueue(c, c->d_x, dW, in_dim, out_dim, batch, c->d_tok, c->d_val, c->stream));
    CK(d2h_sync(c, tokens, c->d_tok, (size_t)batch * sizeof(int)));
    if (logits) CK(d2h_sync(c, logits, c->d_val, (size_t)batch * sizeof(float)));
    return DS_CUDA_OK;
}

extern "C" int ds_cuda_argmax_matvec_bf16_batch_dev(ds_cuda_ctx_t *c, const float *d_x, const uint16_t *d_W,
                                                    int in_dim, int out_dim, int batch, int *d_tokens,
                                                    float *d_logits, void *stream) {
    if (!c || !d_x || !d_W || !d_tokens || !d_logits || batch <= 0 || batch > 512)
        return ctx_fail(c, DS_CUDA_EINVAL, "argmax_batch_dev: bad argument");
    cudaSetDevice(c->device);
    return batch_argmax_enqueue(c, d_x, d_W, in_dim, out_dim, batch, d_tokens, d_logits, pick_stream(c, stream));
}

extern "C" int ds_cuda_matvec_bf16(ds_cuda_ctx_t *c, float *y, const float *x, const uint16_t *W, const float *bias,
                                   int in_dim, int out_dim) {
    if (!c || !y || !x || !W || out_dim <= 0) return ctx_fail(c, DS_CUDA_EINVAL, "matvec: null argument");
    if (in_dim <= 0 || in_dim % 8 || in_dim > 2048) return ctx_fail(c, DS_CUDA_EINVAL, "matvec: in_dim %d unsupported", in_dim);
    cudaSetDevice(c->device);
    const uint16_t *dW = (const uint16_t *)ctx_lookup(c, W, (size_t)out_dim * in_dim * 2, true);
    const float *db = bias ? (const float *)ctx_lookup(c, bias, (size_t)out_dim * 4, true) : nullptr;
    if (!dW || (bias && !db)) return ctx_fail(c, DS_CUDA_ENOTREG, "matvec: weight registration failed");
    CK(stage_vec(c, &c->d_x, &c->x_cap, x, in_dim));
    CK(ctx_grow(c, (void **)&c->d_out, &c->out_cap, (size_t)out_dim * sizeof(float)));
    CK(ctx_cuda(c, launch_matvec_bf16(dW, c->d_x, db, c->d_out, out_dim, in_dim, c->stream, false), "matvec launch"));
    return fetch_vec(c, y, c->d_out, out_dim);
}

extern "C" int ds_cuda_int8_quantize_bf16(ds_cuda_ctx_t *c, const uint16_t *W, int out_dim, int in_dim, int8_t *q,
                                          float *scale, float *off) {
    if (!c || !W || !q || !scale || !off || out_dim <= 0 || in_dim <= 0)
        return ctx_fail(c, DS_CUDA_EINVAL, "int8_quantize: bad argument");
    cudaSetDevice(c->device);
    size_t nW = (size_t)out_dim * in_dim;
    size_t need = nW * 2 + nW + (size_t)out_dim * 8 + 256;
    CK(ctx_grow(c, &c->d_tmp, &c->tmp_cap, need));
    uint16_t *dW = (uint16_t *)c->d_tmp;
    int8_t *dq = (int8_t *)(dW + nW);
    float *ds_ = (float *)(((uintptr_t)(dq + nW) + 15) & ~uintptr_t(15));
    float *dof = ds_ + out_dim;
    CK(ctx_cuda(c, cudaMemcpyAsync(dW, W, nW * 2, cudaMemcpyHostToDevice, c->stream), "copy weights"));
    CK(ctx_cuda(c, launch_quantize_int8(dW, out_dim, in_dim, dq, ds_, dof, c->stream), "quantize launch"));
    CK(ctx_cuda(c, cudaMemcpyAsync(q, dq, nW, cudaMemcpyDeviceToHost, c->stream), "copy q"));
    CK(ctx_cuda(c, cudaMemcpyAsync(scale, ds_, (size_t)out_dim * 4, cudaMemcpyDeviceToHost, c->stream), "copy scale"));
    CK(ctx_cuda(c, cudaMemcpyAsync(off, dof, (size_t)out_dim * 4, cudaMemcpyDeviceToHost, c->stream), "copy offset"));
    return ctx_cuda(c, cudaStreamSynchronize(c->stream), "synchronize");
}
