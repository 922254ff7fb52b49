// mega.cu — the whole greedy decode (ds_decoder_forward, ds_moe_decoder.c:911-
// 1264, repeated for n tokens) as ONE persistent kernel.
//
// One CTA per SM (cooperative launch, so all CTAs are co-resident). The step
// is a fixed sequence of phases separated by grid barriers:
//   per layer:  QKV(+RoPE, KV append) | attention scores | attention PV |
//               O-proj + residual | dense: gate_up, down   or
//               MoE: router + shared gate_up, routed gate_up, down + combine
//   then:       LM head argmax
// Each phase is cut into chunks of at most MK_REGION bytes of weights per
// CTA. Two shared-memory regions form a double buffer: while a chunk is
// computed from one region, one thread has already issued cp.async.bulk
// copies (TMA engine, mbarrier completion) of the CTA's slice of the NEXT
// chunk into the other region — across the grid barrier, so HBM keeps
// streaming while CTAs synchronise. Only the routed experts' weights depend
// on data (the router's top-k): their copies are issued right after the
// barrier that publishes the router scores.
//
// Numerics are those of the multi-kernel path (kernels_moe.cu,
// kernels_decode.cu): F32 FMA accumulation of BF16-widened weights,
// fast-exp softmax and SwiGLU, the reference's combine order, and the
// exact unrolled form of the sequential fast-exp online-softmax attention.
//
// Every wait is bounded: a grid barrier or mbarrier that does not complete
// within its poll budget sets bar[2] and the kernel returns; the host reports
// DS_CUDA_ETIMEOUT.
#include "kernels_moe.cuh"
#include "launch.h"
#include "mega.h"

namespace ds {

constexpr int MK_THREADS = 512;
constexpr int MK_WARPS = MK_THREADS / 32;
constexpr int MK_NREG = 4;             // weight regions in the shared-memory ring
constexpr int MK_REGION = 46 * 1024;  // bytes per weight region
constexpr int MK_XS = 8192;           // floats of vector scratch (also attention scratch)
constexpr int MK_SMEM = MK_NREG * MK_REGION + MK_XS * 4;

enum Phase { PH_QKV, PH_ATTS, PH_ATTV, PH_OPROJ, PH_DGU, PH_DDOWN, PH_RSGU, PH_RGU, PH_MDOWN, PH_LMH, PH_END };

struct Cur {
    int step, layer, phase;
};

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ldcg16(const void *p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ void split_range(int total, int parts, int i, int &a, int &b) {
    a = (int)((long long)total * i / parts);
    b = (int)((long long)total * (i + 1) / parts);
}
__device__ __forceinline__ uint16_t bf16_bits_rne(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Grid-wide barrier over co-resident CTAs, bounded: returns false (and sets
// *err) if it does not complete within its poll budget or another CTA failed.
// bar[0] counts arrivals monotonically (never reset within a launch): the
// n-th barrier completes when it reaches n * gridDim.x. One release-add per
// CTA, then acquire polls; the error flag is checked only every 256 polls.
__device__ bool grid_sync(unsigned *bar, unsigned &epoch) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        epoch++;
        const unsigned target = epoch * gridDim.x;
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(bar), "r"(1u) : "memory");
        int good = 0;
        for (uint32_t it = 0; it < (1u << 24); it++) {
            if ((int)(ld_acquire(bar) - target) >= 0) {
                good = 1;
                break;
            }
            if ((it & 255) == 255 && ld_acquire(bar + 2)) break;
        }
        if (!good) atomicExch(bar + 2, 1u);
        ok = good;
    }
    __syncthreads();
    return ok != 0;
}

// Block-wide exclusive scan (512 threads, one value per thread): warp 0,
// lane l owns 16 consecutive slots, then a shuffle scan of lane totals.
template <typename Op>
__device__ float block_scan512(float v, float ident, Op op, bool reverse, float *buf) {
    const int t = threadIdx.x;
    const int lt = reverse ? MK_THREADS - 1 - t : t;
    buf[lt] = v;
    __syncthreads();
    if (t < 32) {
        float loc[16], acc = ident;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            loc[i] = acc;
            acc = op(acc, buf[t * 16 + i]);
        }
        float inc = acc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            float y = __shfl_up_sync(DS_FULL, inc, o);
            if (t >= o) inc = op(y, inc);
        }
        float excl = __shfl_up_sync(DS_FULL, inc, 1);
        if (t == 0) excl = ident;
#pragma unroll
        for (int i = 0; i < 16; i++) buf[t * 16 + i] = op(excl, loc[i]);
    }
    __syncthreads();
    float r = buf[lt];
    __syncthreads();
    return r;
}

__device__ float block_sum512(float v, float *buf) {
    buf[threadIdx.x] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) s = __fadd_rn(s, buf[threadIdx.x * 16 + i]);
        s = warp_sum(s);
        if (threadIdx.x == 0) buf[MK_THREADS] = s;
    }
    __syncthreads();
    float r = buf[MK_THREADS];
    __syncthreads();
    return r;
}

// xs[0..n) = src (L2-coherent loads: src was written by other CTAs), then
// optionally RMS-normalised in place with the order of block_rms_inv.
__device__ void load_vec(float *xs, const float *src, int n) {
    for (int i = threadIdx.x * 4; i < n; i += MK_THREADS * 4) {
        uint4 u = ldcg16(src + i);
        *reinterpret_cast<uint4 *>(xs + i) = u;
    }
    __syncthreads();
}
__device__ void norm_vec(float *xs, const float *w, int n, float eps) {
    const float inv = block_rms_inv(xs, n, eps);
    for (int i = threadIdx.x; i < n; i += MK_THREADS) xs[i] = __fmul_rn(__fmul_rn(xs[i], w[i]), inv);
    __syncthreads();
}

// ---------------------------------------------------------------------------
// phase geometry: items of this CTA, items per chunk, bytes per item
// ---------------------------------------------------------------------------
struct Geo {
    int a, b;        // item range of this CTA
    int ipc;         // items per chunk
    int nsub;        // chunks
};

__device__ __forceinline__ int item_bytes(const MegaParams &p, int phase) {
    switch (phase) {
        case PH_QKV: case PH_DGU: case PH_RGU: case PH_RSGU: return 4 * p.H;  // gate + up rows
        case PH_OPROJ: return 2 * p.NH * p.HD;
        case PH_DDOWN: return 2 * p.D;
        case PH_MDOWN: return 2 * (p.K * p.I + p.S);
        case PH_LMH: return 2 * p.H;
        default: return 0;
    }
}

__device__ Geo compute_geometry(const MegaParams &p, int phase) {
    Geo g = {0, 0, 1, 1};
    int total = 0;
    switch (phase) {
        case PH_QKV: total = 3 * p.NH * (p.HD / 2); break;
        case PH_OPROJ: case PH_DDOWN: case PH_MDOWN: total = p.H; break;
        case PH_DGU: total = p.D; break;
        case PH_RSGU: total = p.S; break;  // + its router rows (one chunk, checked on the host)
        case PH_RGU: total = p.K * p.I; break;
        case PH_LMH: total = p.V; break;
        default: return g;
    }
    split_range(total, gridDim.x, blockIdx.x, g.a, g.b);
    // the same chunk count on every CTA (balanced by the largest share), so
    // no CTA trails the others into the next barrier by a whole chunk; the
    // router rows of PH_RSGU ride in its last chunk
    const int G = gridDim.x;
    const int cmax = (total + G - 1) / G;
    const int extra = phase == PH_RSGU ? ((p.E + G - 1) / G) * 2 * p.H : 0;
    const int cap = max(1, (MK_REGION - extra) / item_bytes(p, phase));
    g.nsub = max(1, (cmax + cap - 1) / cap);
    g.ipc = max(1, (cmax + g.nsub - 1) / g.nsub);
    return g;
}

// Per-CTA geometry of every phase and this CTA's router rows, computed once
// at kernel start (the issuing thread must not redo integer divisions per
// chunk: it sits on the critical path of its warp).
__shared__ Geo s_geo[PH_END];
__shared__ int s_ea, s_eb;
__device__ __forceinline__ Geo geometry(const MegaParams &, int phase) { return s_geo[phase]; }

__device__ __forceinline__ void next_phase(const MegaParams &p, Cur &c) {
    const MegaLayer &L = p.layers[c.layer];
    switch (c.phase) {
        case PH_QKV: c.phase = PH_ATTS; return;
        case PH_ATTS: c.phase = PH_ATTV; return;
        case PH_ATTV: c.phase = PH_OPROJ; return;
        case PH_OPROJ: c.phase = L.dense ? PH_DGU : PH_RSGU; return;
        case PH_DGU: c.phase = PH_DDOWN; return;
        case PH_RSGU: c.phase = PH_RGU; return;
        case PH_RGU: c.phase = PH_MDOWN; return;
        case PH_DDOWN: case PH_MDOWN:
            if (c.layer + 1 < p.L) { c.layer++; c.phase = PH_QKV; } else c.phase = PH_LMH;
            return;
        case PH_LMH:
            if (c.step + 1 < p.n_steps) { c.step++; c.layer = 0; c.phase = PH_QKV; } else c.phase = PH_END;
            return;
        default: c.phase = PH_END;
    }
}

// ---------------------------------------------------------------------------
// loads: bytes of a chunk (all threads agree) and issuing them (one thread)
// ---------------------------------------------------------------------------
__device__ uint32_t chunk_bytes(const MegaParams &p, const Cur &c, int sub) {
    if (c.phase == PH_ATTS || c.phase == PH_ATTV || c.phase == PH_END) return 0;
    Geo g = geometry(p, c.phase);
    int ia = g.a + sub * g.ipc, ib = min(g.b, ia + g.ipc);
    uint32_t n = ib > ia ? (uint32_t)(ib - ia) * item_bytes(p, c.phase) : 0;
    if (c.phase == PH_RSGU && sub == g.nsub - 1) {
        int ea, eb;
        ea = s_ea;
        eb = s_eb;
        n += (uint32_t)(eb - ea) * 2 * p.H;
    }
    return n;
}

// Issues the bulk copies of chunk (c, sub) into region `dst` completing on
// `bar`. sidx: the layer's routed experts (needed for PH_RGU / PH_MDOWN).
__device__ void issue_chunk(const MegaParams &p, const Cur &c, int sub, uint8_t *dst, uint64_t *bar,
                            const int *sidx) {
    uint32_t total = chunk_bytes(p, c, sub);
    if (total == 0) return;
    mbar_expect_tx(bar, total);
    const MegaLayer &L = p.layers[c.layer];
    Geo g = geometry(p, c.phase);
    const int ia = g.a + sub * g.ipc, ib = min(g.b, ia + g.ipc), cnt = max(0, ib - ia);
    const uint32_t rb = 2 * p.H;  // hidden-length BF16 row
    switch (c.phase) {
        case PH_QKV: {
            // pair t: rows (h*HD + d, h*HD + d + HD/2) of Wq/Wk/Wv; runs of
            // consecutive d within one (matrix, head) are contiguous
            const int half = p.HD / 2, per = p.NH * half;
            int t = ia;
            while (t < ib) {
                int m = t / per, r = t - m * per, h = r / half, d = r - h * half;
                int run = min(ib - t, half - d);
                const uint16_t *W = m == 0 ? L.wq : (m == 1 ? L.wk : L.wv);
                const uint16_t *g0 = W + (size_t)(h * p.HD + d) * p.H;
                bulk_g2s(dst + (size_t)(t - ia) * rb, g0, run * rb, bar);
                bulk_g2s(dst + (size_t)(cnt + t - ia) * rb, g0 + (size_t)half * p.H, run * rb, bar);
                t += run;
            }
            break;
        }
        case PH_DGU:
            bulk_g2s(dst, L.dgate + (size_t)ia * p.H, cnt * rb, bar);
            bulk_g2s(dst + (size_t)cnt * rb, L.dup + (size_t)ia * p.H, cnt * rb, bar);
            break;
        case PH_RSGU: {
            const uint16_t *sgu = L.block + (size_t)p.E * 2 * p.I * p.H;
            if (cnt > 0) {
                bulk_g2s(dst, sgu + (size_t)ia * p.H, cnt * rb, bar);
                bulk_g2s(dst + (size_t)cnt * rb, sgu + (size_t)(p.S + ia) * p.H, cnt * rb, bar);
            }
            if (sub == g.nsub - 1) {
                int ea, eb;
                ea = s_ea;
                eb = s_eb;
                if (eb > ea) bulk_g2s(dst + (size_t)2 * cnt * rb, L.router + (size_t)ea * p.H, (eb - ea) * rb, bar);
            }
            break;
        }
        case PH_RGU: {
            int t = ia;
            while (t < ib) {
                int k = t / p.I, i = t - k * p.I;
                int run = min(ib - t, p.I - i);
                const uint16_t *gu = L.block + (size_t)sidx[k] * 2 * p.I * p.H;
                bulk_g2s(dst + (size_t)(t - ia) * rb, gu + (size_t)i * p.H, run * rb, bar);
                bulk_g2s(dst + (size_t)(cnt + t - ia) * rb, gu + (size_t)(p.I + i) * p.H, run * rb, bar);
                t += run;
            }
            break;
        }
        case PH_OPROJ:
            bulk_g2s(dst, L.wo + (size_t)ia * p.NH * p.HD, cnt * 2 * p.NH * p.HD, bar);
            break;
        case PH_DDOWN:
            bulk_g2s(dst, L.ddown + (size_t)ia * p.D, cnt * 2 * p.D, bar);
            break;
        case PH_MDOWN: {
            for (int k = 0; k < p.K; k++)
                bulk_g2s(dst + (size_t)k * cnt * 2 * p.I,
                         L.down + (size_t)sidx[k] * p.H * p.I + (size_t)ia * p.I, cnt * 2 * p.I, bar);
            bulk_g2s(dst + (size_t)p.K * cnt * 2 * p.I, L.sdown + (size_t)ia * p.S, cnt * 2 * p.S, bar);
            break;
        }
        case PH_LMH:
            bulk_g2s(dst, p.lm_head + (size_t)ia * p.H, cnt * rb, bar);
            break;
        default:
            break;
    }
}

// True when chunk (n, nsub) may be loaded before the barrier that precedes
// it: routed-expert chunks need the router result of their own layer, which
// exists once the CTA is past that layer's router phase.
__device__ __forceinline__ bool loadable_now(const Cur &cur, const Cur &nx) {
    if (nx.phase != PH_RGU && nx.phase != PH_MDOWN) return true;
    return cur.layer == nx.layer && cur.step == nx.step && (cur.phase == PH_RGU || cur.phase == PH_MDOWN);
}

// ---------------------------------------------------------------------------
// compute helpers: dot of a smem BF16 row with the register slice
// ---------------------------------------------------------------------------
template <int CPL>
__device__ __forceinline__ float sdot(const uint16_t *row, int n, const XRegBF16<CPL> &x, int lane) {
    const int nch = n >> 3;
    uint4 w[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        int ch = lane + 32 * c;
        w[c] = ch < nch ? *reinterpret_cast<const uint4 *>(row + 8 * ch) : make_uint4(0, 0, 0, 0);
    }
    // two independent FMA chains (even / odd chunks) for instruction-level parallelism
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        if (c & 1) a1 = dot8_bf16(w[c], x.v[c][0], x.v[c][1], a1);
        else a0 = dot8_bf16(w[c], x.v[c][0], x.v[c][1], a0);
    }
    return __fadd_rn(a0, a1);
}

// Long row (n up to MK_XS) against a vector in shared memory.
__device__ __forceinline__ float sdot_long(const uint16_t *row, const float *xs, int n, int lane) {
    const int nch = n >> 3;
    float acc = 0.f;
    for (int ch = lane; ch < nch; ch += 32) {
        const float4 *xp = reinterpret_cast<const float4 *>(xs + 8 * ch);
        acc = dot8_bf16(*reinterpret_cast<const uint4 *>(row + 8 * ch), xp[0], xp[1], acc);
    }
    return acc;
}

// One KV row slice (16 head-dim elements, hi and lo planes) of key j, or
// zeros when j >= j1; L2-coherent loads (rows are written inside the launch).
__device__ __forceinline__ void kv_row(const uint16_t *hi, const uint16_t *lo, int j, int j1, int lo_start, int hd,
                                       int li, uint4 r[4]) {
    r[0] = r[1] = r[2] = r[3] = make_uint4(0, 0, 0, 0);
    if (j >= j1) return;
    const size_t o = (size_t)j * hd + li * 16;
    r[0] = ldcg16(hi + o);
    r[1] = ldcg16(hi + o + 8);
    if (j >= lo_start) {
        r[2] = ldcg16(lo + o);
        r[3] = ldcg16(lo + o + 8);
    }
}
__device__ __forceinline__ float kv_dot(const uint4 r[4], const float qf[16]) {
    uint32_t hw[8] = {r[0].x, r[0].y, r[0].z, r[0].w, r[1].x, r[1].y, r[1].z, r[1].w};
    uint32_t lw[8] = {r[2].x, r[2].y, r[2].z, r[2].w, r[3].x, r[3].y, r[3].z, r[3].w};
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        s = __fmaf_rn(qf[2 * i], __fadd_rn(bf16_lo(hw[i]), bf16_lo(lw[i])), s);
        s = __fmaf_rn(qf[2 * i + 1], __fadd_rn(bf16_hi(hw[i]), bf16_hi(lw[i])), s);
    }
    return s;
}
__device__ __forceinline__ void kv_axpy(const uint4 r[4], float w, float acc[16]) {
    uint32_t hw[8] = {r[0].x, r[0].y, r[0].z, r[0].w, r[1].x, r[1].y, r[1].z, r[1].w};
    uint32_t lw[8] = {r[2].x, r[2].y, r[2].z, r[2].w, r[3].x, r[3].y, r[3].z, r[3].w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        acc[2 * i] = __fmaf_rn(w, __fadd_rn(bf16_lo(hw[i]), bf16_lo(lw[i])), acc[2 * i]);
        acc[2 * i + 1] = __fmaf_rn(w, __fadd_rn(bf16_hi(hw[i]), bf16_hi(lw[i])), acc[2 * i + 1]);
    }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(MK_THREADS, 1) mega_decode_kernel(const MegaParams *__restrict__ pp) {
    extern __shared__ __align__(128) uint8_t smem[];
    float *xs = reinterpret_cast<float *>(smem + MK_NREG * MK_REGION);
    __shared__ uint64_t full[MK_NREG];
    __shared__ float buf[MK_THREADS + 1];
    __shared__ float ysm[8][8];
    __shared__ int sidx[8];
    __shared__ float swt[8];
    __shared__ float rsc[256];
    __shared__ int s_tok;
    __shared__ unsigned long long cta_best;
    const MegaParams &p = *pp;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned *err = p.bar + 2;
    constexpr int CPL = 5;  // hidden 1280 = 5 x 256 (checked on the host)

    if (tid == 0) {
        for (int i = 0; i < MK_NREG; i++) mbar_init(&full[i], 1);
        mbar_fence_init();
        split_range(p.E, gridDim.x, blockIdx.x, s_ea, s_eb);
    }
    if (tid < PH_END) s_geo[tid] = compute_geometry(p, tid);
    __syncthreads();

    int pos = *p.pos;
    unsigned epoch = 0;  // grid barriers passed
    int tok = 0;
    Cur cur = {0, 0, PH_QKV};
    int chunk_id = 0;    // chunk counter: chunk c computes from region c % MK_NREG
    // optional timing trace: CTA 0 and the last CTA, 5 values per chunk
    const int trace_sel = p.trace == nullptr ? -1 : (blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x - 1 ? 1 : -1));
    long long t_bar0 = 0, t_bar1 = 0;
#define MK_TRACE(slot, val)                                                                                    \
    do {                                                                                                        \
        if (trace_sel >= 0 && tid == 0 && chunk_id < p.trace_cap)                                               \
            p.trace[((size_t)trace_sel * p.trace_cap + chunk_id) * 5 + (slot)] = (val);                         \
    } while (0)
    uint32_t uses = 0;  // one parity bit per region
    // issue cursor (thread 0): the next chunk whose copies are not issued yet
    Cur ic = cur;
    int isub = 0, iid = 0;
    bool first = true;

    while (cur.phase != PH_END) {
        Geo geo = geometry(p, cur.phase);
        const MegaLayer &L = p.layers[cur.layer];
        // ---- barrier that publishes the previous phase's outputs ----
        if (!first) {
            t_bar0 = clock64();
            if (!grid_sync(p.bar, epoch)) return;
            t_bar1 = clock64();
        }
        first = false;
        // new step: decode the previous step's token
        if (cur.phase == PH_QKV && cur.layer == 0 && (cur.step > 0 || p.first_from_token)) {
            if (tid == 0) {
                if (cur.step > 0) {
                    unsigned long long k = atomicAdd(&p.slot[(cur.step - 1) & 1], 0ull);
                    s_tok = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
                    if (blockIdx.x == 0) {
                        p.tok_log[pos] = s_tok;
                        p.slot[cur.step & 1] = 0ull;
                    }
                } else {
                    s_tok = *p.tok;
                }
            }
            __syncthreads();
            tok = s_tok;
            if (tok < 0 || tok >= p.V) tok = 0;  // no winner (all-NaN logits): embed row 0
            if (cur.step > 0) pos++;
        }
        // routed phases: every CTA derives the layer's top-k from the scores
        if (cur.phase == PH_RGU) {
            for (int e = tid; e < p.E; e += MK_THREADS) rsc[e] = __ldcg(p.rscore + e);
            __syncthreads();
            if (tid < 32) router_select(rsc, p.E, p.K, p.renorm, sidx, swt);
            __syncthreads();
        }
        for (int sub = 0; sub < geo.nsub; sub++, chunk_id++) {
            const int r = chunk_id % MK_NREG;
            const uint32_t bytes = chunk_bytes(p, cur, sub);
            // keep up to MK_NREG chunks in flight: issue every chunk up to
            // chunk_id + MK_NREG - 1 whose addresses are known by now (the
            // region of chunk i was last used by chunk i - MK_NREG, done)
            if (tid == 0) {
                while (iid <= chunk_id + MK_NREG - 1 && ic.phase != PH_END && loadable_now(cur, ic)) {
                    const int ir = iid % MK_NREG;
                    if (chunk_bytes(p, ic, isub)) {
                        fence_proxy_async();
                        issue_chunk(p, ic, isub, smem + ir * MK_REGION, &full[ir], sidx);
                    }
                    if (++isub >= geometry(p, ic.phase).nsub) {
                        isub = 0;
                        next_phase(p, ic);
                    }
                    iid++;
                }
            }
            if (bytes) {
                if (!mbar_wait(&full[r], (uses >> r) & 1, err)) return;
                uses ^= 1u << r;
            }
            MK_TRACE(0, (long long)(cur.phase | (sub << 8) | (cur.layer << 16) | ((long long)cur.step << 24)));
            MK_TRACE(1, sub == 0 ? t_bar0 : 0);
            MK_TRACE(2, sub == 0 ? t_bar1 : 0);
            MK_TRACE(3, clock64());
            const uint16_t *W = reinterpret_cast<const uint16_t *>(smem + r * MK_REGION);
            const int ia = geo.a + sub * geo.ipc, ib = min(geo.b, ia + geo.ipc), cnt = max(0, ib - ia);

            switch (cur.phase) {
                case PH_QKV: {
                    // input: the token embedding (layer 0 of a token-fed step) or
                    // xa, normalised once per phase (xs persists across its chunks)
                    if (sub == 0) {
                        if (cur.layer == 0 && (cur.step > 0 || p.first_from_token)) {
                            const uint16_t *e = p.embed + (size_t)tok * p.H;
                            for (int i = tid; i < p.H; i += MK_THREADS) xs[i] = __uint_as_float((uint32_t)e[i] << 16);
                            __syncthreads();
                            int xa0, xa1;
                            split_range(p.H, gridDim.x, blockIdx.x, xa0, xa1);
                            for (int i = xa0 + tid; i < xa1; i += MK_THREADS) p.xa[i] = xs[i];
                        } else {
                            load_vec(xs, p.xa, p.H);
                        }
                        norm_vec(xs, L.in_norm, p.H, p.eps);
                    }
                    XRegBF16<CPL> xr;
                    xr.load(xs, p.H, lane);
                    const int half = p.HD / 2, per = p.NH * half;
                    for (int i = warp; i < cnt; i += MK_WARPS) {
                        float s0 = warp_sum(sdot<CPL>(W + (size_t)i * p.H, p.H, xr, lane));
                        float s1 = warp_sum(sdot<CPL>(W + (size_t)(cnt + i) * p.H, p.H, xr, lane));
                        if (lane == 0) {
                            int t = ia + i, m = t / per, rr = t - m * per, h = rr / half, d = rr - h * half;
                            int row0 = h * p.HD + d;
                            float o0 = s0, o1 = s1;
                            if (m < 2) {
                                const float *cs = p.cos_t + (size_t)pos * p.HD, *sn = p.sin_t + (size_t)pos * p.HD;
                                o0 = __fsub_rn(__fmul_rn(s0, cs[d]), __fmul_rn(s1, sn[d]));
                                o1 = __fadd_rn(__fmul_rn(s0, sn[d + half]), __fmul_rn(s1, cs[d + half]));
                            }
                            if (m == 0) {
                                p.q[row0] = o0;
                                p.q[row0 + half] = o1;
                            } else {
                                size_t idx = ((size_t)h * p.kv_max + pos) * p.HD + d;
                                uint16_t *hi = m == 1 ? L.k_hi : L.v_hi, *lo = m == 1 ? L.k_lo : L.v_lo;
                                uint16_t a0 = bf16_bits_rne(o0), a1 = bf16_bits_rne(o1);
                                hi[idx] = a0;
                                hi[idx + half] = a1;
                                lo[idx] = bf16_bits_rne(__fsub_rn(o0, __uint_as_float((uint32_t)a0 << 16)));
                                lo[idx + half] = bf16_bits_rne(__fsub_rn(o1, __uint_as_float((uint32_t)a1 << 16)));
                            }
                        }
                    }
                    break;
                }
                case PH_ATTS:
                case PH_ATTV: {
                    const int cph = min(16, (int)gridDim.x / p.NH);  // CTAs per head (<= 16 partials)
                    const int h = blockIdx.x / cph, cc = blockIdx.x - h * cph;
                    if (h >= p.NH) break;
                    const int n = pos + 1;
                    const int per = (n + cph - 1) / cph;
                    const int j0 = min(n, cc * per), j1 = min(n, j0 + per);
                    const int g = tid >> 3, li = tid & 7;
                    const size_t hoff = (size_t)h * p.kv_max * p.HD;
                    const uint16_t *khi = L.k_hi + hoff, *klo = L.k_lo + hoff;
                    const uint16_t *vhi = L.v_hi + hoff, *vlo = L.v_lo + hoff;
                    float *wts = xs, *corr = xs + MK_XS / 2;
                    if (cur.phase == PH_ATTS) {
                        // this group's first key and q in one round trip
                        uint4 kr[4];
                        kv_row(khi, klo, j0 + g, j1, L.lo_start, p.HD, li, kr);
                        float qf[16];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            uint4 u = ldcg16(p.q + h * p.HD + li * 16 + 4 * i);
                            qf[4 * i] = __uint_as_float(u.x); qf[4 * i + 1] = __uint_as_float(u.y);
                            qf[4 * i + 2] = __uint_as_float(u.z); qf[4 * i + 3] = __uint_as_float(u.w);
                        }
                        for (int jb = j0; jb < j1; jb += MK_THREADS / 8) {
                            int j = jb + g;
                            if (jb != j0) kv_row(khi, klo, j, j1, L.lo_start, p.HD, li, kr);
                            float s = kv_dot(kr, qf);
                            s += __shfl_xor_sync(DS_FULL, s, 1);
                            s += __shfl_xor_sync(DS_FULL, s, 2);
                            s += __shfl_xor_sync(DS_FULL, s, 4);
                            if (li == 0 && j < j1) p.att_sc[(size_t)h * p.kv_max + j] = __fmul_rn(s, p.scale);
                        }
                    } else {
                        // this group's first V row and every key's score of the head in
                        // one round trip -> exact unrolled weights
                        uint4 vr[4];
                        kv_row(vhi, vlo, j0 + g, j1, L.lo_start, p.HD, li, vr);
                        for (int j = tid; j < n; j += MK_THREADS) wts[j] = __ldcg(p.att_sc + (size_t)h * p.kv_max + j);
                        __syncthreads();
                        const int seg = (n + MK_THREADS - 1) / MK_THREADS;
                        const int s0 = min(n, tid * seg), s1 = min(n, s0 + seg);
                        float lm = -1e30f;
                        for (int j = s0; j < s1; j++) lm = fmaxf(lm, wts[j]);
                        float m = block_scan512(lm, -1e30f, [](float x, float y) { return fmaxf(x, y); }, false, buf);
                        for (int j = s0; j < s1; j++) {
                            float s = wts[j];
                            if (s > m) {
                                corr[j] = fast_expf(__fsub_rn(m, s));
                                wts[j] = 1.0f;
                                m = s;
                            } else {
                                corr[j] = 1.0f;
                                wts[j] = fast_expf(__fsub_rn(s, m));
                            }
                        }
                        float lp = 1.0f;
                        for (int j = s1 - 1; j >= s0; j--) lp = __fmul_rn(lp, corr[j]);
                        float P = block_scan512(lp, 1.0f, [](float x, float y) { return __fmul_rn(x, y); }, true, buf);
                        for (int j = s1 - 1; j >= s0; j--) {
                            wts[j] = __fmul_rn(wts[j], P);
                            P = __fmul_rn(P, corr[j]);
                        }
                        float lsum = 0.f;
                        for (int j = s0; j < s1; j++) lsum = __fadd_rn(lsum, wts[j]);
                        float S = block_sum512(lsum, buf);
                        // this CTA's keys: sum_j w_j v_j
                        float acc[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) acc[i] = 0.f;
                        for (int jb = j0; jb < j1; jb += MK_THREADS / 8) {
                            int j = jb + g;
                            if (jb != j0) kv_row(vhi, vlo, j, j1, L.lo_start, p.HD, li, vr);
                            if (j < j1) kv_axpy(vr, wts[j], acc);
                        }
                        // reduce the 4 groups of each warp, then the 16 warps
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            acc[i] += __shfl_xor_sync(DS_FULL, acc[i], 8);
                            acc[i] += __shfl_xor_sync(DS_FULL, acc[i], 16);
                        }
                        __syncthreads();  // corr is reused as the [16][128] reduction buffer
                        if (lane < 8)
#pragma unroll
                            for (int i = 0; i < 16; i++) corr[warp * 128 + li * 16 + i] = acc[i];
                        __syncthreads();
                        if (tid < 128) {
                            float o = 0.f;
                            for (int w = 0; w < MK_WARPS; w++) o = __fadd_rn(o, corr[w * 128 + tid]);
                            p.att_part[((size_t)h * gridDim.x + cc) * p.HD + tid] = o;
                            if (cc == 0 && tid == 0) p.att_sum[h] = S;
                        }
                    }
                    break;
                }
                case PH_OPROJ: {
                    // attention output = sum of the head's partials / sum of weights
                    const int cph = min(16, (int)gridDim.x / p.NH);  // CTAs per head (<= 16 partials)
                    for (int i = tid; i < p.NH * p.HD; i += MK_THREADS) {
                        int h = i / p.HD, d = i - h * p.HD;
                        // all partials of this element in one round trip, summed in order
                        float v[16];
#pragma unroll
                        for (int cc = 0; cc < 16; cc++)
                            v[cc] = cc < cph ? __ldcg(p.att_part + ((size_t)h * gridDim.x + cc) * p.HD + d) : 0.f;
                        float S = __ldcg(p.att_sum + h);
                        float o = 0.f;
                        for (int cc = 0; cc < cph; cc++) o = __fadd_rn(o, v[cc]);
                        xs[i] = S > 0.f ? __fmul_rn(o, __fdiv_rn(1.0f, S)) : o;
                    }
                    __syncthreads();
                    XRegBF16<CPL> xr;
                    xr.load(xs, p.NH * p.HD, lane);
                    for (int i = warp; i < cnt; i += MK_WARPS) {
                        float s = warp_sum(sdot<CPL>(W + (size_t)i * p.NH * p.HD, p.NH * p.HD, xr, lane));
                        if (lane == 0) p.xb[ia + i] = __fadd_rn(__ldcg(p.xa + ia + i), s);
                    }
                    break;
                }
                case PH_DGU:
                case PH_RSGU:
                case PH_RGU: {
                    if (sub == 0) {
                        load_vec(xs, p.xb, p.H);
                        norm_vec(xs, L.post_norm, p.H, p.eps);
                    }
                    XRegBF16<CPL> xr;
                    xr.load(xs, p.H, lane);
                    const bool sim = p.simulate && cur.phase != PH_DGU;
                    float *hout = cur.phase == PH_RGU ? p.h : (cur.phase == PH_RSGU ? p.h + p.K * p.I : p.h);
                    for (int i = warp; i < cnt; i += MK_WARPS) {
                        float g = warp_sum(sdot<CPL>(W + (size_t)i * p.H, p.H, xr, lane));
                        float u = warp_sum(sdot<CPL>(W + (size_t)(cnt + i) * p.H, p.H, xr, lane));
                        if (lane == 0) {
                            if (sim) { g = bf16_roundtrip(g); u = bf16_roundtrip(u); }
                            float hv = swiglu(g, u);
                            if (sim) hv = bf16_roundtrip(hv);
                            hout[ia + i] = hv;
                        }
                    }
                    if (cur.phase == PH_RSGU && sub == geo.nsub - 1) {
                        int ea, eb;
                        ea = s_ea;
                        eb = s_eb;
                        for (int e = ea + warp; e < eb; e += MK_WARPS) {
                            float s = warp_sum(sdot<CPL>(W + (size_t)(2 * cnt + e - ea) * p.H, p.H, xr, lane));
                            if (lane == 0) p.rscore[e] = s;
                        }
                    }
                    break;
                }
                case PH_DDOWN: {
                    if (sub == 0) load_vec(xs, p.h, p.D);
                    for (int i = warp; i < cnt; i += MK_WARPS) {
                        float s = warp_sum(sdot_long(W + (size_t)i * p.D, xs, p.D, lane));
                        if (lane == 0) p.xa[ia + i] = __fadd_rn(__ldcg(p.xb + ia + i), s);
                    }
                    break;
                }
                case PH_MDOWN: {
                    if (sub == 0) load_vec(xs, p.h, p.K * p.I + p.S);
                    const int half = p.S / 2;
                    const int nslot = p.K + 2;
                    for (int r0 = 0; r0 < cnt; r0 += 8) {
                        const int nr = min(8, cnt - r0);
                        for (int t = warp; t < nr * nslot; t += MK_WARPS) {
                            int rr = t / nslot, sl = t - rr * nslot;
                            int row = r0 + rr;
                            float s;
                            if (sl < p.K) {
                                s = sdot_long(W + (size_t)sl * cnt * p.I + (size_t)row * p.I, xs + sl * p.I, p.I, lane);
                            } else {
                                int hh = sl - p.K;
                                s = sdot_long(W + (size_t)p.K * cnt * p.I + (size_t)row * p.S + hh * half,
                                              xs + p.K * p.I + hh * half, half, lane);
                            }
                            s = warp_sum(s);
                            if (lane == 0) ysm[rr][sl] = s;
                        }
                        __syncthreads();
                        if (tid < nr) {
                            float acc = 0.f;
                            for (int k = 0; k < p.K; k++) {
                                float yk = ysm[tid][k];
                                if (p.simulate) yk = bf16_roundtrip(yk);
                                acc = __fmaf_rn(swt[k], yk, acc);
                            }
                            float sh = __fadd_rn(ysm[tid][p.K], ysm[tid][p.K + 1]);
                            if (p.simulate) sh = bf16_roundtrip(sh);
                            acc = __fadd_rn(acc, sh);
                            int j = ia + r0 + tid;
                            p.xa[j] = __fadd_rn(__ldcg(p.xb + j), acc);
                        }
                        __syncthreads();
                    }
                    break;
                }
                case PH_LMH: {
                    if (sub == 0) {
                        load_vec(xs, p.xa, p.H);
                        norm_vec(xs, p.final_norm, p.H, p.eps);
                        if (p.final_x && blockIdx.x == 0 && cur.step == p.n_steps - 1)
                            for (int i = tid; i < p.H; i += MK_THREADS) p.final_x[i] = xs[i];
                        if (tid == 0) cta_best = 0ull;
                        __syncthreads();
                    }
                    XRegBF16<CPL> xr;
                    xr.load(xs, p.H, lane);
                    float best = -INFINITY;
                    int bi = 0x7fffffff;
                    for (int i = warp; i < cnt; i += MK_WARPS) {
                        float s = warp_sum(sdot<CPL>(W + (size_t)i * p.H, p.H, xr, lane));
                        if (s > best) { best = s; bi = ia + i; }
                    }
                    if (lane == 0 && bi != 0x7fffffff)
                        atomicMax(&cta_best, argmax_key(best, (uint32_t)bi));
                    if (sub == geo.nsub - 1) {
                        __syncthreads();
                        unsigned long long kb = cta_best;
                        if (tid == 0 && kb) atomicMax(&p.slot[cur.step & 1], kb);
                    }
                    break;
                }
                default:
                    break;
            }
            __syncthreads();  // region r and xs are free again
            MK_TRACE(4, clock64());
        }
        next_phase(p, cur);
    }
    // publish the last token
    if (!grid_sync(p.bar, epoch)) return;
    if (tid == 0 && blockIdx.x == 0) {
        unsigned long long k = atomicAdd(&p.slot[(p.n_steps - 1) & 1], 0ull);
        int t = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
        p.tok_log[pos] = t;
        *p.tok = t;
        *p.val = f32_from_ordered((uint32_t)(k >> 32));
        *p.pos = pos + 1;
    }
}

size_t mega_smem_bytes() { return MK_SMEM; }

int mega_grid(int device) {
    static int cached[64] = {0};
    if (device < 0 || device >= 64) return 0;
    if (cached[device]) return cached[device];
    cudaFuncSetAttribute((const void *)mega_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MK_SMEM);
    int per_sm = 0, sms = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mega_decode_kernel, MK_THREADS, MK_SMEM);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaGetLastError();
    cached[device] = per_sm >= 1 ? sms : -1;
    return cached[device];
}

cudaError_t launch_mega(const MegaParams *dparams, int grid, cudaStream_t st) {
    void *args[] = {(void *)&dparams};
    return cudaLaunchCooperativeKernel((const void *)mega_decode_kernel, grid, MK_THREADS, args, MK_SMEM, st);
}

}  // namespace ds
