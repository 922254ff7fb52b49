// moe_step.cu — the MoE block of one batch-1 decode step as ONE kernel
// (moe_forward, ds_moe_decoder.c:131-333, BF16 experts): routing from the
// router terms the O-projection CTAs left behind, the shared expert's and
// the six routed experts' gate/up + SwiGLU, a grid-wide barrier, then every
// expert's down projection, the weighted combine and the residual add.
//
// Why one kernel: the step is a chain of dependent phases whose weights are
// only a few MB each, so the time goes to latency (dependency waits, the
// first bytes of each phase), not to bandwidth. Here every byte that does not
// depend on the routing is in flight before the dependency wait, and every
// byte that does is requested as soon as the routing is known. A producer
// warp issues all of it as TMA bulk copies into shared memory (register loads
// from eight warps cannot keep enough bytes in flight):
//   before the wait  this CTA's rows of the shared down projection, and its
//                    shared-expert gate/up items (a gate row and an up row)
//                    into a ring of item slots;
//   after routing    its rows of the six routed down projections, and its
//                    routed gate/up items into the ring, each slot refilled
//                    as soon as the consumer warp releases it;
//   after the grid dependency (every CTA's part of h counted done) the down
//                    dot products read only shared memory.
// One CTA per SM; the barrier is safe because the grid never exceeds the SM
// count and a CTA always fits on an SM (the kernels around it are small).
//
// Numerics match the per-phase kernels exactly (kernels_moe.cu: same
// association of every dot product, RMS norm, router logits, SwiGLU,
// truncation and combine), so the two paths give bit-identical results.
#include <algorithm>
#include <cstdlib>

#include "kernels_moe.cuh"
#include "launch.h"
#include "moe_step.h"

namespace ds {

constexpr int MS_THREADS = 256;
constexpr int MS_WARPS = MS_THREADS / 32;
constexpr int MS_CPL = 5;      // hidden 1280 = 5 chunks of 8 columns per lane
constexpr int MS_DCPL = 4;     // down rows of 896 columns: 112 chunks <= 4 per lane
constexpr int MS_MAXROWS = 10; // output rows per CTA (hidden / grid, rounded up: 9 on 148 SMs)
constexpr int MS_MAXE = 84;    // experts: 3 (E + 1) threads sum the router terms
constexpr int MS_MAXPART = 32; // router-term parts per summing thread (O-proj CTAs <= 96)
constexpr int MS_NSLOT = 8;    // down dots per output row (one warp each): top_k (6) routed + the shared row's two halves
constexpr int MS_RING = 32;    // gate/up items (a gate row and an up row) in flight in shared memory; one producer lane each

struct MsLayout {
    int i0, i1;   // shared items of this CTA
    int q0, q1;   // routed items
    int j0, j1;   // output rows
    size_t a_bytes, d_bytes;
};

__device__ __forceinline__ MsLayout ms_layout(const MoeStepArgs &a) {
    MsLayout L;
    const int G = gridDim.x, b = blockIdx.x;
    const int nr = a.K * a.I;
    L.i0 = (int)((long long)a.S * b / G);
    L.i1 = (int)((long long)a.S * (b + 1) / G);
    L.q0 = (int)((long long)nr * b / G);
    L.q1 = (int)((long long)nr * (b + 1) / G);
    L.j0 = (int)((long long)a.H * b / G);
    L.j1 = (int)((long long)a.H * (b + 1) / G);
    return L;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier over co-resident CTAs on a counter that only grows: the
// CTA's arrival number picks its generation, the barrier completes when the
// counter reaches the end of that generation. Bounded: gives up after ~2^24
// polls, sets *err and returns false.
__device__ __forceinline__ bool ms_grid_sync(unsigned long long *ctr, unsigned *err) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long old = atomicAdd(ctr, 1ull);
        const unsigned long long target = (old / gridDim.x + 1ull) * gridDim.x;
        int good = 0;
        for (uint32_t it = 0; it < (1u << 24); it++) {
            if (ld_acquire_u64(ctr) >= target) {
                good = 1;
                break;
            }
            if ((it & 1023u) == 1023u && *(volatile unsigned *)err) break;
        }
        if (!good) atomicExch(err, 1u);
        __threadfence();
        ok = good;
    }
    __syncthreads();
    return ok != 0;
}

// This CTA's share of the next layer's Q, K and V weights, asked of L2: the
// HBM is idle while the CTAs synchronise and run the down projection.
__device__ __forceinline__ void prefetch_next(const void *const (&pf)[3], size_t bytes) {
    if (threadIdx.x != 0 || bytes == 0) return;
    const size_t G = gridDim.x, b = blockIdx.x;
    const size_t lo = (bytes * b / G) & ~(size_t)15, hi = b + 1 == G ? bytes : (bytes * (b + 1) / G) & ~(size_t)15;
    for (int m = 0; m < 3; m++)
        if (pf[m] && hi > lo) prefetch_range(static_cast<const uint8_t *>(pf[m]) + lo, hi - lo);
}

// Named barrier over the consumer warps only (the producer warp never joins).
__device__ __forceinline__ void ms_cbar() { asm volatile("bar.sync 1, %0;" :: "r"(MS_THREADS) : "memory"); }

__global__ void __launch_bounds__(MS_THREADS + 32, 1) moe_step_kernel(MoeStepArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar_sd, bar_rd, bar_nw, bar_route, ring_full[MS_RING], ring_empty[MS_RING], ring_drained;
    __shared__ float lg[MS_MAXE + 1];
    __shared__ float lsum[MS_MAXE + 1][3];
    __shared__ float rr[MS_WARPS + 1];
    __shared__ int s_idx[8];
    __shared__ float s_wt[8];
    __shared__ float ysm[MS_MAXROWS][10];
    __shared__ unsigned long long s_epoch;
    TraceScope tr;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = a.H, I = a.I, S = a.S, K = a.K, E = a.E;
    const int nr = K * I;
    const MsLayout L = ms_layout(a);
    const int ns = L.i1 - L.i0, nrows = L.j1 - L.j0;
    // shared memory: the gate/up item ring (then the routed down rows), the
    // shared down rows, xs, norm weight
    uint16_t *ring = reinterpret_cast<uint16_t *>(smem);
    uint16_t *sdn = reinterpret_cast<uint16_t *>(smem + a.a_bytes);
    float *xs = reinterpret_cast<float *>(smem + a.a_bytes + a.d_bytes);
    float *nws = xs + H;
    const uint16_t *sgu = a.block + (size_t)E * 2 * I * H;

    if (tid == 0) {
        // this launch's number (every CTA of a launch adds one): the
        // completion counters below only ever grow
        s_epoch = atomicAdd(a.bar, 1ull) / gridDim.x;
        mbar_init(&bar_sd, 1);
        mbar_init(&bar_rd, 1);
        mbar_init(&bar_nw, 1);
        mbar_init(&bar_route, 1);
        for (int k = 0; k < MS_RING; k++) {
            mbar_init(&ring_full[k], 1);
            mbar_init(&ring_empty[k], 1);
        }
        mbar_init(&ring_drained, MS_RING);
        mbar_fence_init();
    }
    __syncthreads();
    // this CTA's gate/up items: its shared-expert items first (i0 .. i1),
    // then its routed items (q0 .. q1); item n sits in ring slot n % MS_RING
    const int nitems = ns + (L.q1 - L.q0);
    if (warp == MS_WARPS) {
        // producer warp: every TMA copy, so no consumer warp waits behind an
        // issue. At once: the norm weight, this CTA's rows of the shared
        // down projection and its shared-expert items; once warp 0 has the
        // routing: the routed down rows and the routed items. Each ring slot
        // is refilled as soon as its consumer warp has released it.
        // lane l < MS_RING owns ring slot l (items l, l + MS_RING, ...): a
        // bulk copy costs its issuing thread a fixed time, so one thread
        // alone could not keep the slots full
        if (lane == 0) {
            mbar_expect_tx(&bar_nw, (uint32_t)H * 4);
            bulk_g2s(nws, a.norm_w, (uint32_t)H * 4, &bar_nw);
            if (nrows > 0) {
                const uint32_t db = (uint32_t)nrows * S * 2;
                mbar_expect_tx(&bar_sd, db);
                bulk_g2s_stream(sdn, a.sdown + (size_t)L.j0 * S, db, &bar_sd);
            }
        }
        {
            // one warp-uniform polling loop: each pass, every lane whose slot
            // is free (and, for a routed item, whose routing is known) issues
            // its next item; no lane's wait holds up the others (a blocking
            // wait per lane would reconverge the warp behind the slowest slot)
            const uint32_t rb = (uint32_t)H * 2;
            bool routed = false, ok = true;
            int n = lane, last = -1;
            for (uint32_t it = 0; __any_sync(0xffffffffu, n < nitems); it++) {
                if (it >= (1u << 26)) {
                    atomicExch(a.err, 1u);
                    ok = false;
                    break;
                }
                bool go = n < nitems;
                if (go && n >= MS_RING) go = mbar_test(&ring_empty[lane], ((n / MS_RING) - 1) & 1);
                if (go && n >= ns && !routed) go = routed = mbar_test(&bar_route, 0);
                if (go) {
                    const uint16_t *g, *u;
                    if (n < ns) {
                        g = sgu + (size_t)(L.i0 + n) * H;
                        u = sgu + (size_t)(S + L.i0 + n) * H;
                    } else {
                        const int q = L.q0 + n - ns, k = q / I, i = q - k * I;
                        const uint16_t *base = a.block + (size_t)s_idx[k] * 2 * I * H;
                        g = base + (size_t)i * H;
                        u = base + (size_t)(I + i) * H;
                    }
                    uint16_t *d = ring + (size_t)lane * 2 * H;
                    mbar_expect_tx(&ring_full[lane], 2 * rb);
                    bulk_g2s_stream(d, g, rb, &ring_full[lane]);
                    bulk_g2s_stream(d + H, u, rb, &ring_full[lane]);
                    last = n;
                    n += MS_RING;
                }
            }
            // this slot's last item consumed: the ring may take the routed
            // down rows
            if (ok && last >= 0) mbar_wait(&ring_empty[lane], (last / MS_RING) & 1, a.err);
            mbar_arrive(&ring_drained);
        }
        // the routed down rows (the routing is known and the ring drained)
        if (lane == 0 && nrows > 0 && mbar_wait(&bar_route, 0, a.err) && mbar_wait(&ring_drained, 0, a.err)) {
            const uint32_t kb = (uint32_t)nrows * I * 2;
            mbar_expect_tx(&bar_rd, (uint32_t)K * kb);
            for (int k = 0; k < K; k++)
                bulk_g2s_stream(ring + (size_t)k * nrows * I, a.down + ((size_t)s_idx[k] * H + L.j0) * I, kb,
                                &bar_rd);
        }
        return;
    }
    pdl_wait();
    tr.waited();

    // 1. router logits: column e of the O-proj CTAs' terms summed in three
    //    runs of consecutive CTAs (rf_run_sum, as router_fold's last CTA
    //    sums them); the residual stream into xs
    if (tid < 3 * (E + 1)) {
        const int e = tid / 3, part = tid - 3 * e;
        lsum[e][part] = rf_run_sum(a.rpart + (size_t)e * rf_pstride(a.nparts), a.nparts, part);
    }
    {
        // both of a thread's x loads in flight together (H <= 8 * MS_THREADS)
        float4 xv[2];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int i = (tid + u * MS_THREADS) * 4;
            if (i < H) xv[u] = __ldcg(reinterpret_cast<const float4 *>(a.x + i));
        }
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int i = (tid + u * MS_THREADS) * 4;
            if (i < H) *reinterpret_cast<float4 *>(xs + i) = xv[u];
        }
    }
    ms_cbar();
    tr.mark(0);
    // 2. the sum of squares of x (block_rms_inv's order over 8 warps), then
    //    warp 0: routing (softmax and top-k of the logits scaled by the RMS
    //    of x), handed to the producer warp; the others start on the
    //    shared-expert items meanwhile
    float ss = 0.f;
    for (int i = tid; i < H; i += MS_THREADS) ss = __fmaf_rn(xs[i], xs[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) rr[warp] = ss;
    ms_cbar();
    tr.mark(1);
    if (warp == 0) {
        for (int e = lane; e <= E; e += 32) lg[e] = __fadd_rn(__fadd_rn(lsum[e][0], lsum[e][1]), lsum[e][2]);
        __syncwarp();
        const float rinv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(lg[E], (float)H), a.eps)));
        for (int e = lane; e < E; e += 32) {
            lg[e] = __fmul_rn(lg[e], rinv);
            if (blockIdx.x == 0) a.scores[e] = lg[e];
        }
        __syncwarp();
        router_select(lg, E, K, a.renorm, s_idx, s_wt);
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_route);
        tr.mark(6);
        if (blockIdx.x == 0 && lane < K) {
            a.d_idx[lane] = s_idx[lane];
            a.d_wt[lane] = s_wt[lane];
        }
    }
    // post-attention RMSNorm of x (every thread sums the warps' terms in
    // warp order) with the norm weight from shared memory
    float t2 = 0.f;
    for (int w = 0; w < MS_WARPS; w++) t2 = __fadd_rn(t2, rr[w]);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t2, (float)H), a.eps)));
    mbar_wait(&bar_nw, 0, a.err);  // a timeout is recorded in *err; every warp still reaches the barriers
    const bool sim = a.simulate != 0;
    auto swiglu_out = [&](float g, float u) {
        if (sim) {
            g = bf16_roundtrip(g);
            u = bf16_roundtrip(u);
        }
        float hv = swiglu(g, u);
        if (sim) hv = bf16_roundtrip(hv);
        return hv;
    };
    XRegBF16<MS_CPL> xr;
    xr.load_norm(xs, nws, inv, H, lane);
    tr.mark(2);
    // 3. the gate/up items from the ring: item n is warp n % 8's; its gate
    //    and up dot products, SwiGLU, into h; the slot goes back to the
    //    producer
    for (int n = warp; n < nitems; n += MS_WARPS) {
        const int sl = n % MS_RING;
        if (!mbar_wait(&ring_full[sl], (n / MS_RING) & 1, a.err)) break;
        if (n >= ns && n < ns + MS_WARPS) tr.mark(3);
        tr.mark(7);
        const uint16_t *gr = ring + (size_t)sl * 2 * H, *ur = gr + H;
        float g = 0.f, u = 0.f;
#pragma unroll
        for (int c = 0; c < MS_CPL; c++) {
            const int ch = lane + 32 * c;
            g = dot8_bf16(*reinterpret_cast<const uint4 *>(gr + 8 * ch), xr.v[c][0], xr.v[c][1], g);
            u = dot8_bf16(*reinterpret_cast<const uint4 *>(ur + 8 * ch), xr.v[c][0], xr.v[c][1], u);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ring_empty[sl]);
        g = warp_sum(g);
        u = warp_sum(u);
        if (lane == 0) a.h[n < ns ? nr + L.i0 + n : L.q0 + n - ns] = swiglu_out(g, u);
    }
    // this CTA's shared and routed items are in h: count them (release)
    ms_cbar();
    if (tid == 0) {
        __threadfence();
        atomicAdd(a.done + K, 1ull);
        if (L.q1 > L.q0)
            for (int k = L.q0 / I; k < K && k * I < L.q1; k++) atomicAdd(a.done + k, 1ull);
    }
    tr.mark(4);
    // the next kernel may launch now: its prologue loads no longer compete
    // with this kernel's routing and gate/up streams
    pdl_launch();
    prefetch_next(a.pf, a.pf_bytes);
    // 6. down dot products: warp s owns slot s (s < K: routed expert s;
    //    K, K + 1: the two halves of the shared expert's rows). It waits
    //    until every CTA that computes part of its slice of h has counted it
    //    done (no grid-wide barrier: the shared slots start at once, a
    //    routed slot waits only for its own producer CTAs), loads that slice
    //    into registers and walks this CTA's output rows two at a time.
    const int half = S >> 1;
    if (warp < K + 2) {
        const int s = warp;
        const unsigned long long need =
            (s_epoch + 1) * (s < K ? (unsigned long long)a.ncta[s] : (unsigned long long)gridDim.x);
        const unsigned long long *ctr = a.done + (s < K ? s : K);
        bool ok = false;
        for (uint32_t it = 0; it < (1u << 24); it++) {
            if (ld_acquire_u64(ctr) >= need) {
                ok = true;
                break;
            }
            if ((it & 1023u) == 1023u && *(volatile unsigned *)a.err) break;
        }
        if (!ok && lane == 0) atomicExch(a.err, 1u);
        const float *hv = s < K ? a.h + s * I : a.h + nr + (s - K) * half;
        const int nch = I >> 3;
        XRegBF16<MS_DCPL> hr;
#pragma unroll
        for (int c = 0; c < MS_DCPL; c++) {
            const int ch = lane + 32 * c;
            if (ch < nch) {
                hr.v[c][0] = __ldcg(reinterpret_cast<const float4 *>(hv + 8 * ch));
                hr.v[c][1] = __ldcg(reinterpret_cast<const float4 *>(hv + 8 * ch + 4));
            } else {
                hr.v[c][0] = hr.v[c][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        if (nrows > 0) mbar_wait(s < K ? &bar_rd : &bar_sd, 0, a.err);  // timeouts recorded in *err
        auto wrow = [&](int r) {
            return s < K ? ring + ((size_t)s * nrows + r) * I : sdn + (size_t)r * S + (s - K) * half;
        };
        for (int r = 0; r < nrows; r += 2) {
            const bool two = r + 1 < nrows;
            const uint16_t *w0 = wrow(r), *w1 = wrow(two ? r + 1 : r);
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int c = 0; c < MS_DCPL; c++) {
                const int ch = lane + 32 * c;
                if (ch < nch) {
                    a0 = dot8_bf16(*reinterpret_cast<const uint4 *>(w0 + 8 * ch), hr.v[c][0], hr.v[c][1], a0);
                    a1 = dot8_bf16(*reinterpret_cast<const uint4 *>(w1 + 8 * ch), hr.v[c][0], hr.v[c][1], a1);
                }
            }
            a0 = warp_sum(a0);
            a1 = warp_sum(a1);
            if (lane == 0) {
                ysm[r][s] = a0;
                if (two) ysm[r + 1][s] = a1;
            }
        }
    }
    ms_cbar();
    tr.mark(5);
    // 7. combine in the reference's order (ds_expert_combine, then + shared)
    //    and the residual add
    if (tid < nrows) {
        const int j = L.j0 + tid;
        float acc = 0.f;
        for (int k = 0; k < K; k++) {
            float yk = ysm[tid][k];
            if (sim) yk = bf16_roundtrip(yk);
            acc = __fmaf_rn(s_wt[k], yk, acc);
        }
        float sh = __fadd_rn(ysm[tid][K], ysm[tid][K + 1]);
        if (sim) sh = bf16_roundtrip(sh);
        acc = __fadd_rn(acc, sh);
        a.out[j] = __fadd_rn(__ldcg(a.x + j), acc);
    }
    tr.done(10);
}

// ---------------------------------------------------------------------------
// The dense FFN layer (dense_ffn_forward, ds_moe_decoder.c:75-105: gate and
// up [D x H], SwiGLU without truncation, down [H x D], residual add) as ONE
// kernel. No weight depends on the data, so a producer warp streams this
// CTA's gate/up rows (8 items of gate row + up row per stage) through a
// ring of shared-memory stages with the TMA engine, starting before the
// dependency wait; eight consumer warps compute from shared memory. A grid
// barrier separates the SwiGLU outputs from the down projection: once the
// ring has drained, the producer copies this CTA's down rows (one bulk copy;
// an earlier kernel of the step asked L2 for them) into the ring's space
// while the CTAs synchronise; warp w then reads column range w of every
// output row and the eight partial sums of a row are added in warp order.
// The gate/up dot products associate as the per-phase kernel's
// (moe_gate_up_kernel).
// ---------------------------------------------------------------------------
constexpr int DS_CONSUMERS = 8;
constexpr int DS_THREADS = 32 * (DS_CONSUMERS + 1);
constexpr int DS_NST = 4;                         // ring stages
constexpr int DS_ITEMS = DS_CONSUMERS;            // gate/up items per stage (one per consumer warp)

// Consumer-only grid barrier (named barrier 1 over the consumer warps; the
// producer warp keeps streaming): same counter protocol as ms_grid_sync.
__device__ __forceinline__ bool ds_grid_sync_consumers(unsigned long long *ctr, unsigned *err) {
    __shared__ int ok;
    asm volatile("bar.sync 1, %0;" :: "r"(32 * DS_CONSUMERS) : "memory");
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long old = atomicAdd(ctr, 1ull);
        const unsigned long long target = (old / gridDim.x + 1ull) * gridDim.x;
        int good = 0;
        for (uint32_t it = 0; it < (1u << 24); it++) {
            if (ld_acquire_u64(ctr) >= target) {
                good = 1;
                break;
            }
            if ((it & 1023u) == 1023u && *(volatile unsigned *)err) break;
        }
        if (!good) atomicExch(err, 1u);
        __threadfence();
        ok = good;
    }
    asm volatile("bar.sync 1, %0;" :: "r"(32 * DS_CONSUMERS) : "memory");
    return ok != 0;
}

__global__ void __launch_bounds__(DS_THREADS, 1) dense_step_kernel(DenseStepArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar_nw, bar_dn, full[DS_NST], empty[DS_NST];
    __shared__ float red[MS_MAXROWS][DS_CONSUMERS];
    TraceScope tr;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = a.H, D = a.D, G = gridDim.x, b = blockIdx.x;
    const int i0 = (int)((long long)D * b / G), i1 = (int)((long long)D * (b + 1) / G);
    const int j0 = (int)((long long)H * b / G), j1 = (int)((long long)H * (b + 1) / G);
    const int ngu = (i1 - i0 + DS_ITEMS - 1) / DS_ITEMS;  // gate/up stages
    const size_t stage_b = (size_t)DS_ITEMS * 2 * H * 2;
    uint8_t *ring = smem;
    float *xs = reinterpret_cast<float *>(smem + DS_NST * stage_b);
    float *nws = xs + H;
    float *hs = nws + H;
    if (tid == 0) {
        mbar_init(&bar_nw, 1);
        mbar_init(&bar_dn, 1);
        for (int st = 0; st < DS_NST; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], DS_CONSUMERS);
        }
        mbar_fence_init();
        mbar_expect_tx(&bar_nw, (uint32_t)H * 4);
        bulk_g2s(nws, a.norm_w, (uint32_t)H * 4, &bar_nw);
    }
    __syncthreads();
    if (warp == DS_CONSUMERS) {
        // producer: every stage's rows, before and after the dependency wait
        if (lane == 0) {
            for (int q = 0; q < ngu; q++) {
                const int st = q % DS_NST;
                if (q >= DS_NST && !mbar_wait(&empty[st], ((q / DS_NST) - 1) & 1, a.err)) break;
                uint8_t *dst = ring + (size_t)st * stage_b;
                const int ia = i0 + q * DS_ITEMS, cnt = min(DS_ITEMS, i1 - ia);
                const uint32_t rb = (uint32_t)cnt * H * 2;
                mbar_expect_tx(&full[st], 2 * rb);
                bulk_g2s_stream(dst, a.gate + (size_t)ia * H, rb, &full[st]);
                bulk_g2s_stream(dst + (size_t)DS_ITEMS * H * 2, a.up + (size_t)ia * H, rb, &full[st]);
            }
            // the down rows, once every stage has been consumed
            bool ok = true;
            for (int q = max(0, ngu - DS_NST); q < ngu && ok; q++)
                ok = mbar_wait(&empty[q % DS_NST], (q / DS_NST) & 1, a.err);
            if (ok && j1 > j0) {
                const uint32_t db = (uint32_t)(j1 - j0) * D * 2;
                mbar_expect_tx(&bar_dn, db);
                bulk_g2s_stream(ring, a.down + (size_t)j0 * D, db, &bar_dn);
            }
        }
        return;
    }
    pdl_wait();
    pdl_launch();
    tr.waited();
    const int ctid = tid;  // consumers are threads 0 .. 255
    for (int i = ctid * 4; i < H; i += 32 * DS_CONSUMERS * 4)
        *reinterpret_cast<float4 *>(xs + i) = __ldcg(reinterpret_cast<const float4 *>(a.x + i));
    asm volatile("bar.sync 1, %0;" :: "r"(32 * DS_CONSUMERS) : "memory");
    // block_rms_inv's order over the consumer threads
    float inv;
    {
        __shared__ float rr[DS_CONSUMERS + 1];
        float ss = 0.f;
        for (int i = ctid; i < H; i += 32 * DS_CONSUMERS) ss = __fmaf_rn(xs[i], xs[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) rr[warp] = ss;
        asm volatile("bar.sync 1, %0;" :: "r"(32 * DS_CONSUMERS) : "memory");
        if (ctid == 0) {
            float t = 0.f;
            for (int w = 0; w < DS_CONSUMERS; w++) t = __fadd_rn(t, rr[w]);
            rr[DS_CONSUMERS] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)H), a.eps)));
        }
        asm volatile("bar.sync 1, %0;" :: "r"(32 * DS_CONSUMERS) : "memory");
        inv = rr[DS_CONSUMERS];
    }
    if (!mbar_wait(&bar_nw, 0, a.err)) return;
    XRegBF16<MS_CPL> xr;
    xr.load_norm(xs, nws, inv, H, lane);
    tr.mark(0);
    // gate/up stages: warp w takes item w of the stage
    for (int q = 0; q < ngu; q++) {
        const int st = q % DS_NST;
        if (!mbar_wait(&full[st], (q / DS_NST) & 1, a.err)) return;
        const int it = i0 + q * DS_ITEMS + warp;
        if (it < i1) {
            const uint16_t *gr = reinterpret_cast<const uint16_t *>(ring + (size_t)st * stage_b) + (size_t)warp * H;
            const uint16_t *ur = gr + (size_t)DS_ITEMS * H;
            float g = 0.f, u = 0.f;
#pragma unroll
            for (int c = 0; c < MS_CPL; c++) {
                const int ch = lane + 32 * c;
                g = dot8_bf16(*reinterpret_cast<const uint4 *>(gr + 8 * ch), xr.v[c][0], xr.v[c][1], g);
                u = dot8_bf16(*reinterpret_cast<const uint4 *>(ur + 8 * ch), xr.v[c][0], xr.v[c][1], u);
            }
            g = warp_sum(g);
            u = warp_sum(u);
            if (lane == 0) a.h[it] = swiglu(g, u);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    tr.mark(1);
    if (!ds_grid_sync_consumers(a.bar, a.err)) return;
    tr.mark(2);
    for (int i = ctid * 4; i < D; i += 32 * DS_CONSUMERS * 4)
        *reinterpret_cast<float4 *>(hs + i) = __ldcg(reinterpret_cast<const float4 *>(a.h + i));
    asm volatile("bar.sync 1, %0;" :: "r"(32 * DS_CONSUMERS) : "memory");
    tr.mark(3);
    // down rows from shared memory: warp w owns chunk range w of every row
    const int nch = D >> 3;
    const int per = (nch + DS_CONSUMERS - 1) / DS_CONSUMERS;
    const int c0 = warp * per, c1 = min(nch, c0 + per);
    const int nrows = j1 - j0;
    if (nrows > 0 && !mbar_wait(&bar_dn, 0, a.err)) return;
    tr.mark(4);
    // all rows at once (independent accumulators; each h chunk read once)
    {
        const uint16_t *w0 = reinterpret_cast<const uint16_t *>(ring);
        float acc[MS_MAXROWS];
#pragma unroll
        for (int r = 0; r < MS_MAXROWS; r++) acc[r] = 0.f;
        for (int ch = c0 + lane; ch < c1; ch += 32) {
            const float4 *hp = reinterpret_cast<const float4 *>(hs + 8 * ch);
            const float4 h0 = hp[0], h1 = hp[1];
#pragma unroll
            for (int r = 0; r < MS_MAXROWS; r++)
                if (r < nrows) acc[r] = dot8_bf16(*reinterpret_cast<const uint4 *>(w0 + (size_t)r * D + 8 * ch), h0, h1, acc[r]);
        }
#pragma unroll
        for (int r = 0; r < MS_MAXROWS; r++) {
            if (r < nrows) {
                const float v = warp_sum(acc[r]);
                if (lane == 0) red[r][warp] = v;
            }
        }
    }
    tr.mark(5);
    asm volatile("bar.sync 1, %0;" :: "r"(32 * DS_CONSUMERS) : "memory");
    tr.mark(6);
    if (ctid < nrows) {
        float t = 0.f;
        for (int k = 0; k < DS_CONSUMERS; k++) t = __fadd_rn(t, red[ctid][k]);
        const int j = j0 + ctid;
        a.out[j] = __fadd_rn(__ldcg(a.x + j), t);
    }
    tr.mark(7);
    prefetch_next(a.pf, a.pf_bytes);
    tr.done(11);
}

bool dense_step_supported(int H, int D, int sms) {
    const size_t stage_b = (size_t)DS_ITEMS * 2 * H * 2;
    return H == 1280 && D % 8 == 0 && sms >= 1 && (H + sms - 1) / sms <= MS_MAXROWS &&
           (size_t)((H + sms - 1) / sms) * D * 2 <= DS_NST * stage_b &&
           DS_NST * stage_b + (size_t)(2 * H + D) * 4 <= 210 * 1024;
}

cudaError_t launch_dense_step(DenseStepArgs a, int grid, cudaStream_t st, bool pdl) {
    const size_t smem = DS_NST * (size_t)DS_ITEMS * 2 * a.H * 2 + (size_t)(2 * a.H + a.D) * 4;
    static size_t set = 0;
    if (set < smem) {
        cudaError_t e = cudaFuncSetAttribute((const void *)dense_step_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set = smem;
    }
    void *args[] = {&a};
    return launch_ex((const void *)dense_step_kernel, grid, DS_THREADS, smem, st, pdl, args);
}

bool moe_step_supported(int H, int I, int S, int E, int K, int sms) {
    if (H != 1280 || H > 8 * MS_THREADS || I % 8 || S % 16 || I > 8 * 32 * MS_DCPL || S / 2 > 8 * 32 * MS_DCPL) return false;
    if (K != MS_NSLOT - 2 || E > MS_MAXE || E < K || sms < 1 || (H + 15) / 16 > 3 * MS_MAXPART) return false;
    if (2 * S != 2 * I * (S / I) || S / 2 != I) return false;  // the shared row splits into two expert-width halves
    if ((H + sms - 1) / sms > MS_MAXROWS) return false;
    // the routed down rows of a CTA's outputs fit in the drained ring
    if ((size_t)((H + sms - 1) / sms) * K * I * 2 > (size_t)MS_RING * 2 * H * 2) return false;
    return moe_step_smem(H, I, S, K, sms) <= 222 * 1024;  // + about 3 KB of static shared memory
}

size_t moe_step_smem(int H, int I, int S, int K, int G) {
    const int rows_max = (H + G - 1) / G;
    size_t a_bytes = (size_t)MS_RING * 2 * H * 2;  // the ring; later the routed down rows
    size_t d_bytes = (size_t)rows_max * S * 2;      // the shared down rows
    a_bytes = (a_bytes + 127) & ~(size_t)127;
    d_bytes = (d_bytes + 127) & ~(size_t)127;
    return a_bytes + d_bytes + (size_t)H * 8;
}

cudaError_t launch_moe_step(MoeStepArgs a, int grid, cudaStream_t st, bool pdl) {
    const int rows_max = (a.H + grid - 1) / grid;
    a.a_bytes = (size_t)MS_RING * 2 * a.H * 2;
    a.d_bytes = (size_t)rows_max * a.S * 2;
    a.a_bytes = (a.a_bytes + 127) & ~(size_t)127;
    a.d_bytes = (a.d_bytes + 127) & ~(size_t)127;
    const size_t smem = a.a_bytes + a.d_bytes + (size_t)a.H * 8;
    static size_t set = 0;
    if (set < smem) {
        cudaError_t e = cudaFuncSetAttribute((const void *)moe_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        set = smem;
    }
    // CTAs whose routed item range [nr b / G, nr (b + 1) / G) meets slot k's
    // [k I, (k + 1) I): the count slot k's completion counter grows by
    const long long nr = (long long)a.K * a.I;
    for (int k = 0; k < 8; k++) a.ncta[k] = 0;
    for (int b = 0; b < grid; b++) {
        const long long q0 = nr * b / grid, q1 = nr * (b + 1) / grid;
        if (q1 <= q0) continue;
        for (int k = (int)(q0 / a.I); k < a.K && (long long)k * a.I < q1; k++) a.ncta[k]++;
    }
    void *args[] = {&a};
    return launch_ex((const void *)moe_step_kernel, grid, MS_THREADS + 32, smem, st, pdl, args);
}

}  // namespace ds

DS_TRACE_TU(step)
