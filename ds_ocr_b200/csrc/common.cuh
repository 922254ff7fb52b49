// common.cuh — device helpers shared by the ds_cuda kernels (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#define DS_WARP 32
#define DS_FULL 0xffffffffu

namespace ds {

// BF16 weights widen exactly to F32 by a 16-bit shift (the reference does
// the same, ds_kernels_avx.c:49-51).
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Schraudolph fast exp exactly as the compiled reference evaluates it
// (ds_kernels.h:296-302, product-add fused by gcc into one FMA): the FMA is
// rounded to nearest, then truncated to uint32 and reinterpreted.
__device__ __forceinline__ float fast_expf(float x) {
    if (x < -88.0f) return 0.0f;
    if (x > 88.0f) return 1e38f;
    return __uint_as_float(__float2uint_rz(__fmaf_rn(12102203.0f, x, 1064866805.0f)));
}
// The same for x <= 0, where the upper clamp cannot apply.
__device__ __forceinline__ float fast_expf_nonpos(float x) {
    return x < -88.0f ? 0.0f : __uint_as_float(__float2uint_rz(__fmaf_rn(12102203.0f, x, 1064866805.0f)));
}

// F32 -> BF16 -> F32 with the reference's round-half-up on the magnitude
// (ds_kernels.c:2464-2492).
__device__ __forceinline__ float bf16_roundtrip(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x8000u) & 0xffff0000u);
}

// SwiGLU of the reference's non-Apple build (ds_kernels.c:1770-1773).
__device__ __forceinline__ float swiglu(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, fast_expf(-g))), u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(DS_FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(DS_FULL, v, o));
    return v;
}

// L2 policy for data read once per step (weights, KV rows): evicted first,
// so the step's streams do not push the small, reused data (activations,
// router terms, kernel code) out of L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 16-byte streaming load that bypasses L1 and is evicted first from L2
// (weights are read once per step).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(l2_evict_first()));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// Eight BF16 weights (one 16-byte chunk) times eight F32 activations.
__device__ __forceinline__ float dot8_bf16(uint4 w, const float4 &xa, const float4 &xb, float acc) {
    acc = __fmaf_rn(bf16_lo(w.x), xa.x, acc);
    acc = __fmaf_rn(bf16_hi(w.x), xa.y, acc);
    acc = __fmaf_rn(bf16_lo(w.y), xa.z, acc);
    acc = __fmaf_rn(bf16_hi(w.y), xa.w, acc);
    acc = __fmaf_rn(bf16_lo(w.z), xb.x, acc);
    acc = __fmaf_rn(bf16_hi(w.z), xb.y, acc);
    acc = __fmaf_rn(bf16_lo(w.w), xb.z, acc);
    acc = __fmaf_rn(bf16_hi(w.w), xb.w, acc);
    return acc;
}

// Unsigned byte b (0..255) of a word as an exact F32: 0x4B0000bb is
// 2^23 + b, and subtracting 2^23 is exact. Two full-rate ops, no I2F.
__device__ __forceinline__ float ubyte_f(uint32_t w, int b) {
    uint32_t v = __byte_perm(w, 0x4B000000u, 0x7440 + b);  // bytes: [b,4,4,7]
    return __fsub_rn(__uint_as_float(v), 8388608.0f);
}

// Optional launch trace (a debugging aid, off unless a buffer is set): each
// instrumented kernel's CTA appends one 12-word record: kind | block << 16 |
// sm << 40, entry time, time past the dependency wait, exit time, and up to
// eight intermediate marks (globaltimer ns; marks are kept in registers and
// written with the record, so they add no memory traffic while the kernel
// runs). The buffer pointer lives per translation unit; DS_TRACE_TU(tag)
// exports ds_trace_set_<tag>(rec, counter, capacity) to set it (NULL: off).
struct DsTrace {
    unsigned long long *rec;
    unsigned *cnt;
    unsigned cap;
};
static __device__ DsTrace g_ds_trace;
__device__ __forceinline__ unsigned long long ds_gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned ds_smid() {
    unsigned s;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
    return s;
}
struct TraceScope {
    unsigned long long t0 = 0, tw = 0, m[8];
    __device__ __forceinline__ TraceScope() {
        if (g_ds_trace.rec) t0 = ds_gtime();
#pragma unroll
        for (int i = 0; i < 8; i++) m[i] = 0;
    }
    __device__ __forceinline__ void waited() {
        if (t0) tw = ds_gtime();
    }
    __device__ __forceinline__ void mark(int i) {
        if (t0) m[i] = ds_gtime();
    }
    __device__ __forceinline__ void done(int kind) {
        if (t0 && threadIdx.x == 0) {
            const unsigned long long t1 = ds_gtime();
            unsigned i = atomicAdd(g_ds_trace.cnt, 1u);
            if (i < g_ds_trace.cap) {
                unsigned long long *r = g_ds_trace.rec + 12ull * i;
                r[0] = (unsigned long long)kind | ((unsigned long long)blockIdx.x << 16) |
                       ((unsigned long long)ds_smid() << 40);
                r[1] = t0;
                r[2] = tw;
                r[3] = t1;
#pragma unroll
                for (int k = 0; k < 8; k++) r[4 + k] = m[k];
            }
        }
    }
};
#define DS_TRACE_TU(tag)                                                                          \
    extern "C" int ds_trace_set_##tag(void *rec, unsigned *cnt, unsigned cap) {                   \
        ds::DsTrace t = {(unsigned long long *)rec, cnt, cap};                                    \
        return (int)cudaMemcpyToSymbol(ds::g_ds_trace, &t, sizeof(t));                            \
    }

// Programmatic dependent launch (PDL). wait: block until the predecessor
// grid has completed and its memory is visible. launch_dependents: allow the
// next grid in the stream to begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bulk L2 prefetch of [p, p+bytes): p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}
// Prefetch an arbitrary byte range in chunks (addresses rounded to 16 B).
__device__ __forceinline__ void prefetch_range(const void *p, size_t bytes) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
    uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes + 15) & ~uintptr_t(15);
    while (a < e) {
        uintptr_t rem = e - a;
        uint32_t n = rem < (uintptr_t(1) << 20) ? (uint32_t)rem : (1u << 20);
        prefetch_l2(reinterpret_cast<const void *>(a), n);
        a += n;
    }
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA engine, non-tensor form) helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait: gives up after ~2^24 polls (seconds), records the failure in
// *err (if given) and returns false instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *err) {
    for (uint32_t it = 0; it < (1u << 24); it++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, 1u);
    return false;
}
// Orders this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Global -> shared bulk copy completing on `bar` (dst, src 16-byte aligned,
// bytes a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// The same for data read once per step: evicted first from L2.
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(l2_evict_first()) : "memory");
}

// F32 -> BF16 with round-to-nearest-even, as raw bits.
__device__ __forceinline__ uint16_t bf16_rne_bits(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
// Split v into hi + lo BF16 halves (v ~= hi + lo to ~2^-17 relative): the
// decode KV cache stores K and V as two such planes, and the prefill GEMMs
// take their F32 activations as two such planes.
__device__ __forceinline__ void split_bf16(float v, uint16_t &hi, uint16_t &lo) {
    hi = bf16_rne_bits(v);
    lo = bf16_rne_bits(__fsub_rn(v, __uint_as_float((uint32_t)hi << 16)));
}
// Order-preserving map of an F32 to uint32 (larger float -> larger uint).
__device__ __forceinline__ uint32_t f32_ordered(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float f32_from_ordered(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
// Argmax key: larger value wins; on equal values the LOWER index wins
// (the reference's strict '>' scan, ds_kernels_avx.c:223-226).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    return ((unsigned long long)f32_ordered(v) << 32) | (unsigned long long)(0xffffffffu - idx);
}

}  // namespace ds
