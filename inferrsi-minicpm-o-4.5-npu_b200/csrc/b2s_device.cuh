// Device helpers of the B200 sampler: the sampler numerics spec (exp, order keys), the two RNGs, load and
// asynchronous-copy PTX wrappers and CTA-wide primitives (reductions, scans, radix select).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2s {

constexpr int NT = 512;        // threads per CTA of the row kernels
constexpr int NWARP = NT / 32;

// ---------------------------------------------------------------- numerics spec

// exp(x) in fp32: n = rint(x*log2 e), r = x - n*ln2 by a two-constant Cody-Waite reduction, exp(r) by its
// Taylor series to degree 7 in FMA Horner form, then scaled by exact powers of two.  Every operation is
// an explicitly rounded fp32 op, so the CPU oracle (same sequence, -ffp-contract=off) gives the same bits.
// Written without branches (the special cases are selected at the end, the reduction runs on x clamped to
// [-104, 89], where it is the same sequence as for every in-range x) so that independent calls interleave.
__device__ __forceinline__ float b2s_expf(float x) {
    const float xc = fminf(fmaxf(x, -104.0f), 89.0f);
    const float t = __fmul_rn(xc, 1.44269502162933349609375f);
    const float n = rintf(t);
    float r = __fmaf_rn(n, -0.693145751953125f, xc);
    r = __fmaf_rn(n, -1.428606765330187045037746429443359375e-6f, r);
    float p = 1.98412701138295233249664306640625e-4f;
    p = __fmaf_rn(p, r, 1.3888889225199818611145019531250e-3f);
    p = __fmaf_rn(p, r, 8.3333337679505348205566406250000e-3f);
    p = __fmaf_rn(p, r, 4.1666667908430099487304687500000e-2f);
    p = __fmaf_rn(p, r, 1.6666667163372039794921875000000e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ni = (int)n;  // [-150, 128] for x in range
    const bool hi = ni > 127, lo = ni < -126;
    p = hi ? __fmul_rn(p, 2.0f) : p;
    p = lo ? __fmul_rn(p, 5.42101086242752217003726400434970855712890625e-20f) : p;
    ni = hi ? ni - 1 : (lo ? ni + 64 : ni);
    float res = __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
    res = x < -103.97208404541015625f ? 0.0f : res;
    res = x > 88.72283935546875f ? __int_as_float(0x7f800000) : res;
    return x != x ? x : res;
}

// b2s_expf of two arguments x <= 0 (not NaN) at once, with the same results: the range reduction and the
// polynomial in packed fp32x2 arithmetic (each lane one IEEE rn operation).  The scaling by 2^n is taken as
// (p * 2^(n + 64)) * 2^-64: the first product is exact (a normal power-of-two scaling), so the result is p * 2^n
// rounded once, as the scalar form's single or two-step scaling gives it.  (n stays rintf of the rounded product
// t: an add of a rounding constant to t could be fused with the multiply that made t, rounding it differently.)
// For x <= 0 the overflow side of b2s_expf never applies and is left out.
__device__ __forceinline__ float2 b2s_expf2_nonpos(float2 x) {
    const float2 xc = make_float2(fmaxf(x.x, -104.0f), fmaxf(x.y, -104.0f));
    const float2 t = __fmul2_rn(xc, make_float2(1.44269502162933349609375f, 1.44269502162933349609375f));
    const float2 n = make_float2(rintf(t.x), rintf(t.y));
    float2 r = __ffma2_rn(n, make_float2(-0.693145751953125f, -0.693145751953125f), xc);
    r = __ffma2_rn(n, make_float2(-1.428606765330187045037746429443359375e-6f, -1.428606765330187045037746429443359375e-6f), r);
    float2 p = make_float2(1.98412701138295233249664306640625e-4f, 1.98412701138295233249664306640625e-4f);
    p = __ffma2_rn(p, r, make_float2(1.3888889225199818611145019531250e-3f, 1.3888889225199818611145019531250e-3f));
    p = __ffma2_rn(p, r, make_float2(8.3333337679505348205566406250000e-3f, 8.3333337679505348205566406250000e-3f));
    p = __ffma2_rn(p, r, make_float2(4.1666667908430099487304687500000e-2f, 4.1666667908430099487304687500000e-2f));
    p = __ffma2_rn(p, r, make_float2(1.6666667163372039794921875000000e-1f, 1.6666667163372039794921875000000e-1f));
    p = __ffma2_rn(p, r, make_float2(0.5f, 0.5f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    // n + 64 + 127 in the exponent field: n in [-150, 0], so a normal power of two
    const float2 s = make_float2(__uint_as_float((uint32_t)((int)n.x + 191) << 23),
                                 __uint_as_float((uint32_t)((int)n.y + 191) << 23));
    float2 res = __fmul2_rn(__fmul2_rn(p, s), make_float2(5.42101086242752217003726400434970855712890625e-20f,
                                                          5.42101086242752217003726400434970855712890625e-20f));
    res.x = x.x < -103.97208404541015625f ? 0.0f : res.x;
    res.y = x.y < -103.97208404541015625f ? 0.0f : res.y;
    return res;
}

__device__ __forceinline__ float f_inf() { return __int_as_float(0x7f800000); }
__device__ __forceinline__ float f_ninf() { return __int_as_float(0xff800000); }

// Order-preserving 32-bit key of an fp32 value (larger value -> larger key); -0 is keyed as +0 so that
// the two zeros tie exactly as they do under IEEE comparison.
__device__ __forceinline__ uint32_t okey(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) == 0) u = 0;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float okey_to_f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

__device__ __forceinline__ float bf16_bits_to_f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// max(a, b) that returns NaN when either operand is NaN
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// ---------------------------------------------------------------- RNG

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7FEB352Du;
    x ^= x >> 15;
    x *= 0x846CA68Bu;
    x ^= x >> 16;
    return x;
}

// Reference counter uniform of (seed, step): three chained lowbias32 finalisers, 24-bit mantissa.
__device__ __forceinline__ float uniform_counter(int64_t seed, int64_t step) {
    uint64_t s = (uint64_t)seed;
    uint32_t h = mix32((uint32_t)s);
    h = mix32(h ^ (uint32_t)(s >> 32) ^ 0x9E3779B9u);
    h = mix32(h ^ (uint32_t)((uint64_t)step) ^ 0x632BE5ABu);
    return (float)(h >> 8) * (1.0f / 16777216.0f);
}

// Philox4x32-10 (Salmon et al., SC'11); returns the first output word.
__device__ __forceinline__ uint32_t philox4x32_10_w0(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                                     uint32_t k1) {
#pragma unroll
    for (int i = 0; i < 10; ++i) {
        if (i) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    }
    return c0;
}

__device__ __forceinline__ float uniform_philox(int64_t seed, int64_t step, int64_t request) {
    uint64_t s = (uint64_t)seed, t = (uint64_t)step, q = (uint64_t)request;
    uint32_t w = philox4x32_10_w0((uint32_t)t, (uint32_t)(t >> 32), (uint32_t)q, (uint32_t)(q >> 32), (uint32_t)s,
                                  (uint32_t)(s >> 32));
    return (float)(w >> 8) * (1.0f / 16777216.0f);
}

// ---------------------------------------------------------------- PTX: loads and asynchronous copies

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16-byte load of data that stays read-only for the whole kernel, not kept in L1 (it stays in L2 for a later
// pass over the row).  Not volatile: the compiler may batch several of them ahead of their uses.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 q;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(q.x), "=r"(q.y), "=r"(q.z), "=r"(q.w)
        : "l"(p));
    return q;
}

// The same load without the read-only path: it sees data that another CTA of the same launch wrote and
// published before this thread's acquire (the codec head's logits, b2s_head_sample).
__device__ __forceinline__ uint4 ld_stream_coherent(const uint4* p) {
    uint4 q;
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(q.x), "=r"(q.y), "=r"(q.z), "=r"(q.w)
                 : "l"(p)
                 : "memory");
    return q;
}

// Asynchronous 4 / 8-byte copies global -> shared (the issuing thread does not wait for them).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------- PTX: bulk copies (TMA engine) and mbarriers

// mbarrier with `count` expected arrivals (one CTA-local 8-byte word).
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the asynchronous proxy (the bulk-copy engine) and the cluster.
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// One arrival that also announces `bytes` of transactions the phase waits for.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Bulk copy global -> this CTA's shared memory by the TMA engine, completing `bytes` transactions on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Waits for the phase of `bar` with the given parity to complete, for at most `limit_ns`; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// Split cluster barrier: arrive (no ordering of memory) now, wait later; every thread of every CTA of the
// cluster executes both, once per phase.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Named barrier `id` (1..15) of `count` threads (a multiple of 32): sync waits for all of them, arrive only counts
// this warp in.  Both order this thread's earlier memory accesses before the barrier for the others.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialisation may start
// while the previous kernel of the stream is still running.  It first waits for that kernel's completion
// (and the visibility of its writes), then lets the next kernel of the stream start early in turn.  Without
// a programmatic predecessor the wait returns at once.
__device__ __forceinline__ void pdl_wait_then_release() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- warp / CTA primitives

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_incl_scan(double v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        double u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

// CTA-wide helpers use a caller-provided shared scratch of >= NWARP+1 doubles.
__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < NWARP; ++i) r = fmaxf(r, red[i]);
    return r;
}
// Sum of doubles reduced in a fixed order (warp butterfly, then warps in index order).
__device__ __forceinline__ double block_sum(double v, double* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    double r = 0.0;
#pragma unroll
    for (int i = 0; i < NWARP; ++i) r += red[i];
    return r;
}
__device__ __forceinline__ int block_sum_i(int v, int* red) {
    v = warp_sum_i(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    int r = 0;
#pragma unroll
    for (int i = 0; i < NWARP; ++i) r += red[i];
    return r;
}
// Exclusive scan of one double per thread in thread order; returns the exclusive prefix, *total = sum.
__device__ __forceinline__ double block_excl_scan(double v, double* red, double* total) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    double incl = warp_incl_scan(v);
    __syncthreads();
    if (lane == 31) red[w] = incl;
    __syncthreads();
    double off = 0.0, tot = 0.0;
#pragma unroll
    for (int i = 0; i < NWARP; ++i) {
        if (i < w) off += red[i];
        tot += red[i];
    }
    *total = tot;
    return off + incl - v;
}

// Exclusive scan of one int per thread in thread order; *total = sum.  red: NWARP + 1 shared ints.
__device__ __forceinline__ int block_excl_scan_i(int v, int* red, int* total) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    __syncthreads();
    if (lane == 31) red[w] = incl;
    __syncthreads();
    int off = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < NWARP; ++i) {
        off += i < w ? red[i] : 0;
        tot += red[i];
    }
    *total = tot;
    return off + incl - v;
}

// Radix select: the key of the k-th largest (1-based, 1 <= k <= n) of n keys produced by key(i), over 4
// rounds of 8-bit digits, most significant first.  hist: 256 shared words; ctl: 2 shared words.
template <typename KeyFn>
__device__ uint32_t block_kth_largest(int n, int k, KeyFn key, uint32_t* hist, uint32_t* ctl) {
    uint32_t prefix = 0, mask = 0;
    int krem = k;
    const int tid = threadIdx.x;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += NT) hist[i] = 0;
        __syncthreads();
        // whole warps iterate together so equal digits can be aggregated (one atomic per distinct digit)
        for (int base = 0; base < n; base += NT) {
            const int i = base + tid;
            uint32_t d = 256u;
            if (i < n) {
                const uint32_t kk = key(i);
                if ((kk & mask) == prefix) d = (kk >> shift) & 255u;
            }
            const uint32_t same = __match_any_sync(0xffffffffu, d);
            if (d != 256u && (threadIdx.x & 31) == (uint32_t)(__ffs(same) - 1)) atomicAdd(&hist[d], (uint32_t)__popc(same));
        }
        __syncthreads();
        if (tid < 32) {
            // lane l owns digits 255-8l .. 248-8l (descending)
            uint32_t c[8];
            uint32_t s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * tid - j]; s += c[j]; }
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += u;
            }
            uint32_t excl = incl - s;
            if (excl < (uint32_t)krem && (uint32_t)krem <= incl) {
                uint32_t cum = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (cum + c[j] >= (uint32_t)krem) {
                        ctl[0] = (uint32_t)(255 - 8 * tid - j);
                        ctl[1] = (uint32_t)krem - cum;
                        break;
                    }
                    cum += c[j];
                }
            }
        }
        __syncthreads();
        prefix |= ctl[0] << shift;
        mask |= 0xFFu << shift;
        krem = (int)ctl[1];
        __syncthreads();
    }
    return prefix;
}

}  // namespace b2s
