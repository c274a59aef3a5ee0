// The final stage of a row, shared by the candidate path of the sampling kernel and the vocabulary-shard
// merge: from a list of (processed value, vocabulary id) items that contains every element >= the row's
// k-th largest value (ties included), take the top-k values, the top-p cut, the value threshold, and the
// inverse-CDF draw over the kept items in vocabulary order.  One CTA (NT threads) runs it; the short
// sequential parts (top-p, the ordered cumulative mass) run in warp 0 without block barriers.
#pragma once

#include "b2s_device.cuh"

namespace b2s {

constexpr int KLIST = 128;  // largest k the list stage serves (top-p in one warp, 4 values per lane)

// Pointers into the CTA's shared scratch.
struct Scr {
    uint32_t* hist;  // 256 words (radix select)
    uint32_t* rctl;  // 2 words
    int* gather_n;
    int* kn;
    float* thr;
    double* red_d;   // NWARP + 1
    float* red_f;
    int* red_i;
};

// list_topk_values for lists of more than 128 items (kept out of line: decode steps rarely take it).
static __device__ __noinline__ void list_topk_values_large(const float* cv, int n, int k, float* vals, Scr sc);

// The k largest values of cv[0..n) (n >= k), descending with multiplicity, into vals[0..k).  Small lists
// rank every item by counting (value desc, position asc: ranks are a permutation); longer ones find the
// k-th key by radix select first and rank only the items above it.  vals needs 2*KLIST floats; lists of
// at most 128 items use sc.hist for their ranks.
__device__ __forceinline__ void list_topk_values(const float* cv, int n, int k, float* vals, const Scr& sc) {
    const int tid = threadIdx.x;
    if (n > 128) {
        list_topk_values_large(cv, n, k, vals, sc);
        return;
    }
    {
        // every (item, segment of the list) pair in its own thread: S segments of L items per item, partial
        // ranks summed into sc.hist (shared atomics), so no thread walks the whole list
        uint32_t* rk = sc.hist;
        const int S = NT / max(n, 1), L = (n + S - 1) / S;
        for (int i = tid; i < n; i += NT) rk[i] = 0u;
        __syncthreads();
        const int i = tid / S, s0 = (tid % S) * L;
        if (i < n) {
            const float vi = cv[i];
            int part = 0;
            const int s1 = min(n, s0 + L);
            for (int j = s0; j < s1; ++j) {
                const float vj = cv[j];
                part += (vj > vi) | ((vj == vi) & (j < i));
            }
            if (part) atomicAdd(&rk[i], (uint32_t)part);
        }
        __syncthreads();
        for (int a = tid; a < n; a += NT)
            if (rk[a] < (uint32_t)k) vals[rk[a]] = cv[a];
        __syncthreads();
    }
}

static __device__ __noinline__ void list_topk_values_large(const float* cv, int n, int k, float* vals, Scr sc) {
    const int tid = threadIdx.x;
    if (n <= 2 * NT) {
        // cv is 16-byte aligned: four items per shared load, several loads in flight
        const float4* c4 = reinterpret_cast<const float4*>(cv);
        const int n4 = n >> 2;
        for (int i = tid; i < n; i += NT) {
            const float vi = cv[i];
            int rank = 0;
#pragma unroll 4
            for (int j4 = 0; j4 < n4; ++j4) {
                const float4 v = c4[j4];
                const int j = 4 * j4;
                rank += (v.x > vi) | ((v.x == vi) & (j < i));
                rank += (v.y > vi) | ((v.y == vi) & (j + 1 < i));
                rank += (v.z > vi) | ((v.z == vi) & (j + 2 < i));
                rank += (v.w > vi) | ((v.w == vi) & (j + 3 < i));
            }
            for (int j = 4 * n4; j < n; ++j) {
                const float vj = cv[j];
                rank += (vj > vi) | ((vj == vi) & (j < i));
            }
            if (rank < k) vals[rank] = vi;
        }
        __syncthreads();
        return;
    }
    const uint32_t kth = block_kth_largest(n, k, [&](int i) { return okey(cv[i]); }, sc.hist, sc.rctl);
    if (tid == 0) *sc.gather_n = 0;
    __syncthreads();
    for (int i = tid; i < n; i += NT)
        if (okey(cv[i]) > kth) vals[KLIST + atomicAdd(sc.gather_n, 1)] = cv[i];
    __syncthreads();
    const int ng = *sc.gather_n;  // < k
    for (int i = tid; i < ng; i += NT) {
        const float vi = vals[KLIST + i];
        int rank = 0;
        for (int j = 0; j < ng; ++j) {
            const float vj = vals[KLIST + j];
            rank += (vj > vi) | ((vj == vi) & (j < i));
        }
        vals[rank] = vi;
    }
    for (int i = ng + tid; i < k; i += NT) vals[i] = okey_to_f(kth);
    __syncthreads();
}

// Warp 0: the value threshold of the top-p cut over vals[0..k) (hf: probabilities exp(v - lse) of the full
// row; omni: softmax over the k values), kept count clamped to [min(min_keep, k), k]
// (talker_sampler.py:110-115, :127-132).  Returns the threshold in lane 0..31 of warp 0.
static __device__ __noinline__ float warp_topp_threshold(const float* vals, int k, bool hf, float lse, float top_p,
                                                     int min_keep, bool topk_only) {
    const int lane = threadIdx.x & 31;
    float pk[4];
    const float m = vals[0];
    double ls = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int idx = lane * 4 + j;
        float e = 0.0f;
        if (idx < k) e = hf ? b2s_expf(__fsub_rn(vals[idx], lse)) : b2s_expf(__fsub_rn(vals[idx], m));
        pk[j] = e;
        ls += (double)e;
    }
    if (!hf) {
        const float sf = (float)warp_sum(ls);
        ls = 0.0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            pk[j] = (lane * 4 + j < k) ? __fdiv_rn(pk[j], sf) : 0.0f;
            ls += (double)pk[j];
        }
    }
    const double incl = warp_incl_scan(ls);
    double acc = incl - ls;
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int idx = lane * 4 + j;
        if (idx < k) {
            acc += (double)pk[j];
            cnt += __fsub_rn((float)acc, pk[j]) < top_p;
        }
    }
    cnt = warp_sum_i(cnt);
    const int kept = topk_only ? k : max(min(min_keep, k), min(cnt, k));
    return vals[kept - 1];
}

// Warp 0: the draw over kn <= 32 * NPL items (NPL per lane, contiguous) whose values sv[0..kn) are in
// vocabulary order -- softmax over them, fp64 prefix of the probabilities (rounded to fp32 per prefix), the
// first position whose prefix exceeds u * total (talker_sampler.py:168-172).  Returns that position in every lane, or 0x7fffffff when none does.
template <int NPL>
__device__ __forceinline__ int warp_draw_packed(const float* sv, int kn, float u) {
    const int lane = threadIdx.x & 31;
    float pv[NPL];
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int i = lane * NPL + j;
        pv[j] = i < kn ? sv[i] : __int_as_float(0xff800000);
    }
    // the maximum by one redux on order keys (the items are never NaN; a zero maximum of either sign gives the
    // same differences)
    uint32_t key = okey(pv[0]);
#pragma unroll
    for (int j = 1; j < NPL; ++j) key = max(key, okey(pv[j]));
    const float m = okey_to_f(__reduce_max_sync(0xffffffffu, key));
    float e[NPL];
    double es = 0.0;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        e[j] = (lane * NPL + j < kn) ? b2s_expf(__fsub_rn(pv[j], m)) : 0.0f;
        es += (double)e[j];
    }
    const float sf = (float)warp_sum(es);
    double ps = 0.0;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        e[j] = (lane * NPL + j < kn) ? __fdiv_rn(e[j], sf) : 0.0f;
        ps += (double)e[j];
    }
    const double incl = warp_incl_scan(ps);
    const double total = __shfl_sync(0xffffffffu, incl, 31);
    const float target = __fmul_rn(u, (float)total);
    double acc = incl - ps;
    int first = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        acc += (double)e[j];
        if (first == 0x7fffffff && lane * NPL + j < kn && (float)acc > target) first = lane * NPL + j;
    }
    return __reduce_min_sync(0xffffffffu, first);
}
// The draw over 32 < kn <= 128 items in vocabulary order: two items per lane up to 64, four beyond.
__device__ __forceinline__ int warp_draw_sorted(const float* sv, int kn, float u) {
    return kn <= 64 ? warp_draw_packed<2>(sv, kn, u) : warp_draw_packed<4>(sv, kn, u);
}

// Draw over the items >= thr (minus `drop_id` when >= 0): softmax over them, cumulative mass in vocabulary
// order (fp64, rounded per prefix), first id whose mass exceeds u * total, else V - 1
// (talker_sampler.py:168-172).  kv/ki and sv/si: scratch of >= n items each.  Result in every thread.
static __device__ __noinline__ int64_t list_draw(const float* cv, const int* ci, int n, float thr, int drop_id, float u,
                                          int V, float* kv, int* ki, float* sv, int* si, Scr sc) {
    const int tid = threadIdx.x;
    if (tid == 0) *sc.kn = 0;
    __syncthreads();
    for (int i = tid; i < n; i += NT) {
        if (cv[i] >= thr && ci[i] != drop_id) {
            const int pos = atomicAdd(sc.kn, 1);
            kv[pos] = cv[i];
            ki[pos] = ci[i];
        }
    }
    __syncthreads();
    const int kn = *sc.kn;
    for (int i = tid; i < kn; i += NT) {
        int rank = 0;
        const int ii = ki[i];
        for (int j = 0; j < kn; ++j) rank += ki[j] < ii;
        sv[rank] = kv[i];
        si[rank] = ii;
    }
    __syncthreads();
    if (kn <= 128) {
        int first = 0x7fffffff;
        if (tid < 32) first = warp_draw_sorted(sv, kn, u);
        if (tid == 0) *sc.kn = first;
        __syncthreads();
        const int best = *sc.kn;
        return best == 0x7fffffff ? (int64_t)(V - 1) : (int64_t)si[best];
    }
    float lm = __int_as_float(0xff800000);
    for (int i = tid; i < kn; i += NT) lm = fmaxf(lm, sv[i]);
    const float m = block_max(lm, sc.red_f);
    const int per_t = (kn + NT - 1) / NT;
    const int i0 = min(kn, tid * per_t), i1 = min(kn, i0 + per_t);
    double es = 0.0;
    for (int i = i0; i < i1; ++i) es += (double)b2s_expf(__fsub_rn(sv[i], m));
    const float sf = (float)block_sum(es, sc.red_d);
    double ps = 0.0;
    for (int i = i0; i < i1; ++i) ps += (double)__fdiv_rn(b2s_expf(__fsub_rn(sv[i], m)), sf);
    double total;
    double off = block_excl_scan(ps, sc.red_d, &total);
    const float target = __fmul_rn(u, (float)total);
    int first = 0x7fffffff;
    for (int i = i0; i < i1; ++i) {
        const float pi = __fdiv_rn(b2s_expf(__fsub_rn(sv[i], m)), sf);
        off += (double)pi;
        if ((float)off > target) { first = i; break; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    __syncthreads();
    if ((tid & 31) == 0) sc.red_i[tid >> 5] = first;
    __syncthreads();
    int best = 0x7fffffff;
    for (int w = 0; w < NWARP; ++w) best = min(best, sc.red_i[w]);
    return best == 0x7fffffff ? (int64_t)(V - 1) : (int64_t)si[best];
}

// Warp 0, k <= 32: warp_topp_threshold with one value per lane (vals[lane]).  The same fp32 values and
// fp64 accumulation; the fp64 sums only associate differently, which reaches their fp32 rounding only at
// a boundary.
__device__ __forceinline__ float warp_topp_threshold32(const float* vals, int k, bool hf, float lse, float top_p,
                                                       int min_keep, bool topk_only) {
    const int lane = threadIdx.x & 31;
    const bool valid = lane < k;
    const float e = b2s_expf(__fsub_rn(vals[valid ? lane : 0], hf ? lse : vals[0]));
    float pk = valid ? e : 0.0f;
    if (!hf) {
        const float sf = (float)warp_sum((double)pk);
        pk = __fdiv_rn(pk, sf);  // 0 stays 0 (sf >= 1)
    }
    const double incl = warp_incl_scan((double)pk);
    const bool below = valid && __fsub_rn((float)incl, pk) < top_p;
    const int cnt = __popc(__ballot_sync(0xffffffffu, below));
    const int kept = topk_only ? k : max(min(min_keep, k), min(cnt, k));
    return vals[kept - 1];
}

// Warp 0, 32 < k <= 64: warp_topp_threshold with two values per lane (vals[2 * lane], vals[2 * lane + 1]).  The
// same fp32 values and fp64 accumulation, associated in pairs (exact whenever the fp64 sums are, as they are for
// probabilities within 2^29 of each other).
__device__ __forceinline__ float warp_topp_threshold64(const float* vals, int k, bool hf, float lse, float top_p,
                                                       int min_keep, bool topk_only) {
    const int lane = threadIdx.x & 31;
    const float m = vals[0];
    const float2 v2 = reinterpret_cast<const float2*>(vals)[lane];
    float pk[2];
    double ls = 0.0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float v = j ? v2.y : v2.x;
        const float e = 2 * lane + j < k ? b2s_expf(__fsub_rn(v, hf ? lse : m)) : 0.0f;
        pk[j] = e;
        ls += (double)e;
    }
    if (!hf) {
        const float sf = (float)warp_sum(ls);
        ls = 0.0;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            pk[j] = __fdiv_rn(pk[j], sf);  // 0 stays 0 (sf >= 1)
            ls += (double)pk[j];
        }
    }
    const double incl = warp_incl_scan(ls);
    double acc = incl - ls;
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        if (2 * lane + j < k) {
            acc += (double)pk[j];
            cnt += __fsub_rn((float)acc, pk[j]) < top_p;
        }
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    const int kept = topk_only ? k : max(min(min_keep, k), min(cnt, k));
    return vals[kept - 1];
}

// The top-p threshold over the sorted top-k values vals[0..k), in warp 0: one, two or four values per lane.
__device__ __forceinline__ float warp_topp(const float* vals, int k, bool hf, float lse, float top_p, int min_keep,
                                           bool topk_only) {
    return k <= 32 ? warp_topp_threshold32(vals, k, hf, lse, top_p, min_keep, topk_only)
           : k <= 64 ? warp_topp_threshold64(vals, k, hf, lse, top_p, min_keep, topk_only)
                     : warp_topp_threshold(vals, k, hf, lse, top_p, min_keep, topk_only);
}

// Warp 0, kn <= 32 items, lane i holding the value v of the i-th item in vocabulary order (any value past
// kn): warp_draw_sorted with one item per lane.  Returns the position drawn in every lane, or 0x7fffffff.
__device__ __forceinline__ int warp_draw32(float v, int kn, float u) {
    const int lane = threadIdx.x & 31;
    const bool valid = lane < kn;
    // the maximum by one redux on order keys (the items are never NaN; a zero maximum of either sign gives the
    // same differences)
    const float m = okey_to_f(__reduce_max_sync(0xffffffffu, okey(valid ? v : __int_as_float(0xff800000))));
    const float e = valid ? b2s_expf(__fsub_rn(v, m)) : 0.0f;
    const float sf = (float)warp_sum((double)e);
    const float pr = __fdiv_rn(e, sf);  // 0 stays 0
    const double incl = warp_incl_scan((double)pr);
    const double total = __shfl_sync(0xffffffffu, incl, 31);
    const float target = __fmul_rn(u, (float)total);
    const unsigned hit = __ballot_sync(0xffffffffu, valid && (float)incl > target);
    return hit ? __ffs(hit) - 1 : 0x7fffffff;
}

// Bitonic sort, descending, of the warp's 32 * E values: lane l holds elements l * E .. l * E + E - 1 in x.
// Pairs E apart or more are exchanged across lanes by shuffles, nearer pairs inside the lane.  NaN-free input.
template <int E>
__device__ __forceinline__ void warp_bitonic_desc(float (&x)[E]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32 * E; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= E) {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int i = lane * E + e;
                    const float y = __shfl_xor_sync(0xffffffffu, x[e], stride / E);
                    // the lower index of a pair keeps the larger value in a descending block
                    x[e] = (((i & size) == 0) == ((i & stride) == 0)) ? fmaxf(x[e], y) : fminf(x[e], y);
                }
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int f = e ^ stride;
                    if (f > e) {
                        const bool desc = ((lane * E + e) & size) == 0;
                        const float a = x[e], b = x[f];
                        x[e] = desc ? fmaxf(a, b) : fminf(a, b);
                        x[f] = desc ? fminf(a, b) : fmaxf(a, b);
                    }
                }
            }
        }
    }
}

// The sorted top-k values of cv[0..n) (n <= 32 * E, k <= n) into vals[0..k), by one warp.
template <int E>
__device__ __forceinline__ void warp_topk_sorted(const float* cv, int n, int k, float* vals) {
    const int lane = threadIdx.x & 31;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = lane * E + e < n ? cv[lane * E + e] : __int_as_float(0xff800000);
    warp_bitonic_desc<E>(x);
#pragma unroll
    for (int e = 0; e < E; ++e)
        if (lane * E + e < k) vals[lane * E + e] = x[e];
    __syncwarp();
}

// The sorted top-k values of cv[0..n) (n <= 128, NaN-free) into vals[0..k), by one warp.
__device__ __forceinline__ void warp_topk_sorted_n(const float* cv, int n, int k, float* vals) {
    if (n <= 32) warp_topk_sorted<1>(cv, n, k, vals);
    else if (n <= 64) warp_topk_sorted<2>(cv, n, k, vals);
    else warp_topk_sorted<4>(cv, n, k, vals);
}

// One warp (no block barrier), after warp_topk_sorted_n: the rest of the list stage for n <= 128 items already in
// vocabulary order, n >= k -- warp_topp, the kept items (value >= threshold, id != drop_id) compacted by ballot
// into sv / si in list order, which is vocabulary order, and the draw (warp_draw32 / warp_draw_sorted, as
// list_sample).  Returns the position drawn in si in every lane, or 0x7fffffff.
__device__ __forceinline__ int warp_list_kept_draw(const float* cv, const int* ci, int n, int k, bool hf, float lse,
                                                   float top_p, int min_keep, bool topk_only, int drop_id, float u,
                                                   const float* vals, float* sv, int* si) {
    const int lane = threadIdx.x & 31;
    const float thr = warp_topp(vals, k, hf, lse, top_p, min_keep, topk_only);
    int kn = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const float v = i < n ? cv[i] : 0.0f;
        const int id = i < n ? ci[i] : 0;
        const bool keep = i < n && v >= thr && id != drop_id;
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        const int pos = kn + __popc(m & ((1u << lane) - 1u));
        if (keep) {
            sv[pos] = v;
            si[pos] = id;
        }
        kn += __popc(m);
    }
    __syncwarp();
    return kn <= 32 ? warp_draw32(sv[lane < kn ? lane : 0], kn, u) : warp_draw_sorted(sv, kn, u);
}

// The whole list stage: top-k values, top-p threshold (returned in thr_out) and, when `draw`, the token.
// Warp 0 takes the threshold and the draw -- compaction by ballot, vocabulary order by ranking the (distinct)
// kept ids, the same inverse-CDF draw as list_draw -- with no block barrier in between, for up to 32 kept
// items; `in_order` (the list is in vocabulary order already, so the compaction keeps it) skips the ranking
// and serves up to KLIST.  More kept items (heavy ties at the threshold) go to list_draw.  cv must be 16-byte
// aligned.  Result in every thread.
__device__ __forceinline__ int64_t list_sample(const float* cv, const int* ci, int n, int k, bool hf, float lse,
                                               float top_p, int min_keep, bool topk_only, bool draw, int drop_id,
                                               float u, int V, float* vals, float* kv, int* ki, float* sv, int* si,
                                               const Scr& sc, float& thr_out, bool in_order = false) {
    constexpr int FALLBACK = -2;
    list_topk_values(cv, n, k, vals, sc);
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const float t = warp_topp(vals, k, hf, lse, top_p, min_keep, topk_only);
        int res = 0x7fffffff;
        if (draw) {
            // the kept items in list order (in vocabulary order already: straight into sv / si)
            float* ov = in_order ? sv : kv;
            int* oi = in_order ? si : ki;
            int kn = 0;
            for (int i0 = 0; i0 < n; i0 += 32) {
                const int i = i0 + lane;
                const bool keep = i < n && cv[i] >= t && ci[i] != drop_id;
                const unsigned m = __ballot_sync(0xffffffffu, keep);
                const int pos = kn + __popc(m & ((1u << lane) - 1u));
                if (keep && pos < KLIST) {
                    ov[pos] = cv[i];
                    oi[pos] = ci[i];
                }
                kn += __popc(m);
            }
            if (in_order) {
                __syncwarp();
                res = kn <= 32 ? warp_draw32(sv[lane < kn ? lane : 0], kn, u)
                               : kn <= KLIST ? warp_draw_sorted(sv, kn, u) : FALLBACK;
            } else if (kn <= 32) {
                // one kept item per lane: vocabulary order by counting the smaller ids (they are distinct)
                __syncwarp();
                const int id = lane < kn ? ki[lane] : 0x7fffffff;
                const float x = lane < kn ? kv[lane] : 0.0f;
                int rank = 0;
                for (int j = 0; j < kn; ++j) rank += __shfl_sync(0xffffffffu, id, j) < id;
                if (lane < kn) {
                    sv[rank] = x;
                    si[rank] = id;
                }
                __syncwarp();
                res = warp_draw32(sv[lane < kn ? lane : 0], kn, u);
            } else {
                res = FALLBACK;  // more than 32 kept items: the block form below is quicker
            }
        }
        if (lane == 0) {
            *sc.thr = t;
            *sc.kn = res;
        }
    }
    __syncthreads();
    thr_out = *sc.thr;
    const int res = *sc.kn;
    if (res != FALLBACK) return (!draw || res == 0x7fffffff) ? (int64_t)(V - 1) : (int64_t)si[res];
    __syncthreads();  // every thread has read sc.kn before list_draw reuses it
    return list_draw(cv, ci, n, thr_out, drop_id, u, V, kv, ki, sv, si, sc);
}

}  // namespace b2s
