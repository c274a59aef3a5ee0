// Row-level pieces shared by the two sampling kernels (the streaming kernel of b2s_sampler.cu and the
// row-resident kernel of b2s_resident.cu): launch parameters, the per-row shared control block, element
// access for fp32 / bf16 rows, the count-based penalty, the history-aware processed value of an element,
// and the full-row passes (ordered draw, radix select, bucket select) that both kernels fall back on.
#pragma once

#include <cooperative_groups.h>
#include <cuda.h>  // CUtensorMap

#include "../../include/b2s_sampler.h"
#include "b2s_device.cuh"
#include "b2s_list.cuh"

namespace b2s {

constexpr int KFAST = KLIST;     // largest top_k served by the candidate path
#ifndef B2S_CHUNK_BYTES
#define B2S_CHUNK_BYTES 32768
#endif
constexpr int CHUNK = B2S_CHUNK_BYTES;  // bytes of the row a CTA takes per stream iteration
constexpr int VPC = CHUNK / 16;         // 16-byte vectors per stream iteration
constexpr int NBUCKET = 1024;    // buckets per threshold round
constexpr int HPT = 4;           // history positions per thread gathered during the stream
constexpr int MODE_FILTER = 0, MODE_FULL = 1, MODE_FORCED = 2, MODE_SKIP = 3, MODE_FAIL = 4;
constexpr int64_t PAD = -1;
constexpr int RPV = 2048;  // row-resident kernel: 16-byte vectors per piece (32 KB), one bulk copy + mbarrier each
constexpr int RMAXP = 8;   // row-resident kernel: pieces of one CTA's slice at most (256 KB)
constexpr int RSH = RPV / NT;  // row-resident kernel: vectors of a thread's share of a piece
constexpr uint32_t HT_EMPTY = 0xFFFFFFFFu;
constexpr int HT_CNT_BITS = 14;

struct Params {
    const void* logits;
    int64_t lstride;
    int rows, V, W, eos;
    const int64_t* hist;
    int64_t hstride;
    const int64_t* steps;
    const int64_t* seeds;
    const int64_t* requests;
    const float* uvals;
    const uint8_t* active;
    const uint8_t* finished;
    float T, top_p, presence, frequency;
    int top_k, min_keep;
    int64_t min_new, max_new;
    const int64_t* rminn;  // per-row min_new / max_new, or nullptr
    const int64_t* rmaxn;
    const float* rT;
    const float* rP;
    const int32_t* rK;
    const float* alpha;
    int alpha_len, alpha_stride;
    int sem, rng, flags;
    int64_t* tokens;
    float* proc;
    int64_t pstride;
    int64_t* hist_out;
    int64_t hostride;
    int64_t* steps_out;
    uint8_t* fin_out;
    uint32_t* status;
    // vocabulary-shard candidate output (b2s_shard_candidates); cout_n == nullptr otherwise
    float* cout_v;
    int32_t* cout_i;
    int32_t* cout_n;
    int ccap;
    int64_t id_off;  // global id of column 0 of these rows (history ids are global)
    // geometry and shared-memory layout (bytes)
    int lcap, kbuf, nvals;
    int hcap;  // distinct history ids a row can hold (window + the censored EOS)
    uint32_t bitwords;
    uint32_t off_ctl, off_bits, off_pref, off_hcnt, off_hid, off_hpos, off_htv, off_smask, off_hstage, off_atab, off_cand,
        off_candi, off_lst, off_vals, off_hist, off_hraw, off_tmaxc;
    int tmc_chunks;  // chunks whose per-thread maxima fit (rows with more take the exact path)
    int csplit;      // 1: two CTAs per row (a cluster): rank 1 builds the history structures, rank 0 the rest
    uint32_t smem_total;
    // row-resident kernel (b2s_resident.cu): CTAs per row, the merged list's capacity, where the mbarriers and
    // the row slice live, and the slice capacity in 16-byte vectors
    int cl, ltot, slice_vecs;
    uint32_t off_bar, off_slice;
    uint32_t off_ht, ht_slots;  // row-resident kernel, omni order: the owned history ids' (id, count) hash table
    // short-row kernel (b2s_short.cu): one occurrence-count byte per element, 4 per word
    uint32_t off_cnt, cnt_words;
    // several frames in one launch (b2s_sample_frames): logits of frame f start f * fstride elements after frame 0's;
    // tokens and uniform values are [frames, rows]; the state advances in place from frame to frame
    int frames;
    int64_t fstride;
    // codec head in the same launch (b2s_head_sample): CTAs rows .. rows + head_tiles - 1 compute the bf16 logits
    // rows (b2s_head.cuh) from hidden [rows, head_kb * 64] (hid_stride elements apart) into `logits`; the rows'
    // CTAs wait on head_sync (4 words, zero between launches) before reading them
    int head_tiles, head_kb;
    int head_split, head_first;  // CTAs per tile (1, or 2 = a cluster splitting K); first tile CTA (rows, even if split)
    const void* hidden;
    int64_t hid_stride;
    uint32_t* head_sync;
};

struct Ctl {
    int err, gather_n, kn;
    int hd_x;  // distinct history ids, from the helper CTA (two-CTA rows)
    int wcnt[NWARP];  // candidates each warp pushed into its segment of the list
    uint32_t rctl[2];
    uint32_t klo, kcnt;
    float thr;
    float u;
    double red_d[NWARP + 1];
    float red_f[NWARP + 1];
    int red_i[NWARP + 1];
    uint32_t red_u[2 * NWARP + 2];
    int rx_n[8];  // row-resident kernel: candidates each other CTA of the cluster handed over (-1: incomplete)
    int lovf;     // row-resident kernel: a CTA's candidates are incomplete or did not fit rank 0's list
    float rx_tau[8];  // row-resident kernel: each CTA's tau (every one bounds the row's k-th value from below)
    float lse;        // short-row kernel: the normaliser, handed from warp 4 to warp 0
    int hd_n;         // row-resident kernel, omni order: distinct owned history ids appended to the dense list
    int sr_state, sr_n;  // short-row kernel: how the row's token is taken, and the candidates in the list
    int head_ok;         // short-row kernel with the codec head: the row's logits are complete
};

template <typename E>
struct Elem;
template <>
struct Elem<float> {
    static constexpr int SZ = 4, EPV = 4;
    static __device__ __forceinline__ float gld(const void* base, int64_t i) {
        return __ldg(reinterpret_cast<const float*>(base) + i);
    }
    // a plain (coherent) load, for logits written earlier in the same launch (b2s_head_sample)
    static __device__ __forceinline__ float gld_coh(const void* base, int64_t i) {
        return reinterpret_cast<const float*>(base)[i];
    }
    static __device__ __forceinline__ float sld(const unsigned char* s) { return *reinterpret_cast<const float*>(s); }
    static __device__ __forceinline__ float vmax(uint4 q) {
        return fmaxf(fmaxf(__uint_as_float(q.x), __uint_as_float(q.y)), fmaxf(__uint_as_float(q.z), __uint_as_float(q.w)));
    }
    static __device__ __forceinline__ float at(uint4 q, int j) {
        const uint32_t w = j == 0 ? q.x : j == 1 ? q.y : j == 2 ? q.z : q.w;
        return __uint_as_float(w);
    }
    // maximum of the 4 elements, NaN if any is NaN
    static __device__ __forceinline__ float vmax_nan(uint4 q) {
        return fmax_nan(fmax_nan(__uint_as_float(q.x), __uint_as_float(q.y)),
                        fmax_nan(__uint_as_float(q.z), __uint_as_float(q.w)));
    }
    static constexpr uint32_t NEG = 0xff800000u;  // -inf in every element of a word
    static __device__ __forceinline__ void st_ninf(unsigned char* s) { *reinterpret_cast<uint32_t*>(s) = NEG; }
    template <int N>
    static __device__ __forceinline__ float vmaxn(const uint4* q) {
        float m = vmax(q[0]);
#pragma unroll
        for (int t = 1; t < N; ++t) m = fmaxf(m, vmax(q[t]));
        return m;
    }
};
template <>
struct Elem<__nv_bfloat16> {
    static constexpr int SZ = 2, EPV = 8;
    static __device__ __forceinline__ float gld(const void* base, int64_t i) {
        return bf16_bits_to_f(__ldg(reinterpret_cast<const unsigned short*>(base) + i));
    }
    static __device__ __forceinline__ float gld_coh(const void* base, int64_t i) {
        return bf16_bits_to_f(reinterpret_cast<const unsigned short*>(base)[i]);
    }
    static __device__ __forceinline__ float sld(const unsigned char* s) {
        return bf16_bits_to_f(*reinterpret_cast<const uint16_t*>(s));
    }
    static __device__ __forceinline__ float vmax(uint4 q) {
        const __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&q.x), b = *reinterpret_cast<__nv_bfloat162*>(&q.y);
        const __nv_bfloat162 c = *reinterpret_cast<__nv_bfloat162*>(&q.z), d = *reinterpret_cast<__nv_bfloat162*>(&q.w);
        const __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
        return fmaxf(__low2float(m), __high2float(m));
    }
    static __device__ __forceinline__ float at(uint4 q, int j) {
        const uint32_t w = (j >> 1) == 0 ? q.x : (j >> 1) == 1 ? q.y : (j >> 1) == 2 ? q.z : q.w;
        return __uint_as_float((j & 1) ? (w & 0xffff0000u) : (w << 16));
    }
    // maximum of the 8 elements, NaN if any is NaN (bf16 max is exact)
    static __device__ __forceinline__ float vmax_nan(uint4 q) {
        const __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&q.x), b = *reinterpret_cast<__nv_bfloat162*>(&q.y);
        const __nv_bfloat162 c = *reinterpret_cast<__nv_bfloat162*>(&q.z), d = *reinterpret_cast<__nv_bfloat162*>(&q.w);
        const __nv_bfloat162 m = __hmax2_nan(__hmax2_nan(a, b), __hmax2_nan(c, d));
        return fmax_nan(__low2float(m), __high2float(m));
    }
    static constexpr uint32_t NEG = 0xff80ff80u;
    static __device__ __forceinline__ void st_ninf(unsigned char* s) { *reinterpret_cast<uint16_t*>(s) = (uint16_t)0xff80u; }
    // max of N x 8 bf16 values in packed bf16x2 arithmetic
    template <int N>
    static __device__ __forceinline__ float vmaxn(const uint4* q) {
        __nv_bfloat162 r;
#pragma unroll
        for (int t = 0; t < N; ++t) {
            const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&q[t].x);
            const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&q[t].y);
            const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&q[t].z);
            const __nv_bfloat162 d = *reinterpret_cast<const __nv_bfloat162*>(&q[t].w);
            const __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
            r = t == 0 ? m : __hmax2(r, m);
        }
        return fmaxf(__low2float(r), __high2float(r));
    }
};

__device__ __forceinline__ void set_status(const Params& p, uint32_t bits) {
    if (p.status) atomicOr(p.status, bits);
}

// Open-addressing hash of id -> occurrence count, packed as id << 14 | count in one word (ids < 2^18).
__device__ __forceinline__ uint32_t ht_slot(uint32_t id, uint32_t slots) { return (id * 2654435761u) & (slots - 1); }
__device__ __forceinline__ void ht_insert(uint32_t* ht, uint32_t slots, uint32_t id, uint32_t add) {
    uint32_t hs = ht_slot(id, slots);
    for (uint32_t probe = 0; probe < slots; ++probe) {
        uint32_t cur = ht[hs];
        if (cur == HT_EMPTY) {
            cur = atomicCAS(&ht[hs], HT_EMPTY, (id << HT_CNT_BITS) | add);
            if (cur == HT_EMPTY) return;
        }
        if ((cur >> HT_CNT_BITS) == id) {
            if (add) atomicAdd(&ht[hs], add);
            return;
        }
        hs = (hs + 1) & (slots - 1);
    }
}
// ht_insert that also tells its caller the id's slot and whether this call put the id in the table (false for an
// id already there; slot = slots when the table is full, which a table of at least twice the distinct ids never is).
__device__ __forceinline__ bool ht_add(uint32_t* ht, uint32_t slots, uint32_t id, uint32_t add, uint32_t& slot) {
    uint32_t hs = ht_slot(id, slots);
    for (uint32_t probe = 0; probe < slots; ++probe) {
        uint32_t cur = ht[hs];
        if (cur == HT_EMPTY) {
            cur = atomicCAS(&ht[hs], HT_EMPTY, (id << HT_CNT_BITS) | add);
            if (cur == HT_EMPTY) {
                slot = hs;
                return true;
            }
        }
        if ((cur >> HT_CNT_BITS) == id) {
            if (add) atomicAdd(&ht[hs], add);
            slot = hs;
            return false;
        }
        hs = (hs + 1) & (slots - 1);
    }
    slot = slots;
    return false;
}
__device__ __forceinline__ int ht_find(const uint32_t* ht, uint32_t slots, uint32_t id) {
    uint32_t h = ht_slot(id, slots);
    for (uint32_t probe = 0; probe < slots; ++probe) {
        const uint32_t w = ht[h];
        if (w == HT_EMPTY) return -1;
        if ((w >> HT_CNT_BITS) == id) return (int)h;
        h = (h + 1) & (slots - 1);
    }
    return -1;
}

__device__ __forceinline__ float pen_a(float v, int n, float a) {
    if (n <= 0) return v;  // penalty**0 == 1: v * 1 == v / 1 == v
    return v < 0.0f ? __fmul_rn(v, a) : __fdiv_rn(v, a);
}
__device__ __forceinline__ float pen(float v, int n, const float* alpha) { return n <= 0 ? v : pen_a(v, n, alpha[n]); }

// Processed value of a history id seen n times with raw value x, from the row's penalty table atab
// (penalty**n): hf divides by T first, then applies the penalty (talker_sampler.py:149,154); omni applies
// the penalty, then the presence / frequency penalties (subtracted once / n times), then divides by T
// (:146), and a censored EOS is -inf whatever its count.  A count past the table is clamped to its last
// entry and flagged.
__device__ __forceinline__ float hist_proc_value(const Params& p, const float* atab, bool hf, bool censored_eos,
                                                 float T, int n, float x) {
    if (n >= p.alpha_len && n > 0) {
        set_status(p, B2S_STATUS_COUNT_LIMIT);
        n = p.alpha_len - 1;
    }
    const float a = n > 0 ? atab[n] : 1.0f;
    if (hf) return pen_a(__fdiv_rn(x, T), n, a);
    const float z = censored_eos ? __int_as_float(0xff800000) : x;
    float v = pen_a(z, n, a);
    if (n > 0) {
        v = __fsub_rn(v, p.presence);
        v = __fsub_rn(v, __fmul_rn(p.frequency, (float)n));
    }
    return __fdiv_rn(v, T);
}

// Per-row context: where the row's elements live and how an element's processed value is obtained.
template <typename E>
struct Row {
    const unsigned char* rowp;  // element 0 in global memory
    const uint4* gvec;          // interior vector 0 in global memory
    int V, nh, nvec, e0;        // head elements [0, nh); interior vectors; first interior element e0 == nh
    const uint32_t* bits;       // history bitmap (nullptr: no history ids)
    const uint16_t* pref;       // per 4-word group of the bitmap: the history ids below it (exclusive prefix)
    const float* htv;           // processed value of each distinct history id, by rank
    float T;
    bool identity;
    int censor;                 // element whose processed value is -inf regardless (omni censored EOS) or -1
    bool coh = false;           // the row was written earlier in the same launch: coherent loads, not read-only ones

    __device__ __forceinline__ float f(float x) const { return identity ? x : __fdiv_rn(x, T); }
    __device__ __forceinline__ bool hbit(int i) const { return bits && ((bits[i >> 5] >> (i & 31)) & 1u); }
    // bits [i, i + n) of the history bitmap (n <= 8), packed from bit 0
    __device__ __forceinline__ uint32_t hbits(int i, int n) const {
        if (!bits) return 0;
        const int w = i >> 5, o = i & 31;
        uint32_t b = bits[w] >> o;
        if (o + n > 32) b |= bits[w + 1] << (32 - o);
        return b & ((1u << n) - 1u);
    }
    __device__ __forceinline__ float raw(int i) const { return coh ? Elem<E>::gld_coh(rowp, i) : Elem<E>::gld(rowp, i); }
    // rank of a history id i among the row's distinct history ids (ascending id order)
    __device__ __forceinline__ int rank(int i) const {
        const int w = i >> 5, sub = w & 3;
        const uint4 q = reinterpret_cast<const uint4*>(bits)[w >> 2];
        int r = (int)pref[w >> 2];
        r += sub > 0 ? __popc(q.x) : 0;
        r += sub > 1 ? __popc(q.y) : 0;
        r += sub > 2 ? __popc(q.z) : 0;
        const uint32_t wv = sub == 0 ? q.x : sub == 1 ? q.y : sub == 2 ? q.z : q.w;
        return r + __popc(wv & ((1u << (i & 31)) - 1u));
    }
    // processed value of element i (history ids and the censored EOS carry their own value)
    __device__ __forceinline__ float P(int i, float x) const {
        if (hbit(i)) return htv[rank(i)];
        return f(x);
    }
    __device__ __forceinline__ uint4 vec(int v) const { return coh ? gvec[v] : __ldg(gvec + v); }
};

// Visit every element of the row as (index, raw value): interior vectors round-robin over the threads,
// head elements by thread 0, tail elements by thread 1.
template <typename E, typename Fn>
__device__ __forceinline__ void row_visit(const Row<E>& R, Fn fn) {
    const int tid = threadIdx.x;
    constexpr int EPV = Elem<E>::EPV;
    for (int v = tid; v < R.nvec; v += NT) {
        const uint4 q = R.vec(v);
        const int b = R.e0 + v * EPV;
#pragma unroll
        for (int j = 0; j < EPV; ++j) fn(b + j, Elem<E>::at(q, j));
    }
    if (tid == 0)
        for (int i = 0; i < R.nh; ++i) fn(i, R.raw(i));
    if (tid == 1)
        for (int i = R.e0 + R.nvec * EPV; i < R.V; ++i) fn(i, R.raw(i));
}

// Ordered scan of the kept mass: every element i with keep(i, P_i) contributes p_i = fl(expf(P_i - m) / s);
// returns the first index whose fp64 prefix of p, rounded to fp32, exceeds u * total (talker_sampler.py:
// 168-172), or V - 1.  m = max kept P, s = fl(sum expf(P - m)).  Contiguous element ranges per thread keep
// the prefix in index order.
template <typename E, typename Keep>
__device__ int64_t ordered_draw(const Row<E>& R, Keep keep, float u, Ctl* ctl) {
    const int tid = threadIdx.x;
    const int V = R.V;
    const int L = (V + NT - 1) / NT;
    const int i0 = min(V, tid * L), i1 = min(V, i0 + L);
    float lm = f_ninf();
    for (int i = i0; i < i1; ++i) {
        const float P = R.P(i, R.raw(i));
        if (keep(i, P)) lm = fmaxf(lm, P);
    }
    const float m = block_max(lm, ctl->red_f);
    auto e_of = [&](int i) {
        const float P = R.P(i, R.raw(i));
        return keep(i, P) ? b2s_expf(__fsub_rn(P, m)) : 0.0f;
    };
    double es = 0.0;
    for (int i = i0; i < i1; ++i) es += (double)e_of(i);
    const float sf = (float)block_sum(es, ctl->red_d);
    double ps = 0.0;
    for (int i = i0; i < i1; ++i) ps += (double)__fdiv_rn(e_of(i), sf);
    double total;
    double acc = block_excl_scan(ps, ctl->red_d, &total);
    const float target = __fmul_rn(u, (float)total);
    int first = 0x7fffffff;
    for (int i = i0; i < i1; ++i) {
        const float pi = __fdiv_rn(e_of(i), sf);
        if (pi == 0.0f) continue;
        acc += (double)pi;
        if ((float)acc > target) { first = i; break; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    __syncthreads();
    if ((tid & 31) == 0) ctl->red_i[tid >> 5] = first;
    __syncthreads();
    int best = 0x7fffffff;
    for (int w = 0; w < NWARP; ++w) best = min(best, ctl->red_i[w]);
    __syncthreads();
    return best == 0x7fffffff ? (int64_t)(V - 1) : (int64_t)best;
}

// Radix select over the row: the key of the k-th largest processed value (1 <= k <= V).
template <typename E>
__device__ uint32_t row_kth_key(const Row<E>& R, int k, uint32_t* hist, Ctl* ctl) {
    const int tid = threadIdx.x;
    uint32_t prefix = 0, mask = 0;
    int krem = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += NT) hist[i] = 0;
        __syncthreads();
        row_visit<E>(R, [&](int i, float x) {
            const uint32_t kk = okey(R.P(i, x));
            if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 255u], 1u);
        });
        __syncthreads();
        if (tid < 32) {
            uint32_t c[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * tid - j]; s += c[j]; }  // 8-word stride
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += t;
            }
            const uint32_t excl = incl - s;
            if (excl < (uint32_t)krem && (uint32_t)krem <= incl) {
                uint32_t cum = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (cum + c[j] >= (uint32_t)krem) {
                        ctl->rctl[0] = (uint32_t)(255 - 8 * tid - j);
                        ctl->rctl[1] = (uint32_t)krem - cum;
                        break;
                    }
                    cum += c[j];
                }
            }
        }
        __syncthreads();
        prefix |= ctl->rctl[0] << shift;
        mask |= 0xFFu << shift;
        krem = (int)ctl->rctl[1];
        __syncthreads();
    }
    return prefix;
}

// T such that at least k of the n keys produced by key(i) are >= T, found with two rounds of a 1024-bucket
// histogram over [min key, max key]: T is the lower edge of the bucket holding the k-th largest key (the
// key itself when the second round resolves it).  Returns 0 when n < k.  Every thread calls it.
template <typename KeyFn>
__device__ uint32_t kth_key_bucket(int n, int k, KeyFn key, uint32_t* hist, Ctl* ctl) {
    const int tid = threadIdx.x, lane = tid & 31;
    uint32_t kmn = 0xFFFFFFFFu, kmx = 0;
    for (int i = tid; i < n; i += NT) {
        const uint32_t kk = key(i);
        kmn = min(kmn, kk);
        kmx = max(kmx, kk);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        kmn = min(kmn, __shfl_xor_sync(0xffffffffu, kmn, o));
        kmx = max(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    }
    __syncthreads();
    if (lane == 0) {
        ctl->red_u[2 * (tid >> 5)] = kmn;
        ctl->red_u[2 * (tid >> 5) + 1] = kmx;
    }
    __syncthreads();
    uint32_t klo = 0xFFFFFFFFu, khi = 0;
    for (int w = 0; w < NWARP; ++w) {
        klo = min(klo, ctl->red_u[2 * w]);
        khi = max(khi, ctl->red_u[2 * w + 1]);
    }
    if (n < k) return 0u;
    int krem = k;
    for (int round = 0; round < 2 && khi > klo; ++round) {
        const uint32_t range = khi - klo;
        const int nbits = 32 - __clz(range);
        const int sh = nbits > 10 ? nbits - 10 : 0;
        for (int b = tid; b < NBUCKET; b += NT) hist[b] = 0;
        __syncthreads();
        for (int i = tid; i < n; i += NT) {
            const uint32_t kk = key(i);
            if (kk >= klo && kk <= khi) atomicAdd(&hist[(kk - klo) >> sh], 1u);
        }
        __syncthreads();
        if (tid < 32) {
            // lane l owns buckets 1023-32l .. 992-32l (descending); find the lane, then the bucket inside it
            uint32_t sum = 0;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) sum += hist[NBUCKET - 1 - 32 * tid - ((j + tid) & 31)];  // rotated: no bank conflicts
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += t;
            }
            const uint32_t excl = incl - sum;
            const unsigned who = __ballot_sync(0xffffffffu, excl < (uint32_t)krem && (uint32_t)krem <= incl);
            const int L = __ffs(who) - 1;  // who != 0: krem <= the total count
            const uint32_t base = __shfl_sync(0xffffffffu, excl, L);
            const int b = NBUCKET - 1 - 32 * L - tid;
            const uint32_t cb = hist[b];
            uint32_t inc2 = cb;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, inc2, o);
                if (tid >= o) inc2 += t;
            }
            const unsigned who2 = __ballot_sync(0xffffffffu, base + inc2 >= (uint32_t)krem);
            if (tid == __ffs(who2) - 1) {
                ctl->klo = klo + ((uint32_t)b << sh);
                ctl->kcnt = (uint32_t)krem - (base + inc2 - cb);
            }
        }
        __syncthreads();
        const uint32_t nlo = ctl->klo;
        const uint32_t span = (1u << sh) - 1u;
        khi = min(khi, nlo + span);
        klo = nlo;
        krem = (int)ctl->kcnt;
        __syncthreads();
    }
    return klo;
}

// Exact top-k / top-p threshold of a row whose k-th largest processed key is `kth` (row_kth_key): the values
// above the k-th (fewer than k) gathered and sorted, k - count copies of the k-th after them, then the
// top-p cut over the k values -- hf with the full-row normaliser `lse` (talker_sampler.py:110-115), omni
// with a softmax over the k values (:127-132), kept count clamped to [min(min_keep, k), k].  vals holds
// >= max(k, next pow2 of the count above) floats.  Every thread calls it; the same value in every thread.
template <typename E>
__device__ float exact_threshold(const Row<E>& R, uint32_t kth, int k, bool hf, float lse, float top_p, int min_keep,
                                 bool topk_only, float* vals, Ctl* ctl) {
    const int tid = threadIdx.x;
    // values above the k-th (fewer than k), sorted, then k - count copies of the k-th
    if (tid == 0) ctl->gather_n = 0;
    __syncthreads();
    row_visit<E>(R, [&](int i, float x) {
        const float P = R.P(i, x);
        if (okey(P) > kth) vals[atomicAdd(&ctl->gather_n, 1)] = P;
    });
    __syncthreads();
    const int ng = ctl->gather_n;
    int n2 = 1;
    while (n2 < ng) n2 <<= 1;
    for (int i = ng + tid; i < n2; i += NT) vals[i] = f_ninf();
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < n2; i += NT) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const float a = vals[i], b = vals[j];
                    if (desc ? (a < b) : (a > b)) { vals[i] = b; vals[j] = a; }
                }
            }
            __syncthreads();
        }
    }
    for (int i = ng + tid; i < k; i += NT) vals[i] = okey_to_f(kth);
    __syncthreads();
    // top-p over the k values, prefix in order (contiguous chunk per thread)
    const int per_t = (k + NT - 1) / NT;
    const int a0 = min(k, tid * per_t), a1 = min(k, a0 + per_t);
    const float m = vals[0];
    float sf = 1.0f;
    if (!hf) {
        double es = 0.0;
        for (int i = a0; i < a1; ++i) es += (double)b2s_expf(__fsub_rn(vals[i], m));
        sf = (float)block_sum(es, ctl->red_d);
    }
    auto pk = [&](int i) {
        return hf ? b2s_expf(__fsub_rn(vals[i], lse)) : __fdiv_rn(b2s_expf(__fsub_rn(vals[i], m)), sf);
    };
    double ls = 0.0;
    for (int i = a0; i < a1; ++i) ls += (double)pk(i);
    double total;
    double acc = block_excl_scan(ls, ctl->red_d, &total);
    int cnt = 0;
    for (int i = a0; i < a1; ++i) {
        const float pi = pk(i);
        acc += (double)pi;
        cnt += __fsub_rn((float)acc, pi) < top_p;
    }
    cnt = block_sum_i(cnt, ctl->red_i);
    const int kept = topk_only ? k : max(min(min_keep, k), min(cnt, k));
    const float thr = vals[kept - 1];
    __syncthreads();
    return thr;
}

// The row-resident kernel's instantiations (b2s_resident.cu): logits type, omni order fixed at compile time.
using ResKernel = void (*)(const Params);
ResKernel resident_kernel_for(bool bf16, bool omni);

// The short-row kernel (b2s_short.cu): rows of at most SHORT_EPT * NT interior elements, each thread's share held
// in registers; same instantiations.
constexpr int SHORT_EPT = 16;
ResKernel short_kernel_for(bool bf16, bool omni);

// The short-row kernel with the Talker codec head in the same launch (b2s_short.cu, b2s_head.cuh): bf16 logits,
// the head tile's TMA map as the second parameter.
using HeadKernel = void (*)(const Params, const CUtensorMap);
HeadKernel head_kernel_for(bool omni);

}  // namespace b2s
