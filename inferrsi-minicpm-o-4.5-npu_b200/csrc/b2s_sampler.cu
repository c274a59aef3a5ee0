// B200 (sm_100a) token-sampling kernels for MiniCPM-o 4.5 and their C-ABI launchers.
//
// One thread-block cluster of C CTAs owns one logits row; CTA c stages the contiguous slice
// [c*per, min(V, (c+1)*per)) of the row into shared memory with 1-D bulk copies (cp.async.bulk, no
// multicast) and everything after that reads shared memory only:
//
//   history ids -> per-slice hash (id -> count) -> penalised values of those ids, slots set to -inf
//   [hf rows with a filter] full-row logsumexp (cluster max, cluster sum)
//   candidate path: k-th largest of the 512 per-thread slice maxima is a lower bound of the row's k-th
//       largest non-history value; raw values above it (plus history ids above its image) are the
//       candidates; each CTA keeps those >= its local k-th; the leader CTA merges the lists over
//       DSMEM, takes the top-k values, the top-p cut, the value threshold, and draws from the kept set
//       in vocabulary order
//   exact path (top_k > 128, candidate overflow, frame-0 hf rows, draw()): cluster-wide radix select
//       of the k-th key, sorted top-k values, top-p, then a distributed draw (cluster max, cluster sum,
//       per-CTA mass and an ordered scan for the first cumulative mass above u * total)
//
// Selection is done on raw values: for ids outside the history the processed value is fl(x / T),
// monotone in x, so the order and the k-th element carry over; history ids are processed exactly.
#include "b2s_device.cuh"
#include "b2s_list.cuh"

#include <cooperative_groups.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "../../include/b2s_sampler.h"

namespace cg = cooperative_groups;

namespace b2s {

constexpr int KFAST = KLIST;  // largest top_k served by the candidate path
constexpr int CAP = 1024;   // candidate slots per CTA
constexpr int MODE_FILTER = 0, MODE_FULL = 1, MODE_FORCED = 2, MODE_SKIP = 3, MODE_FAIL = 4;
constexpr int64_t PAD = -1;
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
    int64_t id_off;  // global id of this row slice's column 0 (history ids are global)
    // launch geometry and shared-memory layout (bytes)
    int C, per, lcap, mcap, kbuf, candcap;
    uint32_t ht_slots;
    uint32_t off_slice, off_ht, off_htv, off_cand, off_candi, off_list, off_listi, off_vals, off_hist, off_ctl;
    uint32_t smem_total;
};

struct Ctl {
    uint64_t bar;
    int cand_n, list_n, overflow, err, gather_n, kn;
    uint32_t rctl[2];
    uint32_t prefix;
    int krem;
    float thr, lse;
    float xmax1, xmax2;
    double xsum1, xsum2, xq;
    int xfirst;
    int pad_;
    double red_d[NWARP + 1];
    float red_f[NWARP + 1];
    int red_i[NWARP + 1];
};

template <typename E>
struct Elem;
template <>
struct Elem<float> {
    static constexpr int SZ = 4;
    static __device__ __forceinline__ float ld(const unsigned char* s, uint32_t off) {
        return *reinterpret_cast<const float*>(s + off);
    }
    static __device__ __forceinline__ void st_ninf(unsigned char* s, uint32_t off) {
        *reinterpret_cast<uint32_t*>(s + off) = 0xff800000u;
    }
    static __device__ __forceinline__ float gld(const void* base, int64_t i) {
        return __ldg(reinterpret_cast<const float*>(base) + i);
    }
    // max of the 4 values of a 16-byte vector
    static __device__ __forceinline__ float vmax(uint4 q) {
        return fmaxf(fmaxf(__uint_as_float(q.x), __uint_as_float(q.y)), fmaxf(__uint_as_float(q.z), __uint_as_float(q.w)));
    }
    static __device__ __forceinline__ float at(uint4 q, int j) {
        uint32_t w = j == 0 ? q.x : j == 1 ? q.y : j == 2 ? q.z : q.w;
        return __uint_as_float(w);
    }
};
template <>
struct Elem<__nv_bfloat16> {
    static constexpr int SZ = 2;
    static __device__ __forceinline__ float ld(const unsigned char* s, uint32_t off) {
        return bf16_bits_to_f(*reinterpret_cast<const uint16_t*>(s + off));
    }
    static __device__ __forceinline__ void st_ninf(unsigned char* s, uint32_t off) {
        *reinterpret_cast<uint16_t*>(s + off) = (uint16_t)0xff80u;
    }
    static __device__ __forceinline__ float gld(const void* base, int64_t i) {
        return bf16_bits_to_f(__ldg(reinterpret_cast<const unsigned short*>(base) + i));
    }
    static __device__ __forceinline__ float vmax(uint4 q) {
        __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&q.x), b = *reinterpret_cast<__nv_bfloat162*>(&q.y);
        __nv_bfloat162 c = *reinterpret_cast<__nv_bfloat162*>(&q.z), d = *reinterpret_cast<__nv_bfloat162*>(&q.w);
        __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
        return fmaxf(__low2float(m), __high2float(m));
    }
    static __device__ __forceinline__ float at(uint4 q, int j) {
        uint32_t w = (j >> 1) == 0 ? q.x : (j >> 1) == 1 ? q.y : (j >> 1) == 2 ? q.z : q.w;
        return __uint_as_float((j & 1) ? (w & 0xffff0000u) : (w << 16));
    }
};

__device__ __forceinline__ void set_status(const Params& p, uint32_t bits) {
    if (p.status) atomicOr(p.status, bits);
}

// Per-row view of the shared-memory slice and the history hash.
template <typename E>
struct Row {
    unsigned char* slice;  // 16-byte aligned start = floor16(address of element lo)
    uint32_t head;         // byte offset of element lo inside the slice buffer
    int lo, hi;            // element range of this CTA
    uint32_t* ht;          // packed (id - lo) << 14 | count
    float* htv;            // processed value of each hashed id
    uint32_t slots;
    int nvec;              // 16-byte vectors covering [lo, hi)
    float T;
    bool identity;

    __device__ __forceinline__ uint32_t off(int i) const { return head + (uint32_t)(i - lo) * Elem<E>::SZ; }
    __device__ __forceinline__ float raw(int i) const { return Elem<E>::ld(slice, off(i)); }
    __device__ __forceinline__ float f(float x) const { return identity ? x : __fdiv_rn(x, T); }
    // first element index covered by vector v (may be < lo for v = 0)
    __device__ __forceinline__ int vbase(int v) const { return lo + (int)(((int)(v * 16) - (int)head) / Elem<E>::SZ); }
    __device__ __forceinline__ uint32_t hslot(int rel) const { return ((uint32_t)rel * 2654435761u) & (slots - 1); }  // == ht_slot
    // index of the hash slot holding id i, or -1
    __device__ __forceinline__ int find(int i) const {
        if (slots == 0) return -1;
        uint32_t rel = (uint32_t)(i - lo);
        uint32_t h = hslot((int)rel);
        for (uint32_t probe = 0; probe < slots; ++probe) {
            uint32_t w = ht[h];
            if (w == HT_EMPTY) return -1;
            if ((w >> HT_CNT_BITS) == rel) return (int)h;
            h = (h + 1) & (slots - 1);
        }
        return -1;
    }
    // processed value of element i given its raw slice value (history ids carry their own value)
    __device__ __forceinline__ float P(int i, float x) const {
        if (x == f_ninf()) {
            int s = find(i);
            if (s >= 0) return htv[s];
        }
        return f(x);
    }
};

// Open-addressing hash of (id - lo) -> occurrence count, packed as rel << 14 | count in one word.
__device__ __forceinline__ uint32_t ht_slot(uint32_t rel, uint32_t slots) { return (rel * 2654435761u) & (slots - 1); }
__device__ __forceinline__ void ht_insert(uint32_t* ht, uint32_t slots, uint32_t rel) {
    uint32_t hs = ht_slot(rel, slots);
    for (uint32_t probe = 0; probe < slots; ++probe) {
        uint32_t cur = ht[hs];
        if (cur == HT_EMPTY) {
            cur = atomicCAS(&ht[hs], HT_EMPTY, (rel << HT_CNT_BITS) | 1u);
            if (cur == HT_EMPTY) return;
        }
        if ((cur >> HT_CNT_BITS) == rel) {
            atomicAdd(&ht[hs], 1u);
            return;
        }
        hs = (hs + 1) & (slots - 1);
    }
}

__device__ __forceinline__ float pen(float v, int n, const float* alpha) {
    if (n <= 0) return v;
    float a = alpha[n];
    return v < 0.0f ? __fmul_rn(v, a) : __fdiv_rn(v, a);
}

// The whole row program.  Every CTA of a cluster takes the same branches (they depend on row data and
// on values exchanged through distributed shared memory), so the cluster barriers always match.
template <typename E>
__global__ void __launch_bounds__(NT, 2) sample_kernel(const Params p) {
    extern __shared__ __align__(128) unsigned char smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int C = p.C;
    const int crank = (int)cluster.block_rank();
    const int r = (int)(blockIdx.x / C);
    const int tid = threadIdx.x;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + p.off_hist);
    float* cand_v = reinterpret_cast<float*>(smem + p.off_cand);
    int* cand_i = reinterpret_cast<int*>(smem + p.off_candi);
    float* list_v = reinterpret_cast<float*>(smem + p.off_list);
    int* list_i = reinterpret_cast<int*>(smem + p.off_listi);
    float* vals = reinterpret_cast<float*>(smem + p.off_vals);
    const bool leader = crank == 0;
    const int V = p.V;

    // ---------------- row parameters and mode
    const int64_t step = p.steps ? p.steps[r] : 0;
    const bool is_live = (p.active ? p.active[r] != 0 : true) && !(p.finished ? p.finished[r] != 0 : false);
    const bool identity = p.sem == B2S_SEM_IDENTITY;
    const bool hf = p.sem == B2S_SEM_HF;
    const float T = p.rT ? p.rT[r] : p.T;
    const float top_p = p.rP ? p.rP[r] : p.top_p;
    const int top_k = p.rK ? p.rK[r] : p.top_k;
    const bool eos_ok = !identity && p.eos >= 0 && p.eos < V;
    const bool masked_eos = eos_ok && step < p.min_new;
    int mode;
    if (!p.proc && !is_live) mode = MODE_SKIP;
    else if (identity) mode = MODE_FULL;
    else if (step >= p.max_new - 1) mode = MODE_FORCED;
    else if (hf && step <= 0) mode = MODE_FULL;
    else mode = MODE_FILTER;
    int k = 0;
    if (mode == MODE_FILTER) {
        k = min(max(top_k, max(p.min_keep, 1)), V);
        if (k > p.kbuf) {
            mode = MODE_FAIL;
            if (leader && tid == 0) set_status(p, B2S_STATUS_TOPK_LIMIT);
        }
    }
    const int min_keep = p.min_keep;
    const bool topk_only = (p.flags & B2S_FLAG_TOPK_ONLY) != 0;
    const int lo = crank * p.per;
    const int hi = min(V, lo + p.per);

    // state epilogue shared by every mode (leader CTA only)
    // tok_drawn == PAD marks a row that failed on the device: PAD out, state unchanged
    auto finish_row = [&](int64_t tok_drawn) {
        const bool adv = is_live && tok_drawn != PAD;
        const int64_t tok = adv ? tok_drawn : PAD;
        if (tid == 0) {
            if (p.tokens) p.tokens[r] = tok;
            if (p.steps_out) p.steps_out[r] = step + (adv ? 1 : 0);
            if (p.fin_out) {
                bool f0 = p.finished ? p.finished[r] != 0 : false;
                p.fin_out[r] = (uint8_t)(f0 || (adv && tok == (int64_t)p.eos));
            }
        }
        if (p.hist_out && p.W > 0) {
            const int64_t* h = p.hist + (int64_t)r * p.hstride;
            int64_t* ho = p.hist_out + (int64_t)r * p.hostride;
            // read the whole old row before any write: history_out may alias history (W <= 16 * NT)
            int64_t v[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const int j = tid + q * NT;
                if (j < p.W) v[q] = adv ? (j + 1 < p.W ? h[j + 1] : tok) : h[j];
            }
            __syncthreads();
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const int j = tid + q * NT;
                if (j < p.W) ho[j] = v[q];
            }
        }
    };
    auto write_forced = [&]() {
        if (p.proc) {
            float* out = p.proc + (int64_t)r * p.pstride;
            for (int i = lo + tid; i < hi; i += NT) out[i] = (eos_ok && i == p.eos) ? 0.0f : f_ninf();
        }
    };

    if (p.cout_n && mode != MODE_FILTER) {  // a shard row that is not sampled contributes no candidates
        if (leader && tid == 0) p.cout_n[r] = -1;
        return;
    }
    if (mode == MODE_SKIP || mode == MODE_FAIL) {
        if (leader) finish_row(PAD);
        return;
    }
    if (mode == MODE_FORCED) {
        write_forced();
        if (leader) finish_row(eos_ok ? (int64_t)p.eos : (int64_t)(V - 1));
        return;
    }

    // ---------------- stage the slice (bulk copy) and hash the history ids of this slice
    Row<E> R;
    const int ES = Elem<E>::SZ;
    const unsigned char* rowp = reinterpret_cast<const unsigned char*>(p.logits) + (int64_t)r * p.lstride * ES;
    const uintptr_t A = reinterpret_cast<uintptr_t>(rowp) + (uintptr_t)lo * ES;
    const uintptr_t B = reinterpret_cast<uintptr_t>(rowp) + (uintptr_t)hi * ES;
    const uintptr_t Afl = A & ~(uintptr_t)15, Ace = (A + 15) & ~(uintptr_t)15, Bfl = B & ~(uintptr_t)15,
                    Bce = (B + 15) & ~(uintptr_t)15;
    R.slice = smem + p.off_slice;
    R.head = (uint32_t)(A - Afl);
    R.lo = lo;
    R.hi = hi;
    R.nvec = hi > lo ? (int)((Bce - Afl) / 16) : 0;
    R.T = T;
    R.identity = identity;
    const bool use_hist = mode == MODE_FILTER && p.W > 0 && p.hist != nullptr;
    R.ht = reinterpret_cast<uint32_t*>(smem + p.off_ht);
    R.htv = reinterpret_cast<float*>(smem + p.off_htv);
    R.slots = use_hist ? p.ht_slots : 0;
    const bool bulk = hi > lo && Ace < Bfl;
    if (tid == 0) {
        ctl->cand_n = 0;
        ctl->list_n = 0;
        ctl->overflow = 0;
        ctl->err = 0;
        ctl->gather_n = 0;
        ctl->kn = 0;
        mbar_init(&ctl->bar, 1);
        fence_mbar_init();
        if (bulk) {
            const uint32_t bytes = (uint32_t)(Bfl - Ace);
            mbar_arrive_expect_tx(&ctl->bar, bytes);
            const uint32_t chunk = 32768;
            for (uint32_t o = 0; o < bytes; o += chunk)
                bulk_g2s(R.slice + (Ace - Afl) + o, reinterpret_cast<const void*>(Ace + o), min(chunk, bytes - o),
                         &ctl->bar);
        }
    }
    // scalar head / tail elements (or the whole slice when it has no aligned interior)
    if (hi > lo) {
        const int base = lo;
        if (!bulk) {
            for (int i = lo + tid; i < hi; i += NT)
                if (ES == 4) *reinterpret_cast<float*>(R.slice + R.off(i)) = Elem<E>::gld(rowp, i);
                else *reinterpret_cast<uint16_t*>(R.slice + R.off(i)) = __ldg(reinterpret_cast<const unsigned short*>(rowp) + i);
        } else {
            const int nh = (int)((Ace - A) / ES), nt = (int)((B - Bfl) / ES);
            if (tid < nh) {
                const int i = base + tid;
                if (ES == 4) *reinterpret_cast<float*>(R.slice + R.off(i)) = Elem<E>::gld(rowp, i);
                else *reinterpret_cast<uint16_t*>(R.slice + R.off(i)) = __ldg(reinterpret_cast<const unsigned short*>(rowp) + i);
            } else if (tid >= 32 && tid < 32 + nt) {
                const int i = hi - nt + (tid - 32);
                if (ES == 4) *reinterpret_cast<float*>(R.slice + R.off(i)) = Elem<E>::gld(rowp, i);
                else *reinterpret_cast<uint16_t*>(R.slice + R.off(i)) = __ldg(reinterpret_cast<const unsigned short*>(rowp) + i);
            }
        }
    }
    if (use_hist) {
        for (uint32_t s = tid; s < R.slots; s += NT) R.ht[s] = HT_EMPTY;
    }
    __syncthreads();
    if (use_hist) {
        const int64_t* h = p.hist + (int64_t)r * p.hstride;
        for (int j = tid; j < p.W; j += NT) {
            if (h[j] < 0) continue;  // PAD
            const int64_t id = h[j] - p.id_off;
            if (id < 0 || id >= V) {
                // a shard ignores ids of the other shards; an unsharded row flags ids >= vocab
                if (!p.cout_n && crank == 0) set_status(p, B2S_STATUS_HISTORY_RANGE);
                continue;
            }
            if (id < lo || id >= hi) continue;
            ht_insert(R.ht, R.slots, (uint32_t)(id - lo));
        }
    }
    bool ok = true;
    if (bulk) ok = mbar_wait_bounded(&ctl->bar, 0);
    if (!ok) {
        ctl->err = 1;  // benign race: every failing thread writes 1
        set_status(p, B2S_STATUS_WAIT_TIMEOUT);
        mbar_wait_bounded(&ctl->bar, 0);  // give in-flight copies a second bounded chance before reuse
    }
    __syncthreads();

    // ---------------- history ids: exact processed values, then -inf in the slice
    const float* alpha = p.alpha ? p.alpha + (int64_t)r * p.alpha_stride : nullptr;
    if (use_hist) {
        for (uint32_t s = tid; s < R.slots; s += NT) {
            uint32_t w = R.ht[s];
            if (w == HT_EMPTY) continue;
            const int i = lo + (int)(w >> HT_CNT_BITS);
            int n = (int)(w & ((1u << HT_CNT_BITS) - 1));
            if (n >= p.alpha_len) {
                set_status(p, B2S_STATUS_COUNT_LIMIT);
                n = p.alpha_len - 1;
            }
            const float x = R.raw(i);
            float P;
            if (hf) {
                P = pen(__fdiv_rn(x, T), n, alpha);
            } else {
                float z = (masked_eos && i == p.eos) ? f_ninf() : x;
                float v = pen(z, n, alpha);
                if (n > 0) {
                    v = __fsub_rn(v, p.presence);
                    v = __fsub_rn(v, __fmul_rn(p.frequency, (float)n));
                }
                P = __fdiv_rn(v, T);
            }
            R.htv[s] = P;
            Elem<E>::st_ninf(R.slice, R.off(i));
        }
    }
    // omni censors EOS before everything else; hf frame-0 rows drop it from the draw
    if (tid == 0 && masked_eos && p.eos >= lo && p.eos < hi && (!hf || mode == MODE_FULL)) {
        if (R.find(p.eos) < 0) Elem<E>::st_ninf(R.slice, R.off(p.eos));
    }
    __syncthreads();

    // ---------------- per-thread maximum of the raw slice (history slots are -inf now)
    float tmax = f_ninf();
    for (int v = tid; v < R.nvec; v += NT) {
        uint4 q = reinterpret_cast<const uint4*>(R.slice)[v];
        if (v == 0 || v == R.nvec - 1) {
            const int b = R.vbase(v);
#pragma unroll
            for (int j = 0; j < 16 / ES; ++j) {
                const int i = b + j;
                if (i >= lo && i < hi) tmax = fmaxf(tmax, Elem<E>::at(q, j));
            }
        } else {
            tmax = fmaxf(tmax, Elem<E>::vmax(q));
        }
    }

    // ---------------- hf rows with a filter: full-row logsumexp of the penalised values
    float lse = 0.0f;
    if (mode == MODE_FILTER && hf) {
        float hm = f_ninf();
        for (uint32_t s = tid; s < R.slots; s += NT)
            if (R.ht[s] != HT_EMPTY) hm = fmaxf(hm, R.htv[s]);
        float bm = block_max(fmaxf(R.f(tmax), hm), ctl->red_f);
        if (tid == 0) ctl->xmax1 = bm;
        cluster.sync();
        float m = f_ninf();
        for (int c = 0; c < C; ++c) m = fmaxf(m, cluster.map_shared_rank(ctl, c)->xmax1);
        const float mu = (m == f_inf() || m == f_ninf()) ? 0.0f : m;
        double s = 0.0;
        for (int v = tid; v < R.nvec; v += NT) {
            uint4 q = reinterpret_cast<const uint4*>(R.slice)[v];
            const int b = R.vbase(v);
#pragma unroll
            for (int j = 0; j < 16 / ES; ++j) {
                const int i = b + j;
                if (i >= lo && i < hi) s += (double)b2s_expf(__fsub_rn(R.f(Elem<E>::at(q, j)), mu));
            }
        }
        for (uint32_t sl = tid; sl < R.slots; sl += NT)
            if (R.ht[sl] != HT_EMPTY) s += (double)b2s_expf(__fsub_rn(R.htv[sl], mu));
        double bs = block_sum(s, ctl->red_d);
        if (tid == 0) ctl->xsum1 = bs;
        cluster.sync();
        double tot = 0.0;
        for (int c = 0; c < C; ++c) tot += cluster.map_shared_rank(ctl, c)->xsum1;
        lse = __fadd_rn((float)log((double)(float)tot), mu);
    }

    const float u = (p.rng == B2S_RNG_UNIFORM || !p.seeds) ? (p.uvals ? p.uvals[r] : 0.0f)
                    : p.rng == B2S_RNG_PHILOX ? uniform_philox(p.seeds[r], step, p.requests ? p.requests[r] : 0)
                                              : uniform_counter(p.seeds[r], step);
    float thr = f_ninf();
    bool exact = mode == MODE_FILTER;  // exact radix select needed (cleared when the candidate path succeeds)
    int64_t token = V - 1;

    // ---------------- candidate path
    if (mode == MODE_FILTER && k <= KFAST && !(p.flags & B2S_FLAG_FORCE_GENERAL) &&
        (identity || (T >= 1e-6f && T <= 1e6f))) {
        // lower bound on the row's k-th largest non-history raw value
        uint32_t* tkeys = reinterpret_cast<uint32_t*>(cand_v);
        tkeys[tid] = okey(tmax);
        __syncthreads();
        const float t_raw = okey_to_f(block_kth_largest(NT, k, [&](int i) { return tkeys[i]; }, hist, ctl->rctl));
        const bool usable = t_raw != f_ninf() && t_raw == t_raw && R.f(t_raw) != f_inf();
        if (usable) {
            const float t_low = t_raw - fmaxf(fabsf(t_raw) * 9.5367431640625e-7f, 1e-30f);
            const float p_low = R.f(t_low);
            for (int v = tid; v < R.nvec; v += NT) {
                uint4 q = reinterpret_cast<const uint4*>(R.slice)[v];
                if (Elem<E>::vmax(q) < t_low) continue;
                const int b = R.vbase(v);
#pragma unroll
                for (int j = 0; j < 16 / ES; ++j) {
                    const int i = b + j;
                    const float x = Elem<E>::at(q, j);
                    if (i >= lo && i < hi && x >= t_low) {
                        int pos = atomicAdd(&ctl->cand_n, 1);
                        if (pos < p.candcap) { cand_v[pos] = R.f(x); cand_i[pos] = i; }
                    }
                }
            }
            for (uint32_t s = tid; s < R.slots; s += NT) {
                uint32_t w = R.ht[s];
                if (w != HT_EMPTY && R.htv[s] >= p_low) {
                    int pos = atomicAdd(&ctl->cand_n, 1);
                    if (pos < p.candcap) { cand_v[pos] = R.htv[s]; cand_i[pos] = lo + (int)(w >> HT_CNT_BITS); }
                }
            }
        }
        __syncthreads();
        const int nc = ctl->cand_n;
        bool ovf = !usable || nc > p.candcap;
        if (!ovf) {
            uint32_t kth = 0;
            if (nc >= k) kth = block_kth_largest(nc, k, [&](int i) { return okey(cand_v[i]); }, hist, ctl->rctl);
            for (int i = tid; i < nc; i += NT) {
                if (okey(cand_v[i]) >= kth) {
                    int pos = atomicAdd(&ctl->list_n, 1);
                    if (pos < p.lcap) { list_v[pos] = cand_v[i]; list_i[pos] = cand_i[i]; }
                }
            }
            __syncthreads();
            if (ctl->list_n > p.lcap) ovf = true;
        }
        if (tid == 0) ctl->overflow = ovf ? 1 : 0;
        cluster.sync();  // lists published
        bool any_ovf = false, any_err = false;
        for (int c = 0; c < C; ++c) {
            Ctl* rc = cluster.map_shared_rank(ctl, c);
            any_ovf |= rc->overflow != 0;
            any_err |= rc->err != 0;
        }
        int nm = 0;
        if (!any_ovf && leader) {
            // merge every CTA's list into the candidate buffer (no longer needed by this CTA)
            for (int c = 0; c < C; ++c) {
                Ctl* rc = cluster.map_shared_rank(ctl, c);
                const int n = rc->list_n;
                const float* lv = cluster.map_shared_rank(list_v, c);
                const int* li = cluster.map_shared_rank(list_i, c);
                for (int i = tid; i < n; i += NT) { cand_v[nm + i] = lv[i]; cand_i[nm + i] = li[i]; }
                nm += n;
            }
        }
        cluster.sync();  // lists consumed: non-leader shared memory may be reused from here on
        if (!any_ovf) {
            exact = false;
            if (leader) {
                const Scr sc{hist, ctl->rctl, &ctl->gather_n, &ctl->kn, &ctl->thr, ctl->red_d, ctl->red_f, ctl->red_i};
                if (p.cout_n) {
                    // vocabulary shard: hand out every merged item >= this shard's k-th value
                    const uint32_t kthg =
                        block_kth_largest(nm, k, [&](int i) { return okey(cand_v[i]); }, hist, ctl->rctl);
                    if (tid == 0) ctl->kn = 0;
                    __syncthreads();
                    for (int i = tid; i < nm; i += NT) {
                        if (okey(cand_v[i]) >= kthg) {
                            const int pos = atomicAdd(&ctl->kn, 1);
                            if (pos < p.ccap) {
                                p.cout_v[(int64_t)r * p.ccap + pos] = cand_v[i];
                                p.cout_i[(int64_t)r * p.ccap + pos] = (int32_t)(cand_i[i] + p.id_off);
                            }
                        }
                    }
                    __syncthreads();
                    if (tid == 0) p.cout_n[r] = any_err ? -1 : ctl->kn;
                } else {
                    thr = list_threshold(cand_v, nm, k, hf, lse, top_p, min_keep, topk_only, vals, sc);
                    token = list_draw(cand_v, cand_i, nm, thr, masked_eos ? p.eos : -1, u, V, cand_v + p.mcap,
                                      cand_i + p.mcap, list_v, list_i, sc);
                    if (any_err) token = PAD;
                    if (p.proc && tid == 0)
                        for (int c = 1; c < C; ++c) cluster.map_shared_rank(ctl, c)->thr = thr;
                }
            }
            if (p.proc) {
                cluster.sync();  // threshold broadcast
                thr = ctl->thr;
            }
        }
    }

    // ---------------- exact path: cluster-wide radix select of the k-th processed value
    if (exact) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            const uint32_t mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
            const uint32_t prefix = shift == 24 ? 0u : ctl->prefix;
            for (int i = tid; i < 256; i += NT) hist[i] = 0;
            __syncthreads();
            auto count = [&](float P) {
                const uint32_t kk = okey(P);
                if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 255u], 1u);
            };
            for (int v = tid; v < R.nvec; v += NT) {
                uint4 q = reinterpret_cast<const uint4*>(R.slice)[v];
                const int b = R.vbase(v);
#pragma unroll
                for (int j = 0; j < 16 / ES; ++j) {
                    const int i = b + j;
                    if (i < lo || i >= hi) continue;
                    const float x = Elem<E>::at(q, j);
                    if (x == f_ninf() && R.find(i) >= 0) continue;  // history id: counted from the hash
                    count(R.f(x));
                }
            }
            for (uint32_t s = tid; s < R.slots; s += NT)
                if (R.ht[s] != HT_EMPTY) count(R.htv[s]);
            cluster.sync();  // every CTA's histogram is complete
            if (leader && tid < 32) {
                const int krem = shift == 24 ? k : ctl->krem;
                uint32_t c8[8];
                uint32_t s = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t t = 0;
                    for (int c = 0; c < C; ++c) t += cluster.map_shared_rank(hist, c)[255 - 8 * tid - j];
                    c8[j] = t;
                    s += t;
                }
                uint32_t incl = s;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (tid >= o) incl += t;
                }
                const uint32_t excl = incl - s;
                if (excl < (uint32_t)krem && (uint32_t)krem <= incl) {
                    uint32_t cum = excl;
                    for (int j = 0; j < 8; ++j) {
                        if (cum + c8[j] >= (uint32_t)krem) {
                            const uint32_t np = prefix | ((uint32_t)(255 - 8 * tid - j) << shift);
                            for (int c = 0; c < C; ++c) {
                                Ctl* rc = cluster.map_shared_rank(ctl, c);
                                rc->prefix = np;
                                rc->krem = krem - (int)cum;
                            }
                            break;
                        }
                        cum += c8[j];
                    }
                }
            }
            cluster.sync();  // prefix broadcast; histograms may be cleared again
        }
        const uint32_t kth = ctl->prefix;
        if (p.cout_n) {
            // vocabulary shard: every element >= the shard's k-th value, counted in the leader
            int* lkn = &cluster.map_shared_rank(ctl, 0)->kn;
            auto emit = [&](float P, int i) {
                const int pos = atomicAdd(lkn, 1);
                if (pos < p.ccap) {
                    p.cout_v[(int64_t)r * p.ccap + pos] = P;
                    p.cout_i[(int64_t)r * p.ccap + pos] = (int32_t)(i + p.id_off);
                }
            };
            for (int v = tid; v < R.nvec; v += NT) {
                uint4 q = reinterpret_cast<const uint4*>(R.slice)[v];
                const int b = R.vbase(v);
#pragma unroll
                for (int j = 0; j < 16 / ES; ++j) {
                    const int i = b + j;
                    if (i < lo || i >= hi) continue;
                    const float x = Elem<E>::at(q, j);
                    if (x == f_ninf() && R.find(i) >= 0) continue;
                    const float P = R.f(x);
                    if (okey(P) >= kth) emit(P, i);
                }
            }
            for (uint32_t s2 = tid; s2 < R.slots; s2 += NT)
                if (R.ht[s2] != HT_EMPTY && okey(R.htv[s2]) >= kth) emit(R.htv[s2], lo + (int)(R.ht[s2] >> HT_CNT_BITS));
            cluster.sync();  // every CTA has emitted
            if (leader && tid == 0) {
                bool err = false;
                for (int c = 0; c < C; ++c) err |= cluster.map_shared_rank(ctl, c)->err != 0;
                p.cout_n[r] = err ? -1 : ctl->kn;
            }
            cluster.sync();  // the leader has read every CTA's error flag
            return;
        }
        // values above the k-th: gathered into the leader (fewer than k of them)
        float* lvals = cluster.map_shared_rank(vals, 0);
        int* lgn = &cluster.map_shared_rank(ctl, 0)->gather_n;
        for (int v = tid; v < R.nvec; v += NT) {
            uint4 q = reinterpret_cast<const uint4*>(R.slice)[v];
            const int b = R.vbase(v);
#pragma unroll
            for (int j = 0; j < 16 / ES; ++j) {
                const int i = b + j;
                if (i < lo || i >= hi) continue;
                const float x = Elem<E>::at(q, j);
                if (x == f_ninf() && R.find(i) >= 0) continue;
                const float P = R.f(x);
                if (okey(P) > kth) lvals[atomicAdd(lgn, 1)] = P;
            }
        }
        for (uint32_t s = tid; s < R.slots; s += NT)
            if (R.ht[s] != HT_EMPTY && okey(R.htv[s]) > kth) lvals[atomicAdd(lgn, 1)] = R.htv[s];
        cluster.sync();  // gathered
        if (leader) {
            const int ng = ctl->gather_n;
            // bitonic sort of vals[0 .. pow2) descending, padded with -inf
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
            // probabilities of the k values, ordered prefix (contiguous chunk per thread)
            const int per_t = (k + NT - 1) / NT;
            const int i0 = min(k, tid * per_t), i1 = min(k, i0 + per_t);
            const float m = vals[0];
            float sf = 1.0f;
            if (!hf) {
                double es = 0.0;
                for (int i = i0; i < i1; ++i) es += (double)b2s_expf(__fsub_rn(vals[i], m));
                sf = (float)block_sum(es, ctl->red_d);
            }
            auto pk = [&](int i) {
                return hf ? b2s_expf(__fsub_rn(vals[i], lse)) : __fdiv_rn(b2s_expf(__fsub_rn(vals[i], m)), sf);
            };
            double ls = 0.0;
            for (int i = i0; i < i1; ++i) ls += (double)pk(i);
            double total;
            double acc = block_excl_scan(ls, ctl->red_d, &total);
            int cnt = 0;
            for (int i = i0; i < i1; ++i) {
                const float pi = pk(i);
                acc += (double)pi;
                cnt += __fsub_rn((float)acc, pi) < top_p;
            }
            cnt = block_sum_i(cnt, ctl->red_i);
            const int kept = topk_only ? k : max(min(min_keep, k), min(cnt, k));
            const float t = vals[kept - 1];
            if (tid == 0)
                for (int c = 0; c < C; ++c) cluster.map_shared_rank(ctl, c)->thr = t;
        }
        cluster.sync();  // threshold broadcast
        thr = ctl->thr;
    }

    // hf rows with a filter: the censored EOS leaves the kept set only after the filter
    const bool drop_eos_late = mode == MODE_FILTER && hf && masked_eos && p.eos >= lo && p.eos < hi;
    if (drop_eos_late && (exact || p.proc)) {
        if (tid == 0) {
            int s = R.find(p.eos);
            if (s >= 0) R.htv[s] = f_ninf();
            else Elem<E>::st_ninf(R.slice, R.off(p.eos));
        }
        __syncthreads();
    }

    // ---------------- distributed draw over the kept set (exact path and full rows)
    if (mode == MODE_FULL || exact) {
        const bool full = mode == MODE_FULL;
        auto keptP = [&](float P) { return full || P >= thr; };
        // D1: max over the kept set
        float lm = f_ninf();
        for (int v = tid; v < R.nvec; v += NT) {
            uint4 q = reinterpret_cast<const uint4*>(R.slice)[v];
            const int b = R.vbase(v);
#pragma unroll
            for (int j = 0; j < 16 / ES; ++j) {
                const int i = b + j;
                if (i < lo || i >= hi) continue;
                const float P = R.P(i, Elem<E>::at(q, j));
                if (keptP(P)) lm = fmaxf(lm, P);
            }
        }
        float bm = block_max(lm, ctl->red_f);
        if (tid == 0) ctl->xmax2 = bm;
        cluster.sync();
        float m = f_ninf();
        for (int c = 0; c < C; ++c) m = fmaxf(m, cluster.map_shared_rank(ctl, c)->xmax2);
        // contiguous element range per thread (index order for the final scan)
        const int len = hi - lo;
        const int per_t = (len + NT - 1) / NT;
        const int e0 = lo + min(len, tid * per_t), e1 = lo + min(len, tid * per_t + per_t);
        auto ex = [&](int i, float& P) {
            P = R.P(i, R.raw(i));
            return keptP(P) ? b2s_expf(__fsub_rn(P, m)) : 0.0f;
        };
        double es = 0.0;
        for (int i = e0; i < e1; ++i) { float P; es += (double)ex(i, P); }
        double bs = block_sum(es, ctl->red_d);
        if (tid == 0) ctl->xsum2 = bs;
        cluster.sync();
        double stot = 0.0;
        for (int c = 0; c < C; ++c) stot += cluster.map_shared_rank(ctl, c)->xsum2;
        const float sf = (float)stot;
        double qs = 0.0;
        for (int i = e0; i < e1; ++i) { float P; qs += (double)__fdiv_rn(ex(i, P), sf); }
        double qtot;
        double off = block_excl_scan(qs, ctl->red_d, &qtot);
        if (tid == 0) ctl->xq = qtot;
        cluster.sync();
        double before = 0.0, all = 0.0;
        for (int c = 0; c < C; ++c) {
            const double qc = cluster.map_shared_rank(ctl, c)->xq;
            if (c < crank) before += qc;
            all += qc;
        }
        const float target = __fmul_rn(u, (float)all);
        double acc = before + off;
        int first = 0x7fffffff;
        for (int i = e0; i < e1; ++i) {
            float P;
            const float pi = __fdiv_rn(ex(i, P), sf);
            if (pi == 0.0f) continue;
            acc += (double)pi;
            if ((float)acc > target) { first = i; break; }
        }
        int fm = first;
#pragma unroll
        for (int o = 16; o; o >>= 1) fm = min(fm, __shfl_xor_sync(0xffffffffu, fm, o));
        __syncthreads();
        if ((tid & 31) == 0) ctl->red_i[tid >> 5] = fm;
        __syncthreads();
        int best = 0x7fffffff;
        for (int w = 0; w < NWARP; ++w) best = min(best, ctl->red_i[w]);
        if (tid == 0) { ctl->xfirst = best; }
        cluster.sync();
        if (leader) {
            int tokc = 0x7fffffff;
            bool err = false;
            for (int c = 0; c < C; ++c) {
                Ctl* rc = cluster.map_shared_rank(ctl, c);
                tokc = min(tokc, rc->xfirst);
                err |= rc->err != 0;
            }
            token = tokc == 0x7fffffff ? (int64_t)(V - 1) : (int64_t)tokc;
            if (err) token = PAD;
        }
        cluster.sync();  // the leader has read every CTA's exchange slots
    }

    // ---------------- processed row
    if (p.proc) {
        float* out = p.proc + (int64_t)r * p.pstride;
        const bool full = mode == MODE_FULL;
        for (int i = lo + tid; i < hi; i += NT) {
            const float P = R.P(i, R.raw(i));
            out[i] = (full || P >= thr) ? P : f_ninf();
        }
    }
    if (leader) finish_row(token);
}

// ---------------------------------------------------------------- greedy argmax

// Cluster of C CTAs per row; each CTA streams its slice with 16-byte loads and keeps (value, index)
// per thread (first index wins; NaN beats every number), then the leader merges over DSMEM.
template <typename E>
__global__ void __launch_bounds__(NT, 2) argmax_kernel(const void* logits, int V, int64_t stride, int per,
                                                       int64_t* tokens) {
    cg::cluster_group cluster = cg::this_cluster();
    const int C = (int)cluster.num_blocks();
    const int crank = (int)cluster.block_rank();
    const int r = (int)(blockIdx.x / C);
    const int tid = threadIdx.x;
    __shared__ float sv[NWARP];
    __shared__ int si[NWARP];
    __shared__ float cv;
    __shared__ int ci;
    const int ES = Elem<E>::SZ;
    const int lo = crank * per, hi = min(V, lo + per);
    const unsigned char* rowp = reinterpret_cast<const unsigned char*>(logits) + (int64_t)r * stride * ES;
    float bv = f_ninf();
    int bi = 0x7fffffff;
    auto upd = [&](float x, int i) {
        // larger value wins; NaN wins over numbers; equal values keep the lower index
        const bool xn = x != x, bn = bv != bv;
        if (bn) { if (xn && i < bi) bi = i; return; }
        if (xn || x > bv || (x == bv && i < bi)) { bv = x; bi = i; }
    };
    const uintptr_t A = reinterpret_cast<uintptr_t>(rowp) + (uintptr_t)lo * ES;
    const uintptr_t B = reinterpret_cast<uintptr_t>(rowp) + (uintptr_t)hi * ES;
    const uintptr_t Ace = (A + 15) & ~(uintptr_t)15, Bfl = B & ~(uintptr_t)15;
    if (hi > lo) {
        if (Ace < Bfl) {
            const int nh = (int)((Ace - A) / ES), nt = (int)((B - Bfl) / ES);
            if (tid < nh) upd(Elem<E>::gld(rowp, lo + tid), lo + tid);
            if (tid >= 32 && tid < 32 + nt) upd(Elem<E>::gld(rowp, hi - nt + tid - 32), hi - nt + tid - 32);
            const uint4* vp = reinterpret_cast<const uint4*>(Ace);
            const int nv = (int)((Bfl - Ace) / 16);
            const int i0 = lo + nh;
            for (int v = tid; v < nv; v += NT) {
                uint4 q;
                asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(q.x), "=r"(q.y), "=r"(q.z), "=r"(q.w)
                             : "l"(vp + v));
#pragma unroll
                for (int j = 0; j < 16 / ES; ++j) upd(Elem<E>::at(q, j), i0 + v * (16 / ES) + j);
            }
        } else {
            for (int i = lo + tid; i < hi; i += NT) upd(Elem<E>::gld(rowp, i), i);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi != 0x7fffffff) upd(ov, oi);
    }
    if ((tid & 31) == 0) { sv[tid >> 5] = bv; si[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < NWARP; ++w)
            if (si[w] != 0x7fffffff) upd(sv[w], si[w]);
        cv = bv;
        ci = bi;
    }
    cluster.sync();
    if (crank == 0 && tid == 0) {
        for (int c = 1; c < C; ++c) {
            const int oi = *cluster.map_shared_rank(&ci, c);
            if (oi != 0x7fffffff) upd(*cluster.map_shared_rank(&cv, c), oi);
        }
        tokens[r] = bi == 0x7fffffff ? 0 : bi;
    }
    cluster.sync();
}

// ---------------------------------------------------------------- standalone repetition penalty

// grid (chunks, rows): copy the chunk to fp32, then overwrite the history ids of the chunk with their
// penalised value (the same CTA, after a barrier, so the overwrite wins).
template <typename E>
__global__ void __launch_bounds__(NT) penalty_kernel(const void* x, int V, int64_t xstride, const int64_t* hist, int W,
                                                     int64_t hstride, const float* alpha, int alpha_len,
                                                     int alpha_stride, float* out, int64_t ostride, int chunk,
                                                     uint32_t slots, uint32_t* status) {
    extern __shared__ __align__(16) uint32_t ht[];
    const int r = blockIdx.y, tid = threadIdx.x;
    const int lo = blockIdx.x * chunk, hi = min(V, lo + chunk);
    const unsigned char* rowp = reinterpret_cast<const unsigned char*>(x) + (int64_t)r * xstride * Elem<E>::SZ;
    float* orow = out + (int64_t)r * ostride;
    for (int i = lo + tid; i < hi; i += NT) orow[i] = Elem<E>::gld(rowp, i);
    for (uint32_t s = tid; s < slots; s += NT) ht[s] = HT_EMPTY;
    __syncthreads();
    const int64_t* h = hist + (int64_t)r * hstride;
    for (int j = tid; j < W; j += NT) {
        const int64_t id = h[j];
        if (id < 0) continue;
        if (id >= V) {
            if (blockIdx.x == 0 && status) atomicOr(status, B2S_STATUS_HISTORY_RANGE);
            continue;
        }
        if (id >= lo && id < hi) ht_insert(ht, slots, (uint32_t)(id - lo));
    }
    __syncthreads();
    const float* al = alpha + (int64_t)r * alpha_stride;
    for (uint32_t s = tid; s < slots; s += NT) {
        const uint32_t w = ht[s];
        if (w == HT_EMPTY) continue;
        const int i = lo + (int)(w >> HT_CNT_BITS);
        int n = (int)(w & ((1u << HT_CNT_BITS) - 1));
        if (n >= alpha_len) {
            if (status) atomicOr(status, B2S_STATUS_COUNT_LIMIT);
            n = alpha_len - 1;
        }
        orow[i] = pen(Elem<E>::gld(rowp, i), n, al);
    }
}

__global__ void uniform_kernel(const int64_t* seeds, const int64_t* steps, const int64_t* req, int64_t n, int rng,
                               float* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = rng == B2S_RNG_PHILOX ? uniform_philox(seeds[i], steps[i], req ? req[i] : 0)
                                       : uniform_counter(seeds[i], steps[i]);
}

}  // namespace b2s

// ================================================================ host side (C-ABI)

namespace {

thread_local char g_cuda_err[256] = "";

int cuda_fail(cudaError_t e) {
    snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
    return B2S_ERR_CUDA;
}

uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }
int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Cluster size: enough CTAs per row that each slice stays within ~80 KB (two CTAs per SM), and for
// small batches enough CTAs to spread the rows over the SMs.
int choose_cluster(int rows, int64_t row_bytes, int requested) {
    if (requested) return requested;
    int C = 1;
    while (C < 8 && row_bytes / C > 80 * 1024) C <<= 1;
    while (C < 8 && (int64_t)rows * C * 2 <= sm_count() && row_bytes / (C * 2) >= 8 * 1024) C <<= 1;
    return C;
}

template <typename K>
cudaError_t set_smem_attr(K kernel, uint32_t bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

extern "C" {

const char* b2s_error_string(int code) {
    switch (code) {
        case B2S_OK: return "ok";
        case B2S_ERR_INVALID: return "invalid argument";
        case B2S_ERR_UNSUPPORTED: return "unsupported shape";
        case B2S_ERR_CUDA: return "CUDA error";
        default: return "unknown error";
    }
}

const char* b2s_last_cuda_error(void) { return g_cuda_err; }

int b2s_abi_version(void) { return B2S_ABI_VERSION; }

struct ShardOut {
    float* v;
    int32_t* i;
    int32_t* n;
    int cap;
    int64_t offset;
};

static int launch_sample(const b2s_sample_args* a, void* stream, const ShardOut* so) {
    using namespace b2s;
    if (!a || !a->logits || a->rows < 0 || a->vocab <= 0) return B2S_ERR_INVALID;
    if (a->rows == 0) return B2S_OK;
    if (a->logits_dtype != B2S_DTYPE_F32 && a->logits_dtype != B2S_DTYPE_BF16) return B2S_ERR_INVALID;
    if (a->semantics < B2S_SEM_HF || a->semantics > B2S_SEM_IDENTITY) return B2S_ERR_INVALID;
    if (a->rng < B2S_RNG_UNIFORM || a->rng > B2S_RNG_PHILOX) return B2S_ERR_INVALID;
    if (a->logits_row_stride < a->vocab) return B2S_ERR_INVALID;
    const bool identity = a->semantics == B2S_SEM_IDENTITY;
    if (!identity) {
        if (!a->steps) return B2S_ERR_INVALID;
        if (!a->row_temperature && !(a->temperature > 0.0f)) return B2S_ERR_INVALID;
        if (a->window < 0 || (a->window > 0 && !a->history)) return B2S_ERR_INVALID;
        if (a->window > 0 && a->history_row_stride < a->window) return B2S_ERR_INVALID;
        if (a->window > (1 << 13)) return B2S_ERR_UNSUPPORTED;
        if (a->window > 0 && (!a->alpha || a->alpha_len < 1)) return B2S_ERR_INVALID;
        if (!a->row_top_k && a->top_k < 0) return B2S_ERR_INVALID;
    }
    // a uniform source is needed only when the call draws tokens
    const bool draws = a->tokens || a->history_out || a->steps_out || a->finished_out;
    if (draws && a->rng == B2S_RNG_UNIFORM && !a->uniform_values) return B2S_ERR_INVALID;
    if (draws && a->rng != B2S_RNG_UNIFORM && !a->seeds) return B2S_ERR_INVALID;
    if (a->history_out && (a->window <= 0 ? false : a->history_out_row_stride < a->window)) return B2S_ERR_INVALID;
    if (a->processed && a->processed_row_stride < a->vocab) return B2S_ERR_INVALID;
    const int es = a->logits_dtype == B2S_DTYPE_BF16 ? 2 : 4;
    int C = choose_cluster(a->rows, (int64_t)a->vocab * es, a->cluster);
    if (C != 1 && C != 2 && C != 4 && C != 8) return B2S_ERR_INVALID;
    int per = (a->vocab + C - 1) / C;
    per = (per + 15) / 16 * 16;
    while (C > 1 && (int64_t)per * (C - 1) >= a->vocab) {  // every CTA must own at least one element
        C >>= 1;
        per = ((a->vocab + C - 1) / C + 15) / 16 * 16;
    }
    if (per >= (1 << 18)) return B2S_ERR_UNSUPPORTED;

    Params p;
    memset(&p, 0, sizeof(p));
    p.logits = a->logits;
    p.lstride = a->logits_row_stride;
    p.rows = a->rows;
    p.V = a->vocab;
    p.W = identity ? 0 : a->window;
    p.eos = a->eos;
    p.hist = a->history;
    p.hstride = a->history_row_stride;
    p.steps = a->steps;
    p.seeds = a->seeds;
    p.requests = a->requests;
    p.uvals = a->uniform_values;
    p.active = a->active;
    p.finished = a->finished;
    p.T = a->temperature;
    p.top_p = a->top_p;
    p.presence = a->presence_penalty;
    p.frequency = a->frequency_penalty;
    p.top_k = a->top_k;
    p.min_keep = a->min_keep;
    p.min_new = a->min_new_tokens;
    p.max_new = a->max_new_tokens;
    p.rT = a->row_temperature;
    p.rP = a->row_top_p;
    p.rK = a->row_top_k;
    p.alpha = a->alpha;
    p.alpha_len = a->alpha_len;
    p.alpha_stride = a->alpha_row_stride;
    p.sem = a->semantics;
    p.rng = a->rng;
    p.flags = a->flags;
    p.tokens = a->tokens;
    p.proc = a->processed;
    p.pstride = a->processed_row_stride;
    p.hist_out = a->history_out;
    p.hostride = a->history_out_row_stride;
    p.steps_out = a->steps_out;
    p.fin_out = a->finished_out;
    p.status = a->status;
    if (so) {
        p.cout_v = so->v;
        p.cout_i = so->i;
        p.cout_n = so->n;
        p.ccap = so->cap;
        p.id_off = so->offset;
    }
    p.C = C;
    p.per = per;
    int kmax = a->max_top_k > 0 ? a->max_top_k : a->top_k;
    kmax = identity ? 1 : kmax;
    kmax = kmax < a->min_keep ? a->min_keep : kmax;
    kmax = kmax > a->vocab ? a->vocab : kmax;
    kmax = kmax < 1 ? 1 : kmax;
    const int kfast = kmax < KFAST ? kmax : KFAST;
    p.lcap = next_pow2(2 * kfast + 32);
    if (p.lcap > 512) p.lcap = 512;
    p.mcap = C * p.lcap;
    p.candcap = CAP > 2 * p.mcap ? CAP : 2 * p.mcap;
    if (p.candcap < NT) p.candcap = NT;
    // vals: [0, KFAST) sorted top-k of the candidate path, [KFAST, 2*KFAST) its gather area; the exact path
    // sorts up to next_pow2(kmax) values from offset 0
    p.kbuf = kmax;
    const int nvals = next_pow2(kmax) > 2 * KFAST ? next_pow2(kmax) : 2 * KFAST;
    const int hist_ids = a->window < per ? a->window : per;
    p.ht_slots = identity || a->window <= 0 ? 0u : (uint32_t)next_pow2(2 * hist_ids > 32 ? 2 * hist_ids : 32);
    uint32_t off = 0;
    p.off_ctl = off;
    off = align_up(off + (uint32_t)sizeof(Ctl), 128);
    p.off_slice = off;
    off = align_up(off + (uint32_t)per * es + 32, 128);
    p.off_ht = off;
    off = align_up(off + p.ht_slots * 4, 16);
    p.off_htv = off;
    off = align_up(off + p.ht_slots * 4, 16);
    p.off_cand = off;
    off = align_up(off + (uint32_t)p.candcap * 4, 16);
    p.off_candi = off;
    off = align_up(off + (uint32_t)p.candcap * 4, 16);
    p.off_list = off;
    off = align_up(off + (uint32_t)(p.lcap > p.mcap ? p.lcap : p.mcap) * 4, 16);
    p.off_listi = off;
    off = align_up(off + (uint32_t)(p.lcap > p.mcap ? p.lcap : p.mcap) * 4, 16);
    p.off_vals = off;
    off = align_up(off + (uint32_t)nvals * 4, 16);
    p.off_hist = off;
    off = align_up(off + 256 * 4, 16);
    p.smem_total = off;
    if (p.smem_total > 227 * 1024) return B2S_ERR_UNSUPPORTED;

    cudaError_t e;
    void (*kern)(const Params) = a->logits_dtype == B2S_DTYPE_BF16 ? sample_kernel<__nv_bfloat16> : sample_kernel<float>;
    {
        // the attribute is per device: remember which (device, dtype) pairs have it
        static std::mutex mu;
        static uint64_t done[2] = {0, 0};
        int dev = 0;
        e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return cuda_fail(e);
        std::lock_guard<std::mutex> g(mu);
        const int ti = a->logits_dtype == B2S_DTYPE_BF16 ? 1 : 0;
        const uint64_t bit = 1ull << (dev & 63);
        if (!(done[ti] & bit)) {
            e = set_smem_attr(kern, 227 * 1024);
            if (e != cudaSuccess) return cuda_fail(e);
            done[ti] |= bit;
        }
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)(a->rows * C), 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = p.smem_total;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}

int b2s_sample(const b2s_sample_args* a, void* stream) { return launch_sample(a, stream, nullptr); }

int b2s_shard_candidates(const b2s_sample_args* a, int64_t vocab_offset, int32_t cap, float* cand_values,
                         int32_t* cand_ids, int32_t* cand_count, void* stream) {
    if (!a || !cand_values || !cand_ids || !cand_count || cap < 1 || vocab_offset < 0) return B2S_ERR_INVALID;
    if (a->semantics != B2S_SEM_OMNI) return B2S_ERR_UNSUPPORTED;  // hf needs the full-row normaliser
    if (a->processed || a->history_out || a->steps_out || a->finished_out) return B2S_ERR_INVALID;
    if (vocab_offset + a->vocab > (int64_t)INT32_MAX) return B2S_ERR_UNSUPPORTED;
    b2s_sample_args b = *a;
    b.tokens = nullptr;
    b.rng = B2S_RNG_UNIFORM;  // no draw in this stage
    b.uniform_values = nullptr;
    b.eos = (a->eos >= vocab_offset && a->eos < vocab_offset + a->vocab) ? (int32_t)(a->eos - vocab_offset) : -1;
    ShardOut so{cand_values, cand_ids, cand_count, cap, vocab_offset};
    return launch_sample(&b, stream, &so);
}

int b2s_argmax(const void* logits, int32_t dtype, int32_t rows, int32_t vocab, int64_t row_stride, int64_t* tokens,
               void* stream) {
    using namespace b2s;
    if (!logits || !tokens || rows < 0 || vocab <= 0 || row_stride < vocab) return B2S_ERR_INVALID;
    if (dtype != B2S_DTYPE_F32 && dtype != B2S_DTYPE_BF16) return B2S_ERR_INVALID;
    if (rows == 0) return B2S_OK;
    const int es = dtype == B2S_DTYPE_BF16 ? 2 : 4;
    int C = 1;
    const int64_t row_bytes = (int64_t)vocab * es;
    while (C < 8 && (int64_t)rows * C < 2 * sm_count() && row_bytes / (C * 2) >= 16 * 1024) C <<= 1;
    int per = ((vocab + C - 1) / C + 15) / 16 * 16;
    while (C > 1 && (int64_t)per * (C - 1) >= vocab) {
        C >>= 1;
        per = ((vocab + C - 1) / C + 15) / 16 * 16;
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)(rows * C), 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = dtype == B2S_DTYPE_BF16
                        ? cudaLaunchKernelEx(&cfg, argmax_kernel<__nv_bfloat16>, logits, (int)vocab, row_stride, per, tokens)
                        : cudaLaunchKernelEx(&cfg, argmax_kernel<float>, logits, (int)vocab, row_stride, per, tokens);
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}

int b2s_repetition_penalty(const void* x, int32_t x_dtype, int32_t rows, int32_t vocab, int64_t x_row_stride,
                           const int64_t* history, int32_t window, int64_t history_row_stride, const float* alpha,
                           int32_t alpha_len, int32_t alpha_row_stride, float* out, int64_t out_row_stride,
                           uint32_t* status, void* stream) {
    using namespace b2s;
    if (!x || !out || rows < 0 || vocab <= 0 || x_row_stride < vocab || out_row_stride < vocab) return B2S_ERR_INVALID;
    if (x_dtype != B2S_DTYPE_F32 && x_dtype != B2S_DTYPE_BF16) return B2S_ERR_INVALID;
    if (window < 0 || (window > 0 && (!history || history_row_stride < window || !alpha || alpha_len < 1)))
        return B2S_ERR_INVALID;
    if (window > (1 << 13)) return B2S_ERR_UNSUPPORTED;
    if (rows == 0) return B2S_OK;
    const int chunk = 16384;
    const int ids = window < chunk ? window : chunk;
    const uint32_t slots = (uint32_t)next_pow2(2 * ids > 32 ? 2 * ids : 32);
    dim3 grid((unsigned)((vocab + chunk - 1) / chunk), (unsigned)rows);
    const size_t smem = slots * 4;
    cudaStream_t st = (cudaStream_t)stream;
    if (x_dtype == B2S_DTYPE_BF16)
        penalty_kernel<__nv_bfloat16><<<grid, NT, smem, st>>>(x, vocab, x_row_stride, history, window,
                                                              history_row_stride, alpha, alpha_len, alpha_row_stride,
                                                              out, out_row_stride, chunk, slots, status);
    else
        penalty_kernel<float><<<grid, NT, smem, st>>>(x, vocab, x_row_stride, history, window, history_row_stride,
                                                      alpha, alpha_len, alpha_row_stride, out, out_row_stride, chunk,
                                                      slots, status);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}

int b2s_uniform(const int64_t* seeds, const int64_t* steps, const int64_t* requests, int64_t n, int32_t rng, float* out,
                void* stream) {
    if (n < 0 || (n > 0 && (!seeds || !steps || !out))) return B2S_ERR_INVALID;
    if (rng != B2S_RNG_COUNTER && rng != B2S_RNG_PHILOX) return B2S_ERR_INVALID;
    if (n == 0) return B2S_OK;
    const int threads = 256;
    int64_t blocks = (n + threads - 1) / threads;
    if (blocks > 4 * 148) blocks = 4 * 148;
    b2s::uniform_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(seeds, steps, requests, n, rng, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}

}  // extern "C"
