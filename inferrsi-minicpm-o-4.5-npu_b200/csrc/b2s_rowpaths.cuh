// Row paths shared by the two one-launch-per-step kernels (the row-resident kernel of b2s_resident.cu and the
// short-row kernel of b2s_short.cu): the exact full-row path and the hf frame-0 draw (both read the row from
// global memory), the shared-memory history structures those paths read, and the list stage over a candidate
// list.  The full-row paths are kept out of line: decode steps rarely take them, and the instructions a step
// executes stay few and contiguous.
#pragma once

#include "b2s_row.cuh"

namespace b2s {

// The exact full-row path (rank 0, the row read from global memory): radix select of the k-th processed key,
// the top-p threshold over the sorted top-k values, the ordered draw over the elements >= it.
template <typename E>
static __device__ __noinline__ int64_t exact_token(const Row<E> R, int k, bool hf, float lse, float top_p, int min_keep,
                                            bool topk_only, int drop, float u, uint32_t* hist, float* vals, Ctl* ctl) {
    const uint32_t kth = row_kth_key<E>(R, k, hist, ctl);
    const float thr = exact_threshold<E>(R, kth, k, hf, lse, top_p, min_keep, topk_only, vals, ctl);
    return ordered_draw<E>(R, [&](int i, float P) { return i != drop && P >= thr; }, u, ctl);
}

// hf frame 0: the draw over the whole row (talker_sampler.py:155), the masked EOS left out.
template <typename E>
static __device__ __noinline__ int64_t full_token(const Row<E> R, int drop, float u, Ctl* ctl) {
    return ordered_draw<E>(R, [&](int i, float) { return i != drop; }, u, ctl);
}

// Shared-memory structures of the row's penalty history.
struct HistBufs {
    uint32_t* bits;
    uint16_t* pref;
    uint32_t* hcnt;
    int* hid;
    int* hpos;
    float* htv;
    const int64_t* hstage;
    const float* atab;
};

// Ranks and counts of the distinct history ids this CTA owns (their bits set and visible, hcnt zeroed): the rank
// of an id is the exclusive prefix of the popcounts of the bitmap's 4-word groups; one count, id and position per
// rank.  Every thread calls it; returns the number of distinct owned ids (the censored EOS included).
template <typename E, typename Owns>
__device__ __forceinline__ int hist_rank_count(const Params& p, const Row<E>& R, const HistBufs& h, bool pen_hist,
                                               bool censor, Owns owns, Ctl* ctl) {
    const int tid = threadIdx.x;
    const int G = (int)p.bitwords >> 2;
    const int gpt = (G + NT - 1) / NT;
    const int g0 = min(G, tid * gpt), g1 = min(G, g0 + gpt);
    const uint4* b4 = reinterpret_cast<const uint4*>(h.bits);
    int cnt = 0;
    for (int g = g0; g < g1; ++g) {
        const uint4 q = b4[g];
        cnt += __popc(q.x) + __popc(q.y) + __popc(q.z) + __popc(q.w);
    }
    int hd = 0;
    int base = block_excl_scan_i(cnt, ctl->red_i, &hd);
    for (int g = g0; g < g1; ++g) {
        h.pref[g] = (uint16_t)base;
        const uint4 q = b4[g];
        base += __popc(q.x) + __popc(q.y) + __popc(q.z) + __popc(q.w);
    }
    __syncthreads();
    if (pen_hist)
        for (int j = tid; j < p.W; j += NT) {
            const int64_t hv = h.hstage[j];
            if (hv < 0 || hv >= p.V || !owns((int)hv)) continue;
            const int rk = R.rank((int)hv);
            atomicAdd(&h.hcnt[rk], 1u);
            h.hid[rk] = (int)hv;
            h.hpos[rk] = j;
        }
    if (censor && tid == 0 && owns(p.eos)) h.hid[R.rank(p.eos)] = p.eos;
    return hd;
}

// Processed values of the hd distinct history ids (counts complete and visible); raw(id) gives an id's raw value.
template <typename E, typename Raw>
__device__ __forceinline__ void hist_values(const Params& p, const Row<E>& R, const HistBufs& h, int hd, bool hf,
                                            bool pen_hist, bool censor, float T, Raw raw) {
    const int tid = threadIdx.x;
    if (pen_hist) {
        for (int d = tid; d < hd; d += NT) {
            const int id = h.hid[d];
            h.htv[d] = (censor && id == p.eos) ? f_ninf() : hist_proc_value(p, h.atab, hf, false, T, (int)h.hcnt[d], raw(id));
        }
    } else if (censor && tid == 0) {
        for (int d = 0; d < hd; ++d) h.htv[d] = f_ninf();  // the censored EOS alone
    }
}

// The whole-row history structures for a full-row path, built from the staged history (raw values from global
// memory): rank 0 of a multi-CTA row, whose CTAs marked and valued only the history ids of their own slices, and
// the short-row kernel, which keeps per-element occurrence counts instead.
template <typename E>
static __device__ __noinline__ void hist_rebuild(const Params p, const Row<E> R, HistBufs h, bool hf, bool pen_hist,
                                                 bool censor, float T, Ctl* ctl) {
    const int tid = threadIdx.x;
    for (uint32_t g = tid; g < p.bitwords / 4; g += NT) reinterpret_cast<uint4*>(h.bits)[g] = make_uint4(0u, 0u, 0u, 0u);
    for (int d = tid; d < p.hcap; d += NT) h.hcnt[d] = 0u;
    __syncthreads();
    if (pen_hist)
        for (int j = tid; j < p.W; j += NT) {
            const int64_t hv = h.hstage[j];
            if (hv >= 0 && hv < p.V) atomicOr(&h.bits[hv >> 5], 1u << (hv & 31));
        }
    if (censor && tid == 0) atomicOr(&h.bits[p.eos >> 5], 1u << (p.eos & 31));
    __syncthreads();
    const int hd = hist_rank_count<E>(p, R, h, pen_hist, censor, [](int) { return true; }, ctl);
    __syncthreads();
    hist_values<E>(p, R, h, hd, hf, pen_hist, censor, T, [&](int id) { return R.raw(id); });
    __syncthreads();
}

// The list stage in the CTA that draws: narrowing to the items >= the k-th largest value when the list is long,
// then list_sample (b2s_list.cuh).
__device__ __forceinline__ int64_t block_list_token(float* cv, int* ci, float* xv, int* xi, float* sv, int* si,
                                                        int n, int k, bool hf, float lse, float top_p, int min_keep,
                                                        bool topk_only, int drop, float u, int V, float* vals,
                                                        uint32_t* hist, Ctl* ctl) {
    const int tid = threadIdx.x;
    if (n > 256) {
        const uint32_t kk = kth_key_bucket(n, k, [&](int i) { return okey(cv[i]); }, hist, ctl);
        if (tid == 0) ctl->kn = 0;
        __syncthreads();
        for (int i = tid; i < n; i += NT)
            if (okey(cv[i]) >= kk) {
                const int pos = atomicAdd(&ctl->kn, 1);
                xv[pos] = cv[i];
                xi[pos] = ci[i];
            }
        __syncthreads();
        n = ctl->kn;
        float* tv = cv;
        int* ti = ci;
        cv = xv;
        ci = xi;
        xv = tv;
        xi = ti;
    }
    const Scr sc{hist, ctl->rctl, &ctl->gather_n, &ctl->kn, &ctl->thr, ctl->red_d, ctl->red_f, ctl->red_i};
    float thr;
    return list_sample(cv, ci, n, k, hf, lse, top_p, min_keep, topk_only, true, drop, u, V, vals, xv, xi, sv, si, sc,
                       thr);
}

}  // namespace b2s
