// Vocabulary-sharded Thinker head, stages 2 and 3 (no counterpart in the reference, which runs on one device).
//
// Stage 1 (b2s_shard_candidates, the sampling kernel) leaves, per shard and row, every processed element above the
// shard's k-th value (fewer than k) and then elements equal to it while `cap` >= k allows, plus the count of every
// element >= the shard's k-th value.  The lists are all-gathered.  The elements a shard did not send are ties at its
// k-th value, which is never above the row's k-th value; they are known by value and count alone.
//
// Stage 2 (merge, on every rank, identical results): the row's top-k values (the sent values plus the unsent ties'
// copies), the top-p cut and value threshold thr; the kept set is every element >= thr.  Its softmax normaliser and
// each shard's kept mass follow from the sent elements and the tie counts, so the shard holding the draw (the first
// element, in vocabulary order, whose cumulative mass exceeds u * total) is known on every rank.  When every kept
// element of that shard was sent, the token is found among them; otherwise the row is left to that shard's rank.
//
// Stage 3 (resolve, on every rank): the rank of the pending shard scans its shard row in vocabulary order from the
// mass before it and finds the token; every other rank contributes -1, and resolved rows carry the merged token,
// so one max-all-reduce of [rows] int64 publishes the same tokens everywhere.  They equal the unsharded kernel's.
#include <stdio.h>
#include <string.h>

#include "../../include/b2s_sampler.h"
#include "b2s_device.cuh"
#include "b2s_list.cuh"
#include "b2s_row.cuh"

namespace b2s {

int cuda_fail(cudaError_t e);  // b2s_sampler.cu

constexpr int MAXSH = 64;  // shards

struct MergeParams {
    const float* cv;
    const int32_t* ci;
    const int32_t* cn;
    int shards, rows, cap, V;
    int top_k, min_keep;
    float top_p;
    const int32_t* rK;
    const float* rP;
    int rng, flags;
    const int64_t* seeds;
    const int64_t* steps;
    const int64_t* requests;
    const float* uvals;
    int64_t* tokens;
    b2s_shard_pending* pending;
    uint32_t* status;
    int nmax;  // shards * cap + shards * KLIST
};

struct MergeCtl {
    uint32_t rctl[2];
    int gather_n, kn, n, ntot, bad;
    float thr;
    double red_d[NWARP + 1];
    float red_f[NWARP + 1];
    int red_i[NWARP + 1];
    int offs[MAXSH + 1];   // listed items of shard s: [offs[s], offs[s + 1])
    int miss[MAXSH];       // unsent ties of shard s (value tval[s])
    float tval[MAXSH];
    double mass[MAXSH];    // kept mass of shard s
    int kcnt[MAXSH];       // kept listed items of shard s (sorted by id at the start of its region in sv / si)
    int star;
    double base;
    float target, sf, pt;
};

__global__ void __launch_bounds__(NT, 1) shard_merge_kernel(const MergeParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    MergeCtl* ctl = reinterpret_cast<MergeCtl*>(smem);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + ((sizeof(MergeCtl) + 15) / 16 * 16));
    float* vals = reinterpret_cast<float*>(hist + 256);
    float* cv = vals + 2 * KLIST;
    int* ci = reinterpret_cast<int*>(cv + p.nmax);
    float* sv = reinterpret_cast<float*>(ci + p.nmax);
    int* si = reinterpret_cast<int*>(sv + p.nmax);
    const int top_k = p.rK ? p.rK[r] : p.top_k;
    const int k = min(max(top_k, max(p.min_keep, 1)), p.V);
    if (tid == 0) {
        int off = 0, bad = 0;
        for (int s = 0; s < p.shards; ++s) {
            const int c = p.cn[(int64_t)s * p.rows + r];
            ctl->offs[s] = off;
            if (c < 0) bad = 1;
            const int nl = max(0, min(c, p.cap));
            ctl->miss[s] = max(0, c - p.cap);
            off += nl;
        }
        ctl->offs[p.shards] = off;
        ctl->n = off;
        ctl->bad = bad;
    }
    __syncthreads();
    const int n = ctl->n;
    b2s_shard_pending rec;
    memset(&rec, 0, sizeof(rec));
    rec.shard = -1;
    if (ctl->bad || n < 1 || k > KLIST) {
        if (tid == 0) {
            p.tokens[r] = -1;
            if (p.pending) p.pending[r] = rec;
            if (p.status) atomicOr(p.status, k > KLIST ? B2S_STATUS_TOPK_LIMIT : B2S_STATUS_SHARD_INCOMPLETE);
        }
        return;
    }
    for (int s = 0; s < p.shards; ++s) {
        const int o = ctl->offs[s], c = ctl->offs[s + 1] - o;
        const float* src_v = p.cv + ((int64_t)s * p.rows + r) * p.cap;
        const int32_t* src_i = p.ci + ((int64_t)s * p.rows + r) * p.cap;
        for (int i = tid; i < c; i += NT) {
            cv[o + i] = src_v[i];
            ci[o + i] = src_i[i];
        }
    }
    __syncthreads();
    // a shard that did not send all its ties: their value is its k-th value, the smallest it sent
    for (int s = warp; s < p.shards; s += NWARP) {
        float m = f_inf();
        for (int i = ctl->offs[s] + lane; i < ctl->offs[s + 1]; i += 32) m = fminf(m, cv[i]);
        m = -warp_max(-m);
        if (lane == 0) ctl->tval[s] = m;
    }
    __syncthreads();
    // the value multiset of the top-k: the sent values, plus up to k copies of each shard's unsent ties
    if (tid == 0) {
        int off = n;
        for (int s = 0; s < p.shards; ++s) {
            const int c = min(ctl->miss[s], k);
            for (int i = 0; i < c; ++i) {
                cv[off + i] = ctl->tval[s];
                ci[off + i] = -1;
            }
            off += c;
        }
        ctl->ntot = off;
    }
    __syncthreads();
    const int ntot = ctl->ntot;
    const Scr sc{hist, ctl->rctl, &ctl->gather_n, &ctl->kn, &ctl->thr, ctl->red_d, ctl->red_f, ctl->red_i};
    const float top_p = p.rP ? p.rP[r] : p.top_p;
    const bool topk_only = (p.flags & B2S_FLAG_TOPK_ONLY) != 0;
    const int kk = min(k, ntot);  // (every shard sends min(k, its columns) at least, so ntot >= k in practice)
    list_topk_values(cv, ntot, kk, vals, sc);
    if (tid < 32) {
        const float t = warp_topp(vals, kk, false, 0.0f, top_p, p.min_keep, topk_only);
        if (tid == 0) ctl->thr = t;
    }
    __syncthreads();
    const float thr = ctl->thr, vmax = vals[0];
    const float et = b2s_expf(__fsub_rn(thr, vmax));  // each unsent kept tie (value thr)
    // the kept sent items of each shard, ordered by id (ranks by counting within the shard), into sv / si
    for (int i = tid; i < n; i += NT) {
        if (!(cv[i] >= thr)) continue;
        int s = 0;
        while (ctl->offs[s + 1] <= i) ++s;
        const int id = ci[i];
        int rk = 0;
        for (int j = ctl->offs[s]; j < ctl->offs[s + 1]; ++j) rk += (cv[j] >= thr) & (ci[j] < id);
        sv[ctl->offs[s] + rk] = cv[i];
        si[ctl->offs[s] + rk] = id;
    }
    for (int s = warp; s < p.shards; s += NWARP) {
        int c = 0;
        for (int i = ctl->offs[s] + lane; i < ctl->offs[s + 1]; i += 32) c += cv[i] >= thr;
        c = warp_sum_i(c);
        if (lane == 0) ctl->kcnt[s] = c;
    }
    __syncthreads();
    // softmax normaliser of the kept set: the kept sent items and the unsent ties at thr (value thr, count miss[s])
    double es = 0.0;
    for (int i = tid; i < n; i += NT)
        if (cv[i] >= thr) es += (double)b2s_expf(__fsub_rn(cv[i], vmax));
    if (tid == 0)
        for (int s = 0; s < p.shards; ++s)
            if (ctl->miss[s] > 0 && ctl->tval[s] >= thr) es += (double)ctl->miss[s] * (double)et;
    const float sf = (float)block_sum(es, ctl->red_d);
    const float pt = __fdiv_rn(et, sf);
    // each shard's kept mass: its sent items in id order, then its unsent ties
    for (int s = warp; s < p.shards; s += NWARP) {
        const int o = ctl->offs[s], c = ctl->kcnt[s];
        double acc = 0.0;
        for (int i0 = 0; i0 < c; i0 += 32) {
            const double pi = i0 + lane < c ? (double)__fdiv_rn(b2s_expf(__fsub_rn(sv[o + i0 + lane], vmax)), sf) : 0.0;
            acc += __shfl_sync(0xffffffffu, warp_incl_scan(pi), 31);
        }
        if (ctl->miss[s] > 0 && ctl->tval[s] >= thr) acc += (double)ctl->miss[s] * (double)pt;
        if (lane == 0) ctl->mass[s] = acc;
    }
    __syncthreads();
    const int64_t step = p.steps ? p.steps[r] : 0;
    if (tid == 0) {
        const float u = p.rng == B2S_RNG_UNIFORM ? p.uvals[r]
                        : p.rng == B2S_RNG_PHILOX ? uniform_philox(p.seeds[r], step, p.requests ? p.requests[r] : 0)
                                                  : uniform_counter(p.seeds[r], step);
        double total = 0.0;
        for (int s = 0; s < p.shards; ++s) total += ctl->mass[s];
        const float target = __fmul_rn(u, (float)total);
        double c = 0.0;
        int star = -1;
        double base = 0.0;
        for (int s = 0; s < p.shards; ++s) {
            const double c2 = c + ctl->mass[s];
            if ((float)c2 > target) {
                star = s;
                base = c;
                break;
            }
            c = c2;
        }
        ctl->star = star;
        ctl->base = base;
        ctl->target = target;
        ctl->sf = sf;
        ctl->pt = pt;
    }
    __syncthreads();
    const int star = ctl->star;
    if (star < 0) {  // no cumulative mass exceeds u * total: the last id (searchsorted clamp)
        if (tid == 0) {
            p.tokens[r] = p.V - 1;
            if (p.pending) p.pending[r] = rec;
        }
        return;
    }
    const bool ties_out = ctl->miss[star] > 0 && ctl->tval[star] >= thr;
    if (ties_out) {  // the shard holding the draw did not send all its kept elements: its rank resolves the row
        if (tid == 0) {
            rec.base = ctl->base;
            rec.thr = thr;
            rec.vmax = vmax;
            rec.sf = sf;
            rec.target = ctl->target;
            rec.shard = star;
            if (p.pending) {
                p.pending[r] = rec;
                p.tokens[r] = -2;
            } else {  // no stage 3 to hand the row to
                p.tokens[r] = -1;
                if (p.status) atomicOr(p.status, B2S_STATUS_SHARD_INCOMPLETE);
            }
        }
        return;
    }
    if (warp == 0) {
        // among the shard's kept sent items, in id order, from the mass before the shard
        const int o = ctl->offs[star], c = ctl->kcnt[star];
        const float target = ctl->target;
        double acc = ctl->base;
        int found = -1;
        for (int i0 = 0; i0 < c && found < 0; i0 += 32) {
            const double pi = i0 + lane < c ? (double)__fdiv_rn(b2s_expf(__fsub_rn(sv[o + i0 + lane], vmax)), sf) : 0.0;
            const double incl = warp_incl_scan(pi);
            const unsigned hit = __ballot_sync(0xffffffffu, i0 + lane < c && (float)(acc + incl) > target);
            if (hit) found = si[o + i0 + __ffs(hit) - 1];
            acc += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (found < 0) found = c > 0 ? si[o + c - 1] : p.V - 1;  // rounding at the shard's last item
        if (lane == 0) {
            p.tokens[r] = found;
            if (p.pending) p.pending[r] = rec;
        }
    }
}

// Stage 3: a row pending on this shard is finished by scanning the shard row's processed elements in vocabulary
// order; other pending rows get -1, resolved rows their merged token.
struct ResolveParams {
    Params p;  // this shard's launch (logits, history, penalties, temperature, EOS rule), V = the shard's columns
    int shard, bf16;
    uint32_t slots;
    const b2s_shard_pending* pending;
    const int64_t* merged;
    int64_t* out;
};

__global__ void __launch_bounds__(NT, 1) shard_resolve_kernel(const ResolveParams rp) {
    extern __shared__ __align__(16) uint32_t ht[];
    const Params& p = rp.p;
    const int r = blockIdx.x, tid = threadIdx.x;
    __shared__ double red_d[NWARP + 1];
    __shared__ int red_i[NWARP], red_j[NWARP];
    pdl_wait_then_release();
    const b2s_shard_pending rec = rp.pending[r];
    if (rec.shard != rp.shard) {
        if (tid == 0) rp.out[r] = rec.shard < 0 ? rp.merged[r] : -1;
        return;
    }
    // this shard's history ids -> occurrence counts (open addressing, ids local to the shard)
    for (uint32_t s = tid; s < rp.slots; s += NT) ht[s] = HT_EMPTY;
    __syncthreads();
    const int Vs = p.V;
    if (p.hist && p.W > 0) {
        const int64_t* h = p.hist + (int64_t)r * p.hstride;
        for (int j = tid; j < p.W; j += NT) {
            const int64_t id = h[j] - p.id_off;
            if (h[j] >= 0 && id >= 0 && id < Vs) ht_insert(ht, rp.slots, (uint32_t)id, 1u);
        }
    }
    __syncthreads();
    const int64_t step = p.steps ? p.steps[r] : 0;
    const int64_t min_new = p.rminn ? p.rminn[r] : p.min_new;
    const int cens = (p.eos >= 0 && p.eos < Vs && step < min_new) ? p.eos : -1;  // omni: a masked EOS is -inf
    const float T = p.rT ? p.rT[r] : p.T;
    const float* atab = p.alpha ? p.alpha + (int64_t)r * p.alpha_stride : nullptr;
    const unsigned char* rowp = reinterpret_cast<const unsigned char*>(p.logits);
    const bool bf16 = rp.bf16 != 0;
    auto raw = [&](int i) {
        return bf16 ? bf16_bits_to_f(__ldg(reinterpret_cast<const unsigned short*>(rowp) + (int64_t)r * p.lstride + i))
                    : __ldg(reinterpret_cast<const float*>(rowp) + (int64_t)r * p.lstride + i);
    };
    auto P = [&](int i) {
        const float x = raw(i);
        const int slot = ht_find(ht, rp.slots, (uint32_t)i);
        if (slot >= 0 || i == cens) {
            const int n = slot >= 0 ? (int)(ht[slot] & ((1u << HT_CNT_BITS) - 1)) : 0;
            return hist_proc_value(p, atab, false, i == cens, T, n, x);
        }
        return __fdiv_rn(x, T);
    };
    auto prob = [&](float v) { return __fdiv_rn(b2s_expf(__fsub_rn(v, rec.vmax)), rec.sf); };
    // contiguous ranges per thread keep the prefix in id order
    const int L = (Vs + NT - 1) / NT;
    const int i0 = min(Vs, tid * L), i1 = min(Vs, i0 + L);
    double ps = 0.0;
    int last = -1;
    for (int i = i0; i < i1; ++i) {
        const float v = P(i);
        if (v >= rec.thr) {
            ps += (double)prob(v);
            last = i;
        }
    }
    double total;
    double acc = rec.base + block_excl_scan(ps, red_d, &total);
    int first = 0x7fffffff;
    for (int i = i0; i < i1 && first == 0x7fffffff; ++i) {
        const float v = P(i);
        if (!(v >= rec.thr)) continue;
        acc += (double)prob(v);
        if ((float)acc > rec.target) first = i;
    }
    int f = first;
#pragma unroll
    for (int o = 16; o; o >>= 1) f = min(f, __shfl_xor_sync(0xffffffffu, f, o));
    int lmax = last;
#pragma unroll
    for (int o = 16; o; o >>= 1) lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    __syncthreads();
    if ((tid & 31) == 0) {
        red_i[tid >> 5] = f;
        red_j[tid >> 5] = lmax;
    }
    __syncthreads();
    if (tid == 0) {
        int best = 0x7fffffff, lm = -1;
        for (int w = 0; w < NWARP; ++w) {
            best = min(best, red_i[w]);
            lm = max(lm, red_j[w]);
        }
        // rounding at the shard's end: its last kept element
        rp.out[r] = (best != 0x7fffffff ? best : lm) + p.id_off;
    }
}

}  // namespace b2s

extern "C" int b2s_shard_merge(const float* cand_values, const int32_t* cand_ids, const int32_t* cand_count, int32_t shards,
                               int32_t rows, int32_t cap, int32_t vocab, const b2s_sample_args* a,
                               b2s_shard_pending* pending, void* stream) {
    using namespace b2s;
    if (!cand_values || !cand_ids || !cand_count || !a || !a->tokens) return B2S_ERR_INVALID;
    if (shards < 1 || shards > MAXSH || rows < 0 || cap < 1 || vocab < 1) return B2S_ERR_INVALID;
    if (a->rng == B2S_RNG_UNIFORM ? !a->uniform_values : !a->seeds) return B2S_ERR_INVALID;
    if (a->rng != B2S_RNG_UNIFORM && !a->steps) return B2S_ERR_INVALID;  // the counter / Philox draw is keyed by the step
    if (rows == 0) return B2S_OK;
    MergeParams p;
    memset(&p, 0, sizeof(p));
    p.cv = cand_values;
    p.ci = cand_ids;
    p.cn = cand_count;
    p.shards = shards;
    p.rows = rows;
    p.cap = cap;
    p.V = vocab;
    p.top_k = a->top_k;
    p.min_keep = a->min_keep < 1 ? 1 : a->min_keep;
    p.top_p = a->top_p;
    p.rK = a->row_top_k;
    p.rP = a->row_top_p;
    p.rng = a->rng;
    p.flags = a->flags;
    p.seeds = a->seeds;
    p.steps = a->steps;
    p.requests = a->requests;
    p.uvals = a->uniform_values;
    p.tokens = a->tokens;
    p.pending = pending;
    p.status = a->status;
    p.nmax = shards * cap + shards * KLIST;
    const size_t smem = (sizeof(MergeCtl) + 15) / 16 * 16 + 256 * 4 + 2 * KLIST * 4 + (size_t)p.nmax * 4 * 4;
    if (smem > 227 * 1024) return B2S_ERR_UNSUPPORTED;
    cudaError_t e = cudaFuncSetAttribute(shard_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e);
    shard_merge_kernel<<<(unsigned)rows, NT, smem, (cudaStream_t)stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}

extern "C" int b2s_shard_resolve(const b2s_sample_args* a, int64_t vocab_offset, int32_t shard,
                                 const b2s_shard_pending* pending, const int64_t* merged, int64_t* tokens_out,
                                 void* stream) {
    using namespace b2s;
    if (!a || !a->logits || !pending || !merged || !tokens_out || shard < 0 || vocab_offset < 0) return B2S_ERR_INVALID;
    if (a->rows < 0 || a->vocab <= 0 || a->logits_row_stride < a->vocab) return B2S_ERR_INVALID;
    if (a->logits_dtype != B2S_DTYPE_F32 && a->logits_dtype != B2S_DTYPE_BF16) return B2S_ERR_INVALID;
    if (!a->row_temperature && !(a->temperature > 0.0f)) return B2S_ERR_INVALID;
    if (a->window < 0 || (a->window > 0 && (!a->history || !a->alpha || a->alpha_len < 1 ||
                                            a->history_row_stride < a->window)))
        return B2S_ERR_INVALID;
    if (a->window > (1 << 13)) return B2S_ERR_UNSUPPORTED;
    if (a->vocab > (1 << 18)) return B2S_ERR_UNSUPPORTED;  // packed hash ids
    if (a->rows == 0) return B2S_OK;
    ResolveParams rp;
    memset(&rp, 0, sizeof(rp));
    Params& p = rp.p;
    p.logits = a->logits;
    p.lstride = a->logits_row_stride;
    p.rows = a->rows;
    p.V = a->vocab;
    p.W = a->window;
    p.eos = (a->eos >= vocab_offset && a->eos < vocab_offset + a->vocab) ? (int)(a->eos - vocab_offset) : -1;
    p.hist = a->history;
    p.hstride = a->history_row_stride;
    p.steps = a->steps;
    p.T = a->temperature;
    p.rT = a->row_temperature;
    p.presence = a->presence_penalty;
    p.frequency = a->frequency_penalty;
    p.min_new = a->min_new_tokens;
    p.rminn = a->row_min_new_tokens;
    p.alpha = a->alpha;
    p.alpha_len = a->alpha_len;
    p.alpha_stride = a->alpha_row_stride;
    p.status = a->status;
    p.id_off = vocab_offset;
    p.sem = B2S_SEM_OMNI;
    rp.bf16 = a->logits_dtype == B2S_DTYPE_BF16 ? 1 : 0;
    rp.shard = shard;
    rp.pending = pending;
    rp.merged = merged;
    rp.out = tokens_out;
    uint32_t slots = 32;
    while (slots < 2u * (uint32_t)(a->window > 0 ? a->window : 1)) slots <<= 1;
    rp.slots = slots;
    const size_t smem = slots * 4;
    cudaError_t e = cudaFuncSetAttribute(shard_resolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e);
    shard_resolve_kernel<<<(unsigned)a->rows, NT, smem, (cudaStream_t)stream>>>(rp);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}
