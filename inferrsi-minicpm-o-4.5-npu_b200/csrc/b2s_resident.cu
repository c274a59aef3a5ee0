// Row-resident sampling kernel (sm_100a): the decode-step form of b2s_sample for batches that fit the GPU in
// one wave and rows that fit a cluster's shared memory.
//
// A cluster of CL CTAs (CL = 1, 2, 4 or 8) owns one logits row.  Each CTA copies its slice of the row's
// 16-byte interior into shared memory with bulk copies on the TMA engine (32 KB pieces, one mbarrier
// each, no multicast), so the whole slice is in flight at once instead of the few KB a thread's registers
// can hold.  While the pieces land, the threads stage the penalty history, build the history bitmap, mark
// the piece shares that hold a history id, and (rank 0) count the ids and take their processed values.
// Then, per CTA and from shared memory:
//
//   maxima:  each thread's largest value of its share of every piece (RSH vectors), taken as the piece lands;
//   tau:     the k-th largest of the warps' ceil(k/16) largest per-thread maxima over shares without a
//            history id -- a lower bound of the slice's (hence the row's) k-th largest non-history value;
//   pass 2:  the shares whose maximum clears tau are re-read from shared memory; every non-history element
//            >= tau (less a rounding margin) joins the CTA's candidate list.
//
// The other CTAs hand their lists to rank 0 through distributed shared memory (one cluster barrier); rank 0
// adds the history ids whose processed value clears f(tau) and runs the list stage of b2s_list.cuh (top-k
// values, top-p cut, value threshold, inverse-CDF draw in vocabulary order), then the state epilogue.  Each
// CTA's list holds every element of its slice >= the row's k-th largest processed value, so their union
// does, and the result is the same as the streaming kernel's.  Rows the list cannot serve (a segment
// overflow from heavy ties, NaN or unusable tau) take the exact full-row path of b2s_row.cuh in rank 0,
// reading the row from global memory; hf frame-0 rows take the ordered scan.  Those paths, and the slow
// side of the mbarrier waits, are out of line: the instructions a decode step executes stay few and
// contiguous (a launch is short enough that instruction fetch is a large part of it).
//
// hf's full-row normaliser (talker_sampler.py:112) is taken from the resident row (one CTA per row for hf).
// Every mbarrier wait is bounded (WAIT_NS); a wait that gives up marks the row (PAD, B2S_STATUS_WAIT_TIMEOUT)
// and the CTA waits once more, bounded, for its copies before it exits.  The only wait between CTAs is the
// hardware cluster barrier, two phases per row, reached by every CTA of the cluster.
#include "b2s_rowpaths.cuh"

namespace cg = cooperative_groups;

namespace b2s {

constexpr uint64_t WAIT_NS = 250ull * 1000 * 1000;  // bound of every mbarrier wait
constexpr int ERR_TIMEOUT = 2;

static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity) {
    return mbar_wait_bounded(bar, parity, WAIT_NS);
}
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity) {
    return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity);
}

// hf's full-row normaliser from the resident row (one CTA per row): max over the candidates (or, when the
// list failed, the row), then the fp64 sum of exp(P - max) in row_visit's thread layout, so the same partial
// sums.  Inlined: as an out-of-line call it measured about 0.7 us slower per Talker launch.
template <typename E>
__device__ __forceinline__ float resident_lse(const Row<E>& R, const uint4* slice, int nv, const float* cv, int n,
                                              bool from_list, Ctl* ctl) {
    constexpr int EPV = Elem<E>::EPV;
    const int tid = threadIdx.x, V = R.V;
    float lm = f_ninf();
    if (from_list) {
        for (int i = tid; i < n; i += NT) lm = fmaxf(lm, cv[i]);
    } else {
        for (int v = tid; v < nv; v += NT) {
            const uint4 q = slice[v];
#pragma unroll
            for (int j = 0; j < EPV; ++j) lm = fmaxf(lm, R.P(R.e0 + v * EPV + j, Elem<E>::at(q, j)));
        }
        if (tid == 0)
            for (int i = 0; i < R.nh; ++i) lm = fmaxf(lm, R.P(i, Elem<E>::gld(R.rowp, i)));
        if (tid == 1)
            for (int i = R.e0 + R.nvec * EPV; i < V; ++i) lm = fmaxf(lm, R.P(i, Elem<E>::gld(R.rowp, i)));
    }
    const float m = block_max(lm, ctl->red_f);
    const float mu = (m == f_inf() || m == f_ninf()) ? 0.0f : m;
    double sacc = 0.0;
    for (int v = tid; v < nv; v += NT) {
        const uint4 q = slice[v];
        const int e = R.e0 + v * EPV;
#pragma unroll
        for (int j = 0; j < EPV; ++j) sacc += (double)b2s_expf(__fsub_rn(R.P(e + j, Elem<E>::at(q, j)), mu));
    }
    if (tid == 0)
        for (int i = 0; i < R.nh; ++i) sacc += (double)b2s_expf(__fsub_rn(R.P(i, Elem<E>::gld(R.rowp, i)), mu));
    if (tid == 1)
        for (int i = R.e0 + R.nvec * EPV; i < V; ++i)
            sacc += (double)b2s_expf(__fsub_rn(R.P(i, Elem<E>::gld(R.rowp, i)), mu));
    return __fadd_rn((float)log((double)(float)block_sum(sacc, ctl->red_d)), mu);
}

template <typename E, int SEM>
__global__ void __launch_bounds__(NT, 1) resident_kernel(const Params p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int CL = p.cl;
    const int crank = CL > 1 ? (int)cg::this_cluster().block_rank() : 0;
    const bool lead = crank == 0;
    const int r = (int)blockIdx.x / CL;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + p.off_bar);
    const uint4* slice = reinterpret_cast<const uint4*>(smem + p.off_slice);
    HistBufs hb;
    hb.bits = reinterpret_cast<uint32_t*>(smem + p.off_bits);
    hb.pref = reinterpret_cast<uint16_t*>(smem + p.off_pref);
    hb.hcnt = reinterpret_cast<uint32_t*>(smem + p.off_hcnt);
    hb.hid = reinterpret_cast<int*>(smem + p.off_hid);
    hb.hpos = reinterpret_cast<int*>(smem + p.off_hpos);
    hb.htv = reinterpret_cast<float*>(smem + p.off_htv);
    int64_t* hstage = reinterpret_cast<int64_t*>(smem + p.off_hstage);
    float* atab = reinterpret_cast<float*>(smem + p.off_atab);
    hb.hstage = hstage;
    hb.atab = atab;
    uint32_t* bits = hb.bits;
    uint32_t* smask = reinterpret_cast<uint32_t*>(smem + p.off_smask);  // [thread] bit pc: share holds a history id
    float* cand_v = reinterpret_cast<float*>(smem + p.off_cand);  // rank 0: the merged list, filtered by tau*
    int* cand_i = reinterpret_cast<int*>(smem + p.off_candi);
    float* kv = reinterpret_cast<float*>(smem + p.off_lst);  // this CTA's list; rank 0: every CTA's, by region
    int* ki = reinterpret_cast<int*>(kv + p.ltot);
    float* sv = kv + 2 * p.ltot;
    int* si = reinterpret_cast<int*>(kv + 3 * p.ltot);
    float* vals = reinterpret_cast<float*>(smem + p.off_vals);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + p.off_hist);
    constexpr int ES = Elem<E>::SZ, EPV = Elem<E>::EPV;
    const int V = p.V;
    // ---------------- before the wait for the previous kernel (nothing global is read): the first phase of the
    // cluster barrier (arrived here, waited on just before the first remote store, so that no CTA writes into
    // another's shared memory before that one runs), the row's geometry, the mbarriers, the zeroed history
    // structures -- set-up a CTA that starts early does while the previous kernel finishes
    if (CL > 1) cluster_arrive_relaxed();
    Row<E> R;
    R.rowp = reinterpret_cast<const unsigned char*>(p.logits) + (int64_t)r * p.lstride * ES;
    R.V = V;
    {
        const uintptr_t a = reinterpret_cast<uintptr_t>(R.rowp), b = a + (uintptr_t)V * ES;
        const uintptr_t ace = (a + 15) & ~(uintptr_t)15, bfl = b & ~(uintptr_t)15;
        if (ace < bfl) {
            R.nh = (int)((ace - a) / ES);
            R.nvec = (int)((bfl - ace) / 16);
        } else {
            R.nh = V;
            R.nvec = 0;
        }
        R.gvec = reinterpret_cast<const uint4*>(ace);
        R.e0 = R.nh;
    }
    const int per = (R.nvec + CL - 1) / CL;  // <= p.slice_vecs (the launcher sized it for the widest row)
    const int v0 = min(R.nvec, crank * per), nv = min(R.nvec, v0 + per) - v0;
    const int npc = (nv + RPV - 1) / RPV;
    if (tid == 0) {
        for (int i = 0; i < npc; ++i) mbar_init(&bar[i], 1u);
        fence_mbar_init();
        ctl->err = 0;
        ctl->kn = 0;
    }
    // omni order (the Thinker's): the owned history ids go into an (id, count) hash table and a dense list instead
    // of bitmap ranks -- the fast path reads them by list position; a row taking a full-row path rebuilds the ranks
    constexpr bool HASH = SEM == B2S_SEM_OMNI;
    uint32_t* ht = reinterpret_cast<uint32_t*>(smem + p.off_ht);
    const bool may_ht = (p.W > 0 && p.hist != nullptr) || (p.eos >= 0 && p.eos < V);  // a superset of use_ht below
    if (may_ht) {
        for (uint32_t g = tid; g < p.bitwords / 4; g += NT) reinterpret_cast<uint4*>(bits)[g] = make_uint4(0u, 0u, 0u, 0u);
        for (int d = tid; d < p.hcap; d += NT) hb.hcnt[d] = 0u;
        if (HASH)
            for (uint32_t g = tid; g < p.ht_slots; g += NT) ht[g] = HT_EMPTY;
    }
    if (HASH && tid == 0) ctl->hd_n = 0;
    smask[tid] = 0u;
    pdl_wait_then_release();  // nothing global is read before the previous kernel of the stream is done

    // ---------------- the history, the penalty table and the row's parameters are requested first; then the row
    // slice's bulk copies
    const int64_t* hrow = p.hist ? p.hist + (int64_t)r * p.hstride : nullptr;
    if (hrow && p.W > 0) {
        for (int j = tid; j < p.W; j += NT) cp_async8(&hstage[j], &hrow[j]);
        const float* alpha = p.alpha ? p.alpha + (int64_t)r * p.alpha_stride : nullptr;
        if (alpha)
            for (int j = tid; j < p.alpha_len; j += NT) cp_async4(&atab[j], &alpha[j]);
    }
    const int64_t step = p.steps ? p.steps[r] : 0;
    const bool is_live = (p.active ? p.active[r] != 0 : true) && !(p.finished ? p.finished[r] != 0 : false);
    const float T = p.rT ? p.rT[r] : p.T;
    const float top_p = p.rP ? p.rP[r] : p.top_p;
    const int top_k = p.rK ? p.rK[r] : p.top_k;
    const int64_t min_new = p.rminn ? p.rminn[r] : p.min_new, max_new = p.rmaxn ? p.rmaxn[r] : p.max_new;
    if (tid == 0)
        for (int i = 0; i < npc; ++i) {
            const uint32_t bytes = (uint32_t)min(RPV, nv - i * RPV) * 16u;
            mbar_arrive_expect_tx(&bar[i], bytes);
            bulk_g2s(const_cast<uint4*>(slice) + (size_t)i * RPV, R.gvec + v0 + (size_t)i * RPV, bytes, &bar[i]);
        }
    // the ids this CTA is responsible for: its slice, and (rank 0) the elements outside the 16-byte interior
    const int e_lo = R.e0 + v0 * EPV, e_hi = e_lo + nv * EPV, i_end = R.e0 + R.nvec * EPV;
    auto owns = [&](int id) { return (id >= e_lo && id < e_hi) || (lead && (id < R.e0 || id >= i_end)); };

    // ---------------- mode
    const bool hf = SEM >= 0 ? SEM == B2S_SEM_HF : p.sem == B2S_SEM_HF;
    const bool eos_ok = p.eos >= 0 && p.eos < V;
    const bool masked_eos = eos_ok && step < min_new;
    int mode;
    if (!is_live) mode = MODE_SKIP;
    else if (step >= max_new - 1) mode = MODE_FORCED;
    else if (hf && step <= 0) mode = MODE_FULL;
    else mode = MODE_FILTER;
    int k = 0;
    if (mode == MODE_FILTER) {
        k = min(max(top_k, max(p.min_keep, 1)), V);
        if (k > p.kbuf) {
            mode = MODE_FAIL;
            if (tid == 0 && lead) set_status(p, B2S_STATUS_TOPK_LIMIT);
        }
    }
    if (tid == 32 && lead) {
        ctl->u = (p.rng == B2S_RNG_UNIFORM || !p.seeds) ? (p.uvals ? p.uvals[r] : 0.0f)
                 : p.rng == B2S_RNG_PHILOX ? uniform_philox(p.seeds[r], step, p.requests ? p.requests[r] : 0)
                                           : uniform_counter(p.seeds[r], step);
    }
    R.T = T;
    R.identity = false;
    const bool pen_hist = mode == MODE_FILTER && p.W > 0 && hrow != nullptr;
    const bool censor = mode == MODE_FILTER && !hf && masked_eos;  // omni: EOS is -inf before anything else
    const bool use_ht = pen_hist || censor;
    R.bits = use_ht ? bits : nullptr;
    R.pref = hb.pref;
    R.htv = hb.htv;
    R.censor = censor ? p.eos : -1;
    // rank 0: the elements outside the 16-byte interior, one per lane of the last warp's lanes 16..31 (head in
    // 16..23, tail in 24..31; a row with no interior vector has at most 15 elements, all in lanes 16..31)
    int edge_i = -1;
    float edge_x = 0.0f;
    if (lead && tid >= NT - 16) {
        const int t = tid - (NT - 16);
        const bool whole = R.nvec == 0;
        const int i = (whole || t < 8) ? t : i_end + (t - 8);
        if ((!whole && t < 8) ? i < R.nh : i < V) {
            edge_i = i;
            edge_x = Elem<E>::gld(R.rowp, i);
        }
    }
    cp_async_wait_all();
    __syncthreads();  // the history has landed; the mbarriers are initialised

    // global id -> (piece, owner thread) of this slice: bit pc of smask[owner]
    auto mark_share = [&](int id) {
        const int v = (id - R.e0) / EPV - v0;
        atomicOr(&smask[(v % RPV) % NT], 1u << (v / RPV));
    };
    int hd = 0;  // distinct owned history ids (the censored EOS included)
    if (use_ht) {
        if (pen_hist)
            for (int j = tid; j < p.W; j += NT) {
                const int64_t hv = hstage[j];
                if (hv < 0) continue;
                if (hv >= V) {
                    if (lead) set_status(p, B2S_STATUS_HISTORY_RANGE);
                    continue;
                }
                const int id = (int)hv;
                if (!owns(id)) continue;
                atomicOr(&bits[id >> 5], 1u << (id & 31));
                if (id >= e_lo && id < e_hi) mark_share(id);
                if (HASH) {
                    uint32_t slot;
                    if (ht_add(ht, p.ht_slots, (uint32_t)id, 1u, slot)) hb.hpos[atomicAdd(&ctl->hd_n, 1)] = (int)slot;
                }
            }
        if (censor && tid == 0 && owns(p.eos)) {
            atomicOr(&bits[p.eos >> 5], 1u << (p.eos & 31));
            if (p.eos >= e_lo && p.eos < e_hi) mark_share(p.eos);
            if (HASH) {
                uint32_t slot;
                if (ht_add(ht, p.ht_slots, (uint32_t)p.eos, 0u, slot)) hb.hpos[atomicAdd(&ctl->hd_n, 1)] = (int)slot;
            }
        }
        __syncthreads();
        if (HASH)
            hd = ctl->hd_n;  // hpos[0, hd): the slots of the distinct owned ids
        else
            hd = hist_rank_count<E>(p, R, hb, pen_hist, censor, owns, ctl);
    }

    // ---------------- the slice lands piece by piece: each thread's maximum of its share of every piece
    float tm[RMAXP];
    bool timed_out = false;
#pragma unroll
    for (int pc = 0; pc < RMAXP; ++pc) {
        tm[pc] = f_ninf();
        if (pc < npc) {
            if (!mbar_wait_fast(&bar[pc], 0u)) timed_out = true;
            const int n = min(RPV, nv - pc * RPV);
            const uint4* s = slice + (size_t)pc * RPV;
            uint4 q[RSH];
#pragma unroll
            for (int h = 0; h < RSH; ++h)
                q[h] = tid + h * NT < n ? s[tid + h * NT] : make_uint4(Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG);
            tm[pc] = Elem<E>::template vmaxn<RSH>(q);
        }
    }
    if (timed_out) {
        atomicOr(&ctl->err, ERR_TIMEOUT);
        set_status(p, B2S_STATUS_WAIT_TIMEOUT);
    }
    __syncthreads();  // smask and the counts are complete; every piece has landed
    // the owned history ids' processed values, their raw values from the resident slice (edges: global memory)
    auto raw_of = [&](int id) {
        if (id >= e_lo && id < e_hi) {
            const int rel = id - e_lo;
            return Elem<E>::at(slice[rel / EPV], rel % EPV);
        }
        return Elem<E>::gld(R.rowp, id);
    };
    if (use_ht && HASH) {
        // the dense list's ids and processed values from the table's (id, count) words
        for (int d = tid; d < hd; d += NT) {
            const uint32_t wd = ht[hb.hpos[d]];
            const int id = (int)(wd >> HT_CNT_BITS), n = (int)(wd & ((1u << HT_CNT_BITS) - 1u));
            hb.hid[d] = id;
            hb.htv[d] = (censor && id == p.eos) ? f_ninf()
                        : pen_hist ? hist_proc_value(p, atab, hf, false, T, n, raw_of(id)) : f_ninf();
        }
    } else if (use_ht) {
        hist_values<E>(p, R, hb, hd, hf, pen_hist, censor, T, raw_of);
    }

    // ---------------- tau of this CTA's slice
    const bool cand_path = mode == MODE_FILTER && k <= KFAST && !(p.flags & B2S_FLAG_FORCE_GENERAL) && T >= 1e-6f &&
                           T <= 1e6f;
    const int jw = (k + NWARP - 1) / NWARP;
    const int ng = NWARP * jw;  // gathered maxima: a multiple of 16, <= 128
    if (cand_path) {
        // this thread's largest value over its shares that hold no history id (each such maximum is a distinct
        // non-history element, so the k-th largest of them bounds the slice's k-th largest from below)
        const uint32_t hm = smask[tid];
        float tmax_nh = f_ninf();
#pragma unroll
        for (int pc = 0; pc < RMAXP; ++pc)
            if (!((hm >> pc) & 1u)) tmax_nh = fmaxf(tmax_nh, tm[pc]);
        if (edge_i >= 0 && !R.hbit(edge_i)) tmax_nh = fmaxf(tmax_nh, edge_x);
        // the warp's jw largest, one redux on order keys each (tmax_nh is never NaN: fmaxf keeps the other operand)
        uint32_t key = okey(tmax_nh);
        for (int t = 0; t < jw; ++t) {
            const uint32_t mk = __reduce_max_sync(0xffffffffu, key);
            const unsigned who = __ballot_sync(0xffffffffu, key == mk);
            if (lane == __ffs(who) - 1) key = 0u;  // below every key: taken
            if (lane == 0) vals[warp * jw + t] = okey_to_f(mk);
        }
    }
    __syncthreads();
    float tau = f_ninf();
    if (cand_path) {
        // every warp finds the k-th largest of the ng gathered values (each lane ranks up to 4 of them)
        const float4* v4 = reinterpret_cast<const float4*>(vals);
        float found = f_ninf();
        for (int b = 0; b < ng; b += 32) {
            const float x = b + lane < ng ? vals[b + lane] : f_ninf();
            int gt = 0, eq = 0;
#pragma unroll 4
            for (int j4 = 0; j4 < ng / 4; ++j4) {
                const float4 y = v4[j4];
                gt += (y.x > x) + (y.y > x) + (y.z > x) + (y.w > x);
                eq += (y.x == x) + (y.y == x) + (y.z == x) + (y.w == x);
            }
            const unsigned who = __ballot_sync(0xffffffffu, b + lane < ng && x > f_ninf() && gt < k && k <= gt + eq);
            if (who) found = __shfl_sync(0xffffffffu, x, __ffs(who) - 1);
        }
        tau = found;
    }
    bool ovf = !cand_path;
    float tau_low = f_inf();
    if (cand_path) {
        if (nv == 0 && !lead && hd == 0) {
            tau_low = f_inf();  // an empty slice has nothing to hand over
        } else if (!(tau > f_ninf()) || tau == f_inf() || R.f(tau) == f_inf()) {
            ovf = true;
        } else {
            tau_low = tau - fmaxf(fabsf(tau) * 9.5367431640625e-7f, 1e-30f);  // margin for collisions of fl(x / T)
        }
    }

    // ---------------- pass 2: this CTA's candidates (processed values) into its list
    const int hshare = p.ltot / CL;  // a CTA's share of rank 0's merged list
    // every lane of the warp calls it with its count: one shared atomic per warp, the lane's first position back
    auto warp_reserve = [&](int cnt) {
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        int base = 0;
        if (lane == 31 && incl > 0) base = atomicAdd(&ctl->kn, incl);
        return __shfl_sync(0xffffffffu, base, 31) + incl - cnt;
    };
    if (cand_path && !ovf) {
        // the thread's shares whose maximum clears tau, one per round of its warp; their non-history elements >=
        // tau_low
        uint32_t hits = 0u;
#pragma unroll
        for (int pc = 0; pc < RMAXP; ++pc) hits |= (uint32_t)(tm[pc] >= tau_low) << pc;
        while (__any_sync(0xffffffffu, hits != 0u)) {
            uint32_t em[RSH];
            uint4 q[RSH];
            int cnt = 0, eb = 0;
#pragma unroll
            for (int h = 0; h < RSH; ++h) {
                em[h] = 0u;
                q[h] = make_uint4(0u, 0u, 0u, 0u);
            }
            if (hits) {
                const int pc = __ffs(hits) - 1;
                hits &= hits - 1u;
                const int n = min(RPV, nv - pc * RPV);
                eb = R.e0 + (v0 + pc * RPV + tid) * EPV;  // element 0 of the share's first vector
#pragma unroll
                for (int h = 0; h < RSH; ++h) {
                    const int vl = tid + h * NT;
                    if (vl < n) {
                        q[h] = slice[(size_t)pc * RPV + vl];
                        if (Elem<E>::vmax(q[h]) >= tau_low) {
                            const uint32_t hbm = R.hbits(eb + h * NT * EPV, EPV);
#pragma unroll
                            for (int j = 0; j < EPV; ++j)
                                if (Elem<E>::at(q[h], j) >= tau_low && !((hbm >> j) & 1u)) em[h] |= 1u << j;
                        }
                    }
                    cnt += __popc(em[h]);
                }
            }
            int pos = warp_reserve(cnt);
#pragma unroll
            for (int h = 0; h < RSH; ++h) {
                uint32_t m = em[h];
                while (m) {
                    const int j = __ffs(m) - 1;
                    m &= m - 1u;
                    if (pos < hshare) {  // past it: counted, and the list is flagged as overflowed below
                        kv[pos] = R.f(Elem<E>::at(q[h], j));
                        ki[pos] = eb + h * NT * EPV + j;
                    }
                    ++pos;
                }
            }
        }
        if (warp == NWARP - 1) {  // the ragged head / tail (rank 0)
            const bool eh = edge_i >= 0 && edge_x >= tau_low && !R.hbit(edge_i);
            const int pos = warp_reserve(eh ? 1 : 0);
            if (eh && pos < hshare) {
                kv[pos] = R.f(edge_x);
                ki[pos] = edge_i;
            }
        }
        // the owned history ids whose processed value clears f(tau_low)
        const float p_low = R.f(tau_low);
        for (int d0 = 0; d0 < hd; d0 += NT) {
            const int d = d0 + tid;
            const float hv = d < hd ? hb.htv[d] : f_ninf();
            const bool ok = d < hd && hv >= p_low;
            if (!__any_sync(0xffffffffu, ok)) continue;
            const int pos = warp_reserve(ok ? 1 : 0);
            if (ok && pos < hshare) {
                kv[pos] = hv;
                ki[pos] = hb.hid[d];
            }
        }
    }
    __syncthreads();
    int n = ctl->kn;
    if (cand_path && n > hshare) ovf = true;

    // ---------------- the other CTAs hand their lists and taus to rank 0 (region c: positions from c * hshare)
    if (CL > 1) {
        cg::cluster_group cl = cg::this_cluster();
        cluster_wait();  // every CTA of the cluster runs
        if (!lead) {
            const bool bad = !cand_path || ovf || (ctl->err != 0);
            if (!bad) {
                float* dv = cl.map_shared_rank(kv, 0) + crank * hshare;
                int* di = cl.map_shared_rank(ki, 0) + crank * hshare;
                for (int i = tid; i < n; i += NT) {
                    dv[i] = kv[i];
                    di[i] = ki[i];
                }
            }
            if (tid == 0) {
                *cl.map_shared_rank(&ctl->rx_n[crank], 0) = bad ? -1 : n;
                *cl.map_shared_rank(&ctl->rx_tau[crank], 0) = tau_low;
            }
        }
        cl.sync();  // every list is in rank 0's shared memory
        if (!lead) {
            if (ctl->err && tid == 0)
                for (int i = 0; i < npc; ++i) mbar_wait_bounded(&bar[i], 0u, WAIT_NS);
            return;
        }
    }

    // ---------------- rank 0: every CTA's list, one after the other, into cand_v / cand_i
    const bool row_err = ctl->err != 0;
    if (cand_path && !ovf && !row_err) {
        int off[8];
        int tot = 0;
        for (int c = 0; c < CL; ++c) {
            const int nc = c == 0 ? n : ctl->rx_n[c];
            if (nc < 0) ovf = true;
            off[c] = tot;
            tot += max(nc, 0);
        }
        if (!ovf) {
            for (int c = 0; c < CL; ++c) {
                const int nc = (c + 1 < CL ? off[c + 1] : tot) - off[c];
                for (int i = tid; i < nc; i += NT) {
                    cand_v[off[c] + i] = kv[c * hshare + i];
                    cand_i[off[c] + i] = ki[c * hshare + i];
                }
            }
            n = tot;
        }
    }
    __syncthreads();
    if (cand_path && !ovf && !row_err) ovf = n < k;

    // ---------------- rank 0: the row's token
    int64_t token = V - 1;
    float lse = 0.0f;
    const int drop = (hf && masked_eos) ? p.eos : -1;
    if (mode == MODE_FILTER && !row_err && (CL > 1 || HASH) && ovf)
        hist_rebuild<E>(p, R, hb, hf, pen_hist, censor, T, ctl);  // the full-row path reads every history value
    if (mode == MODE_FILTER && hf && !row_err) lse = resident_lse<E>(R, slice, nv, cand_v, n, !ovf, ctl);
    const bool topk_only = (p.flags & B2S_FLAG_TOPK_ONLY) != 0;
    if (mode == MODE_FILTER && !row_err) {
        if (!ovf) {
            token = block_list_token(cand_v, cand_i, kv, ki, sv, si, n, k, hf, lse, top_p, p.min_keep, topk_only, drop,
                                     ctl->u, V, vals, hist, ctl);
        } else {
            token = exact_token<E>(R, k, hf, lse, top_p, p.min_keep, topk_only, drop, ctl->u, hist, vals, ctl);
        }
    }
    if (mode == MODE_FORCED) token = eos_ok ? (int64_t)p.eos : (int64_t)(V - 1);
    if (mode == MODE_FULL && !row_err) token = full_token<E>(R, drop, ctl->u, ctl);

    // ---------------- state epilogue (a failed row: PAD out, state unchanged)
    const int64_t tok_drawn = (row_err || mode == MODE_SKIP || mode == MODE_FAIL) ? PAD : token;
    const bool adv = is_live && tok_drawn != PAD;
    const int64_t tok = adv ? tok_drawn : PAD;
    if (tid == 0) {
        if (p.tokens) p.tokens[r] = tok;
        if (p.steps_out) p.steps_out[r] = step + (adv ? 1 : 0);
        if (p.fin_out) {
            const bool f0 = p.finished ? p.finished[r] != 0 : false;
            p.fin_out[r] = (uint8_t)(f0 || (adv && tok == (int64_t)p.eos));
        }
    }
    if (p.hist_out && p.W > 0) {
        int64_t* ho = p.hist_out + (int64_t)r * p.hostride;
        for (int j = tid; j < p.W; j += NT) ho[j] = adv ? (j + 1 < p.W ? hstage[j + 1] : tok) : hstage[j];
    }
    if (row_err && tid == 0)
        for (int i = 0; i < npc; ++i) mbar_wait_bounded(&bar[i], 0u, WAIT_NS);
}


// The instantiations: general (hf or omni from the parameters) and omni fixed at compile time.
ResKernel resident_kernel_for(bool bf16, bool omni) {
    static const ResKernel k[2][2] = {
        {resident_kernel<float, -1>, resident_kernel<float, B2S_SEM_OMNI>},
        {resident_kernel<__nv_bfloat16, -1>, resident_kernel<__nv_bfloat16, B2S_SEM_OMNI>}};
    return k[bf16 ? 1 : 0][omni ? 1 : 0];
}

}  // namespace b2s
