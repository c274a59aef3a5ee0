// Row-resident sampling kernel (sm_100a): the decode-step form of b2s_sample for batches that fit the GPU in
// one wave and rows that fit a cluster's shared memory.
//
// A cluster of CL CTAs (CL = 1, 2, 4 or 8) owns one logits row.  Each CTA copies its slice of the row's
// 16-byte interior into shared memory with bulk copies on the TMA engine (16 KB pieces, one mbarrier
// each, no multicast), so the whole slice is in flight at once instead of the few KB a thread's registers
// can hold.  While the pieces land, the threads stage the penalty history, build the history bitmap and
// (rank 0) the per-id counts and processed values.  Then, per CTA and from shared memory:
//
//   maxima:  each thread's largest value of each piece share (2 vectors), taken as the piece lands;
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
// overflow from heavy ties, NaN or unusable tau, top_k beyond the list stage) take the exact full-row path
// of b2s_row.cuh in rank 0, reading the row from global memory; hf frame-0 rows take the ordered scan.
//
// hf's full-row normaliser (talker_sampler.py:112) is taken from the resident row (one CTA per row for hf).
// Every mbarrier wait is bounded (WAIT_NS); a wait that gives up marks the row (PAD, B2S_STATUS_WAIT_TIMEOUT)
// and the CTA waits once more, bounded, for its copies before it exits.  The only wait between CTAs is the
// hardware cluster barrier, reached once per row by every CTA of the cluster.
#include "b2s_row.cuh"

namespace cg = cooperative_groups;

namespace b2s {

constexpr uint64_t WAIT_NS = 250ull * 1000 * 1000;  // bound of every mbarrier wait
constexpr int ERR_TIMEOUT = 2;

template <typename E, int SEM>
__global__ void __launch_bounds__(NT, 1) resident_kernel(const Params p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31;
    const int CL = p.cl;
    const int crank = CL > 1 ? (int)cg::this_cluster().block_rank() : 0;
    const bool lead = crank == 0;
    const int r = (int)blockIdx.x / CL;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + p.off_bar);
    const uint4* slice = reinterpret_cast<const uint4*>(smem + p.off_slice);
    uint32_t* bits = reinterpret_cast<uint32_t*>(smem + p.off_bits);
    uint16_t* pref = reinterpret_cast<uint16_t*>(smem + p.off_pref);
    uint32_t* hcnt = reinterpret_cast<uint32_t*>(smem + p.off_hcnt);
    int* hid = reinterpret_cast<int*>(smem + p.off_hid);
    int* hpos = reinterpret_cast<int*>(smem + p.off_hpos);
    float* htv = reinterpret_cast<float*>(smem + p.off_htv);
    int64_t* hstage = reinterpret_cast<int64_t*>(smem + p.off_hstage);
    float* hraw = reinterpret_cast<float*>(smem + p.off_hraw);
    float* atab = reinterpret_cast<float*>(smem + p.off_atab);
    float* cand_v = reinterpret_cast<float*>(smem + p.off_cand);  // warp segments, then list-stage scratch
    int* cand_i = reinterpret_cast<int*>(smem + p.off_candi);
    float* kv = reinterpret_cast<float*>(smem + p.off_lst);  // the compacted list (rank 0: every CTA's)
    int* ki = reinterpret_cast<int*>(kv + p.ltot);
    float* sv = kv + 2 * p.ltot;
    int* si = reinterpret_cast<int*>(kv + 3 * p.ltot);
    float* vals = reinterpret_cast<float*>(smem + p.off_vals);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + p.off_hist);
    constexpr int ES = Elem<E>::SZ, EPV = Elem<E>::EPV;
    const int V = p.V;
    const Scr sc{hist, ctl->rctl, &ctl->gather_n, &ctl->kn, &ctl->thr, ctl->red_d, ctl->red_f, ctl->red_i};
    pdl_wait_then_release();  // nothing global is read before the previous kernel of the stream is done
    // first phase of the cluster barrier: arrived here, waited on just before the first remote store, so that
    // no CTA writes into another's shared memory before that one runs
    if (CL > 1) cluster_arrive_relaxed();

    // ---------------- geometry: the row's 16-byte interior, this CTA's slice of it; its bulk copies go out first
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
        for (int i = 0; i < npc; ++i) {
            const uint32_t bytes = (uint32_t)min(RPV, nv - i * RPV) * 16u;
            mbar_arrive_expect_tx(&bar[i], bytes);
            bulk_g2s(const_cast<uint4*>(slice) + (size_t)i * RPV, R.gvec + v0 + (size_t)i * RPV, bytes, &bar[i]);
        }
        ctl->err = 0;
        ctl->thr = f_ninf();
        ctl->kn = 0;
    }
    // the history and (rank 0) the penalty table, asynchronously, before the row's parameters are known
    const int64_t* hrow = p.hist ? p.hist + (int64_t)r * p.hstride : nullptr;
    const float* alpha = p.alpha ? p.alpha + (int64_t)r * p.alpha_stride : nullptr;
    if (hrow && p.W > 0) {
        for (int j = tid; j < p.W; j += NT) cp_async8(&hstage[j], &hrow[j]);
        if (alpha && lead)
            for (int j = tid; j < p.alpha_len; j += NT) cp_async4(&atab[j], &alpha[j]);
    }

    // ---------------- row parameters and mode
    const int64_t step = p.steps ? p.steps[r] : 0;
    const bool is_live = (p.active ? p.active[r] != 0 : true) && !(p.finished ? p.finished[r] != 0 : false);
    const bool hf = SEM >= 0 ? SEM == B2S_SEM_HF : p.sem == B2S_SEM_HF;
    const float T = p.rT ? p.rT[r] : p.T;
    const float top_p = p.rP ? p.rP[r] : p.top_p;
    const int top_k = p.rK ? p.rK[r] : p.top_k;
    const bool eos_ok = p.eos >= 0 && p.eos < V;
    const int64_t min_new = p.rminn ? p.rminn[r] : p.min_new, max_new = p.rmaxn ? p.rmaxn[r] : p.max_new;
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
    const bool topk_only = (p.flags & B2S_FLAG_TOPK_ONLY) != 0;
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
    R.pref = pref;
    R.htv = htv;
    R.censor = censor ? p.eos : -1;
    if (use_ht) {
        for (uint32_t g = tid; g < p.bitwords / 4; g += NT) reinterpret_cast<uint4*>(bits)[g] = make_uint4(0u, 0u, 0u, 0u);
        if (lead)
            for (int d = tid; d < p.hcap; d += NT) hcnt[d] = 0u;
    }
    // rank 0: the elements outside the 16-byte interior, one per lane of the last warp's lanes 16..31 (head in
    // 16..23, tail in 24..31; a row with no interior vector has at most 15 elements, all in lanes 16..31)
    int edge_i = -1;
    float edge_x = 0.0f;
    if (lead && tid >= NT - 16) {
        const int t = tid - (NT - 16);
        const bool whole = R.nvec == 0;
        const int i = (whole || t < 8) ? t : R.e0 + R.nvec * EPV + (t - 8);
        if ((!whole && t < 8) ? i < R.nh : i < V) {
            edge_i = i;
            edge_x = Elem<E>::gld(R.rowp, i);
        }
    }
    cp_async_wait_all();
    __syncthreads();  // the history has landed; the mbarriers are initialised

    auto hist_id = [&](int j) -> int {
        const int64_t hv = hstage[j];
        return (hv >= 0 && hv < V) ? (int)hv : -1;
    };
    const uintptr_t row_lo = reinterpret_cast<uintptr_t>(R.rowp), row_hi = row_lo + (uintptr_t)V * ES;
    // rank 0: the raw 4-byte word holding each history id's value, gathered from global memory under the copies
    if (pen_hist && lead)
        for (int j = tid; j < min(p.W, HPT * NT); j += NT) {
            const int id = hist_id(j);
            if (id < 0) continue;
            const uintptr_t wa = (row_lo + (uintptr_t)id * ES) & ~(uintptr_t)3;
            if (wa >= row_lo && wa + 4 <= row_hi) cp_async4(&hraw[j], reinterpret_cast<const void*>(wa));
        }
    int hd = 0;  // distinct history ids (the censored EOS included), rank 0
    if (use_ht) {
        if (pen_hist)
            for (int j = tid; j < p.W; j += NT) {
                const int id = hist_id(j);
                if (id < 0) {
                    if (hstage[j] >= 0 && lead) set_status(p, B2S_STATUS_HISTORY_RANGE);
                    continue;
                }
                atomicOr(&bits[id >> 5], 1u << (id & 31));
            }
        if (censor && tid == 0) atomicOr(&bits[p.eos >> 5], 1u << (p.eos & 31));
        __syncthreads();
        if (lead) {
            // rank of an id = the distinct ids below it: exclusive prefix of the popcounts of 4-word groups
            const int G = (int)p.bitwords >> 2;
            const int gpt = (G + NT - 1) / NT;
            const int g0 = min(G, tid * gpt), g1 = min(G, g0 + gpt);
            const uint4* b4 = reinterpret_cast<const uint4*>(bits);
            int cnt = 0;
            for (int g = g0; g < g1; ++g) {
                const uint4 q = b4[g];
                cnt += __popc(q.x) + __popc(q.y) + __popc(q.z) + __popc(q.w);
            }
            int base = block_excl_scan_i(cnt, ctl->red_i, &hd);
            for (int g = g0; g < g1; ++g) {
                pref[g] = (uint16_t)base;
                const uint4 q = b4[g];
                base += __popc(q.x) + __popc(q.y) + __popc(q.z) + __popc(q.w);
            }
            __syncthreads();
            if (pen_hist)
                for (int j = tid; j < p.W; j += NT) {
                    const int id = hist_id(j);
                    if (id < 0) continue;
                    const int rk = R.rank(id);
                    atomicAdd(&hcnt[rk], 1u);
                    hid[rk] = id;
                    hpos[rk] = j;
                }
            if (censor && tid == 0) hid[R.rank(p.eos)] = p.eos;
        }
    }

    // ---------------- the slice lands piece by piece: each thread's maximum of its share of every piece
    float tm[RMAXP];
    bool timed_out = false;
#pragma unroll
    for (int pc = 0; pc < RMAXP; ++pc) {
        tm[pc] = f_ninf();
        if (pc < npc) {
            if (!mbar_wait_bounded(&bar[pc], 0u, WAIT_NS)) timed_out = true;
            const int n = min(RPV, nv - pc * RPV);
            const uint4* s = slice + (size_t)pc * RPV;
            float m = f_ninf();
            if (tid < n) m = Elem<E>::vmax(s[tid]);
            if (tid + NT < n) m = fmaxf(m, Elem<E>::vmax(s[tid + NT]));
            tm[pc] = m;
        }
    }
    if (timed_out) {
        atomicOr(&ctl->err, ERR_TIMEOUT);
        set_status(p, B2S_STATUS_WAIT_TIMEOUT);
    }
    // rank 0: the history ids' processed values, once their raw words have landed
    cp_async_wait_all();
    __syncthreads();
    if (lead) {
        if (pen_hist) {
            for (int d = tid; d < hd; d += NT) {
                const int id = hid[d];
                if (censor && id == p.eos) {
                    htv[d] = f_ninf();
                    continue;
                }
                const int j = hpos[d];
                const uintptr_t ea = row_lo + (uintptr_t)id * ES, wa = ea & ~(uintptr_t)3;
                float x;
                if (j < HPT * NT && wa >= row_lo && wa + 4 <= row_hi) {
                    const uint32_t w = __float_as_uint(hraw[j]);
                    x = ES == 4 ? __uint_as_float(w) : bf16_bits_to_f((uint16_t)(w >> (8 * (unsigned)(ea - wa))));
                } else {
                    x = Elem<E>::gld(R.rowp, id);
                }
                htv[d] = hist_proc_value(p, atab, hf, false, T, (int)hcnt[d], x);
            }
        } else if (censor && tid == 0) {
            htv[R.rank(p.eos)] = f_ninf();
        }
    }

    // ---------------- candidates of this CTA's slice
    const bool cand_path = mode == MODE_FILTER && k <= KFAST && !(p.flags & B2S_FLAG_FORCE_GENERAL) && T >= 1e-6f &&
                           T <= 1e6f;
    bool ovf = !cand_path;
    float tau_low = f_inf();
    auto margin = [](float t) { return t - fmaxf(fabsf(t) * 9.5367431640625e-7f, 1e-30f); };
    const int seg = p.lcap / NWARP;
    const int hshare = p.ltot / CL;  // this CTA's share of rank 0's merged list
    float* wv = cand_v + (tid >> 5) * seg;
    int* wi = cand_i + (tid >> 5) * seg;
    int wn = 0;  // this warp's candidates (same in every lane)
    auto seg_reserve = [&](int cnt) {
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const int first = wn + incl - cnt;
        wn += __shfl_sync(0xffffffffu, incl, 31);
        return first;
    };
    auto place = [&](float x, int id, int pos) {
        if (pos < seg) {
            wv[pos] = x;
            wi[pos] = id;
        }
    };
    // global element index of element 0 of vector `v` of this slice
    auto elem_of = [&](int v) { return R.e0 + (v0 + v) * EPV; };
    if (cand_path) {
        // this thread's largest value over its shares that hold no history id (each such maximum is a distinct
        // non-history element, so the k-th largest of them bounds the slice's k-th largest from below)
        float tmax_nh = f_ninf();
#pragma unroll
        for (int pc = 0; pc < RMAXP; ++pc) {
            if (pc < npc) {
                const int n = min(RPV, nv - pc * RPV);
                const int va = pc * RPV + tid, vb = va + NT;
                uint32_t hb = 0u;
                if (tid < n) hb |= R.hbits(elem_of(va), EPV);
                if (tid + NT < n) hb |= R.hbits(elem_of(vb), EPV);
                if (!hb) tmax_nh = fmaxf(tmax_nh, tm[pc]);
            }
        }
        if (edge_i >= 0 && !R.hbit(edge_i)) tmax_nh = fmaxf(tmax_nh, edge_x);
        const int jw = (k + NWARP - 1) / NWARP;
        float v = tmax_nh;
        for (int t = 0; t < jw; ++t) {
            const float mj = warp_max(v);
            const unsigned who = __ballot_sync(0xffffffffu, v == mj);
            if (who && lane == __ffs(who) - 1) v = f_ninf();
            if (lane == 0) kv[(tid >> 5) * jw + t] = mj;
        }
    }
    __syncthreads();
    if (cand_path) {
        const int ng = NWARP * ((k + NWARP - 1) / NWARP);
        if (tid < ng) {
            const float x = kv[tid];
            int gt = 0, eq = 0;
            for (int j = 0; j < ng; ++j) {
                const float y = kv[j];
                gt += y > x;
                eq += y == x;
            }
            if (x > f_ninf() && gt < k && k <= gt + eq) ctl->thr = x;
        }
    }
    __syncthreads();
    if (cand_path) {
        const float t0 = ctl->thr;
        if (nv == 0 && !lead) {
            tau_low = f_inf();  // an empty slice has nothing to hand over
        } else if (!(t0 > f_ninf()) || t0 == f_inf() || R.f(t0) == f_inf()) {
            ovf = true;
        } else {
            tau_low = margin(t0);
        }
    }
    if (cand_path && !ovf) {
        // pass 2 over the resident slice: shares whose maximum clears tau; non-history elements >= tau_low
#pragma unroll
        for (int pc = 0; pc < RMAXP; ++pc) {
            if (pc < npc) {
                const bool hit = tm[pc] >= tau_low;
                if (__any_sync(0xffffffffu, hit)) {
                    const int n = min(RPV, nv - pc * RPV);
                    uint4 q[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
                    uint32_t hm = 0u;
                    int vv[2] = {pc * RPV + tid, pc * RPV + tid + NT};
                    if (hit) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            if (vv[h] - pc * RPV < n) {
                                q[h] = slice[vv[h]];
                                if (Elem<E>::vmax(q[h]) >= tau_low) {
                                    const uint32_t hb = R.hbits(elem_of(vv[h]), EPV);
#pragma unroll
                                    for (int j = 0; j < EPV; ++j)
                                        if (Elem<E>::at(q[h], j) >= tau_low && !((hb >> j) & 1u)) hm |= 1u << (h * EPV + j);
                                }
                            }
                        }
                    }
                    int pos = seg_reserve(__popc(hm));
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t m = (hm >> (h * EPV)) & ((1u << EPV) - 1u);
                        while (m) {
                            const int j = __ffs(m) - 1;
                            m &= m - 1u;
                            place(Elem<E>::at(q[h], j), elem_of(vv[h]) + j, pos++);
                        }
                    }
                }
            }
        }
        if ((tid >> 5) == NWARP - 1) {  // the ragged head / tail (rank 0)
            const bool eh = edge_i >= 0 && edge_x >= tau_low && !R.hbit(edge_i);
            const int pos = seg_reserve(eh ? 1 : 0);
            if (eh) place(edge_x, edge_i, pos);
        }
    }
    if (lane == 0) ctl->wcnt[tid >> 5] = wn;
    __syncthreads();
    if (cand_path && !ovf)
        for (int w = 0; w < NWARP; ++w)
            if (ctl->wcnt[w] > seg) ovf = true;  // a warp's segment overflowed (heavy ties): full-row path
    // compaction: processed values of the candidates >= tau_low (rank 0 adds the history ids clearing f(tau_low))
    int n = 0;
    if (cand_path && !ovf) {
        const float tl = tau_low;
        for (int i = tid; i < p.lcap; i += NT) {
            if (i % seg < ctl->wcnt[i / seg] && cand_v[i] >= tl) {
                const int pos = atomicAdd(&ctl->kn, 1);
                if (pos < hshare) {
                    kv[pos] = R.f(cand_v[i]);
                    ki[pos] = cand_i[i];
                }
            }
        }
        if (lead && use_ht) {
            const float p_low = R.f(tl);
            for (int d = tid; d < hd; d += NT) {
                if (htv[d] >= p_low) {
                    const int pos = atomicAdd(&ctl->kn, 1);
                    if (pos < hshare) {
                        kv[pos] = htv[d];
                        ki[pos] = hid[d];
                    }
                }
            }
        }
        __syncthreads();
        n = ctl->kn;
        if (n > hshare) ovf = true;
    }

    // ---------------- the other CTAs hand their lists to rank 0 (positions [c * hshare, c * hshare + n) of its list)
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
            if (tid == 0) *cl.map_shared_rank(&ctl->rx_n[crank], 0) = bad ? -1 : n;
        }
        cl.sync();  // every list is in rank 0's shared memory
        if (!lead) {
            if (ctl->err && tid == 0)
                for (int i = 0; i < npc; ++i) mbar_wait_bounded(&bar[i], 0u, WAIT_NS);
            return;
        }
        if (cand_path && !ovf) {
            // close the gaps: rank c's items move down behind the ones before them
            int off = n;
            for (int c = 1; c < CL; ++c) {
                const int nc = ctl->rx_n[c];
                if (nc < 0) {
                    ovf = true;
                    break;
                }
                for (int i = tid; i < nc; i += NT) {  // staged: the destination may overlap the source
                    sv[i] = kv[c * hshare + i];
                    si[i] = ki[c * hshare + i];
                }
                __syncthreads();
                for (int i = tid; i < nc; i += NT) {
                    kv[off + i] = sv[i];
                    ki[off + i] = si[i];
                }
                __syncthreads();
                off += nc;
            }
            n = off;
        }
    }

    // ---------------- rank 0: the row's token
    const bool row_err = ctl->err != 0;
    float thr = f_ninf();
    int64_t token = V - 1;
    float lse = 0.0f;
    if (mode == MODE_FILTER && cand_path && !ovf && n < k) ovf = true;
    if (mode == MODE_FILTER && hf && !row_err) {
        // full-row logsumexp of the processed values (talker_sampler.py:112), from the resident row (one CTA per
        // row for hf): the same thread layout as row_visit, so the same fp64 partial sums
        float lm = f_ninf();
        if (cand_path && !ovf) {
            for (int i = tid; i < n; i += NT) lm = fmaxf(lm, kv[i]);
        } else {
            for (int v = tid; v < nv; v += NT) {
                const uint4 q = slice[v];
#pragma unroll
                for (int j = 0; j < EPV; ++j) lm = fmaxf(lm, R.P(elem_of(v) + j, Elem<E>::at(q, j)));
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
#pragma unroll
            for (int j = 0; j < EPV; ++j)
                sacc += (double)b2s_expf(__fsub_rn(R.P(elem_of(v) + j, Elem<E>::at(q, j)), mu));
        }
        if (tid == 0)
            for (int i = 0; i < R.nh; ++i) sacc += (double)b2s_expf(__fsub_rn(R.P(i, Elem<E>::gld(R.rowp, i)), mu));
        if (tid == 1)
            for (int i = R.e0 + R.nvec * EPV; i < V; ++i)
                sacc += (double)b2s_expf(__fsub_rn(R.P(i, Elem<E>::gld(R.rowp, i)), mu));
        lse = __fadd_rn((float)log((double)(float)block_sum(sacc, ctl->red_d)), mu);
    }
    bool full = mode == MODE_FULL;
    if (mode == MODE_FILTER && !row_err) {
        if (cand_path && !ovf) {
            float* cv = kv;
            int* ci = ki;
            float* xv = cand_v;
            int* xi = cand_i;
            if (n > 256) {
                // narrow to the items >= the k-th largest processed value (ties kept)
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
            token = list_sample(cv, ci, n, k, hf, lse, top_p, p.min_keep, topk_only, true,
                                (hf && masked_eos) ? p.eos : -1, ctl->u, V, vals, xv, xi, sv, si, sc, thr);
        } else {
            // the exact full-row path, from global memory
            const uint32_t kth = row_kth_key<E>(R, k, hist, ctl);
            thr = exact_threshold<E>(R, kth, k, hf, lse, top_p, p.min_keep, topk_only, vals, ctl);
            full = true;
        }
    }
    if (mode == MODE_FORCED) token = eos_ok ? (int64_t)p.eos : (int64_t)(V - 1);
    if (full && !row_err) {
        const bool filt = mode == MODE_FILTER;
        const int drop = (hf && masked_eos) ? p.eos : -1;
        token = ordered_draw<E>(R, [&](int i, float P) { return i != drop && (!filt || P >= thr); }, ctl->u, ctl);
    }

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
