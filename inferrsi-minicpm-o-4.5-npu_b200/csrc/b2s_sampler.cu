// B200 (sm_100a) streaming sampling kernel, the greedy argmax, the standalone penalty and uniform kernels, and the
// C-ABI launchers of include/b2s_sampler.h (the row-resident kernel is in b2s_resident.cu, the vocabulary-shard
// merge and resolve in b2s_shard.cu).
//
// Streaming kernel: one 512-thread CTA owns one logits row at a time (a loop over rows when the batch is larger than
// the grid; over a row's frames for b2s_sample_frames).  The row's 16-byte-aligned interior streams through
// registers in 32 KB chunks (4 x 16 bytes per thread, two register buffers in turn, plain loads kept out of L1); the
// ragged head and tail are single loads.  Per row:
//
//   prologue: the history ids and penalty table by cp.async; a bitmap of the history ids, the rank of each distinct
//             id from a prefix of the bitmap's group popcounts, its count, and per-thread masks of the chunk shares
//             that hold one;
//   pass 1:   each (chunk, thread) share's maximum, kept in shared memory;
//   tau:      the k-th largest of the warps' ceil(k/16) largest per-thread maxima over shares without a history id
//             (a lower bound of the row's k-th largest non-history value);
//   pass 2:   the shares whose maximum clears tau are re-read from L2 (listed per warp, dealt over its lanes); every
//             non-history element >= tau goes to the candidate list, history ids by their processed values;
//   list:     top-k values, top-p cut, value threshold and the inverse-CDF draw in vocabulary order (b2s_list.cuh);
//   exact:    rows the list cannot serve (k > 128, overflowing lists, NaN or unusable tau) take a radix select of the
//             k-th processed key over the row and an ordered scan; hf frame-0 rows and draw() take the ordered scan;
//   state:    token, steps, finished and the shifted history (in place when the outputs alias the inputs).
//
// For batches of at most half the SMs with a penalty history, the rows of the thinker shape run as CTA pairs: the
// second CTA builds the history structures beside pass 1 and hands them over through distributed shared memory.
// Selection runs on raw values: outside the history the processed value is fl(x / T), monotone in x.  No block in
// this file waits on another block except at the hardware cluster barrier.
#include "b2s_row.cuh"
#include "b2s_head.cuh"

#include <cooperative_groups.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "../../include/b2s_sampler.h"

namespace cg = cooperative_groups;

namespace b2s {

// The whole row program; with a grid smaller than the batch each CTA loops over rows.
// LEAN: a launch with neither processed output nor vocabulary-shard output (the decode step); the code of
// those outputs is left out of that instantiation.  SEM >= 0: the launch's semantics fixed at compile time, so
// the other orders' code is left out too (only the omni decode step uses it: an hf-only build measured slower
// on the batched Talker shape); -1: read from the parameters.
template <typename E, bool LEAN, int SEM>
__global__ void __launch_bounds__(NT, 1) sample_kernel(const Params p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const bool has_proc = !LEAN && p.proc != nullptr;  // processed-logits output
    int32_t* const cout_n = LEAN ? nullptr : p.cout_n;  // vocabulary-shard output
    const int tid = threadIdx.x, lane = tid & 31;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
    uint32_t* bits = reinterpret_cast<uint32_t*>(smem + p.off_bits);
    uint16_t* pref = reinterpret_cast<uint16_t*>(smem + p.off_pref);
    uint32_t* hcnt = reinterpret_cast<uint32_t*>(smem + p.off_hcnt);  // occurrences of each distinct id, by rank
    int* hid = reinterpret_cast<int*>(smem + p.off_hid);              // the id of each rank
    int* hpos = reinterpret_cast<int*>(smem + p.off_hpos);            // a history position of each rank
    float* htv = reinterpret_cast<float*>(smem + p.off_htv);
    unsigned long long* smask = reinterpret_cast<unsigned long long*>(smem + p.off_smask);  // [thread] chunk bits
    int64_t* hstage = reinterpret_cast<int64_t*>(smem + p.off_hstage);
    float* hraw = reinterpret_cast<float*>(smem + p.off_hraw);  // raw words of the history positions
    float* tmaxc = reinterpret_cast<float*>(smem + p.off_tmaxc);  // [chunk][thread] maximum of the pass 1
    float* atab = reinterpret_cast<float*>(smem + p.off_atab);
    float* cand_v = reinterpret_cast<float*>(smem + p.off_cand);
    int* cand_i = reinterpret_cast<int*>(smem + p.off_candi);
    float* kv = reinterpret_cast<float*>(smem + p.off_lst);
    int* ki = reinterpret_cast<int*>(kv + p.lcap);
    float* sv = kv + 2 * p.lcap;
    int* si = reinterpret_cast<int*>(kv + 3 * p.lcap);
    float* vals = reinterpret_cast<float*>(smem + p.off_vals);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + p.off_hist);
    constexpr int ES = Elem<E>::SZ, EPV = Elem<E>::EPV;
    const int V = p.V;
    const Scr sc{hist, ctl->rctl, &ctl->gather_n, &ctl->kn, &ctl->thr, ctl->red_d, ctl->red_f, ctl->red_i};
    pdl_wait_then_release();  // nothing global is read before the previous kernel of the stream is done

    // logits row of work item w: frame w / rows (p.fstride elements apart), row w % rows
    auto row_of = [&](int w) {
        return reinterpret_cast<const unsigned char*>(p.logits) +
               ((int64_t)(w / p.rows) * p.fstride + (int64_t)(w % p.rows) * p.lstride) * ES;
    };
    // 16-byte-aligned interior of work item w's row: head elements before it, vectors in it
    auto geometry = [&](int w, int& nh, int& nvec, const uint4*& gvec) {
        const unsigned char* rowp = row_of(w);
        const uintptr_t a = reinterpret_cast<uintptr_t>(rowp);
        const uintptr_t b = a + (uintptr_t)V * ES;
        const uintptr_t ace = (a + 15) & ~(uintptr_t)15, bfl = b & ~(uintptr_t)15;
        if (ace < bfl) {
            nh = (int)((ace - a) / ES);
            nvec = (int)((bfl - ace) / 16);
        } else {
            nh = V;
            nvec = 0;
        }
        gvec = reinterpret_cast<const uint4*>(ace);
    };
    // chunk c of a row's stream: vectors c * VPC + it * NT + tid, it < ITS, loaded straight into registers
    // (16-byte loads that skip L1; the row stays in L2 for any later pass); -inf past the row's end
    constexpr int ITS = VPC / NT;
    auto load_chunk_of = [&](const uint4* gvec, int nvec, int c, uint4* q) {
        const int vn = min(VPC, nvec - c * VPC);
        const uint4* g = gvec + (size_t)c * VPC;
#pragma unroll
        for (int it = 0; it < ITS; ++it) {
            const int vl = it * NT + tid;
            q[it] = vl < vn ? ldg_stream(g + vl) : make_uint4(Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG);
        }
    };
    // Two register buffers in turn: chunk c + 1 is in flight while chunk c is processed.  They are named,
    // never copied into one another, so a load that has not landed never stalls a register move.
    uint4 nq[ITS], nq2[ITS];  // even / odd chunks
    bool next_row_in = false;  // nq already holds chunk 0 of this CTA's next row

    // Two-CTA rows (p.csplit): the cluster's rank 1 stages the history, builds the bitmap, slice masks, ranks
    // and counts, gathers the history ids' raw values, and copies all of it into rank 0's shared memory,
    // while rank 0 streams pass 1.  They meet at a cluster barrier; rank 0 does the rest of the row.  A second
    // cluster barrier ends each row, so the helper never overwrites structures still in use.
    const bool split = p.csplit != 0;
    const bool helper = split && cg::this_cluster().block_rank() == 1;
    // Work items w = frame * rows + row.  With several frames (b2s_sample_frames) the grid has one CTA per row, so a
    // CTA takes its row's frames in order and the state each frame writes in place is the next frame's input.
    const int rstep = split ? (int)gridDim.x / 2 : (int)gridDim.x;
    const int nwork = p.rows * p.frames;
    for (int w = split ? (int)blockIdx.x / 2 : (int)blockIdx.x; w < nwork; w += rstep) {
        const int r = w % p.rows;
        // ---------------- geometry; the first chunk's loads go out before anything else
        Row<E> R;
        R.rowp = row_of(w);
        R.V = V;
        geometry(w, R.nh, R.nvec, R.gvec);
        R.e0 = R.nh;
        const int nchunks = (R.nvec + VPC - 1) / VPC;
        auto load_chunk = [&](int c, uint4* q) { load_chunk_of(R.gvec, R.nvec, c, q); };
        if (!helper) {
            if (!next_row_in && nchunks > 0) load_chunk(0, nq);
            if (nchunks > 1) load_chunk(1, nq2);
        }
        next_row_in = false;
        if (tid == 0) ctl->err = 0;
        // the history and the penalty table, asynchronously, before the row's parameters are known (a row that
        // turns out not to need them just does not read them)
        const int64_t* hrow = p.hist ? p.hist + (int64_t)r * p.hstride : nullptr;
        const float* alpha = p.alpha ? p.alpha + (int64_t)r * p.alpha_stride : nullptr;
        if (hrow && p.W > 0 && (!split || helper)) {  // two-CTA rows: the helper's copy arrives later
            for (int j = tid; j < p.W; j += NT) cp_async8(&hstage[j], &hrow[j]);
            if (alpha)
                for (int j = tid; j < p.alpha_len; j += NT) cp_async4(&atab[j], &alpha[j]);
        }

        // ---------------- row parameters and mode (global loads overlap the stream)
        const int64_t step = p.steps ? p.steps[r] : 0;
        const bool is_live = (p.active ? p.active[r] != 0 : true) && !(p.finished ? p.finished[r] != 0 : false);
        const bool identity = SEM >= 0 ? false : p.sem == B2S_SEM_IDENTITY;
        const bool hf = SEM >= 0 ? SEM == B2S_SEM_HF : p.sem == B2S_SEM_HF;
        const float T = p.rT ? p.rT[r] : p.T;
        const float top_p = p.rP ? p.rP[r] : p.top_p;
        const int top_k = p.rK ? p.rK[r] : p.top_k;
        const bool eos_ok = !identity && p.eos >= 0 && p.eos < V;
        const int64_t min_new = p.rminn ? p.rminn[r] : p.min_new, max_new = p.rmaxn ? p.rmaxn[r] : p.max_new;
        const bool masked_eos = eos_ok && step < min_new;
        int mode;
        if (!has_proc && !cout_n && !is_live) mode = MODE_SKIP;
        else if (identity) mode = MODE_FULL;
        else if (step >= max_new - 1) mode = MODE_FORCED;
        else if (hf && step <= 0) mode = MODE_FULL;
        else mode = MODE_FILTER;
        int k = 0;
        if (mode == MODE_FILTER) {
            k = min(max(top_k, max(p.min_keep, 1)), V);
            if (k > p.kbuf) {
                mode = MODE_FAIL;
                if (tid == 0) set_status(p, B2S_STATUS_TOPK_LIMIT);
            }
        }
        if (cout_n && mode != MODE_FILTER) mode = MODE_FAIL;
        const bool topk_only = (p.flags & B2S_FLAG_TOPK_ONLY) != 0;
        if (tid == 32) {  // one thread: the row's uniform (read after the next barrier)
            ctl->u = (p.rng == B2S_RNG_UNIFORM || !p.seeds) ? (p.uvals ? p.uvals[w] : 0.0f)
                     : p.rng == B2S_RNG_PHILOX ? uniform_philox(p.seeds[r], step, p.requests ? p.requests[r] : 0)
                                               : uniform_counter(p.seeds[r], step);
        }
        R.T = T;
        R.identity = identity;
        const bool pen_hist = mode == MODE_FILTER && p.W > 0 && hrow != nullptr;
        const bool censor = mode == MODE_FILTER && !hf && masked_eos;  // omni: EOS is -inf before anything else
        const bool use_ht = pen_hist || censor;
        R.bits = use_ht ? bits : nullptr;
        R.pref = pref;
        R.htv = htv;
        R.censor = censor ? p.eos : -1;

        // ---------------- prologue: once the staged history has landed, mark its ids in a bitmap and in
        // per-thread slice masks; rank the distinct ids and count them
        const bool own_hist = !split || helper;  // this CTA builds the history structures
        if (use_ht && own_hist) {
            for (uint32_t g = tid; g < p.bitwords / 4; g += NT) reinterpret_cast<uint4*>(bits)[g] = make_uint4(0u, 0u, 0u, 0u);
            for (int d = tid; d < p.hcap; d += NT) hcnt[d] = 0u;
        }
        if (own_hist) smask[tid] = 0ull;
        // the elements outside the 16-byte interior, one per lane of the last warp's lanes 16..31: the head
        // (at most 7) in lanes 16..23 and the tail (at most 7) in lanes 24..31 -- or, for a row with no
        // interior vector (under 32 bytes, so at most 15 elements), the whole row in lanes 16..31
        int edge_i = -1;
        float edge_x = 0.0f;
        if (tid >= NT - 16) {
            const int t = tid - (NT - 16);
            const bool whole = R.nvec == 0;
            const int i = (whole || t < 8) ? t : R.e0 + R.nvec * EPV + (t - 8);
            if ((!whole && t < 8) ? i < R.nh : i < V) {
                edge_i = i;
                edge_x = Elem<E>::gld(R.rowp, i);
            }
        }
        if (tid == 0) {
            ctl->thr = f_ninf();
            ctl->red_u[0] = 0u;
        }
        cp_async_wait_all();
        __syncthreads();
        // history id of position j (or -1 when it has no value here: PAD, another shard, out of range)
        auto hist_id = [&](int j) -> int {
            const int64_t hv = hstage[j];
            const int64_t id = hv - p.id_off;
            return (hv >= 0 && id >= 0 && id < V) ? (int)id : -1;
        };
        // raw value of history position j: the aligned 4-byte word holding it, copied asynchronously into
        // hraw[j] (positions tid + u * NT, u < HPT, one per chunk so the gathers do not queue up together)
        const uintptr_t row_lo = reinterpret_cast<uintptr_t>(R.rowp), row_hi = row_lo + (uintptr_t)V * ES;
        auto gather_hist = [&](int j) {
            if (!pen_hist || j >= p.W) return;
            const int id = hist_id(j);
            if (id < 0) return;
            const uintptr_t wa = (row_lo + (uintptr_t)id * ES) & ~(uintptr_t)3;
            if (wa >= row_lo && wa + 4 <= row_hi) cp_async4(&hraw[j], reinterpret_cast<const void*>(wa));
        };
        if (helper)  // all of them at once, under the marking and ranking below
            for (int u = 0; u < HPT; ++u) gather_hist(tid + u * NT);
        // interior element e lies in the pass-1 share of thread v % NT in chunk v / VPC (v: its vector)
        auto mark_slice = [&](int e) {
            const int rel = e - R.e0;
            if (rel < 0) return;
            const int v = rel / EPV;
            const int c = v / VPC;  // (the low word of smask[t] holds chunks 0..31)
            if (v < R.nvec && c < 64) atomicOr(reinterpret_cast<uint32_t*>(&smask[v % NT]) + (c >> 5), 1u << (c & 31));
        };
        int hd = 0;  // distinct history ids of the row (the censored EOS included)
        if (use_ht && own_hist) {
            if (pen_hist)
                for (int j = tid; j < p.W; j += NT) {
                    const int id = hist_id(j);
                    if (id < 0) {
                        // a vocabulary shard ignores ids of the other shards; an unsharded row flags ids >= vocab
                        if (hstage[j] >= 0 && !cout_n) set_status(p, B2S_STATUS_HISTORY_RANGE);
                        continue;
                    }
                    atomicOr(&bits[id >> 5], 1u << (id & 31));
                    mark_slice(id);
                }
            if (censor && tid == 0) {
                atomicOr(&bits[p.eos >> 5], 1u << (p.eos & 31));
                mark_slice(p.eos);
            }
            __syncthreads();
            // rank of an id = the distinct ids below it: exclusive prefix of the popcounts of the bitmap's
            // 4-word groups (contiguous groups per thread, 16-byte shared loads)
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
                    hid[rk] = id;  // every occurrence writes the same id
                    hpos[rk] = j;  // and one of them its position
                }
            if (censor && tid == 0) hid[R.rank(p.eos)] = p.eos;
            // hcnt / hid are read after the next barrier
        } else {
            __syncthreads();
        }
        // processed value of history id `id`, seen n times, with raw value x
        auto hist_value = [&](int id, int n, float x) {
            if (n >= p.alpha_len && n > 0) {
                set_status(p, B2S_STATUS_COUNT_LIMIT);
                n = p.alpha_len - 1;
            }
            const float a = n > 0 ? atab[n] : 1.0f;
            if (hf) return pen_a(__fdiv_rn(x, T), n, a);
            const float z = (censor && id == p.eos) ? f_ninf() : x;
            float v = pen_a(z, n, a);
            if (n > 0) {
                v = __fsub_rn(v, p.presence);
                v = __fsub_rn(v, __fmul_rn(p.frequency, (float)n));
            }
            return __fdiv_rn(v, T);
        };
        // processed values of the history ids (hcnt and the raw values gathered during pass 1)
        // (once per distinct id, with the raw value gathered at one of its positions)
        auto compute_htv = [&]() {
            if (pen_hist) {
                if (!split)
                    for (int u = nchunks; u < HPT; ++u) gather_hist(tid + u * NT);  // short rows
                cp_async_wait_all();
                __syncthreads();  // every thread's gathers have landed
                for (int d = tid; d < hd; d += NT) {
                    const int id = hid[d];
                    if (censor && id == p.eos) {  // omni: EOS is -inf (a history id or not)
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
                    htv[d] = hist_value(id, (int)hcnt[d], x);
                }
            } else if (censor && tid == 0) {
                htv[R.rank(p.eos)] = f_ninf();  // omni: EOS is -inf (no history ids)
            }
        };
        if (helper) {
            // the history's processed values too; then hand rank 0 what the rest of its row reads -- history
            // ids, bitmap, processed values and ids by rank, slice masks -- in 16-byte pieces (every region is
            // 16-byte aligned and padded).  Ranks and counts stay here: rank 0 reads those remotely, and only
            // on its rare full-row paths.
            compute_htv();
            __syncthreads();
            cg::cluster_group cl = cg::this_cluster();
            auto copy_region = [&](uint32_t off, uint32_t bytes) {
                uint4* dst = cl.map_shared_rank(reinterpret_cast<uint4*>(smem + off), 0);
                const uint4* src = reinterpret_cast<const uint4*>(smem + off);
                for (uint32_t i = tid; i < (bytes + 15u) / 16u; i += NT) dst[i] = src[i];
            };
            if (hrow && p.W > 0) copy_region(p.off_hstage, (uint32_t)p.W * 8u);
            if (use_ht) {
                copy_region(p.off_bits, p.bitwords * 4u);
                copy_region(p.off_htv, (uint32_t)hd * 4u);
                copy_region(p.off_hid, (uint32_t)hd * 4u);
            }
            copy_region(p.off_smask, NT * 8u);
            if (tid == 0) *cl.map_shared_rank(&ctl->hd_x, 0) = hd;
            cl.sync();  // the structures are in rank 0's shared memory
            cl.sync();  // rank 0 is done with this row
            continue;
        }

        // ---------------- candidate path, in two passes over the row.
        //   pass 1 (HBM, every element once): each thread's largest non-history value, and the largest value
        //           (history included) of each of its chunks, kept in shared memory;
        //   tau:    the k-th largest of the warps' ceil(k / 16) largest per-thread maxima -- k distinct
        //           non-history elements are >= tau, so tau is a lower bound of the row's k-th largest
        //           non-history raw value;
        //   pass 2 (L2, only the thread-chunks whose maximum clears tau): every non-history element >= tau, less
        //           a margin for collisions of fl(x / T), goes to the candidate list.
        const bool cand_path = mode == MODE_FILTER && k <= KFAST && !(p.flags & B2S_FLAG_FORCE_GENERAL) &&
                               T >= 1e-6f && T <= 1e6f && nchunks <= p.tmc_chunks;
        bool ovf = !cand_path;
        float tau_low = f_inf();
        auto margin = [](float t) { return t - fmaxf(fabsf(t) * 9.5367431640625e-7f, 1e-30f); };
        // Each warp appends to its own segment of the candidate list (seg entries at cand_v + warp * seg), with
        // a warp-uniform count in a register: no returning atomic.
        const int seg = p.lcap / NWARP;
        float* wv = cand_v + (tid >> 5) * seg;
        int* wi = cand_i + (tid >> 5) * seg;
        int wn = 0;  // this warp's candidates (same in every lane)
        // every lane of the warp calls it with its own count; returns the lane's first position
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
        // bit it * EPV + j: element j of vector it is >= tau_low and not a history id
        auto hit_mask = [&](const uint4* q, int cbase, int t) {
            uint32_t hm = 0u;
#pragma unroll
            for (int it = 0; it < ITS; ++it) {
                if (Elem<E>::vmax(q[it]) >= tau_low) {
                    const uint32_t hb = R.hbits(cbase + (it * NT + t) * EPV, EPV);
#pragma unroll
                    for (int j = 0; j < EPV; ++j)
                        if (Elem<E>::at(q[it], j) >= tau_low && !((hb >> j) & 1u)) hm |= 1u << (it * EPV + j);
                }
            }
            return hm;
        };
        static_assert(ITS >= 1 && ITS * NT == VPC, "whole vectors per thread per chunk");
        static_assert(ITS * EPV <= 32, "one mask bit per element of a thread's chunk share");
        // this thread's largest value over its chunk shares that hold no history id (a share that holds one
        // is left out whole: the value stays a lower bound of a distinct non-history element)
        float tmax_nh = f_ninf();
        if (cand_path) {
            const unsigned long long hmask = split ? 0ull : smask[tid];  // two-CTA rows: applied below
            // the bookkeeping of chunk c, once its maximum is known (its registers are refilled first)
            auto pass1_account = [&](int c, float vm) {
                if (!split && c < HPT) gather_hist(tid + c * NT);
                tmaxc[c * NT + tid] = vm;
                if (!split && !((hmask >> c) & 1ull)) tmax_nh = fmaxf(tmax_nh, vm);
            };
            // chunk c in nq (even) or nq2 (odd); each buffer is refilled as soon as its chunk's maximum is taken
            for (int c = 0; c < nchunks; c += 2) {
                const float vm0 = Elem<E>::template vmaxn<ITS>(nq);
                if (c + 2 < nchunks) load_chunk(c + 2, nq);
                pass1_account(c, vm0);
                if (c + 1 < nchunks) {
                    const float vm1 = Elem<E>::template vmaxn<ITS>(nq2);
                    if (c + 3 < nchunks) load_chunk(c + 3, nq2);
                    pass1_account(c + 1, vm1);
                }
            }
        } else if (!split) {
            for (int u = 0; u < HPT; ++u) gather_hist(tid + u * NT);
        }
        if (split) {
            // the helper's structures are complete: read them where they are (distributed shared memory)
            cg::cluster_group cl = cg::this_cluster();
            cl.sync();
            R.pref = cl.map_shared_rank(pref, 1);  // the ranks stayed with the helper
            hd = ctl->hd_x;
            if (cand_path) {
                const unsigned long long hm = smask[tid];
                for (int c = 0; c < nchunks; ++c)
                    if (!((hm >> c) & 1ull)) tmax_nh = fmaxf(tmax_nh, tmaxc[c * NT + tid]);
            }
        }
        if (cand_path) {
            // the ragged head / tail (one element in each of the last warp's lanes 16..31)
            if (edge_i >= 0 && !R.hbit(edge_i)) tmax_nh = fmaxf(tmax_nh, edge_x);
            // the warp's jw largest per-thread maxima (distinct lanes): take the maximum out jw times
            const int jw = (k + NWARP - 1) / NWARP;
            float v = tmax_nh;
            for (int t = 0; t < jw; ++t) {
                const float mj = warp_max(v);
                const unsigned who = __ballot_sync(0xffffffffu, v == mj);
                if (who && lane == __ffs(who) - 1) v = f_ninf();
                if (lane == 0) kv[(tid >> 5) * jw + t] = mj;
            }
        }
        // this row's stream is done: start the first chunk of the CTA's next row
        if (w + rstep < nwork) {
            int nh2, nvec2;
            const uint4* g2;
            geometry(w + rstep, nh2, nvec2, g2);
            if (nvec2 > 0) load_chunk_of(g2, nvec2, 0, nq);
            next_row_in = true;
        }
        __syncthreads();
        if (cand_path) {
            // tau = the k-th largest of the gathered values (each one a distinct non-history element)
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
            if (!(t0 > f_ninf()) || t0 == f_inf() || R.f(t0) == f_inf()) {
                ovf = true;
            } else {
                tau_low = margin(t0);
            }
        }
        bool htv_done = false;
        if (cand_path && !ovf) {
            // pass 2: the (chunk, thread) shares whose maximum clears tau are re-read from L2.  Each warp first
            // lists its hit shares and deals them out over its lanes, two per lane per round, so a warp needs a
            // single round trip unless it holds more than 64 hits, however they fall among its threads.
            uint64_t hits = 0ull;
            for (int c = 0; c < nchunks; ++c) hits |= (uint64_t)(tmaxc[c * NT + tid] >= tau_low) << c;
            const int wcap = p.lcap / 2;  // kv, ki, sv, si (16 * lcap bytes, free until compaction) per warp
            uint16_t* const wl = reinterpret_cast<uint16_t*>(kv) + (tid >> 5) * wcap;
            const int cnt = __popcll((long long)hits);
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            const int tot = __shfl_sync(0xffffffffu, incl, 31);
            const int nh = tot <= wcap ? tot : 0;  // more (flat rows): the warp's segment is flagged as overflowed
            if (tot <= wcap) {
                int pos = incl - cnt;
                for (uint64_t h = hits; h; h &= h - 1ull)
                    wl[pos++] = (uint16_t)(((__ffsll((long long)h) - 1) << 9) | tid);
            }
            __syncwarp();
            static_assert(NT == 512, "list entries pack (chunk << 9) | thread");
            // list entry i: its share's global position and owner thread; its vectors into q
            auto load_share = [&](int i, uint4* q, int& cbase, int& t) {
                int c = -1;
                t = 0;
                if (i < nh) {
                    const int e = wl[i];
                    c = e >> 9;
                    t = e & (NT - 1);
                }
                cbase = c >= 0 ? R.e0 + c * VPC * EPV : -1;
                const int vn = c >= 0 ? min(VPC, R.nvec - c * VPC) : 0;
#pragma unroll
                for (int it = 0; it < ITS; ++it) {
                    const int vl = it * NT + t;
                    q[it] = vl < vn ? __ldg(R.gvec + (size_t)c * VPC + vl)
                                    : make_uint4(Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG);
                }
            };
            auto place_all = [&](const uint4* q, uint32_t hm, int cbase, int t, int pos) {
#pragma unroll
                for (int it = 0; it < ITS; ++it) {
                    uint32_t m = (hm >> (it * EPV)) & ((1u << EPV) - 1u);
                    while (m) {
                        const int j = __ffs(m) - 1;
                        m &= m - 1u;
                        place(Elem<E>::at(q[it], j), cbase + (it * NT + t) * EPV + j, pos++);
                    }
                }
            };
            int i1 = lane, i2 = lane + 32;
            int cb1, cb2, t1, t2;
            uint4 q1[ITS], q2[ITS];
            load_share(i1, q1, cb1, t1);
            load_share(i2, q2, cb2, t2);
            // the history values are computed while the first round's loads are in flight
            if (!split) compute_htv();
            htv_done = true;
            for (;;) {
                const uint32_t h1 = cb1 >= 0 ? hit_mask(q1, cb1, t1) : 0u;
                const uint32_t h2 = cb2 >= 0 ? hit_mask(q2, cb2, t2) : 0u;
                const int pos = seg_reserve(__popc(h1) + __popc(h2));
                if (h1) place_all(q1, h1, cb1, t1, pos);
                if (h2) place_all(q2, h2, cb2, t2, pos + __popc(h1));
                i1 += 64;
                i2 += 64;
                if (i1 - lane >= nh) break;  // the round's first entry: the same in every lane
                load_share(i1, q1, cb1, t1);
                load_share(i2, q2, cb2, t2);
            }
            if (tot > wcap) wn = seg + 1;
            // the ragged head / tail
            if ((tid >> 5) == NWARP - 1) {
                const bool eh = edge_i >= 0 && edge_x >= tau_low && !R.hbit(edge_i);
                const int pos = seg_reserve(eh ? 1 : 0);
                if (eh) place(edge_x, edge_i, pos);
            }
        }
        if (!htv_done && !split) compute_htv();
        if (lane == 0) ctl->wcnt[tid >> 5] = wn;
        if (tid == 0) ctl->kn = 0;  // the candidate count of the compaction below
        __syncthreads();
        const bool row_err = ctl->err != 0;
        if (cand_path && !ovf)
            for (int w = 0; w < NWARP; ++w)
                if (ctl->wcnt[w] > seg) ovf = true;  // a warp's segment overflowed (heavy ties)

        // state epilogue (tok_drawn == PAD: the row failed on the device -> PAD out, state unchanged)
        auto finish_row = [&](int64_t tok_drawn) {
            const bool adv = is_live && tok_drawn != PAD;
            const int64_t tok = adv ? tok_drawn : PAD;
            if (tid == 0) {
                if (p.tokens) p.tokens[w] = tok;
                if (p.steps_out) p.steps_out[r] = step + (adv ? 1 : 0);
                if (p.fin_out) {
                    const bool f0 = p.finished ? p.finished[r] != 0 : false;
                    p.fin_out[r] = (uint8_t)(f0 || (adv && tok == (int64_t)p.eos));
                }
            }
            if (p.hist_out && p.W > 0) {
                int64_t* ho = p.hist_out + (int64_t)r * p.hostride;
                // the old row was staged before any write (history_out may alias history)
                for (int j = tid; j < p.W; j += NT) ho[j] = adv ? (j + 1 < p.W ? hstage[j + 1] : tok) : hstage[j];
            }
        };

        float thr = f_ninf();
        int64_t token = V - 1;
        bool exact = mode == MODE_FILTER;
        bool full = mode == MODE_FULL;
        float lse = 0.0f;
        const bool wants_draw = p.tokens || p.hist_out || p.steps_out || p.fin_out;

        // ---------------- candidate list: the items >= the final tau (processed), plus the history ids whose
        // processed value clears f(tau)
        // (compacted into kv / ki, which then hold the list; cand_v / cand_i become scratch)
        int n = 0;
        float* cv = kv;
        int* ci = ki;
        float* xv = cand_v;
        int* xi = cand_i;
        if (cand_path && !ovf && !row_err) {
            const float tl = tau_low;
            for (int i = tid; i < p.lcap; i += NT) {
                if (i % seg < ctl->wcnt[i / seg] && cand_v[i] >= tl) {
                    const int pos = atomicAdd(&ctl->kn, 1);
                    if (pos < p.lcap) {
                        kv[pos] = R.f(cand_v[i]);
                        ki[pos] = cand_i[i];
                    }
                }
            }
            if (use_ht) {
                const float p_low = R.f(tl);
                for (int d = tid; d < hd; d += NT) {
                    if (htv[d] >= p_low) {
                        const int pos = atomicAdd(&ctl->kn, 1);
                        if (pos < p.lcap) {
                            kv[pos] = htv[d];
                            ki[pos] = hid[d];
                        }
                    }
                }
            }
            __syncthreads();
            n = ctl->kn;
            if (n > p.lcap || n < k) ovf = true;
        }

        if (mode == MODE_FILTER && hf && !row_err) {
            // full-row logsumexp of the penalised values (talker_sampler.py:112); the row maximum is a candidate
            float lm = f_ninf();
            if (cand_path && !ovf) {
                for (int i = tid; i < n; i += NT) lm = fmaxf(lm, cv[i]);
            } else {
                row_visit<E>(R, [&](int i, float x) { lm = fmaxf(lm, R.P(i, x)); });
            }
            const float m = block_max(lm, ctl->red_f);
            const float mu = (m == f_inf() || m == f_ninf()) ? 0.0f : m;
            double sacc = 0.0;
            row_visit<E>(R, [&](int i, float x) { sacc += (double)b2s_expf(__fsub_rn(R.P(i, x), mu)); });
            lse = __fadd_rn((float)log((double)(float)block_sum(sacc, ctl->red_d)), mu);
        }

        // ---------------- candidate path: finish from the candidate list
        if (cand_path && !ovf && !row_err) {
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
                // the narrowed list is the list now; the old one is scratch
                float* tv = cv;
                int* ti = ci;
                cv = xv;
                ci = xi;
                xv = tv;
                xi = ti;
            }
            exact = false;
            if (cout_n) {
                // vocabulary shard: every candidate above this shard's k-th value (fewer than k <= cap), then the ones
                // equal to it while room is left; the count is of every element >= the k-th value
                list_topk_values(cv, n, k, vals, sc);
                const float kth = vals[k - 1];
                if (tid == 0) ctl->kn = 0;
                __syncthreads();
                for (int pass = 0; pass < 2; ++pass) {
                    for (int i = tid; i < n; i += NT) {
                        if (pass == 0 ? cv[i] > kth : cv[i] == kth) {
                            const int pos = atomicAdd(&ctl->kn, 1);
                            if (pos < p.ccap) {
                                p.cout_v[(int64_t)r * p.ccap + pos] = cv[i];
                                p.cout_i[(int64_t)r * p.ccap + pos] = (int32_t)(ci[i] + p.id_off);
                            }
                        }
                    }
                    __syncthreads();
                }
                if (tid == 0) cout_n[r] = ctl->kn;
            } else {
                const int64_t t = list_sample(cv, ci, n, k, hf, lse, top_p, p.min_keep, topk_only, wants_draw,
                                              (hf && masked_eos) ? p.eos : -1, ctl->u, V, vals, xv, xi, sv, si, sc,
                                              thr);
                if (wants_draw) token = t;
            }
        }

        // ---------------- exact path: radix select of the k-th processed key over the row
        if (exact && !row_err && mode == MODE_FILTER) {
            const uint32_t kth = row_kth_key<E>(R, k, hist, ctl);
            if (cout_n) {
                // as above: the elements above the k-th key first, then the ones equal to it
                if (tid == 0) ctl->kn = 0;
                __syncthreads();
                for (int pass = 0; pass < 2; ++pass) {
                    row_visit<E>(R, [&](int i, float x) {
                        const float P = R.P(i, x);
                        if (pass == 0 ? okey(P) > kth : okey(P) == kth) {
                            const int pos = atomicAdd(&ctl->kn, 1);
                            if (pos < p.ccap) {
                                p.cout_v[(int64_t)r * p.ccap + pos] = P;
                                p.cout_i[(int64_t)r * p.ccap + pos] = (int32_t)(i + p.id_off);
                            }
                        }
                    });
                    __syncthreads();
                }
                if (tid == 0) cout_n[r] = ctl->kn;
            } else {
                thr = exact_threshold<E>(R, kth, k, hf, lse, top_p, p.min_keep, topk_only, vals, ctl);
                full = true;  // draw by the ordered scan over the elements >= thr
            }
        }

        if (mode == MODE_FORCED) token = eos_ok ? (int64_t)p.eos : (int64_t)(V - 1);
        if (full && !row_err && wants_draw) {
            const bool filt = mode == MODE_FILTER;
            const int drop = (hf && masked_eos) ? p.eos : -1;
            token = ordered_draw<E>(R, [&](int i, float P) { return i != drop && (!filt || P >= thr); }, ctl->u, ctl);
        }

        // ---------------- processed row
        if (has_proc && !cout_n) {
            float* out = p.proc + (int64_t)r * p.pstride;
            const int drop = (hf && masked_eos) ? p.eos : -1;
            if (mode == MODE_FORCED) {
                for (int i = tid; i < V; i += NT) out[i] = (eos_ok && i == p.eos) ? 0.0f : f_ninf();
            } else {
                const bool filt = mode == MODE_FILTER;
                row_visit<E>(R, [&](int i, float x) {
                    const float P = R.P(i, x);
                    out[i] = (i == drop || (filt && !(P >= thr))) ? f_ninf() : P;
                });
            }
        }
        if (cout_n && (mode != MODE_FILTER || row_err) && tid == 0) cout_n[r] = -1;
        if (!cout_n) finish_row((row_err || mode == MODE_SKIP || mode == MODE_FAIL) ? PAD : token);
        if (split) cg::this_cluster().sync();  // the helper may overwrite the history structures now
        __syncthreads();  // the row's shared state is dead: the next row may reuse it
    }
}

// ---------------------------------------------------------------- greedy argmax

// Cluster of C CTAs per row; each CTA streams its slice with 16-byte loads and keeps (value, index)
// per thread (first index wins; NaN beats every number), then the leader merges over DSMEM.
template <typename E>
__global__ void __launch_bounds__(NT, 2) argmax_kernel(const void* logits, int V, int64_t stride, int per,
                                                       int64_t* tokens) {
    pdl_wait_then_release();
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
            // Per vector only its NaN-propagating maximum; the thread keeps the first vector holding its best
            // value (NaN first, then larger; an equal later vector never replaces it) and finds the element in
            // it at the end.  Vectors of a thread come in increasing index order.
            constexpr int U = 4, STEP = U * NT;
            float vb = f_ninf();
            int vbi = -1;
            uint4 bq = make_uint4(0u, 0u, 0u, 0u);
            auto ld = [&](int v0, uint4* q) {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int v = v0 + u * NT + tid;
                    q[u] = v < nv ? ldg_stream(vp + v) : make_uint4(0u, 0u, 0u, 0u);
                }
            };
            auto scan = [&](const uint4* q, int v0) {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int v = v0 + u * NT + tid;
                    if (v < nv) {
                        const float vm = Elem<E>::vmax_nan(q[u]);
                        if (vbi < 0 || vm > vb || (vm != vm && vb == vb)) {
                            vb = vm;
                            vbi = v;
                            bq = q[u];
                        }
                    }
                }
            };
            // two register buffers in turn: one in flight while the other is scanned
            uint4 qa[U], qb[U];
            if (nv > 0) ld(0, qa);
            if (nv > STEP) ld(STEP, qb);
            for (int v0 = 0; v0 < nv; v0 += 2 * STEP) {
                scan(qa, v0);
                if (v0 + 2 * STEP < nv) ld(v0 + 2 * STEP, qa);
                if (v0 + STEP < nv) {
                    scan(qb, v0 + STEP);
                    if (v0 + 3 * STEP < nv) ld(v0 + 3 * STEP, qb);
                }
            }
            if (vbi >= 0) {
                const bool want_nan = vb != vb;
                int jb = 16 / ES - 1;
#pragma unroll
                for (int j = 16 / ES - 1; j >= 0; --j) {
                    const float x = Elem<E>::at(bq, j);
                    if (want_nan ? x != x : x == vb) jb = j;
                }
                upd(Elem<E>::at(bq, jb), i0 + vbi * (16 / ES) + jb);
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
    if (crank == 0 && tid < 32) {
        // lane c reads rank c's result (the remote reads overlap), then the warp reduces
        bv = f_ninf();
        bi = 0x7fffffff;
        if (tid < C) {
            const int oi = *cluster.map_shared_rank(&ci, tid);
            if (oi != 0x7fffffff) upd(*cluster.map_shared_rank(&cv, tid), oi);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff) upd(ov, oi);
        }
        if (tid == 0) tokens[r] = bi == 0x7fffffff ? 0 : bi;
    }
    cluster.sync();
}

// ---------------------------------------------------------------- standalone repetition penalty

// grid (chunks, row groups): copy the chunk to fp32, then overwrite the history ids of the chunk with their
// penalised value (the same CTA, after a barrier, so the overwrite wins).  A CTA takes the rows
// blockIdx.y, blockIdx.y + gridDim.y, ... so that any row count fits the grid's y limit.
template <typename E>
__global__ void __launch_bounds__(NT) penalty_kernel(const void* x, int rows, int V, int64_t xstride,
                                                     const int64_t* hist, int W, int64_t hstride, const float* alpha,
                                                     int alpha_len, int alpha_stride, float* out, int64_t ostride,
                                                     int chunk, uint32_t slots, uint32_t* status) {
    extern __shared__ __align__(16) uint32_t ht[];
    const int tid = threadIdx.x;
    const int lo = blockIdx.x * chunk, hi = min(V, lo + chunk);
    for (int r = blockIdx.y; r < rows; r += gridDim.y) {
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
            if (id >= lo && id < hi) ht_insert(ht, slots, (uint32_t)(id - lo), 1u);
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
        __syncthreads();  // the table is reset for the next row
    }
}

// The numerics spec's exp on the device: y[i] = b2s_expf(x[i]); y2[i] = the paired non-positive form where
// x[i] <= 0 (pairs (2j, 2j+1) when both qualify, else the scalar form).
__global__ void expf_spec_kernel(const float* x, int64_t n, float* y, float* y2) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; 2 * j < n; j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = 2 * j;
        const float a = x[i], b = i + 1 < n ? x[i + 1] : 0.0f;
        y[i] = b2s_expf(a);
        if (i + 1 < n) y[i + 1] = b2s_expf(b);
        const bool pa = a <= 0.0f, pb = b <= 0.0f;
        if (pa && pb) {
            const float2 e = b2s_expf2_nonpos(make_float2(a, b));
            y2[i] = e.x;
            if (i + 1 < n) y2[i + 1] = e.y;
        } else {
            y2[i] = b2s_expf(a);
            if (i + 1 < n) y2[i + 1] = b2s_expf(b);
        }
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
}  // namespace

namespace b2s {
// Records a failed CUDA runtime call for b2s_last_cuda_error() (every launcher of the library reports
// through it) and returns B2S_ERR_CUDA.
int cuda_fail(cudaError_t e) {
    snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
    return B2S_ERR_CUDA;
}
}  // namespace b2s

namespace {
using b2s::cuda_fail;

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

// Shared-memory layout of the row-resident kernel with CL CTAs per row (b2s_resident.cu); false when the row
// slice and the structures beside it do not fit one CTA.  Fills p's resident fields and list sizes.
static bool resident_layout(b2s::Params& p, const b2s_sample_args* a, int CL, int es, int kmax) {
    using namespace b2s;
    const int64_t nvec_max = (int64_t)a->vocab * es / 16;  // the widest 16-byte interior of a row
    const int64_t sv = (nvec_max + CL - 1) / CL;
    if (sv > (int64_t)RMAXP * RPV) return false;
    const int kfast = kmax < KFAST ? kmax : KFAST;
    int lcap = next_pow2(4 * kfast + 128);
    lcap = lcap < 256 ? 256 : (lcap > 2048 ? 2048 : lcap);
    p.cl = CL;
    p.slice_vecs = (int)sv;
    p.lcap = lcap;
    // the merged list: an equal share per CTA (a CTA with more candidates than its share sends the row to the
    // full-row path)
    p.ltot = CL * lcap < 1024 ? CL * lcap : (lcap > 1024 ? lcap : 1024);
    p.csplit = 0;
    uint32_t off = 0;
    p.off_ctl = off;
    off = align_up(off + (uint32_t)sizeof(Ctl), 128);
    p.off_bar = off;
    off = align_up(off + RMAXP * 8, 128);
    p.off_slice = off;
    off = align_up(off + (uint32_t)sv * 16, 128);
    p.off_bits = off;
    off = align_up(off + p.bitwords * 4, 16);
    p.off_pref = off;
    off = align_up(off + p.bitwords / 4 * 2, 16);
    p.off_hcnt = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_hid = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_hpos = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_htv = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_smask = off;
    off = align_up(off + NT * 4, 16);
    // omni rows: the owned history ids' hash table, at most half full
    p.ht_slots = (a->semantics == B2S_SEM_OMNI && p.hcap > 0) ? (uint32_t)next_pow2(2 * p.hcap) : 0u;
    p.off_ht = off;
    off = align_up(off + p.ht_slots * 4, 16);
    p.off_hraw = off;  // unused: the history ids' raw values are read from the resident slice
    p.off_hstage = off;
    off = align_up(off + (uint32_t)a->window * 8, 16);
    p.off_atab = off;
    off = align_up(off + (uint32_t)(a->window <= 0 ? 0 : a->alpha_len) * 4, 16);
    p.off_cand = off;
    off = align_up(off + (uint32_t)p.ltot * 4, 16);
    p.off_candi = off;
    off = align_up(off + (uint32_t)p.ltot * 4, 16);
    p.off_lst = off;
    off = align_up(off + (uint32_t)p.ltot * 16, 16);
    p.off_vals = off;
    off = align_up(off + (uint32_t)p.nvals * 4, 16);
    p.off_hist = off;
    off = align_up(off + NBUCKET * 4, 16);
    p.smem_total = off;
    return off <= 227 * 1024;
}

// Shared-memory layout of the short-row kernel (b2s_short.cu); false when the rows are not short: more interior
// elements than its threads hold in registers, under 64 bytes (no interior vector), or a window longer than
// 255 (one position per thread, counted by scanning the window).  Fills p's short-row fields and list sizes.
static bool short_layout(b2s::Params& p, const b2s_sample_args* a, int es, int kmax) {
    using namespace b2s;
    const int64_t row_bytes = (int64_t)a->vocab * es;
    if (row_bytes < 64 || row_bytes / 16 > (int64_t)(SHORT_EPT * es / 16) * NT || a->window > 255) return false;
    const int kfast = kmax < KFAST ? kmax : KFAST;
    int lcap = next_pow2(4 * kfast + 128);
    lcap = lcap < 256 ? 256 : (lcap > 2048 ? 2048 : lcap);
    p.cl = 1;
    p.lcap = lcap;
    p.ltot = lcap;
    p.csplit = 0;
    p.cnt_words = (uint32_t)((a->vocab + 16 + 15) / 16 * 4);  // count bytes: id - e0 + EPV < vocab + 16, whole 16-byte groups
    uint32_t off = 0;
    p.off_ctl = off;
    off = align_up(off + (uint32_t)sizeof(Ctl), 128);
    p.off_cnt = off;
    off = align_up(off + p.cnt_words * 4, 16);
    p.off_bits = off;
    off = align_up(off + p.bitwords * 4, 16);
    p.off_pref = off;
    off = align_up(off + p.bitwords / 4 * 2, 16);
    p.off_hcnt = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_hid = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_hpos = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_htv = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_hraw = off;  // the history ids' processed values, indexed like the count bytes
    off = align_up(off + p.cnt_words * 16, 16);
    p.off_hstage = off;
    off = align_up(off + (uint32_t)a->window * 8, 16);
    p.off_atab = off;
    off = align_up(off + (uint32_t)(a->window <= 0 ? 0 : a->alpha_len) * 4, 16);
    p.off_cand = off;
    off = align_up(off + (uint32_t)p.ltot * 4, 16);
    p.off_candi = off;
    off = align_up(off + (uint32_t)p.ltot * 4, 16);
    p.off_lst = off;
    off = align_up(off + (uint32_t)p.ltot * 16, 16);
    p.off_vals = off;
    off = align_up(off + (uint32_t)p.nvals * 4, 16);
    p.off_hist = off;
    off = align_up(off + NBUCKET * 4, 16);
    p.smem_total = off;
    return off <= 227 * 1024;
}

// The codec head of b2s_head_sample: the head tiles' TMA map and operands (the rows' CTAs read `logits`).
struct HeadLaunch {
    CUtensorMap map;
    int tiles, kb;
    const void* hidden;
    int64_t hid_stride;
    uint32_t* sync;
    void* logits;
};

static int launch_sample(const b2s_sample_args* a, void* stream, const ShardOut* so, int frames = 1,
                         int64_t fstride = 0, const HeadLaunch* hl = nullptr) {
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
    if (!identity && a->window > 0 && a->vocab > (1 << 18)) return B2S_ERR_UNSUPPORTED;  // packed hash ids

    Params p;
    memset(&p, 0, sizeof(p));
    p.frames = frames;
    p.fstride = fstride;
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
    p.rminn = a->row_min_new_tokens;
    p.rmaxn = a->row_max_new_tokens;
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
    int kmax = a->max_top_k > 0 ? a->max_top_k : a->top_k;
    kmax = identity ? 1 : kmax;
    kmax = kmax < a->min_keep ? a->min_keep : kmax;
    kmax = kmax > a->vocab ? a->vocab : kmax;
    kmax = kmax < 1 ? 1 : kmax;
    const int kfast = kmax < KFAST ? kmax : KFAST;
    // candidates pushed during the stream: ~k from the first chunk, then ~k / (c + 1) from chunk c as the
    // threshold rises, plus the values sharing its histogram bucket; more means heavy ties
    p.lcap = next_pow2(8 * kfast + 256);
    if (p.lcap > 2048) p.lcap = 2048;
    p.kbuf = kmax;
    p.nvals = next_pow2(kmax) > 2 * KFAST ? next_pow2(kmax) : 2 * KFAST;
    const bool hashed = !identity && (a->window > 0 || (a->eos >= 0 && a->eos < a->vocab));
    const int hist_ids = (a->window < a->vocab ? a->window : a->vocab) + 1;  // distinct ids: window + EOS
    p.hcap = hashed ? hist_ids : 0;
    p.bitwords = hashed ? (uint32_t)(((a->vocab + 31) / 32 + 3) / 4 * 4) : 0u;  // whole 4-word groups
    uint32_t off = 0;
    p.off_ctl = off;
    off = align_up(off + (uint32_t)sizeof(Ctl), 128);
    p.off_bits = off;
    off = align_up(off + p.bitwords * 4, 16);
    p.off_pref = off;  // one 16-bit rank per 4-word group: hcap <= 2^13 + 1
    off = align_up(off + p.bitwords / 4 * 2, 16);
    p.off_hcnt = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_hid = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_hpos = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_htv = off;
    off = align_up(off + (uint32_t)p.hcap * 4, 16);
    p.off_smask = off;
    off = align_up(off + NT * 8, 16);
    p.off_hraw = off;  // the 4-byte word holding the raw value of each of the first 4 * NT history positions
    off = align_up(off + (uint32_t)(identity ? 0 : (a->window < 4 * NT ? a->window : 4 * NT)) * 4, 16);
    p.off_hstage = off;
    off = align_up(off + (uint32_t)(identity ? 0 : a->window) * 8, 16);
    p.off_atab = off;
    off = align_up(off + (uint32_t)(identity || a->window <= 0 ? 0 : a->alpha_len) * 4, 16);
    p.off_cand = off;
    off = align_up(off + (uint32_t)p.lcap * 4, 16);
    p.off_candi = off;
    off = align_up(off + (uint32_t)p.lcap * 4, 16);
    p.off_lst = off;
    off = align_up(off + (uint32_t)p.lcap * 16, 16);
    p.off_vals = off;
    off = align_up(off + (uint32_t)p.nvals * 4, 16);
    p.off_hist = off;
    off = align_up(off + NBUCKET * 4, 16);
    const uint32_t limit = 227 * 1024;
    p.off_tmaxc = off;
    {
        const int row_chunks = (int)(((int64_t)a->vocab * es / 16 + VPC - 1) / VPC);
        int fit = off < limit ? (int)((limit - off) / (NT * 4)) : 0;
        fit = fit < 64 ? fit : 64;  // pass 2 keeps one bit per chunk
        p.tmc_chunks = row_chunks < fit ? row_chunks : fit;
        off = align_up(off + (uint32_t)p.tmc_chunks * NT * 4, 16);
    }
    p.smem_total = off;
    if (p.smem_total > limit) return B2S_ERR_UNSUPPORTED;

    cudaError_t e;
    const bool lean = !so && !a->processed;
    // Row-resident kernel: decode steps (no processed / shard output) of up to 128 candidates, one wave of
    // clusters, and one CTA per row for hf (its full-row normaliser is taken from the resident row).
    // `cluster` > 0 asks for it with that many CTAs per row; 0 lets the launcher pick the smallest that fits.
    {
        const bool streamed = (a->flags & B2S_FLAG_STREAM) != 0 || frames > 1;
        if (a->cluster != 0 && (streamed || !(a->cluster == 1 || a->cluster == 2 || a->cluster == 4 || a->cluster == 8)))
            return B2S_ERR_INVALID;
        const bool res_ok = lean && draws && !identity && !streamed && kmax <= KLIST;
        int CL = 0;
        Params rp = p;
        // the short-row kernel also takes K frames per launch (one CTA per row, frames in order)
        const bool short_ok = lean && draws && !identity && (a->flags & B2S_FLAG_STREAM) == 0 && kmax <= KLIST;
        if (hl) {
            // the codec head and the sampling step in one launch: rows' CTAs first, then the head tiles
            if (!(a->cluster == 0 && short_ok && frames == 1 && short_layout(rp, a, es, kmax)))
                return B2S_ERR_UNSUPPORTED;
            // the rows wait on the tiles: one wave.  Two CTAs per tile (K split over a cluster) where they fit
            const int even_rows = (a->rows + 1) & ~1;
            const int split = (hl->kb % 2 == 0 && even_rows + 2 * hl->tiles <= sm_count()) ? 2 : 1;
            if (a->rows + hl->tiles > sm_count()) return B2S_ERR_UNSUPPORTED;
            rp.head_split = split;
            rp.head_first = split > 1 ? even_rows : a->rows;
            rp.head_tiles = hl->tiles;
            rp.head_kb = hl->kb;
            rp.hidden = hl->hidden;
            rp.hid_stride = hl->hid_stride;
            rp.head_sync = hl->sync;
            rp.logits = hl->logits;
            const uint32_t smem = rp.smem_total > HEAD_SMEM ? rp.smem_total : HEAD_SMEM;
            const bool omni = a->semantics == B2S_SEM_OMNI;
            HeadKernel kern = head_kernel_for(omni);
            {
                static std::mutex mu;
                static uint64_t done[2] = {0, 0};
                int dev = 0;
                e = cudaGetDevice(&dev);
                if (e != cudaSuccess) return cuda_fail(e);
                std::lock_guard<std::mutex> g(mu);
                const uint64_t bit = 1ull << (dev & 63);
                if (!(done[omni ? 1 : 0] & bit)) {
                    e = set_smem_attr(kern, 227 * 1024);
                    if (e != cudaSuccess) return cuda_fail(e);
                    done[omni ? 1 : 0] |= bit;
                }
            }
            cudaLaunchConfig_t cfg;
            memset(&cfg, 0, sizeof(cfg));
            cfg.gridDim = dim3((unsigned)(rp.head_first + split * hl->tiles), 1, 1);
            cfg.blockDim = dim3(NT, 1, 1);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = (cudaStream_t)stream;
            cudaLaunchAttribute attrs[2];
            attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attrs[0].val.programmaticStreamSerializationAllowed = 1;
            attrs[1].id = cudaLaunchAttributeClusterDimension;
            attrs[1].val.clusterDim.x = 2;
            attrs[1].val.clusterDim.y = 1;
            attrs[1].val.clusterDim.z = 1;
            cfg.attrs = attrs;
            cfg.numAttrs = split > 1 ? 2 : 1;
            e = cudaLaunchKernelEx(&cfg, kern, rp, hl->map);
            if (e != cudaSuccess) return cuda_fail(e);
            return B2S_OK;
        }
        if (a->cluster == 0 && short_ok && short_layout(rp, a, es, kmax)) {
            // short rows: one CTA per row, the row's elements in its threads' registers (b2s_short.cu)
            const bool omni = a->semantics == B2S_SEM_OMNI;
            ResKernel kern = short_kernel_for(a->logits_dtype == B2S_DTYPE_BF16, omni);
            {
                static std::mutex mu;
                static uint64_t done[4] = {0, 0, 0, 0};
                int dev = 0;
                e = cudaGetDevice(&dev);
                if (e != cudaSuccess) return cuda_fail(e);
                std::lock_guard<std::mutex> g(mu);
                const int ti = (a->logits_dtype == B2S_DTYPE_BF16 ? 2 : 0) + (omni ? 1 : 0);
                const uint64_t bit = 1ull << (dev & 63);
                if (!(done[ti] & bit)) {
                    e = set_smem_attr(kern, 227 * 1024);
                    if (e != cudaSuccess) return cuda_fail(e);
                    done[ti] |= bit;
                }
            }
            cudaLaunchConfig_t cfg;
            memset(&cfg, 0, sizeof(cfg));
            cfg.gridDim = dim3((unsigned)a->rows, 1, 1);
            cfg.blockDim = dim3(NT, 1, 1);
            cfg.dynamicSmemBytes = rp.smem_total;
            cfg.stream = (cudaStream_t)stream;
            cudaLaunchAttribute attr;
            attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr.val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            e = cudaLaunchKernelEx(&cfg, kern, rp);
            if (e != cudaSuccess) return cuda_fail(e);
            return B2S_OK;
        }
        rp = p;
        if (a->cluster != 0) {
            if (!res_ok || (a->semantics == B2S_SEM_HF && a->cluster > 1) || !resident_layout(rp, a, a->cluster, es, kmax))
                return B2S_ERR_UNSUPPORTED;
            CL = a->cluster;
        } else if (res_ok) {
            for (int c = 1; c <= 8; c <<= 1) {
                if (a->semantics == B2S_SEM_HF && c > 1) break;
                if ((int64_t)a->rows * c > sm_count()) break;
                if (resident_layout(rp, a, c, es, kmax)) {
                    CL = c;
                    break;
                }
            }
        }
        if (CL > 0) {
            const bool omni = a->semantics == B2S_SEM_OMNI;
            ResKernel kern = resident_kernel_for(a->logits_dtype == B2S_DTYPE_BF16, omni);
            {
                static std::mutex mu;
                static uint64_t done[4] = {0, 0, 0, 0};
                int dev = 0;
                e = cudaGetDevice(&dev);
                if (e != cudaSuccess) return cuda_fail(e);
                std::lock_guard<std::mutex> g(mu);
                const int ti = (a->logits_dtype == B2S_DTYPE_BF16 ? 2 : 0) + (omni ? 1 : 0);
                const uint64_t bit = 1ull << (dev & 63);
                if (!(done[ti] & bit)) {
                    e = set_smem_attr(kern, 227 * 1024);
                    if (e != cudaSuccess) return cuda_fail(e);
                    done[ti] |= bit;
                }
            }
            cudaLaunchConfig_t cfg;
            memset(&cfg, 0, sizeof(cfg));
            cfg.gridDim = dim3((unsigned)((int64_t)a->rows * CL), 1, 1);
            cfg.blockDim = dim3(NT, 1, 1);
            cfg.dynamicSmemBytes = rp.smem_total;
            cfg.stream = (cudaStream_t)stream;
            cudaLaunchAttribute attrs[2];
            attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attrs[0].val.programmaticStreamSerializationAllowed = 1;
            attrs[1].id = cudaLaunchAttributeClusterDimension;
            attrs[1].val.clusterDim.x = (unsigned)CL;
            attrs[1].val.clusterDim.y = 1;
            attrs[1].val.clusterDim.z = 1;
            cfg.attrs = attrs;
            cfg.numAttrs = CL > 1 ? 2 : 1;
            e = cudaLaunchKernelEx(&cfg, kern, rp);
            if (e != cudaSuccess) return cuda_fail(e);
            return B2S_OK;
        }
    }
    const bool bf16 = a->logits_dtype == B2S_DTYPE_BF16;
    // variant: 0 general, 1 lean, 2 lean with the omni order fixed at compile time
    const int var = !lean ? 0 : a->semantics == B2S_SEM_OMNI ? 2 : 1;
    using K = void (*)(const Params);
    static const K kernels[2][3] = {
        {sample_kernel<float, false, -1>, sample_kernel<float, true, -1>, sample_kernel<float, true, B2S_SEM_OMNI>},
        {sample_kernel<__nv_bfloat16, false, -1>, sample_kernel<__nv_bfloat16, true, -1>,
         sample_kernel<__nv_bfloat16, true, B2S_SEM_OMNI>}};
    K kern = kernels[bf16 ? 1 : 0][var];
    {
        // the attribute is per device: remember which (device, kernel) pairs have it
        static std::mutex mu;
        static uint64_t done[6] = {0, 0, 0, 0, 0, 0};
        int dev = 0;
        e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return cuda_fail(e);
        std::lock_guard<std::mutex> g(mu);
        const int ti = (bf16 ? 3 : 0) + var;
        const uint64_t bit = 1ull << (dev & 63);
        if (!(done[ti] & bit)) {
            e = set_smem_attr(kern, 227 * 1024);
            if (e != cudaSuccess) return cuda_fail(e);
            done[ti] |= bit;
        }
    }
    // Two CTAs per row when every pair fits on the SMs at once (one 512-thread CTA per SM), the row streams
    // several chunks and has a penalty history: the history work then runs beside pass 1.
    {
        const int64_t row_chunks = ((int64_t)a->vocab * es / 16 + VPC - 1) / VPC;
        p.csplit = (!so && !a->processed && !identity && p.W > 0 && row_chunks >= 4 && row_chunks <= p.tmc_chunks &&
                    (int64_t)a->rows * 2 <= sm_count() && frames == 1) ? 1 : 0;
    }
    // several frames: one CTA per row, which takes the row's frames in order (b2s_sample_frames checks the size)
    const int64_t grid_rows = frames > 1 ? a->rows : (a->rows < 65535 * 8 ? a->rows : 65535 * 8);
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)(p.csplit ? 2 * grid_rows : grid_rows), 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = p.smem_total;
    cfg.stream = (cudaStream_t)stream;
    // the launch may overlap the tail of the stream's previous kernel (the kernel waits for it before any read)
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = 2;
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = p.csplit ? 2 : 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}

int b2s_sample(const b2s_sample_args* a, void* stream) { return launch_sample(a, stream, nullptr); }

int b2s_sample_frames(const b2s_sample_args* a, int32_t frames, int64_t frame_stride, void* stream) {
    if (!a || frames < 1 || !a->tokens) return B2S_ERR_INVALID;
    if (frames == 1) return launch_sample(a, stream, nullptr);
    if (a->semantics == B2S_SEM_IDENTITY || a->processed || a->cluster != 0) return B2S_ERR_INVALID;
    // the state carries from frame to frame in place
    if (!a->steps_out || a->steps_out != a->steps || !a->finished || a->finished_out != a->finished) return B2S_ERR_INVALID;
    if (a->window > 0 && a->history_out != a->history) return B2S_ERR_INVALID;
    if (a->window > 0 && a->history_out_row_stride != a->history_row_stride) return B2S_ERR_INVALID;
    if (frame_stride < (int64_t)a->rows * a->logits_row_stride) return B2S_ERR_INVALID;
    if (a->rows > 65535 * 8 || (int64_t)a->rows * frames > INT32_MAX) return B2S_ERR_UNSUPPORTED;
    return launch_sample(a, stream, nullptr, frames, frame_stride);
}

// cuTensorMapEncodeTiled from the driver, through the runtime (no link against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

int b2s_head_sample(const b2s_head_args* h, const b2s_sample_args* a, void* stream) {
    using namespace b2s;
    if (!h || !a || !h->hidden || !h->head || !h->logits || !h->sync) return B2S_ERR_INVALID;
    if (a->rows < 1 || a->vocab < 1 || a->logits_dtype != B2S_DTYPE_BF16) return B2S_ERR_INVALID;
    if (a->logits && a->logits != h->logits) return B2S_ERR_INVALID;
    if (a->logits_row_stride < a->vocab) return B2S_ERR_INVALID;
    if (h->hidden_dim < HEAD_KB || h->hidden_dim % HEAD_KB != 0 || h->hidden_row_stride < h->hidden_dim)
        return B2S_ERR_INVALID;
    // the hidden rows are read as 16-byte vectors, the head by TMA: 16-byte aligned rows; the sync words as one block
    if (h->hidden_row_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(h->hidden) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(h->head) & 15) != 0 || (reinterpret_cast<uintptr_t>(h->sync) & 15) != 0)
        return B2S_ERR_INVALID;
    if (a->rows > HEAD_N || h->hidden_dim > HEAD_MAX_KB * HEAD_KB) return B2S_ERR_UNSUPPORTED;
    HeadLaunch hl;
    memset(&hl, 0, sizeof(hl));
    hl.tiles = (a->vocab + HEAD_M - 1) / HEAD_M;
    hl.kb = h->hidden_dim / HEAD_KB;
    hl.hidden = h->hidden;
    hl.hid_stride = h->hidden_row_stride;
    hl.sync = h->sync;
    hl.logits = h->logits;
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return cuda_fail(cudaErrorNotSupported);
    // head [vocab, hidden_dim] bf16, rows hidden_dim elements apart; boxes of [128 ids x 64] in the 128-byte
    // swizzle (the MMA's K-major operand layout); ids past the vocabulary read as zero
    const cuuint64_t dims[2] = {(cuuint64_t)h->hidden_dim, (cuuint64_t)a->vocab};
    const cuuint64_t strides[1] = {(cuuint64_t)h->hidden_dim * 2};
    const cuuint32_t box[2] = {(cuuint32_t)HEAD_KB, (cuuint32_t)HEAD_M};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&hl.map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(h->head), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return B2S_ERR_INVALID;
    b2s_sample_args a2 = *a;
    a2.logits = h->logits;
    return launch_sample(&a2, stream, nullptr, 1, 0, &hl);
}

static int lmhead_common(const void* hidden, int64_t hidden_row_stride, const void* head, int32_t hidden_dim,
                         int32_t vocab, int32_t rows, int64_t* tokens, uint64_t* keys, uint32_t* status, void* stream,
                         int64_t offset, int64_t* keys_out) {
    using namespace b2s;
    if (!hidden || !head || !(tokens || keys_out) || !keys || vocab < 1 || rows < 1) return B2S_ERR_INVALID;
    if (offset < 0 || offset + (int64_t)vocab > (int64_t)0xfffffffe) return B2S_ERR_INVALID;
    if (hidden_dim < 64 || hidden_dim % 64 != 0 || hidden_row_stride < hidden_dim || hidden_row_stride % 8 != 0)
        return B2S_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(hidden) & 15) != 0 || (reinterpret_cast<uintptr_t>(head) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(keys) & 7) != 0)
        return B2S_ERR_INVALID;
    if (rows > LMHEAD_MAX_ROWS) return B2S_ERR_UNSUPPORTED;
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return cuda_fail(cudaErrorNotSupported);
    // head [vocab, hidden_dim]: boxes of [128 ids x 64]; hidden [rows, hidden_dim]: boxes of [64 rows x 64] (rows
    // past the batch read as zero); both in the 128-byte swizzle
    CUtensorMap amap, bmap;
    const cuuint64_t adims[2] = {(cuuint64_t)hidden_dim, (cuuint64_t)vocab};
    const cuuint64_t astr[1] = {(cuuint64_t)hidden_dim * 2};
    const cuuint32_t abox[2] = {64, 128};
    const cuuint64_t bdims[2] = {(cuuint64_t)hidden_dim, (cuuint64_t)rows};
    const cuuint64_t bstr[1] = {(cuuint64_t)hidden_row_stride * 2};
    const cuuint32_t bbox[2] = {64, 64};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(head), adims, astr, abox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(hidden), bdims, bstr, bbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return B2S_ERR_INVALID;
    const cudaError_t e = lmhead_argmax_launch(amap, bmap, vocab, rows, hidden_dim / 64, tokens,
                                               reinterpret_cast<unsigned long long*>(keys), status, stream, offset,
                                               keys_out);
    return e == cudaSuccess ? B2S_OK : cuda_fail(e);
}

int b2s_lmhead_argmax(const void* hidden, int64_t hidden_row_stride, const void* head, int32_t hidden_dim,
                      int32_t vocab, int32_t rows, int64_t* tokens, uint64_t* keys, uint32_t* status, void* stream) {
    if (!tokens) return B2S_ERR_INVALID;
    return lmhead_common(hidden, hidden_row_stride, head, hidden_dim, vocab, rows, tokens, keys, status, stream, 0,
                         nullptr);
}

int b2s_lmhead_argmax_keys(const void* hidden, int64_t hidden_row_stride, const void* head_shard, int32_t hidden_dim,
                           int32_t shard_vocab, int64_t vocab_offset, int32_t rows, int64_t* keys_out, uint64_t* keys,
                           uint32_t* status, void* stream) {
    if (!keys_out) return B2S_ERR_INVALID;
    return lmhead_common(hidden, hidden_row_stride, head_shard, hidden_dim, shard_vocab, rows, nullptr, keys, status,
                         stream, vocab_offset, keys_out);
}

// ---------------------------------------------------------------- the codec head without caller scratch
// b2s_head_sample needs two device buffers beyond its inputs and outputs: the bf16 logits rows that the head's
// tiles hand to the rows, and four control words.  A caller that cannot allocate device memory -- an embedding
// whose allocator is fixed at start-up, a host runtime that passes in only the buffers it owns (weights, hidden
// rows, decode state, tokens), or a decode loop that must not call cudaMalloc / cudaFree, which can synchronise
// the device, while other work is in flight -- uses this variant instead.  Its scratch is one file-scope device
// array of a fixed size, which every process that loads this library holds on every GPU it uses until it exits.
// Host code must not use the array's name as a device address: it is a host-side stand-in, so the device address
// is looked up once per device (cudaGetSymbolAddress, with that device current) and passed to the kernel.
static __device__ __align__(256) unsigned char g_head_scratch[B2S_NOALLOC_SCRATCH_BYTES];
static_assert(B2S_NOALLOC_SCRATCH_BYTES == B2S_NOALLOC_MAX_ROWS * B2S_NOALLOC_MAX_VOCAB * 2 + 256,
              "the scratch holds the bf16 logits rows, then the control words");

static int head_scratch_address(unsigned char** out) {
    static std::mutex mu;
    static unsigned char* addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= 64) return B2S_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> g(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_head_scratch);
        if (e != cudaSuccess) return cuda_fail(e);
        addr[dev] = static_cast<unsigned char*>(p);
    }
    *out = addr[dev];
    return B2S_OK;
}

int b2s_head_sample_noalloc(const void* hidden, int64_t hidden_row_stride, const void* head, int32_t hidden_dim,
                            const b2s_sample_args* a, void* stream) {
    if (!a || a->logits) return B2S_ERR_INVALID;  // the logits live in the library's scratch
    if (a->rows > B2S_NOALLOC_MAX_ROWS || a->vocab > B2S_NOALLOC_MAX_VOCAB) return B2S_ERR_UNSUPPORTED;
    unsigned char* scratch = nullptr;
    int rc = head_scratch_address(&scratch);
    if (rc != B2S_OK) return rc;
    // the control words start at zero (a completed launch leaves them so; one that gave up may not)
    uint32_t* sync = reinterpret_cast<uint32_t*>(scratch + (size_t)B2S_NOALLOC_MAX_ROWS * B2S_NOALLOC_MAX_VOCAB * 2);
    cudaError_t e = cudaMemsetAsync(sync, 0, 4 * sizeof(uint32_t), (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e);
    b2s_head_args h;
    memset(&h, 0, sizeof(h));
    h.hidden = hidden;
    h.hidden_row_stride = hidden_row_stride;
    h.head = head;
    h.hidden_dim = hidden_dim;
    h.logits = scratch;
    h.sync = sync;
    b2s_sample_args a2 = *a;
    a2.logits = nullptr;
    a2.logits_dtype = B2S_DTYPE_BF16;
    a2.logits_row_stride = a->vocab;
    return b2s_head_sample(&h, &a2, stream);
}

int b2s_shard_candidates(const b2s_sample_args* a, int64_t vocab_offset, int32_t cap, float* cand_values,
                         int32_t* cand_ids, int32_t* cand_count, void* stream) {
    if (!a || !cand_values || !cand_ids || !cand_count || cap < 1 || vocab_offset < 0) return B2S_ERR_INVALID;
    {
        const int kb = a->max_top_k > 0 ? a->max_top_k : a->top_k;
        if (cap < (kb > a->min_keep ? kb : a->min_keep)) return B2S_ERR_INVALID;  // every element above the k-th fits
    }
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
    // split rows over up to 8 CTAs while the grid stays within one wave (two CTAs per SM)
    while (C < 8 && (int64_t)rows * C * 2 <= 2 * sm_count() && row_bytes / (C * 2) >= 16 * 1024) C <<= 1;
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
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see b2s_sample
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
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
    dim3 grid((unsigned)((vocab + chunk - 1) / chunk), (unsigned)(rows < 65535 ? rows : 65535));
    const size_t smem = slots * 4;
    cudaStream_t st = (cudaStream_t)stream;
    if (x_dtype == B2S_DTYPE_BF16)
        penalty_kernel<__nv_bfloat16><<<grid, NT, smem, st>>>(x, rows, vocab, x_row_stride, history, window,
                                                              history_row_stride, alpha, alpha_len, alpha_row_stride,
                                                              out, out_row_stride, chunk, slots, status);
    else
        penalty_kernel<float><<<grid, NT, smem, st>>>(x, rows, vocab, x_row_stride, history, window, history_row_stride,
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

int b2s_expf_spec(const float* x, int64_t n, float* y, float* y_pair, void* stream) {
    if (n < 0 || (n > 0 && (!x || !y || !y_pair))) return B2S_ERR_INVALID;
    if (n == 0) return B2S_OK;
    const int threads = 256;
    int64_t blocks = ((n + 1) / 2 + threads - 1) / threads;
    if (blocks > 4 * 148) blocks = 4 * 148;
    b2s::expf_spec_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(x, n, y, y_pair);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}

}  // extern "C"
