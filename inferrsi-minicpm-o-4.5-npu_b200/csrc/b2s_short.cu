// Short-row sampling kernel (sm_100a): the decode-step form of b2s_sample (and of b2s_sample_frames: the CTA takes
// its row's K frames in order, the state advancing in place) for rows of at most SHORT_EPT * NT interior elements
// -- the Talker's codec vocabulary (6,562 ids) in fp32 or bf16 -- one CTA per row.
//
// Such a row is a few tens of KB: its step is as long as its chain of dependent phases, not as its bytes.
// The kernel keeps that chain short and its instructions few:
//
//   loads:    every thread requests its interior vectors (tid, tid + NT, ...: the thread layout of the other
//             row kernels, so the same fp64 partial sums) into registers; threads 0 / 1 the head / tail
//             elements outside the 16-byte interior, as one more vector (slot); thread j < W its history id;
//             the penalty table goes to shared memory by asynchronous copies.
//   history:  as soon as its id lands, thread j adds one to the id's byte in a packed count array (zeroed
//             while the previous kernel still ran) and requests the id's raw value; once the counts are
//             complete it writes the id's processed value into a table indexed like the counts (byte
//             id - e0 + EPV, so that one aligned shared word holds the counts of a vector).  No bitmap, no ranks.
//   values:   meanwhile every thread divides its elements by T in registers; then an element with a non-zero
//             count takes its value from the table, and each thread keeps its maximum.
//   gather:   the processed row goes to shared memory; each warp gathers its ceil(k/16) largest thread maxima
//             (each a distinct element) and its maximum.
//   split:    warps 0..3 take tau -- the k-th largest of the gathered maxima, so a lower bound of the row's
//             k-th largest processed value, exactly (the comparison is on processed values: no rounding
//             margin) -- and put every element >= tau into the candidate list in vocabulary order (two passes
//             over contiguous runs of the row in shared memory, one scan); meanwhile warps 4..15 take the fp64
//             sum of exp(P - max) for hf's full-row normaliser (talker_sampler.py:112).
//
// Then the list stage of b2s_list.cuh in one warp -- a bitonic sort of up to 128 candidate values, the top-p
// cut, and the draw over the kept items, which the list already holds in vocabulary order -- and the state
// epilogue.  A row the list cannot serve (NaN, an unusable tau, more candidates
// than the list holds) builds the history structures and takes the exact full-row path; hf frame-0 rows take
// the ordered scan: both shared with the row-resident kernel (b2s_rowpaths.cuh) and out of line.  The kernel
// waits on nothing but its own loads and block barriers -- except in head_kernel (below), where the rows' CTAs
// wait (bounded) for the codec-head tiles of the same launch to publish their logits.
#include <type_traits>

#include "b2s_head.cuh"
#include "b2s_rowpaths.cuh"

namespace b2s {

// The flagged elements of one vector (ids e .. e + EPV - 1, the first `valid` real): an element whose count byte
// in cw is non-zero takes its processed value from hval[c + j] (c: the table index of element e); the censored
// EOS (omni) is -inf whatever its history.  Then the thread's maximum.
template <typename E>
__device__ __forceinline__ void short_patch(const float* hval, int cens, uint64_t cw, int e, int c, int valid,
                                            float* out, float& tmax) {
    constexpr int EPV = Elem<E>::EPV;
    if (cw != 0u) {
#pragma unroll
        for (int j = 0; j < EPV; ++j)
            if ((cw >> (8 * j)) & 255u) out[j] = hval[c + j];
    }
    if ((unsigned)(cens - e) < (unsigned)valid) {
#pragma unroll
        for (int j = 0; j < EPV; ++j)
            if (e + j == cens) out[j] = f_ninf();
    }
#pragma unroll
    for (int j = 0; j < EPV; ++j) tmax = fmaxf(tmax, out[j]);
}

// The exact full-row path of a short row: the whole-row history structures first (the register pass keeps
// only counts), then the radix select, threshold and ordered draw that every row kernel falls back on.
template <typename E>
static __device__ __noinline__ int64_t short_exact(const Params p, Row<E> R, HistBufs hb, int k, bool hf, float lse,
                                                   float top_p, bool topk_only, int drop, bool pen_hist, bool censor,
                                                   float T, float u, uint32_t* hist, float* vals, Ctl* ctl) {
    const bool use_ht = pen_hist || censor;
    R.bits = use_ht ? hb.bits : nullptr;
    R.pref = hb.pref;
    R.htv = hb.htv;
    R.censor = censor ? p.eos : -1;
    if (use_ht) hist_rebuild<E>(p, R, hb, hf, pen_hist, censor, T, ctl);
    return exact_token<E>(R, k, hf, lse, top_p, p.min_keep, topk_only, drop, u, hist, vals, ctl);
}

// One row per CTA (blockIdx.x).  HEAD: the row's logits are written by the codec-head CTAs of the same launch
// (b2s_head.cuh); the row waits for them after its history loads and reads them with coherent loads.
template <typename E, int SEM, bool HEAD>
__device__ __forceinline__ void short_rows(const Params& p, unsigned char* smem) {
    constexpr int EPV = Elem<E>::EPV, ES = Elem<E>::SZ, SV = SHORT_EPT / EPV;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = (int)blockIdx.x;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
    uint32_t* cnts = reinterpret_cast<uint32_t*>(smem + p.off_cnt);  // byte id - e0 + EPV: the id's occurrences
    float* hval = reinterpret_cast<float*>(smem + p.off_hraw);       // [id - e0 + EPV]: its processed value
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
    float* cand_v = reinterpret_cast<float*>(smem + p.off_cand);
    int* cand_i = reinterpret_cast<int*>(smem + p.off_candi);
    float* kv = reinterpret_cast<float*>(smem + p.off_lst);
    int* ki = reinterpret_cast<int*>(kv + p.ltot);
    float* sv = kv + 2 * p.ltot;
    int* si = reinterpret_cast<int*>(kv + 3 * p.ltot);
    float* vals = reinterpret_cast<float*>(smem + p.off_vals);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + p.off_hist);
    const int V = p.V;
    // several frames (b2s_sample_frames): this CTA takes its row's frames in order, each one's state written in
    // place being the next one's input
    for (int f = 0; f < p.frames; ++f) {
    const int w = f * p.rows + r;  // work item: tokens and uniform values are [frames, rows]
    if (f > 0) __syncthreads();  // the previous frame's state is visible to the CTA; its shared memory is free
    // (frame 0: before the wait for the previous kernel -- nothing global is read) the count bytes zeroed, tau's slot
    if (p.hist && p.W > 0)
        for (uint32_t g = tid; g < p.cnt_words / 4; g += NT) reinterpret_cast<uint4*>(cnts)[g] = make_uint4(0u, 0u, 0u, 0u);
    if (tid == 0) ctl->thr = f_ninf();  // tau, until a rank finds it
    __syncthreads();
    if (f == 0) pdl_wait_then_release();  // nothing global is read before the previous kernel of the stream is done

    // ---------------- loads: this thread's row elements and history id (registers), the penalty table
    Row<E> R;
    R.rowp = reinterpret_cast<const unsigned char*>(p.logits) + ((int64_t)f * p.fstride + (int64_t)r * p.lstride) * ES;
    R.V = V;
    R.coh = HEAD;  // the codec head's logits are written in this launch: no read-only-path loads of the row
    {
        const uintptr_t a = reinterpret_cast<uintptr_t>(R.rowp), b = a + (uintptr_t)V * ES;
        const uintptr_t ace = (a + 15) & ~(uintptr_t)15, bfl = b & ~(uintptr_t)15;
        // the launcher sends only rows of >= 64 bytes: the interior holds at least one vector
        R.nh = (int)((ace - a) / ES);
        R.nvec = (int)((bfl - ace) / 16);
        R.gvec = reinterpret_cast<const uint4*>(ace);
        R.e0 = R.nh;
    }
    const int64_t* hrow = p.hist ? p.hist + (int64_t)r * p.hstride : nullptr;
    const bool hthread = hrow != nullptr && tid < p.W;  // W <= 255 < NT: one history position per thread
    const int64_t hv = hthread ? hrow[tid] : -1;
    if (hrow && p.W > 0 && p.alpha)
        for (int j = tid; j < p.alpha_len; j += NT) cp_async4(&atab[j], p.alpha + (int64_t)r * p.alpha_stride + j);
    bool head_ok = true;
    if constexpr (HEAD) {
        // the codec-head tiles publish their logits with a release increment; the last row to see them all
        // zeroes the control words for the next launch (which touches them only after this one has completed)
        if (tid == 0) {
            const bool seen = wait_geq_acquire(p.head_sync + HS_TILES, (uint32_t)p.head_tiles, HEAD_WAIT_NS);
            const bool ok = seen && ld_acquire_u32(p.head_sync + HS_ERR) == 0u;
            if (!ok) set_status(p, B2S_STATUS_WAIT_TIMEOUT);
            ctl->head_ok = ok ? 1 : 0;
            if (atomicAdd(p.head_sync + HS_ROWS, 1u) == (uint32_t)p.rows - 1u) {
                p.head_sync[HS_TILES] = 0u;
                p.head_sync[HS_ERR] = 0u;
                p.head_sync[HS_ROWS] = 0u;
            }
        }
        __syncthreads();
        head_ok = ctl->head_ok != 0;
    }
    uint4 q[SV + 1];  // interior vectors tid + s * NT, then (threads 0 / 1) the head / tail as one more vector
#pragma unroll
    for (int s = 0; s < SV; ++s) {
        const int v = tid + s * NT;
        if constexpr (HEAD)
            q[s] = v < R.nvec ? ld_stream_coherent(R.gvec + v)
                              : make_uint4(Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG);
        else
            q[s] = v < R.nvec ? ldg_stream(R.gvec + v) : make_uint4(Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG);
    }
    const int i_end = R.e0 + R.nvec * EPV;
    const int x0 = tid == 0 ? 0 : i_end;                       // first element of the edge slot
    const int nx = tid == 0 ? R.nh : tid == 1 ? V - i_end : 0;  // < EPV
    uint32_t ex[EPV - 1];  // the edge elements' bits, packed into q[SV] once they are needed
#pragma unroll
    for (int j = 0; j < EPV - 1; ++j) ex[j] = j < nx ? __float_as_uint(R.raw(x0 + j)) : 0u;
    const int64_t step = p.steps ? p.steps[r] : 0;
    const bool is_live = (p.active ? p.active[r] != 0 : true) && !(p.finished ? p.finished[r] != 0 : false);
    const float T = p.rT ? p.rT[r] : p.T;
    const float top_p = p.rP ? p.rP[r] : p.top_p;
    const int top_k = p.rK ? p.rK[r] : p.top_k;
    const int64_t min_new = p.rminn ? p.rminn[r] : p.min_new, max_new = p.rmaxn ? p.rmaxn[r] : p.max_new;

    // ---------------- mode
    const bool hf = SEM >= 0 ? SEM == B2S_SEM_HF : p.sem == B2S_SEM_HF;
    const bool eos_ok = p.eos >= 0 && p.eos < V;
    const bool masked_eos = eos_ok && step < min_new;
    int mode;
    if (!is_live) mode = MODE_SKIP;
    else if (step >= max_new - 1) mode = MODE_FORCED;
    else if (hf && step <= 0) mode = MODE_FULL;
    else mode = MODE_FILTER;
    if (!head_ok && mode != MODE_SKIP) mode = MODE_FAIL;  // the head tiles did not all complete: PAD
    int k = 0;
    if (mode == MODE_FILTER) {
        k = min(max(top_k, max(p.min_keep, 1)), V);
        if (k > p.kbuf) {
            mode = MODE_FAIL;
            if (tid == 0) set_status(p, B2S_STATUS_TOPK_LIMIT);
        }
    }
    if (tid == 32) {
        ctl->u = (p.rng == B2S_RNG_UNIFORM || !p.seeds) ? (p.uvals ? p.uvals[w] : 0.0f)
                 : p.rng == B2S_RNG_PHILOX ? uniform_philox(p.seeds[r], step, p.requests ? p.requests[r] : 0)
                                           : uniform_counter(p.seeds[r], step);
    }
    R.T = T;
    R.identity = false;
    R.bits = nullptr;  // the register pass keeps counts; the full-row paths build their own structures
    R.pref = nullptr;
    R.htv = nullptr;
    R.censor = -1;
    const bool pen_hist = mode == MODE_FILTER && p.W > 0 && hrow != nullptr;
    const bool censor = mode == MODE_FILTER && !hf && masked_eos;  // omni: EOS is -inf before anything else
    const int cens = censor ? p.eos : -1;

    // ---------------- history: each position counts its id (one shared atomic) and requests the id's raw value
    const bool hvalid = pen_hist && hthread && hv >= 0 && hv < V;
    const int hc = (int)hv - R.e0 + EPV;  // the id's byte in the count array and its slot in hval
    float hx = 0.0f;
    if (hthread) {
        hstage[tid] = hv;
        if (pen_hist && hv >= V) set_status(p, B2S_STATUS_HISTORY_RANGE);
    }
    if (hvalid) {
        atomicAdd(&cnts[hc >> 2], 1u << ((hc & 3) * 8));
        hx = R.raw(hv);
    }
    cp_async_wait_all();
    __syncthreads();  // the counts are complete; the window and the penalty table are staged

    // ---------------- processed values: the history ids' into hval (history threads), x / T into registers (all)
    if (hvalid)  // every position of the id writes the same value
        hval[hc] = hv == cens ? f_ninf()
                              : hist_proc_value(p, atab, hf, false, T,
                                                (int)((cnts[hc >> 2] >> ((hc & 3) * 8)) & 255u), hx);
    if (nx > 0) {
        uint32_t w[4] = {Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG};
#pragma unroll
        for (int j = 0; j < EPV - 1; ++j) {
            if (j < nx) {
                if constexpr (ES == 4) {
                    w[j] = ex[j];
                } else {  // element j is the low (even j) or high (odd j) half of word j / 2
                    w[j >> 1] = (j & 1) ? ((w[j >> 1] & 0x0000ffffu) | (ex[j] & 0xffff0000u))
                                        : ((w[j >> 1] & 0xffff0000u) | (ex[j] >> 16));
                }
            }
        }
        q[SV] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        q[SV] = make_uint4(Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG, Elem<E>::NEG);
    }
    float P[(SV + 1) * EPV];
#pragma unroll
    for (int s = 0; s <= SV; ++s) {
        const int valid = s < SV ? (tid + s * NT < R.nvec ? EPV : 0) : nx;
#pragma unroll
        for (int j = 0; j < EPV; ++j) P[s * EPV + j] = j < valid ? R.f(Elem<E>::at(q[s], j)) : f_ninf();
    }
    __syncthreads();  // the history ids' values are in hval

    // ---------------- the flagged elements patched from hval; the thread's maximum
    float tmax = f_ninf();
    auto counts_at = [&](int b) -> uint64_t {  // the EPV count bytes from byte b (a multiple of EPV)
        if (!pen_hist) return 0u;
        if constexpr (EPV == 4) return (uint64_t)cnts[b >> 2];
        else return reinterpret_cast<const uint64_t*>(cnts)[b >> 3];
    };
#pragma unroll
    for (int s = 0; s < SV; ++s) {
        const int v = tid + s * NT;
        const int valid = v < R.nvec ? EPV : 0;
        const uint64_t cw = valid ? counts_at((v + 1) * EPV) : 0u;
        short_patch<E>(hval, cens, cw, R.e0 + v * EPV, (v + 1) * EPV, valid, &P[s * EPV], tmax);
    }
    {
        // the head's counts end at byte EPV, the tail's start at the vector boundary after the interior
        uint64_t cw = 0u;
        if (nx > 0) cw = tid == 0 ? counts_at(0) >> (8 * (EPV - R.nh)) : counts_at((R.nvec + 1) * EPV);
        short_patch<E>(hval, cens, cw, x0, x0 - R.e0 + EPV, nx, &P[SV * EPV], tmax);
    }
    // the processed row into shared memory (over hval, indexed alike: each slot is read and rewritten by its owner
    // only): element id at hval[id + EPV - nh], where the candidates and the normaliser's exponentials are taken
    const bool want_lse = mode == MODE_FILTER && hf;
    if (mode == MODE_FILTER) {
#pragma unroll
        for (int s = 0; s < SV; ++s) {
            const int v = tid + s * NT;
            if (v < R.nvec) {
                float4* d = reinterpret_cast<float4*>(hval + (v + 1) * EPV);
#pragma unroll
                for (int j = 0; j < EPV; j += 4)
                    d[j / 4] = make_float4(P[s * EPV + j], P[s * EPV + j + 1], P[s * EPV + j + 2], P[s * EPV + j + 3]);
            }
        }
#pragma unroll
        for (int j = 0; j < EPV - 1; ++j)
            if (j < nx) hval[x0 - R.e0 + EPV + j] = P[SV * EPV + j];
    }

    // ---------------- tau: the k-th largest of the warps' jw largest thread maxima; the row's maximum
    const bool cand_path = mode == MODE_FILTER && k <= KFAST && !(p.flags & B2S_FLAG_FORCE_GENERAL) && T >= 1e-6f &&
                           T <= 1e6f;
    const int jw = (k + NWARP - 1) / NWARP;
    const int ng = NWARP * jw;  // gathered maxima, a multiple of 16, <= 128
    int ngp = 16;
    while (ngp < ng) ngp <<= 1;  // ranked as ngp values (the rest -inf)
    bool has_nan = false;
#pragma unroll
    for (int j = 0; j < (SV + 1) * EPV; ++j) has_nan |= P[j] != P[j];
    {
        uint32_t key = okey(tmax);  // tmax is never NaN (fmaxf keeps the other operand)
        const int jx = cand_path ? jw : 1;
        for (int t = 0; t < jx; ++t) {
            const uint32_t mk = __reduce_max_sync(0xffffffffu, key);
            const unsigned who = __ballot_sync(0xffffffffu, key == mk);
            if (lane == __ffs(who) - 1) key = 0u;  // below every key: taken
            if (lane == 0) {
                if (cand_path) vals[warp * jw + t] = okey_to_f(mk);
                if (t == 0) ctl->red_u[warp] = mk;
            }
        }
        if (cand_path && tid < ngp - ng) vals[ng + tid] = f_ninf();
    }
    has_nan = __syncthreads_or(has_nan) != 0;
    uint32_t mkey = ctl->red_u[0];
#pragma unroll
    for (int w = 1; w < NWARP; ++w) mkey = max(mkey, ctl->red_u[w]);
    const float m = okey_to_f(mkey);  // the row's largest processed value (NaN aside)
    // hf's full-row normaliser: the fp64 sum of exp(P - max) over the row in shared memory (a row with a NaN sums
    // to NaN, one whose maximum is +inf to +inf: taken without the exponentials; every other row's arguments
    // P - max are <= 0, the paired form's domain)
    const float mu = (m == f_inf() || m == f_ninf()) ? 0.0f : m;
    const bool lse_sum = want_lse && !has_nan && m != f_inf();
    // this thread's part of the normaliser's sum: the row's vectors t, t + nthr, ... (t = tid - first), then the
    // head (t == 0) and the tail (t == 1); the warp's sum in red_d[warp]
    auto lse_part = [&](int first, int nthr) {
        const int t = tid - first;
        double sacc = 0.0;
        const float2 nmu = make_float2(-mu, -mu);
        for (int v = t; v < R.nvec; v += nthr) {
            const float4* pv = reinterpret_cast<const float4*>(hval + (v + 1) * EPV);
#pragma unroll
            for (int j = 0; j < EPV / 4; ++j) {
                const float4 q4 = pv[j];
                const float2 e0 = b2s_expf2_nonpos(__fadd2_rn(make_float2(q4.x, q4.y), nmu));
                const float2 e1 = b2s_expf2_nonpos(__fadd2_rn(make_float2(q4.z, q4.w), nmu));
                sacc += (double)e0.x;
                sacc += (double)e0.y;
                sacc += (double)e1.x;
                sacc += (double)e1.y;
            }
        }
        if (t < 2) {
            const int c0 = t == 0 ? EPV - R.nh : (R.nvec + 1) * EPV, ne = t == 0 ? R.nh : V - i_end;
            for (int j = 0; j < ne; ++j) sacc += (double)b2s_expf(__fsub_rn(hval[c0 + j], mu));
        }
        sacc = warp_sum(sacc);
        if (lane == 0) ctl->red_d[warp] = sacc;
    };
    auto lse_of = [&](double sum) { return __fadd_rn((float)log((double)(float)sum), mu); };
    const float lse_special = has_nan ? __int_as_float(0x7fffffff) : f_inf();

    // ---------------- the row's token
    int64_t token = V - 1;
    const int drop = (hf && masked_eos) ? p.eos : -1;
    const bool topk_only = (p.flags & B2S_FLAG_TOPK_ONLY) != 0;
    float lse = 0.0f;
    if (mode == MODE_FILTER && cand_path && !has_nan) {
        // Two groups of warps from here.  Warps 0..3 rank tau, put every element >= tau (from the row in shared
        // memory) into the list in vocabulary order, and warp 0 runs the list stage; warps 4..15 meanwhile take
        // the normaliser's sum, which warp 4 hands to warp 0.  Barriers: 1 = warps 0 and 4, 2 = warps 4..15,
        // 3 = warps 0..3.
        constexpr int NL = 128;  // threads of warps 0..3
        if (warp < 4) {
            {
                // value i of the ngp ranked by S threads of one warp, each over L of the values
                const int S = min(NL / ngp, ngp), L = ngp / S;
                const int i = tid / S, sg = tid % S;
                const float x = vals[i];
                int gt = 0, eq = 0;
                for (int j = sg * L; j < sg * L + L; ++j) {
                    const float y = vals[j];
                    gt += y > x;
                    eq += y == x;
                }
                for (int o = 1; o < S; o <<= 1) {
                    gt += __shfl_xor_sync(0xffffffffu, gt, o);
                    eq += __shfl_xor_sync(0xffffffffu, eq, o);
                }
                if (sg == 0 && x > f_ninf() && gt < k && k <= gt + eq) ctl->thr = x;  // ties: the same value
            }
            named_bar_sync(3, NL);
            const float tau = ctl->thr;
            bool ok = tau > f_ninf() && tau != f_inf();
            int n = 0;
            if (ok) {
                // 4-element groups covering [cb, cb + V) (element id at cb + id), in contiguous runs per thread:
                // a count pass, a scan over the 128 threads, a write pass
                const int cb = EPV - R.nh;
                const int g0 = cb >> 2, g1 = (cb + V + 3) >> 2;
                const int per = (g1 - g0 + NL - 1) / NL;
                const int ga = g0 + tid * per, gb = min(g1, ga + per);
                const float4* pv4 = reinterpret_cast<const float4*>(hval);
                auto take = [&](int c, float v) { return c >= cb && c < cb + V && v >= tau; };
                int cnt = 0;
                for (int g = ga; g < gb; ++g) {
                    const float4 q4 = pv4[g];
                    const int c = 4 * g;
                    cnt += take(c, q4.x) + take(c + 1, q4.y) + take(c + 2, q4.z) + take(c + 3, q4.w);
                }
                int incl = cnt;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t;
                }
                int* tot = reinterpret_cast<int*>(hist);
                if (lane == 31) tot[warp] = incl;
                named_bar_sync(3, NL);
                int base = 0;
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const int x = tot[w];
                    n += x;
                    base += w < warp ? x : 0;
                }
                if (n <= p.ltot && cnt > 0) {
                    int pos = base + incl - cnt;
                    for (int g = ga; g < gb; ++g) {
                        const float4 q4 = pv4[g];
                        const float w4[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int c = 4 * g + j;
                            if (take(c, w4[j])) {
                                cand_v[pos] = w4[j];
                                cand_i[pos] = c - cb;
                                ++pos;
                            }
                        }
                    }
                }
                ok = n <= p.ltot && n >= k;
            }
            named_bar_sync(3, NL);  // the list is complete
            if (warp == 0) {
                const bool one_warp = ok && n <= KLIST;
                if (one_warp) warp_topk_sorted_n(cand_v, n, k, vals);
                if (want_lse) {
                    named_bar_sync(1, 64);
                    lse = ctl->lse;
                }
                int pos = 0x7fffffff;
                if (one_warp)
                    pos = warp_list_kept_draw(cand_v, cand_i, n, k, hf, lse, top_p, p.min_keep, topk_only, drop, ctl->u,
                                              vals, sv, si);
                if (lane == 0) {
                    ctl->kn = pos;
                    ctl->sr_state = one_warp ? 1 : ok ? 2 : 0;
                    ctl->sr_n = n;
                }
            }
        } else if (want_lse) {
            if (lse_sum) {
                lse_part(NL, NT - NL);
                named_bar_sync(2, NT - NL);
            }
            if (warp == 4) {
                double sum = 0.0;
#pragma unroll
                for (int w = 4; w < NWARP; ++w) sum += ctl->red_d[w];
                if (lane == 0) ctl->lse = lse_sum ? lse_of(sum) : lse_special;
                named_bar_arrive(1, 64);
            }
        }
        __syncthreads();
        // 1: warp 0 drew; 2: the list is complete but longer than one warp's; 0: the full-row path
        const int state = ctl->sr_state, n = ctl->sr_n;
        if (want_lse) lse = ctl->lse;
        if (state == 1) {
            const int pos = ctl->kn;
            token = pos == 0x7fffffff ? (int64_t)(V - 1) : (int64_t)si[pos];
        } else if (state == 2 && n <= 2 * KLIST) {
            __syncthreads();  // every thread has read the state before the list stage reuses ctl
            const Scr sc{hist, ctl->rctl, &ctl->gather_n, &ctl->kn, &ctl->thr, ctl->red_d, ctl->red_f, ctl->red_i};
            float thr;
            token = list_sample(cand_v, cand_i, n, k, hf, lse, top_p, p.min_keep, topk_only, true, drop, ctl->u, V, vals,
                                kv, ki, sv, si, sc, thr, true);
        } else if (state == 2) {
            __syncthreads();
            token = block_list_token(cand_v, cand_i, kv, ki, sv, si, n, k, hf, lse, top_p, p.min_keep, topk_only, drop,
                                     ctl->u, V, vals, hist, ctl);
        } else {
            __syncthreads();
            token = short_exact<E>(p, R, hb, k, hf, lse, top_p, topk_only, drop, pen_hist, censor, T, ctl->u, hist,
                                   vals, ctl);
        }
    } else if (mode == MODE_FILTER) {
        // NaN, the exact path asked for, top_k beyond the list stage or an extreme temperature: the full-row path
        if (lse_sum) {
            lse_part(0, NT);
            __syncthreads();
            double sum = 0.0;
#pragma unroll
            for (int w = 0; w < NWARP; ++w) sum += ctl->red_d[w];
            lse = lse_of(sum);
            __syncthreads();
        } else if (want_lse) {
            lse = lse_special;
        }
        token = short_exact<E>(p, R, hb, k, hf, lse, top_p, topk_only, drop, pen_hist, censor, T, ctl->u, hist, vals,
                               ctl);
    }
    if (mode == MODE_FORCED) token = eos_ok ? (int64_t)p.eos : (int64_t)(V - 1);
    if (mode == MODE_FULL) token = full_token<E>(R, drop, ctl->u, ctl);

    // ---------------- state epilogue
    const int64_t tok_drawn = (mode == MODE_SKIP || mode == MODE_FAIL) ? PAD : token;
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
        for (int j = tid; j < p.W; j += NT) ho[j] = adv ? (j + 1 < p.W ? hstage[j + 1] : tok) : hstage[j];
    }
    }  // frames
}

template <typename E, int SEM>
__global__ void __launch_bounds__(NT, 1) short_kernel(const Params p) {
    extern __shared__ __align__(128) unsigned char smem[];
    short_rows<E, SEM, false>(p, smem);
}

// The codec head and the sampling step in one launch: CTAs [0, rows) take the rows (above), CTAs
// [head_first, head_first + head_split * head_tiles) the vocabulary tiles of the head (b2s_head.cuh), one or two
// (a cluster splitting K) per tile.
template <int SEM>
__global__ void __launch_bounds__(NT, 1) head_kernel(const Params p, const __grid_constant__ CUtensorMap amap) {
    extern __shared__ __align__(128) unsigned char smem[];
    if ((int)blockIdx.x >= p.rows) {
        if ((int)blockIdx.x < p.head_first) return;  // the pad CTA of an odd row count (clusters of two)
        const int tt = (int)blockIdx.x - p.head_first;
        head_tile(tt / p.head_split, p.head_split, p.head_split > 1 ? (int)cluster_ctarank() : 0, p.rows, p.V,
                  p.head_kb, p.hidden, p.hid_stride, static_cast<uint16_t*>(const_cast<void*>(p.logits)), p.lstride,
                  p.head_sync, p.status, &amap, smem);
        return;
    }
    short_rows<__nv_bfloat16, SEM, true>(p, smem);
}

HeadKernel head_kernel_for(bool omni) { return omni ? head_kernel<B2S_SEM_OMNI> : head_kernel<-1>; }

ResKernel short_kernel_for(bool bf16, bool omni) {
    static const ResKernel k[2][2] = {
        {short_kernel<float, -1>, short_kernel<float, B2S_SEM_OMNI>},
        {short_kernel<__nv_bfloat16, -1>, short_kernel<__nv_bfloat16, B2S_SEM_OMNI>}};
    return k[bf16 ? 1 : 0][omni ? 1 : 0];
}

}  // namespace b2s
