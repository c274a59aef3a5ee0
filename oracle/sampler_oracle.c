/*
 * CPU oracle for the MiniCPM-o 4.5 token-sampling path.  TEST INFRASTRUCTURE ONLY:
 * the product never links, loads or calls this file.  It is the checker that the CUDA
 * path in the package is compared against (tests/, __graft_entry__.smoke(), and the
 * cpu_baseline / --impl reference legs of bench.py).
 *
 * It restates, row by row and over the full vocabulary (no candidate tricks), the
 * algorithm of the reference module engine/talker_sampler.py:
 *   uniform / _mix32 ............ engine/talker_sampler.py:60-76
 *   repetition_penalty .......... engine/talker_sampler.py:79-84
 *   top_p_top_k_filter (hf) ..... engine/talker_sampler.py:101-116
 *   top_k_top_p_filter (omni) ... engine/talker_sampler.py:119-133
 *   processed_logits ............ engine/talker_sampler.py:136-158
 *   draw ........................ engine/talker_sampler.py:161-172
 * plus the Thinker greedy step (argmax, lowest index wins; engine/runtime/thinker_decode.py:107)
 * and two extensions the reference does not have (parity unpinned for those):
 * Philox4x32-10 uniforms and presence/frequency penalties.
 *
 * Floating-point contract shared with the CUDA kernels (the "sampler numerics spec"):
 *  - every fp32 op that the reference does element-wise (x/T, x*alpha, x/alpha, v-lse,
 *    e/s, u*S) is one IEEE fp32 operation, round to nearest even;
 *  - exp is b2s_expf below (Cody-Waite reduction + degree-7 Taylor polynomial by FMA
 *    Horner); the CUDA side evaluates the identical operation sequence;
 *  - sums that torch accumulates (sum, cumsum) accumulate in fp64 and round once to fp32;
 *  - log is the fp64 log rounded to fp32.
 * torch's CPU softmax/exp use their own vectorised exp, so against the reference itself
 * results agree up to last-ulp rounding; tokens then agree except where the uniform or
 * the top-p mass lands within float rounding of a boundary.  Those margins are returned
 * per row (orc_meta) so every disagreement can be classified.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_HF 0
#define ORC_OMNI 1
#define ORC_RNG_UNIFORM 0 /* caller-supplied uniforms (draw(uniform_values=...)) */
#define ORC_RNG_COUNTER 1 /* reference lowbias32 counter hash */
#define ORC_RNG_PHILOX 2  /* Philox4x32-10 keyed on (seed, step, request) */

typedef struct {
    int32_t vocab;
    int32_t window;
    int32_t eos;       /* column index; outside [0, vocab) means "no EOS column" */
    int32_t semantics; /* ORC_HF / ORC_OMNI */
    int32_t top_k;
    int32_t min_keep;  /* hf only; omni always uses 1 (talker_sampler.py:147) */
    float temperature;
    float top_p;
    float presence;    /* extension: subtract presence once for seen tokens (omni order only) */
    float frequency;   /* extension: subtract frequency*count (omni order only) */
    int64_t min_new;
    int64_t max_new;
    int32_t apply_filter_at_step0; /* hf: 0 (reference); kept for completeness */
    int32_t pad_;
} orc_cfg;

typedef struct {
    int32_t kept;        /* number of kept values in the top-k list (value threshold rank) */
    int32_t mode;        /* 0 filtered, 1 full row (hf frame 0), 2 forced EOS */
    float thr;           /* value threshold (processed domain) */
    float lse;           /* hf full-row logsumexp */
    double topp_margin;  /* min_j |above_j - top_p| (absolute, probabilities) */
    double draw_margin;  /* min_j |cdf_j - target| / cdf_last over kept boundaries */
    float target;        /* u * cdf_last */
    float cdf_last;
    int64_t token;
} orc_meta;

/* ---------------------------------------------------------------- exp / log */

static inline float f_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t bits_from_f(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* exp(x) for fp32: n = rint(x*log2 e); r = x - n*ln2 in two FMA steps (Cody & Waite,
 * "Software Manual for the Elementary Functions", 1980); exp(r) by the Taylor series to
 * degree 7 evaluated with FMA Horner (|r| <= 0.347 so the truncation term r^8/8! is
 * below 6e-9); scale by 2^n through exact power-of-two multiplies. */
float b2s_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    float t = x * 1.44269502162933349609375f;
    float n = rintf(t);
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.428606765330187045037746429443359375e-6f, r);
    float p = 1.98412701138295233249664306640625e-4f; /* 1/5040 */
    p = fmaf(p, r, 1.3888889225199818611145019531250e-3f);  /* 1/720 */
    p = fmaf(p, r, 8.3333337679505348205566406250000e-3f);  /* 1/120 */
    p = fmaf(p, r, 4.1666667908430099487304687500000e-2f);  /* 1/24 */
    p = fmaf(p, r, 1.6666667163372039794921875000000e-1f);  /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) { p = p * 2.0f; ni -= 1; }
    if (ni < -126) { p = p * 5.42101086242752217003726400434970855712890625e-20f; ni += 64; } /* 2^-64 */
    return p * f_from_bits((uint32_t)(ni + 127) << 23);
}

static inline float logf_via_double(float s) { return (float)log((double)s); }

/* ---------------------------------------------------------------- RNG */

static inline uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7FEB352Du;
    x ^= x >> 15;
    x *= 0x846CA68Bu;
    x ^= x >> 16;
    return x;
}

/* talker_sampler.py:70-76: the three chained finalisers over seed lo, seed hi, step. */
float orc_uniform_counter(int64_t seed, int64_t step) {
    uint64_t s = (uint64_t)seed;
    uint32_t h = mix32((uint32_t)(s & 0xFFFFFFFFu));
    h = mix32(h ^ (uint32_t)((s >> 32) & 0xFFFFFFFFu) ^ 0x9E3779B9u);
    h = mix32(h ^ (uint32_t)((uint64_t)step & 0xFFFFFFFFu) ^ 0x632BE5ABu);
    return (float)(h >> 8) * (1.0f / 16777216.0f);
}

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy as 1, 2,
 * 3", SC'11): 10 rounds of the 4x32 S-box with multipliers 0xD2511F53 / 0xCD9E8D57 and
 * Weyl key increments 0x9E3779B9 / 0xBB67AE85. */
void orc_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int i = 0; i < 10; ++i) {
        if (i) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

float orc_uniform_philox(int64_t seed, int64_t step, int64_t request) {
    uint32_t key[2] = {(uint32_t)((uint64_t)seed & 0xFFFFFFFFu), (uint32_t)((uint64_t)seed >> 32)};
    uint32_t ctr[4] = {(uint32_t)((uint64_t)step & 0xFFFFFFFFu), (uint32_t)((uint64_t)step >> 32),
                       (uint32_t)((uint64_t)request & 0xFFFFFFFFu), (uint32_t)((uint64_t)request >> 32)};
    uint32_t out[4];
    orc_philox4x32_10(ctr, key, out);
    return (float)(out[0] >> 8) * (1.0f / 16777216.0f);
}

void orc_uniform_batch(const int64_t* seeds, const int64_t* steps, const int64_t* requests, int64_t n, int32_t rng,
                       float* out) {
    for (int64_t i = 0; i < n; ++i)
        out[i] = rng == ORC_RNG_PHILOX ? orc_uniform_philox(seeds[i], steps[i], requests ? requests[i] : 0)
                                       : orc_uniform_counter(seeds[i], steps[i]);
}

/* ---------------------------------------------------------------- top-k (values) */

/* k largest values of y[0..n) in descending order (ties kept with multiplicity), via a
 * bounded min-heap: the value list torch.topk returns (talker_sampler.py:111, :128). */
static void topk_values(const float* y, int32_t n, int32_t k, float* vals) {
    float* h = vals; /* min-heap in place, size k */
    int32_t sz = 0;
    for (int32_t i = 0; i < n; ++i) {
        float v = y[i];
        if (sz < k) {
            int32_t j = sz++;
            h[j] = v;
            while (j > 0) {
                int32_t p = (j - 1) >> 1;
                if (h[p] <= h[j]) break;
                float t = h[p]; h[p] = h[j]; h[j] = t; j = p;
            }
        } else if (v > h[0]) {
            h[0] = v;
            int32_t j = 0;
            for (;;) {
                int32_t l = 2 * j + 1, r = l + 1, m = j;
                if (l < sz && h[l] < h[m]) m = l;
                if (r < sz && h[r] < h[m]) m = r;
                if (m == j) break;
                float t = h[m]; h[m] = h[j]; h[j] = t; j = m;
            }
        }
    }
    /* heap-sort the k values into descending order */
    for (int32_t end = sz - 1; end > 0; --end) {
        float t = h[0]; h[0] = h[end]; h[end] = t;
        int32_t j = 0;
        for (;;) {
            int32_t l = 2 * j + 1, r = l + 1, m = j;
            if (l < end && h[l] < h[m]) m = l;
            if (r < end && h[r] < h[m]) m = r;
            if (m == j) break;
            float t2 = h[m]; h[m] = h[j]; h[j] = t2; j = m;
        }
    }
}

/* Shared tail of both filters: exclusive-above cumulative mass of the descending top-k
 * probabilities p[], cut at top_p, clamped to [min(min_keep,k), k]; returns kept count.
 * talker_sampler.py:113-114 / :130-131 (cumsum accumulates in fp64 on CPU). */
static int32_t topp_cut(const float* p, int32_t k, float top_p, int32_t min_keep, double* margin) {
    double acc = 0.0;
    int32_t cnt = 0;
    double mg = INFINITY;
    for (int32_t j = 0; j < k; ++j) {
        acc += (double)p[j];
        float cum = (float)acc;
        float above = cum - p[j];
        if (above < top_p) cnt++;
        double d = fabs((double)above - (double)top_p);
        if (d < mg) mg = d;
    }
    int32_t lo = min_keep < k ? min_keep : k;
    if (cnt < lo) cnt = lo;
    if (cnt > k) cnt = k;
    if (margin) *margin = mg;
    return cnt;
}

/* ---------------------------------------------------------------- processed_logits */

static inline float penalise(float v, int32_t n, const float* alpha) {
    if (n <= 0) return v; /* alpha = penalty**0 = 1 exactly: v*1 == v/1 == v */
    float a = alpha[n];
    return v < 0.0f ? v * a : v / a;
}

/* One row of processed_logits (talker_sampler.py:136-158).  counts[V] is scratch. */
static void process_row(const float* x, const int64_t* hist, int64_t step, const float* alpha, int32_t alpha_len,
                        const orc_cfg* c, float* y, int32_t* counts, float* vals, float* pk, orc_meta* meta,
                        int32_t* bad_history) {
    const int32_t V = c->vocab;
    const int eos_ok = c->eos >= 0 && c->eos < V;
    memset(counts, 0, sizeof(int32_t) * (size_t)V);
    for (int32_t j = 0; j < c->window; ++j) {
        int64_t id = hist[j];
        if (id < 0) continue;
        if (id >= V) { *bad_history = 1; continue; }
        counts[id]++;
    }
    for (int32_t i = 0; i < V; ++i)
        if (counts[i] >= alpha_len) { *bad_history = 1; counts[i] = alpha_len - 1; }
    meta->mode = 0;
    meta->kept = 0;
    meta->thr = -INFINITY;
    meta->lse = NAN;
    meta->topp_margin = INFINITY;
    const float T = c->temperature;
    const int masked_eos = eos_ok && step < c->min_new;
    if (c->semantics == ORC_OMNI) {
        for (int32_t i = 0; i < V; ++i) {
            float z = (masked_eos && i == c->eos) ? -INFINITY : x[i];
            float v = penalise(z, counts[i], alpha);
            if (counts[i] > 0) {
                v = v - c->presence;
                v = v - c->frequency * (float)counts[i];
            }
            y[i] = v / T;
        }
        int32_t k = c->top_k > 1 ? c->top_k : 1;
        if (k > V) k = V;
        topk_values(y, V, k, vals);
        /* softmax over the k values (talker_sampler.py:129) */
        float m = vals[0];
        double s = 0.0;
        for (int32_t j = 0; j < k; ++j) { pk[j] = b2s_expf(vals[j] - m); s += (double)pk[j]; }
        float sf = (float)s;
        for (int32_t j = 0; j < k; ++j) pk[j] = pk[j] / sf;
        int32_t kept = topp_cut(pk, k, c->top_p, 1, &meta->topp_margin);
        float thr = vals[kept - 1];
        for (int32_t i = 0; i < V; ++i)
            if (y[i] < thr) y[i] = -INFINITY;
        meta->kept = kept;
        meta->thr = thr;
    } else {
        for (int32_t i = 0; i < V; ++i) y[i] = x[i] / T;
        if (step > 0 || c->apply_filter_at_step0) {
            for (int32_t i = 0; i < V; ++i) y[i] = penalise(y[i], counts[i], alpha);
            int32_t k = c->top_k > c->min_keep ? c->top_k : c->min_keep;
            if (k > V) k = V;
            topk_values(y, V, k, vals);
            /* torch.logsumexp: max, then log(sum(exp(y - max))) + max (infinite max -> 0) */
            float m = -INFINITY;
            for (int32_t i = 0; i < V; ++i) if (y[i] > m) m = y[i];
            float mu = isinf(m) ? 0.0f : m;
            double s = 0.0;
            for (int32_t i = 0; i < V; ++i) s += (double)b2s_expf(y[i] - mu);
            float lse = logf_via_double((float)s) + mu;
            for (int32_t j = 0; j < k; ++j) pk[j] = b2s_expf(vals[j] - lse);
            int32_t kept = topp_cut(pk, k, c->top_p, c->min_keep, &meta->topp_margin);
            float thr = vals[kept - 1];
            for (int32_t i = 0; i < V; ++i)
                if (y[i] < thr) y[i] = -INFINITY;
            meta->kept = kept;
            meta->thr = thr;
            meta->lse = lse;
        } else {
            meta->mode = 1;
        }
        if (masked_eos) y[c->eos] = -INFINITY;
    }
    if (step >= c->max_new - 1) {
        meta->mode = 2;
        for (int32_t i = 0; i < V; ++i) y[i] = -INFINITY;
        if (eos_ok) y[c->eos] = 0.0f;
    }
}

/* ---------------------------------------------------------------- draw */

/* talker_sampler.py:161-172: softmax over the row, cumsum in vocabulary order (fp64
 * accumulation), target u*cdf[-1], searchsorted(right=True) = first index whose cdf
 * exceeds the target, clamped to V-1 (also the result for an all -inf / NaN row). */
static int64_t draw_row(const float* y, int32_t V, float u, float* e, orc_meta* meta) {
    float m = -INFINITY;
    for (int32_t i = 0; i < V; ++i) if (y[i] > m) m = y[i];
    double s = 0.0;
    for (int32_t i = 0; i < V; ++i) { e[i] = b2s_expf(y[i] - m); s += (double)e[i]; }
    float sf = (float)s;
    double acc = 0.0;
    /* first pass: cdf_last */
    for (int32_t i = 0; i < V; ++i) acc += (double)(e[i] / sf);
    float last = (float)acc;
    float target = u * last;
    int64_t tok = V - 1;
    double mg = INFINITY;
    int found = 0;
    acc = 0.0;
    for (int32_t i = 0; i < V; ++i) {
        float p = e[i] / sf;
        if (p == 0.0f) continue;
        acc += (double)p;
        float cdf = (float)acc;
        double d = fabs((double)cdf - (double)target);
        if (d < mg) mg = d;
        if (!found && cdf > target) { tok = i; found = 1; }
    }
    if (meta) {
        meta->target = target;
        meta->cdf_last = last;
        meta->draw_margin = last > 0.0f ? mg / (double)last : INFINITY;
        meta->token = tok;
    }
    return tok;
}

/* ---------------------------------------------------------------- batch entry points */

typedef struct {
    const void* logits;     /* [rows, vocab] fp32 (dtype 0) or bf16 bits (dtype 1) */
    int32_t logits_dtype;
    int32_t rows;
    int64_t logits_row_stride;
    const int64_t* history; /* [rows, window] */
    int64_t history_row_stride;
    const int64_t* steps;   /* [rows] */
    const int64_t* seeds;   /* [rows] */
    const int64_t* requests;/* [rows] or NULL */
    const float* uniforms;  /* [rows] (rng == ORC_RNG_UNIFORM) */
    const float* alpha;     /* [rows or 1][alpha_len] */
    int32_t alpha_len;
    int32_t alpha_row_stride;
    const float* row_temperature; /* per-row overrides or NULL */
    const float* row_top_p;
    const int32_t* row_top_k;
    int32_t rng;
    int32_t threads;
    float* processed;       /* [rows, vocab] or NULL */
    int64_t* tokens;        /* [rows] or NULL */
    orc_meta* meta;         /* [rows] or NULL */
    int32_t* bad_history;   /* out flag or NULL */
    const int64_t* row_min_new; /* per-row min_new_tokens / max_new_tokens overrides or NULL */
    const int64_t* row_max_new;
} orc_batch;

static inline float bf16_to_f(uint16_t b) { return f_from_bits((uint32_t)b << 16); }

int orc_sample_batch(const orc_batch* b, const orc_cfg* cfg) {
    const int32_t V = cfg->vocab;
    int32_t bad = 0;
#ifdef _OPENMP
    if (b->threads > 0) omp_set_num_threads(b->threads);
#pragma omp parallel reduction(| : bad)
#endif
    {
        float* x = (float*)malloc(sizeof(float) * (size_t)V);
        float* y = (float*)malloc(sizeof(float) * (size_t)V);
        float* e = (float*)malloc(sizeof(float) * (size_t)V);
        int32_t* counts = (int32_t*)malloc(sizeof(int32_t) * (size_t)V);
        float* vals = (float*)malloc(sizeof(float) * (size_t)V);
        float* pk = (float*)malloc(sizeof(float) * (size_t)V);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int32_t r = 0; r < b->rows; ++r) {
            if (b->logits_dtype == 1) {
                const uint16_t* src = (const uint16_t*)b->logits + (size_t)r * (size_t)b->logits_row_stride;
                for (int32_t i = 0; i < V; ++i) x[i] = bf16_to_f(src[i]);
            } else {
                const float* src = (const float*)b->logits + (size_t)r * (size_t)b->logits_row_stride;
                memcpy(x, src, sizeof(float) * (size_t)V);
            }
            orc_cfg c = *cfg;
            if (b->row_temperature) c.temperature = b->row_temperature[r];
            if (b->row_top_p) c.top_p = b->row_top_p[r];
            if (b->row_top_k) c.top_k = b->row_top_k[r];
            if (b->row_min_new) c.min_new = b->row_min_new[r];
            if (b->row_max_new) c.max_new = b->row_max_new[r];
            orc_meta m;
            memset(&m, 0, sizeof(m));
            int32_t bh = 0;
            process_row(x, b->history + (size_t)r * (size_t)b->history_row_stride, b->steps[r],
                        b->alpha + (size_t)r * (size_t)b->alpha_row_stride, b->alpha_len, &c, y, counts, vals, pk,
                        &m, &bh);
            bad |= bh;
            if (b->processed) memcpy(b->processed + (size_t)r * (size_t)V, y, sizeof(float) * (size_t)V);
            if (b->tokens || b->meta) {
                float u;
                if (b->rng == ORC_RNG_UNIFORM) u = b->uniforms[r];
                else if (b->rng == ORC_RNG_PHILOX)
                    u = orc_uniform_philox(b->seeds[r], b->steps[r], b->requests ? b->requests[r] : 0);
                else u = orc_uniform_counter(b->seeds[r], b->steps[r]);
                int64_t tok = draw_row(y, V, u, e, &m);
                if (b->tokens) b->tokens[r] = tok;
            }
            if (b->meta) b->meta[r] = m;
        }
        free(x); free(y); free(e); free(counts); free(vals); free(pk);
    }
    if (b->bad_history) *b->bad_history = bad;
    return 0;
}

/* draw() on given fp32 rows (talker_sampler.py:161-172). */
int orc_draw_batch(const float* x, int32_t rows, int32_t V, int64_t row_stride, const float* uniforms, int64_t* tokens,
                   orc_meta* meta, int32_t threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
    {
        float* e = (float*)malloc(sizeof(float) * (size_t)V);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int32_t r = 0; r < rows; ++r) {
            orc_meta m;
            memset(&m, 0, sizeof(m));
            tokens[r] = draw_row(x + (size_t)r * (size_t)row_stride, V, uniforms[r], e, &m);
            if (meta) meta[r] = m;
        }
        free(e);
    }
    return 0;
}

/* Thinker greedy step: argmax over the row, first index among equal maxima; NaN is the
 * maximum (torch.argmax semantics), engine/runtime/thinker_decode.py:107. */
int orc_argmax_batch(const void* logits, int32_t dtype, int32_t rows, int32_t V, int64_t row_stride,
                     int64_t* tokens) {
    for (int32_t r = 0; r < rows; ++r) {
        int64_t best = 0;
        float bv = -INFINITY;
        int have = 0;
        for (int32_t i = 0; i < V; ++i) {
            float v = dtype == 1 ? bf16_to_f(((const uint16_t*)logits)[(size_t)r * (size_t)row_stride + (size_t)i])
                                 : ((const float*)logits)[(size_t)r * (size_t)row_stride + (size_t)i];
            if (v != v) { best = i; break; }
            if (!have || v > bv) { bv = v; best = i; have = 1; }
        }
        tokens[r] = best;
    }
    return 0;
}

/* exposed for the accuracy test of b2s_expf against fp64 exp */
void orc_expf_batch(const float* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = b2s_expf(x[i]);
}
