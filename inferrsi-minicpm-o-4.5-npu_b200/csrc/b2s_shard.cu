// Vocabulary-sharded Thinker head, stage 2: every rank holds the all-gathered candidate lists of all shards
// ([shards][rows][cap] values / global ids, plus the count each shard produced) and draws the row's token.
// A shard's list holds every element >= that shard's k-th value, so their union holds every element >= the
// row's k-th value; the list stage (b2s_list.cuh) then gives the same top-k values, threshold and token as
// the unsharded sampling kernel.
#include <stdio.h>
#include <string.h>

#include "../../include/b2s_sampler.h"
#include "b2s_device.cuh"
#include "b2s_list.cuh"

namespace b2s {

int cuda_fail(cudaError_t e);  // b2s_sampler.cu

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
    uint32_t* status;
    int nmax;  // shards * cap
};

struct MergeCtl {
    uint32_t rctl[2];
    int gather_n, kn, n, bad;
    float thr;
    double red_d[NWARP + 1];
    float red_f[NWARP + 1];
    int red_i[NWARP + 1];
    int offs[65];
};

__global__ void __launch_bounds__(NT, 1) shard_merge_kernel(const MergeParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int r = blockIdx.x, tid = threadIdx.x;
    MergeCtl* ctl = reinterpret_cast<MergeCtl*>(smem);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + ((sizeof(MergeCtl) + 15) / 16 * 16));
    float* vals = reinterpret_cast<float*>(hist + 256);
    float* cv = vals + 2 * KLIST;
    int* ci = reinterpret_cast<int*>(cv + p.nmax);
    float* kv = reinterpret_cast<float*>(ci + p.nmax);
    int* ki = reinterpret_cast<int*>(kv + p.nmax);
    float* sv = reinterpret_cast<float*>(ki + p.nmax);
    int* si = reinterpret_cast<int*>(sv + p.nmax);
    if (tid == 0) {
        int off = 0, bad = 0;
        for (int s = 0; s < p.shards; ++s) {
            const int c = p.cn[(int64_t)s * p.rows + r];
            ctl->offs[s] = off;
            if (c < 0 || c > p.cap) bad = 1;
            off += max(0, min(c, p.cap));
        }
        ctl->offs[p.shards] = off;
        ctl->n = off;
        ctl->bad = bad;
    }
    __syncthreads();
    const int n = ctl->n;
    const int top_k = p.rK ? p.rK[r] : p.top_k;
    const int k = min(max(top_k, max(p.min_keep, 1)), p.V);
    if (ctl->bad || n < k || k > KLIST) {
        if (tid == 0) {
            p.tokens[r] = -1;
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
    const Scr sc{hist, ctl->rctl, &ctl->gather_n, &ctl->kn, &ctl->thr, ctl->red_d, ctl->red_f, ctl->red_i};
    const float top_p = p.rP ? p.rP[r] : p.top_p;
    const int64_t step = p.steps ? p.steps[r] : 0;
    const float u = p.rng == B2S_RNG_UNIFORM ? p.uvals[r]
                    : p.rng == B2S_RNG_PHILOX ? uniform_philox(p.seeds[r], step, p.requests ? p.requests[r] : 0)
                                              : uniform_counter(p.seeds[r], step);
    float thr;
    const int64_t tok = list_sample(cv, ci, n, k, false, 0.0f, top_p, p.min_keep, (p.flags & B2S_FLAG_TOPK_ONLY) != 0,
                                    true, -1, u, p.V, vals, kv, ki, sv, si, sc, thr);
    if (tid == 0) p.tokens[r] = tok;
}

}  // namespace b2s

extern "C" int b2s_shard_merge(const float* cand_values, const int32_t* cand_ids, const int32_t* cand_count,
                               int32_t shards, int32_t rows, int32_t cap, int32_t vocab, const b2s_sample_args* a,
                               void* stream) {
    using namespace b2s;
    if (!cand_values || !cand_ids || !cand_count || !a || !a->tokens) return B2S_ERR_INVALID;
    if (shards < 1 || shards > 64 || rows < 0 || cap < 1 || vocab < 1) return B2S_ERR_INVALID;
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
    p.status = a->status;
    p.nmax = shards * cap;
    const size_t smem = (sizeof(MergeCtl) + 15) / 16 * 16 + 256 * 4 + 2 * KLIST * 4 + (size_t)p.nmax * 4 * 6;
    if (smem > 227 * 1024) return B2S_ERR_UNSUPPORTED;
    cudaError_t e = cudaFuncSetAttribute(shard_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e);
    shard_merge_kernel<<<(unsigned)rows, NT, smem, (cudaStream_t)stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return B2S_OK;
}
