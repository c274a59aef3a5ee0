// The Thinker's greedy step from its LM head on the tensor cores (sm_100a): token[n] = argmax_m
// bf16(sum_k hidden[n, k] * head[m, k]) -- the F.linear(hidden, lm_head) -> .float() -> argmax(-1) of
// engine/runtime/thinker_decode.py:83,107 and engine/runtime/backend_s.py:893 -- without writing the logits.
//
// One CTA per 128-id tile of the vocabulary (three per SM): a ring of LM_STAGES shared-memory stages, each one TMA load of the
// head's [128 ids x 64] block and one of the hidden rows' [64 rows x 64] block (128-byte swizzle, K-major; rows
// beyond the batch read as zero), filled by one thread and drained by another that issues tcgen05.mma (M = 128
// ids, N = 64 batch rows, K = 16) into a 64-column fp32 accumulator in tensor memory; each MMA group frees its
// stage through tcgen05.commit.  The epilogue reads the accumulator back (lane = id, column = batch row), rounds
// every logit to bf16 as F.linear's bf16 output is rounded, and reduces each row over the tile's ids to one
// 64-bit key -- the order key of the value above the complement of the id, so the maximum key is the largest value
// at its first id, NaN above every number (torch's argmax) -- which one atomicMax merges into the row's key in
// global memory.  A one-block kernel then turns the keys into tokens and zeroes them for the next call.
//
// The head (V x H x 2 bytes, 1.24 GB for Qwen3-8B) crosses DRAM once; the hidden rows are re-read from L2 by every
// tile.  Every wait is bounded; a wait that gives up records B2S_STATUS_WAIT_TIMEOUT.
#include <string.h>

#include "b2s_head.cuh"

namespace b2s {

constexpr int LM_M = 128, LM_N = 64, LM_KB = 64, LM_STAGES = 3, LM_THREADS = 128;
constexpr uint32_t LM_A_BYTES = LM_M * LM_KB * 2;  // 16 KB: the head's block of a stage
constexpr uint32_t LM_B_BYTES = LM_N * LM_KB * 2;  // 8 KB: the hidden rows' block
constexpr uint32_t LM_STAGE_BYTES = LM_A_BYTES + LM_B_BYTES;
constexpr uint32_t LM_TMEM_COLS = 64;
// 1 KB alignment slack, the stages (the warps' keys [4][64] reuse them once the MMAs are done), the mbarriers /
// TMEM address / flags: 75 KB, so that three CTAs share an SM -- 444 per wave on 148 SMs, 2.7 waves for the
// Thinker's 1,187 tiles, the last of them still enough CTAs to keep HBM busy
constexpr uint32_t LM_SMEM = 1024 + LM_STAGES * LM_STAGE_BYTES + 256;
constexpr uint32_t LM_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(LM_N >> 3) << 17) |
                              ((uint32_t)(LM_M >> 4) << 24);

// order key of a logit: NaN above every number, -0 as +0 (equal values keep the first id)
__device__ __forceinline__ uint32_t argmax_key(float x) {
    if (x != x) return 0xffffffffu;
    return okey(x == 0.0f ? 0.0f : x);
}

__global__ void __launch_bounds__(LM_THREADS, 3)
    lmhead_argmax_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, int V,
                         int rows, int nkb, unsigned long long* keys, uint32_t* status) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = (int)blockIdx.x * LM_M;
    const uint32_t base_u = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((base_u + 1023u) & ~1023u) - base_u);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + LM_STAGES * LM_STAGE_BYTES);
    uint64_t* empty = full + LM_STAGES;
    uint64_t* done = empty + LM_STAGES;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* fail = reinterpret_cast<volatile int*>(tslot + 1);
    volatile int* issued = fail + 1;    // stage loads the producer issued
    volatile int* consumed = fail + 2;  // stage loads the MMA thread saw land
    unsigned long long* wkey = reinterpret_cast<unsigned long long*>(sm);  // the stages are free once `done`

    if (tid == 0) {
        prefetch_tensormap(&amap);
        prefetch_tensormap(&bmap);
        for (int s = 0; s < LM_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        *fail = 0;
        *issued = 0;
        *consumed = 0;
    }
    if (warp == 2) tmem_alloc(tslot, LM_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_wait_then_release();  // the hidden rows are the previous kernel's output

    if (tid == 0) {  // producer: fill the ring
        int n = 0;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % LM_STAGES;
            if (kb >= LM_STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)((kb / LM_STAGES) - 1) & 1u, HEAD_WAIT_NS)) {
                *fail = 1;
                break;
            }
            if (*fail) break;
            unsigned char* st = sm + s * LM_STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], LM_STAGE_BYTES);
            tma_load_2d(st, &amap, kb * LM_KB, m0, &full[s]);                // ids >= V read as zero
            tma_load_2d(st + LM_A_BYTES, &bmap, kb * LM_KB, 0, &full[s]);    // rows >= `rows` read as zero
            n = kb + 1;
        }
        *issued = n;
    } else if (tid == 32) {  // MMA issuer: drain the ring
        int n = 0;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % LM_STAGES;
            if (!mbar_wait_bounded(&full[s], (uint32_t)(kb / LM_STAGES) & 1u, HEAD_WAIT_NS)) {
                *fail = 1;
                break;
            }
            n = kb + 1;
            tc_fence_after();
            const uint32_t a0 = smem_u32(sm + s * LM_STAGE_BYTES), b0 = a0 + LM_A_BYTES;
#pragma unroll
            for (int k = 0; k < LM_KB / 16; ++k)
                umma_bf16(tmem, umma_desc_sw128(a0 + 32u * k), umma_desc_sw128(b0 + 32u * k), LM_IDESC,
                          (kb | k) != 0 ? 1u : 0u);
            umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        *consumed = n;
        umma_commit(done);
    }

    const bool ready = mbar_wait_bounded(done, 0u, HEAD_WAIT_NS);
    tc_fence_after();
    uint32_t v[LM_N];
#pragma unroll
    for (int q = 0; q < LM_N / 16; ++q) {
        uint32_t part[16];
        tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + 16u * q, part);  // lane = id, column = batch row
#pragma unroll
        for (int j = 0; j < 16; ++j) v[16 * q + j] = part[j];
    }
    tc_fence_before();
    __syncthreads();  // the flags are visible; every thread has read its accumulator
    const bool good = ready && *fail == 0;
    const int m = m0 + warp * 32 + lane;
#pragma unroll
    for (int n = 0; n < LM_N; ++n) {
        if (n < rows) {
            const float x = __bfloat162float(__float2bfloat16_rn(__uint_as_float(v[n])));
            const uint32_t k = (good && m < V) ? argmax_key(x) : 0u;
            const uint32_t km = __reduce_max_sync(0xffffffffu, k);
            const uint32_t im = __reduce_min_sync(0xffffffffu, (k == km && km != 0u) ? (uint32_t)m : 0xffffffffu);
            if (lane == 0) wkey[warp * LM_N + n] = km ? ((unsigned long long)km << 32) | (0xffffffffu - im) : 0ull;
        }
    }
    __syncthreads();
    if (tid < rows) {
        unsigned long long best = wkey[tid];
#pragma unroll
        for (int w = 1; w < 4; ++w) best = max(best, wkey[w * LM_N + tid]);
        if (best) atomicMax(&keys[tid], best);
    }
    if (tid == 0 && !good) {
        if (status) atomicOr(status, B2S_STATUS_WAIT_TIMEOUT);
        // loads that were issued but not seen landing still write this CTA's shared memory: wait for them
        for (int kb = *consumed; kb < *issued; ++kb)
            mbar_wait_bounded(&full[kb % LM_STAGES], (uint32_t)(kb / LM_STAGES) & 1u, HEAD_WAIT_NS);
    }
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, LM_TMEM_COLS);
    }
}

// The rows' keys -> tokens (PAD for a row no tile reached), the keys zeroed for the next call.
__global__ void lmhead_finish_kernel(unsigned long long* keys, int rows, int64_t* tokens) {
    const int r = (int)threadIdx.x;
    if (r < rows) {
        const unsigned long long k = keys[r];
        tokens[r] = k ? (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull)) : (int64_t)-1;  // -1: PAD
        keys[r] = 0ull;
    }
}

// Vocabulary shards: the rows' keys with the shard's first global id added, in an order that a signed 64-bit
// maximum preserves (the top bit flipped), INT64_MIN for a row no tile reached; the keys zeroed for the next call.
// A max-all-reduce of these words over the shards leaves every rank with the global maximum's key.
__global__ void lmhead_keys_kernel(unsigned long long* keys, int rows, int64_t offset, int64_t* keys_out) {
    const int r = (int)threadIdx.x;
    if (r < rows) {
        const unsigned long long k = keys[r];
        int64_t out = INT64_MIN;
        if (k) {
            const uint64_t id = (uint64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull)) + (uint64_t)offset;
            const uint64_t g = (k & 0xffffffff00000000ull) | (0xffffffffull - id);
            out = (int64_t)(g ^ 0x8000000000000000ull);
        }
        keys_out[r] = out;
        keys[r] = 0ull;
    }
}

// Launches the tiles and the finishing block on `stream` (the argument checks and TMA maps are the caller's).
cudaError_t lmhead_argmax_launch(const CUtensorMap& amap, const CUtensorMap& bmap, int vocab, int rows, int nkb,
                                 int64_t* tokens, unsigned long long* keys, uint32_t* status, void* stream,
                                 int64_t offset, int64_t* keys_out) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        e = cudaFuncSetAttribute(lmhead_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LM_SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)((vocab + LM_M - 1) / LM_M), 1, 1);
    cfg.blockDim = dim3(LM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = LM_SMEM;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, lmhead_argmax_kernel, amap, bmap, vocab, rows, nkb, keys, status);
    if (e != cudaSuccess) return e;
    if (keys_out)
        lmhead_keys_kernel<<<1, LM_N, 0, (cudaStream_t)stream>>>(keys, rows, offset, keys_out);
    else
        lmhead_finish_kernel<<<1, LM_N, 0, (cudaStream_t)stream>>>(keys, rows, tokens);
    return cudaGetLastError();
}

}  // namespace b2s
