// The Talker codec head on the tensor cores (sm_100a): logits[n, m] = bf16(sum_k hidden[n, k] * head[m, k]) for
// one 128-id tile of the vocabulary per CTA -- the F.linear(hidden, head) of the Talker's decode step
// (engine/runtime/talker_decode.py:120, engine/runtime/talker_post_graph.py:58) whose bf16 output the sampler reads.
//
// One tile is one tcgen05 MMA chain: M = 128 vocabulary ids (A = the head tile, K-major, straight from the
// [vocab, hidden] weight), N = 16 batch rows (B = the hidden rows, K-major, rows >= B zero), K = hidden_dim in
// steps of 16, split over a cluster of two CTAs where the SMs allow it.  A CTA's whole share of K (at most 12
// blocks of 64) sits in shared memory at once: every block of the head tile is one TMA load of [128 ids x 64] in
// the 128-byte swizzled layout, all requested before the wait for the previous kernel (the head is a constant
// weight).  The hidden rows -- the previous kernel's output -- are read after that wait by all threads and
// stored in the same swizzled layout.  One thread issues the MMAs as the blocks land; the fp32 accumulator (128
// lanes x 16 columns of tensor memory) is read back by warps 0..3 (the partner's added through distributed shared
// memory), rounded to bf16 (round to nearest even, as the bf16 output of F.linear) and stored to the logits rows,
// which stay in L2 for the rows' CTAs of the same launch.
#pragma once

#include <cuda.h>  // CUtensorMap

#include "../../include/b2s_sampler.h"
#include "b2s_device.cuh"

namespace b2s {

constexpr int HEAD_M = 128;      // vocabulary ids per tile (the MMA's M)
constexpr int HEAD_N = 16;       // batch rows per tile (the MMA's N; B <= 16)
constexpr int HEAD_KB = 64;      // K elements per block: one 128-byte row of the swizzle atom
constexpr int HEAD_MAX_KB = 12;  // hidden_dim <= 768
constexpr uint32_t HEAD_A_BYTES = HEAD_M * HEAD_KB * 2;  // 16 KB per block of the head tile
constexpr uint32_t HEAD_B_BYTES = HEAD_N * HEAD_KB * 2;  // 2 KB per block of the hidden rows
constexpr uint32_t HEAD_TMEM_COLS = 32;                  // smallest allocation; the accumulator uses 16 columns
// shared memory of a tile CTA: 1 KB of alignment slack (the swizzle atoms want 1024-byte alignment), the
// head and hidden blocks, the mbarriers (one per block, the accumulator's, the partner's), the TMEM address and
// failure flags; rank 0 of a split tile receives the partner's accumulator in head blocks it does not use
constexpr uint32_t HEAD_SMEM = 1024 + HEAD_MAX_KB * (HEAD_A_BYTES + HEAD_B_BYTES) + 256;
constexpr uint64_t HEAD_WAIT_NS = 250ull * 1000 * 1000;  // bound of every wait of the head path

// Instruction descriptor of tcgen05.mma kind::f16: fp32 accumulator (bits 4-5 = 1), A and B bf16 (bits 7-9,
// 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t HEAD_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(HEAD_N >> 3) << 17) |
                                ((uint32_t)(HEAD_M >> 4) << 24);

// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzled layout: start address >> 4
// (bits 0-13), leading-dimension offset 1 (unused by swizzled K-major layouts, bits 16-29), stride between
// 8-row groups 1024 B >> 4 (bits 32-45), descriptor version 1 (bits 46-47), swizzle mode 2 = 128 B (bits 61-63).
// The k-th 16-element slice of a 64-element block starts 32 * k bytes further (the swizzle is applied to the
// address bits, so the advance is a plain offset inside the 1024-byte-aligned atom).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// 2-D tiled TMA load global -> this CTA's shared memory (no multicast): the box at (x = K element, y = id).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Makes this thread's generic-proxy shared-memory writes visible to the asynchronous proxy (the tensor cores).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Tensor memory: allocation (one warp, the address written to shared memory), release, fences and loads.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, both bf16 K-major, fp32 accumulator; `acc` = 0 overwrites D.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// Arrives on `bar` once every MMA this thread issued before it has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// This warp's 32 lanes (lane quarter warp % 4) x 16 columns of fp32 from tensor memory, waited for in the same
// statement so no use of the registers can be scheduled before the data is there.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Waits until *p >= target, for at most limit_ns (false on timeout): relaxed polls, then one acquire fence, so
// that this thread's later reads see what the releasing threads wrote before their increments.
__device__ __forceinline__ bool wait_geq_acquire(const uint32_t* p, uint32_t target, uint64_t limit_ns) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (ld_relaxed_u32(p) >= target) {
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                return true;
            }
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// Distributed shared memory of a CTA pair (split K): the partner's address of a shared word, a 16-byte store
// there, a remote arrival (release at cluster scope) on the partner's mbarrier, and a wait with cluster-scope
// acquire on this CTA's own.
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// The control words of one head launch (4 x u32, zero between launches): [0] tiles whose logits are stored,
// [1] a tile failed, [2] rows that have seen the logits (the last one zeroes the words for the next launch).
enum { HS_TILES = 0, HS_ERR = 1, HS_ROWS = 2 };

// One vocabulary tile, or one half of its K when split == 2 (a cluster of two CTAs per tile, rank = the CTA's
// rank in it): the MMA chain over this CTA's K blocks, then -- split: rank 1 hands its fp32 accumulator to rank 0
// through distributed shared memory and rank 0 adds it to its own -- the bf16 logits of every batch row at the
// tile's ids, stored by rank 0, which then counts the tile in.  `logits` rows are `lstride` elements apart.
// Every thread of the CTA calls it.
//
// Why split: the tensor cores stream the head tile out of shared memory at a fixed rate per SM, and the tile's
// loads land at a rate per SM too, so the head's bytes per CTA set the tile's time; two CTAs per tile halve them
// and use 104 SMs instead of 52 for the Talker's 6,562 ids.
__device__ __forceinline__ void head_tile(int tile, int split, int rank, int rows, int V, int nkb_all,
                                          const void* hidden, int64_t hid_stride, uint16_t* logits, int64_t lstride,
                                          uint32_t* sync, uint32_t* status, const CUtensorMap* amap,
                                          unsigned char* smem_raw) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = tile * HEAD_M;
    const int nkb = nkb_all / split, kb0 = rank * nkb;  // this CTA's K blocks
    const uint32_t base_u = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((base_u + 1023u) & ~1023u) - base_u);
    unsigned char* A = sm;                                // nkb blocks of [128 ids x 64] (16 KB each)
    unsigned char* Bm = sm + HEAD_MAX_KB * HEAD_A_BYTES;  // nkb blocks of [16 rows x 64] (2 KB each)
    // [0, nkb): blocks; HEAD_MAX_KB: MMAs; HEAD_MAX_KB + 1: the partner's accumulator (split, rank 0)
    uint64_t* bars = reinterpret_cast<uint64_t*>(Bm + HEAD_MAX_KB * HEAD_B_BYTES);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + HEAD_MAX_KB + 2);
    volatile int* fail = reinterpret_cast<volatile int*>(tslot + 1);
    volatile int* pfail = reinterpret_cast<volatile int*>(tslot + 2);  // [4]: the partner's warps failed (split)
    // rank 0's receive buffer for the partner's [128 ids x 16 rows] fp32 accumulator: head blocks this CTA does
    // not use (split: nkb <= HEAD_MAX_KB / 2)
    float* part = reinterpret_cast<float*>(A + (HEAD_MAX_KB / 2) * HEAD_A_BYTES);
    uint64_t* mma_bar = &bars[HEAD_MAX_KB];
    uint64_t* part_bar = &bars[HEAD_MAX_KB + 1];

    // (before the wait for the previous kernel: no global memory is written and only the constant head is read)
    if (tid == 0) {
        prefetch_tensormap(amap);
        for (int i = 0; i < nkb; ++i) mbar_init(&bars[i], 1);
        mbar_init(mma_bar, 1);
        mbar_init(part_bar, 128);  // the partner's 128 epilogue threads
        fence_mbar_init();
        *fail = 0;
    }
    if (warp == 1) tmem_alloc(tslot, HEAD_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    if (split > 1) cluster_arrive_relaxed();  // the partner may arrive on part_bar once both have passed the wait
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (tid == 0)
        for (int kb = 0; kb < nkb; ++kb) {
            mbar_arrive_expect_tx(&bars[kb], HEAD_A_BYTES);
            tma_load_2d(A + kb * HEAD_A_BYTES, amap, (kb0 + kb) * HEAD_KB, m0, &bars[kb]);  // ids >= vocab: zero
        }
    pdl_wait_then_release();

    // the hidden rows into the B blocks: 16-byte chunk j of row n of block kb at row n's 128-byte line, position
    // j ^ (n % 8) (the 128-byte swizzle); rows >= `rows` are zero
    const int nchunks = nkb * HEAD_N * 8;
    for (int c = tid; c < nchunks; c += NT) {
        const int kb = c / (HEAD_N * 8), n = (c >> 3) % HEAD_N, j = c & 7;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (n < rows)
            v = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(hidden) + (int64_t)n * hid_stride +
                                                (kb0 + kb) * HEAD_KB + j * 8);
        *reinterpret_cast<uint4*>(Bm + kb * HEAD_B_BYTES + (n >> 3) * 1024 + (n & 7) * 128 + ((j ^ (n & 7)) << 4)) = v;
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (split > 1) cluster_wait();

    if (tid == 0) {
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait_bounded(&bars[kb], 0u, HEAD_WAIT_NS)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(A + kb * HEAD_A_BYTES), b0 = smem_u32(Bm + kb * HEAD_B_BYTES);
#pragma unroll
            for (int k = 0; k < HEAD_KB / 16; ++k)
                umma_bf16(tmem, umma_desc_sw128(a0 + 32u * k), umma_desc_sw128(b0 + 32u * k), HEAD_IDESC,
                          (kb | k) != 0 ? 1u : 0u);
        }
        umma_commit(mma_bar);  // arrives once the MMAs above have completed
        if (!ok) {
            *fail = 1;
            // the block loads still in flight land in this CTA's shared memory: wait for them (bounded) before
            // the CTA can exit
            for (int kb = 0; kb < nkb; ++kb) mbar_wait_bounded(&bars[kb], 0u, HEAD_WAIT_NS);
        }
    }
    if (warp < 4) {
        const bool done = mbar_wait_bounded(mma_bar, 0u, HEAD_WAIT_NS);
        tc_fence_after();
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16), v);  // lane = id m0 + 32 * warp + lane, column = batch row
        tc_fence_before();
        named_bar_sync(1, 128);  // thread 0's failure flag is visible; the accumulator is read
        bool good = done && *fail == 0;
        const int ml = warp * 32 + lane;  // this thread's id in the tile
        if (split > 1 && rank == 1) {
            // hand the partial sums to rank 0: 64 bytes per id, then one arrival per thread (release, cluster)
            const uint32_t dst = mapa_shared(smem_u32(part + ml * HEAD_N), 0);
#pragma unroll
            for (int q = 0; q < HEAD_N / 4; ++q) st_cluster_v4(dst + 16u * q, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            if (lane == 0)
                asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(mapa_shared(smem_u32(const_cast<int*>(pfail + warp)), 0)),
                             "r"(good ? 0u : 1u)
                             : "memory");
            mbar_arrive_remote(mapa_shared(smem_u32(part_bar), 0));
            if (!good && lane == 0) atomicOr(&sync[HS_ERR], 1u);
            if (!good && tid == 0 && status) atomicOr(status, B2S_STATUS_WAIT_TIMEOUT);
        } else {
            if (split > 1) {
                // the partner's half of K: K blocks kb0 + nkb .. of the same ids (a NaN word marks a failed partner)
                good = mbar_wait_cluster_bounded(part_bar, 0u, HEAD_WAIT_NS) && good;
                const float4* pp = reinterpret_cast<const float4*>(part + ml * HEAD_N);
#pragma unroll
                for (int q = 0; q < HEAD_N / 4; ++q) {
                    const float4 o = pp[q];
                    v[4 * q] = __float_as_uint(__uint_as_float(v[4 * q]) + o.x);
                    v[4 * q + 1] = __float_as_uint(__uint_as_float(v[4 * q + 1]) + o.y);
                    v[4 * q + 2] = __float_as_uint(__uint_as_float(v[4 * q + 2]) + o.z);
                    v[4 * q + 3] = __float_as_uint(__uint_as_float(v[4 * q + 3]) + o.w);
                }
                if (pfail[0] | pfail[1] | pfail[2] | pfail[3]) good = false;
            }
            const int m = m0 + ml;
            if (good && m < V) {
#pragma unroll
                for (int n = 0; n < HEAD_N; ++n)
                    if (n < rows)
                        logits[(int64_t)n * lstride + m] =
                            __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[n])));
            }
            if (!good && lane == 0) atomicOr(&sync[HS_ERR], 1u);
            named_bar_sync(1, 128);  // every store of the tile precedes thread 0's release below (cumulative)
            if (tid == 0) {
                if (!good && status) atomicOr(status, B2S_STATUS_WAIT_TIMEOUT);
                red_release_add(&sync[HS_TILES], 1u);
            }
        }
        if (warp == 1) {
            tc_fence_after();
            tmem_dealloc(tmem, HEAD_TMEM_COLS);
        }
    }
}

// The Thinker LM head's greedy step (b2s_lmhead.cu): tiles + finishing block on `stream`.
constexpr int LMHEAD_MAX_ROWS = 64;
// With keys_out: the shard's ordered keys (global ids from `offset`) instead of tokens.
cudaError_t lmhead_argmax_launch(const CUtensorMap& amap, const CUtensorMap& bmap, int vocab, int rows, int nkb,
                                 int64_t* tokens, unsigned long long* keys, uint32_t* status, void* stream,
                                 int64_t offset = 0, int64_t* keys_out = nullptr);

}  // namespace b2s
