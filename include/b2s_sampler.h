/*
 * b2s_sampler.h -- C-ABI of the B200 token-sampling engine for MiniCPM-o 4.5 (sm_100a).
 *
 * Every entry point takes plain device pointers and sizes plus a CUDA stream handle
 * (cudaStream_t passed as void*), enqueues its kernels on that stream, never synchronises,
 * never allocates, and returns B2S_OK or a B2S_ERR_* code for invalid arguments or launch
 * failures.  Conditions that can only be seen on the device are OR-ed into an optional device
 * status word (B2S_STATUS_*); there are no device traps.  A history id >= vocab is ignored (the
 * row is sampled as if that position were PAD; the reference's scatter_add would raise), a
 * repetition count beyond the penalty table is clamped to its last entry; a per-row top_k above
 * the declared bound, an incomplete vocabulary shard or a bounded wait that gave up make the
 * affected row yield token PAD (-1) with its state unchanged.
 *
 * The interface replaces the reference module engine/talker_sampler.py (pure torch in the
 * reference; the reference has no native library) and the greedy argmax of the Thinker call
 * sites.  Each function below cites the reference interface it replaces.
 */
#ifndef B2S_SAMPLER_H
#define B2S_SAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2S_ABI_VERSION 5

/* return codes */
#define B2S_OK 0
#define B2S_ERR_INVALID 1     /* bad argument (null pointer, size, dtype, parameter range) */
#define B2S_ERR_UNSUPPORTED 2 /* shape outside what the kernels are built for (e.g. row too large) */
#define B2S_ERR_CUDA 3        /* a CUDA runtime call failed (see b2s_last_cuda_error) */

/* logits element types */
#define B2S_DTYPE_F32 0
#define B2S_DTYPE_BF16 1

/* processing order (engine/talker_sampler.py:142-156) */
#define B2S_SEM_HF 0       /* x/T -> penalty -> top-p(min_keep) -> top-k; frame 0 unfiltered */
#define B2S_SEM_OMNI 1     /* EOS censor -> penalty -> /T -> top-k -> top-p (min_keep 1) */
#define B2S_SEM_IDENTITY 2 /* rows are already processed: draw() only */

/* where the per-row uniform comes from */
#define B2S_RNG_UNIFORM 0 /* caller-provided uniform_values (draw(uniform_values=...)) */
#define B2S_RNG_COUNTER 1 /* the reference counter hash of (seed, step), talker_sampler.py:60-76 */
#define B2S_RNG_PHILOX 2  /* Philox4x32-10: key = seed, counter = (step, request) */

/* bits of the device status word */
#define B2S_STATUS_HISTORY_RANGE 1u /* a history id >= vocab was ignored (the row is still sampled) */
#define B2S_STATUS_TOPK_LIMIT 2u    /* a row's top_k exceeded max_top_k; the row returned PAD */
#define B2S_STATUS_WAIT_TIMEOUT 4u  /* a bounded device wait gave up; the row returned PAD */
#define B2S_STATUS_COUNT_LIMIT 8u   /* a token repeated more than alpha_len-1 times; its count was clamped */
#define B2S_STATUS_SHARD_INCOMPLETE 16u /* a shard's candidate list overflowed `cap` or failed; the row returned PAD */

/* flags */
#define B2S_FLAG_FORCE_GENERAL 1 /* take the exact radix-select path even when the candidate path applies */
#define B2S_FLAG_TOPK_ONLY 2     /* no top-p cut: keep every value >= the k-th largest (top_k_filter) */
#define B2S_FLAG_STREAM 4        /* use the streaming kernel even where the row-resident one applies */

typedef struct b2s_sample_args {
    /* logits [rows, vocab], row-major with logits_row_stride elements between rows */
    const void* logits;
    int32_t logits_dtype;
    int32_t rows;
    int32_t vocab;
    /* CTAs per row of the row-resident kernel (1, 2, 4 or 8), or 0 for the launcher's choice.  The
     * row-resident kernel serves decode steps (tokens and/or state out, no processed or shard output, hf or
     * omni order, k = max(top_k, min_keep) <= 128); hf takes one CTA per row.  A nonzero value for a launch
     * it cannot serve, or whose row slice does not fit a CTA's shared memory, is B2S_ERR_UNSUPPORTED. */
    int32_t cluster;
    int64_t logits_row_stride;
    /* penalty history [rows, window] int64 (most recent last); ids < 0 are empty (PAD) */
    const int64_t* history;
    int64_t history_row_stride;
    int32_t window;
    int32_t eos; /* EOS column; outside [0, vocab) = no EOS column */
    const int64_t* steps;        /* [rows] frame index of the token being sampled */
    const int64_t* seeds;        /* [rows] request seeds (B2S_RNG_COUNTER / B2S_RNG_PHILOX) */
    const int64_t* requests;     /* [rows] Philox counter words 2-3, or NULL (= 0) */
    const float* uniform_values; /* [rows] (B2S_RNG_UNIFORM) */
    const uint8_t* active;       /* [rows] bool or NULL (= all active) */
    const uint8_t* finished;     /* [rows] bool or NULL (= none finished) */
    /* parameters; the per-row arrays override the scalars when non-NULL */
    float temperature;
    float top_p;
    float presence_penalty;  /* omni order only: subtracted once from seen tokens */
    float frequency_penalty; /* omni order only: subtracted count times from seen tokens */
    int32_t top_k;
    int32_t min_keep; /* k = max(top_k, min_keep) and the top-p cut keeps >= min_keep (omni callers pass 1) */
    int64_t min_new_tokens;
    int64_t max_new_tokens;
    const float* row_temperature;
    const float* row_top_p;
    const int32_t* row_top_k;
    /* alpha[n] = penalty**n for n in [0, alpha_len); alpha_row_stride 0 = one table for all rows */
    const float* alpha;
    int32_t alpha_len;
    int32_t alpha_row_stride;
    int32_t max_top_k; /* bound on every row's top_k (sizes on-chip buffers); 0 = use top_k */
    int32_t semantics;
    int32_t rng;
    int32_t flags;
    /* outputs, each optional */
    int64_t* tokens;                 /* [rows]; PAD (-1) for inactive / finished rows */
    float* processed;                /* [rows, vocab] processed logits */
    int64_t processed_row_stride;
    int64_t* history_out;            /* [rows, window] state after the step (may alias history) */
    int64_t history_out_row_stride;
    int64_t* steps_out;              /* [rows] (may alias steps) */
    uint8_t* finished_out;           /* [rows] (may alias finished) */
    uint32_t* status;                /* device status word (bits OR-ed), or NULL */
    /* per-row min_new_tokens / max_new_tokens ([rows] int64) overriding the scalars, or NULL (ABI 2) */
    const int64_t* row_min_new_tokens;
    const int64_t* row_max_new_tokens;
} b2s_sample_args;

/*
 * Fused sampling step: per row, processed_logits (temperature, count-based repetition penalty,
 * optional presence/frequency penalties, EOS min/max rules, top-k/top-p value threshold) and the
 * inverse-CDF draw in vocabulary order, optionally writing the processed row and advancing the
 * step() state.
 * Replaces: engine/talker_sampler.py:136-158 processed_logits, :161-172 draw, :234-249 step
 * (and :252-254 decode_k as K calls), and the graph bodies engine/runtime/talker_decode.py:120-128,
 * engine/runtime/talker_post_graph.py:56-76.  With semantics B2S_SEM_IDENTITY it is draw() alone.
 */
int b2s_sample(const b2s_sample_args* args, void* stream);

/*
 * K frames of the step() state machine in one launch (the K-frame device block of the Talker decode loop):
 * frame f samples from the rows of logits + f * frame_stride elements, writes tokens[f * rows + row] (PAD for
 * rows that are not live), and advances the state in place -- history_out == history, steps_out == steps and
 * finished_out == finished (non-NULL) are required -- so that frame f + 1 sees it; a row that draws EOS is
 * frozen for the frames after it.  uniform_values (B2S_RNG_UNIFORM) are [frames, rows].  The tokens and the
 * final state equal `frames` calls of b2s_sample.  No processed output; cluster must be 0 (one CTA per row
 * takes the row's frames in order, prefetching the next frame's logits under the current frame's draw).
 * Replaces: engine/talker_sampler.py:252-254 decode_k and the K-frame graph bodies of
 * engine/runtime/talker_decode.py:120-128, engine/runtime/talker_block_graph.py:70-89.
 */
int b2s_sample_frames(const b2s_sample_args* args, int32_t frames, int64_t frame_stride, void* stream);

/*
 * The Talker codec head and the sampling step in one launch (ABI 5):
 *     logits = bf16(hidden[rows, hidden_dim] x head[vocab, hidden_dim]^T)   (fp32 accumulation, tensor cores)
 * then b2s_sample's step on those logits.  The logits equal the bf16 output of F.linear up to the order of the
 * fp32 accumulation; they are written to `logits` (args->logits_row_stride elements apart, args->logits NULL or
 * equal) so that the caller can check them, and the rows' CTAs of the same launch read them there.
 * Replaces: the head and the sampler of engine/runtime/talker_post_graph.py:58-63 (F.linear(hidden, head).float(),
 * processed_logits, draw) and engine/runtime/talker_decode.py:120-121.
 * Limits: rows <= 16, hidden_dim a multiple of 64 and at most 768, rows + ceil(vocab / 128) <= the GPU's SM count,
 * bf16 only; args must be a decode step the short-row kernel takes (tokens and/or state out, no processed
 * output, cluster 0, k <= 128, window <= 255, vocab <= 8192 * 16 / element size) -- else B2S_ERR_UNSUPPORTED.
 * `head` is read before the launch waits for the stream's previous kernel: that kernel must not write it.
 * `sync`: 4 words of device memory, zero before the first call, left zero by every call that completes; calls
 * sharing one `sync` block must not overlap on the GPU (one block per stream).
 */
typedef struct b2s_head_args {
    const void* hidden;        /* [rows, hidden_dim] bf16, 16-byte aligned */
    int64_t hidden_row_stride; /* elements, a multiple of 8 */
    const void* head;          /* [vocab, hidden_dim] bf16, contiguous rows, 16-byte aligned */
    int32_t hidden_dim;
    void* logits;              /* [rows, vocab] bf16 out */
    uint32_t* sync;            /* 4 words, 16-byte aligned */
} b2s_head_args;
int b2s_head_sample(const b2s_head_args* head, const b2s_sample_args* args, void* stream);

/*
 * The Thinker's greedy step from its LM head (ABI 5): tokens[n] = argmax_m bf16(hidden[n, :] . head[m, :]) (fp32
 * accumulation on the tensor cores, each logit rounded to bf16 like F.linear's bf16 output, first index among equal
 * maxima, NaN above every number) without writing the logits.  `keys`: `rows` 64-bit device words, zero before the
 * first call and left zero by every call (one block per stream); `status` (optional) gets
 * B2S_STATUS_WAIT_TIMEOUT if a bounded wait gave up (the row then returns PAD or a partial maximum).
 * Replaces: F.linear(h, lm_head).float().argmax(-1) at engine/runtime/thinker_decode.py:83,107,
 * engine/runtime/backend_s.py:893, engine/runtime/backend.py:238, engine/runtime/track_s.py:60.
 * Limits: rows <= 64 (else B2S_ERR_UNSUPPORTED), hidden_dim a multiple of 64, hidden rows and head 16-byte aligned
 * with row strides a multiple of 8 elements (the head's rows contiguous).
 */
int b2s_lmhead_argmax(const void* hidden, int64_t hidden_row_stride, const void* head, int32_t hidden_dim,
                      int32_t vocab, int32_t rows, int64_t* tokens, uint64_t* keys, uint32_t* status, void* stream);

/*
 * The same over one vocabulary shard (ABI 5; no counterpart in the reference, which has no multi-device code):
 * head_shard holds ids vocab_offset .. vocab_offset + shard_vocab - 1.  Writes, per row, a 64-bit word whose signed
 * maximum over the shards -- one max-all-reduce of `rows` int64 (NCCL) -- is the key of the global argmax: the
 * order key of its bf16 value in the high word, the complement of its global id in the low word, the top bit
 * flipped; INT64_MIN for a row that no tile reached.  The token is 0xffffffff - (word & 0xffffffff) after the top
 * bit is flipped back.  `keys` as for b2s_lmhead_argmax.
 */
int b2s_lmhead_argmax_keys(const void* hidden, int64_t hidden_row_stride, const void* head_shard, int32_t hidden_dim,
                           int32_t shard_vocab, int64_t vocab_offset, int32_t rows, int64_t* keys_out, uint64_t* keys,
                           uint32_t* status, void* stream);

/*
 * b2s_head_sample for callers that cannot allocate device memory: no counterpart in the reference, whose
 * callers allocate through torch.  Some hosts of this library cannot call cudaMalloc on this path -- an embedding
 * whose device allocator is fixed at start-up, a runtime that hands the library only the buffers it owns, or a
 * decode loop that must not call cudaMalloc / cudaFree (which can synchronise the device) while other work is in
 * flight.  The caller passes the inputs and outputs as for b2s_head_sample (args->logits must be NULL; the dtype
 * and row stride of the logits are set here); the logits rows and the control words live in one fixed device
 * array of B2S_NOALLOC_SCRATCH_BYTES inside the library, held on every GPU that uses it until the process exits.
 * Allocates nothing and calls no allocating routine.  Limits: rows <= B2S_NOALLOC_MAX_ROWS and vocab <=
 * B2S_NOALLOC_MAX_VOCAB, else B2S_ERR_UNSUPPORTED before anything is launched; the other limits of
 * b2s_head_sample apply.  Each call clears the control words on `stream` (cudaMemsetAsync) before its launch.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress): make that first call
 * before any stream capture.  Every call on a device shares the one array, which keeps the last call's contents:
 * calls that overlap on the GPU (other streams, other threads) race and must be serialised by the caller.
 */
#define B2S_NOALLOC_MAX_ROWS 16
#define B2S_NOALLOC_MAX_VOCAB 8192
#define B2S_NOALLOC_SCRATCH_BYTES (B2S_NOALLOC_MAX_ROWS * B2S_NOALLOC_MAX_VOCAB * 2 + 256)
int b2s_head_sample_noalloc(const void* hidden, int64_t hidden_row_stride, const void* head, int32_t hidden_dim,
                            const b2s_sample_args* args, void* stream);

/*
 * Greedy next token: argmax over each row (first index among equal maxima, NaN wins).
 * Replaces the Thinker sampling step F.linear(h, lm_head).float().argmax(-1) at
 * engine/runtime/thinker_decode.py:83,107, engine/runtime/backend_s.py:893,
 * engine/runtime/backend.py:238, engine/runtime/backend_npu.py:890, engine/runtime/track_s.py:60.
 */
int b2s_argmax(const void* logits, int32_t logits_dtype, int32_t rows, int32_t vocab, int64_t row_stride,
               int64_t* tokens, void* stream);

/*
 * Per-row U[0,1) from (seed, step[, request]): rng B2S_RNG_COUNTER is the reference counter hash
 * (engine/talker_sampler.py:60-76 _mix32/uniform), B2S_RNG_PHILOX is Philox4x32-10.
 */
int b2s_uniform(const int64_t* seeds, const int64_t* steps, const int64_t* requests, int64_t n, int32_t rng,
                float* out, void* stream);

/*
 * The sampler's fp32 exp (its numerics spec: every exponential the kernels take) evaluated on the device, for
 * verification against a CPU restatement (no counterpart in the reference, whose exponentials are torch's):
 * y[i] = exp(x[i]) in the scalar form; y_pair[i] the same through the paired form the kernels use for x[i] <= 0
 * (the scalar form elsewhere).  The two must agree bit for bit.
 */
int b2s_expf_spec(const float* x, int64_t n, float* y, float* y_pair, void* stream);

/*
 * Vocabulary-sharded head, stage 1 (no counterpart in the reference, which has no multi-device code).
 * `args` describes this rank's shard: logits [rows, shard_vocab] are the columns
 * [vocab_offset, vocab_offset + shard_vocab) of the full head; history ids and eos are global ids.
 * Omni order only.  Per row it writes, as (value fp32, global id int32) pairs into cand_values /
 * cand_ids [rows][cap], every processed element above the shard's k-th largest value
 * (k = max(top_k, min_keep); there are fewer than k, and cap >= k is required), then elements equal to
 * it while room is left; cand_count[rows] is the number of elements >= the k-th value (above cap: the
 * unsent ones are ties at the k-th value, the smallest value sent; -1: the row failed on the device).
 */
int b2s_shard_candidates(const b2s_sample_args* args, int64_t vocab_offset, int32_t cap, float* cand_values,
                         int32_t* cand_ids, int32_t* cand_count, void* stream);

/* A row whose draw falls among ties that its shard did not send (stage 2 -> stage 3). */
typedef struct b2s_shard_pending {
    double base;   /* cumulative mass of the kept elements before the shard, in vocabulary order */
    float thr;     /* the row's value threshold: kept elements are >= thr */
    float vmax;    /* the largest kept value */
    float sf;      /* softmax normaliser of the kept set */
    float target;  /* u * total mass: the token is the first element whose cumulative mass exceeds it */
    int32_t shard; /* the shard holding the token, or -1 when stage 2 resolved the row */
    int32_t pad_;
} b2s_shard_pending;

/*
 * Vocabulary-sharded head, stage 2: from the all-gathered stage-1 outputs of `shards` shards
 * (layout [shards][rows][cap], counts [shards][rows]) each row's top-k values (the sent values and the
 * unsent ties), top-p cut and value threshold over the full vocabulary `vocab`, and the shard whose
 * range holds the draw.  args->tokens[row] receives the token when every kept element of that shard
 * was sent, else -2 with the row's pending[row] record naming the shard (pending may be NULL: such rows
 * then get PAD and B2S_STATUS_SHARD_INCOMPLETE).  Uses args->top_k / top_p / min_keep / row_* / rng /
 * seeds / steps / requests / uniform_values / tokens / status / flags; k must be <= 128.
 */
int b2s_shard_merge(const float* cand_values, const int32_t* cand_ids, const int32_t* cand_count, int32_t shards,
                    int32_t rows, int32_t cap, int32_t vocab, const b2s_sample_args* args,
                    b2s_shard_pending* pending, void* stream);

/*
 * Vocabulary-sharded head, stage 3, on the rank of shard `shard` (args and vocab_offset as in stage 1):
 * tokens_out[row] = merged[row] for rows stage 2 resolved, the global id of the row's token for rows
 * pending on this shard (a scan of the shard row's processed elements in vocabulary order from the
 * record's mass), -1 for rows pending on other shards.  A max-all-reduce of tokens_out over the shards'
 * ranks gives every rank the tokens of b2s_sample on the unsharded row.
 */
int b2s_shard_resolve(const b2s_sample_args* args, int64_t vocab_offset, int32_t shard,
                      const b2s_shard_pending* pending, const int64_t* merged, int64_t* tokens_out, void* stream);

/*
 * Count-based repetition penalty on its own: out = x * penalty**n where x < 0, x / penalty**n otherwise,
 * n = occurrences of the column in the row's history (ids < 0 ignored), alpha[n] = penalty**n.
 * Replaces engine/talker_sampler.py:79-84 repetition_penalty (out is fp32 [rows, vocab]).
 */
int b2s_repetition_penalty(const void* x, int32_t x_dtype, int32_t rows, int32_t vocab, int64_t x_row_stride,
                           const int64_t* history, int32_t window, int64_t history_row_stride, const float* alpha,
                           int32_t alpha_len, int32_t alpha_row_stride, float* out, int64_t out_row_stride,
                           uint32_t* status, void* stream);

/* Human-readable text of a B2S_ERR_* code, and of the last CUDA error seen by this library. */
const char* b2s_error_string(int code);
const char* b2s_last_cuda_error(void);
int b2s_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B2S_SAMPLER_H */
