// torch custom-op layer: TORCH_LIBRARY(minicpmo_sampler) ops whose CUDA kernels call the C-ABI of
// libb2s.so (include/b2s_sampler.h) on torch's current stream, plus Meta kernels so shapes are known
// without running anything.  Outputs come from the caching allocator (graph-capture pools included);
// nothing here synchronises with the host.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <tuple>

#include "../../include/b2s_sampler.h"

using at::Tensor;
using c10::optional;

namespace {

void check_rc(int rc, const char* what) {
    TORCH_CHECK(rc == B2S_OK, what, " failed: ", b2s_error_string(rc),
                rc == B2S_ERR_CUDA ? std::string(" (") + b2s_last_cuda_error() + ")" : std::string());
}

template <typename T>
const T* opt_ptr(const optional<Tensor>& t, at::ScalarType st, int64_t numel, const Tensor& like, const char* name) {
    if (!t.has_value() || !t->defined()) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->device() == like.device(), name, " must be on ", like.device());
    TORCH_CHECK(t->scalar_type() == st, name, " must be ", c10::toString(st), ", got ", t->scalar_type());
    TORCH_CHECK(t->is_contiguous(), name, " must be contiguous");
    TORCH_CHECK(numel < 0 || t->numel() == numel, name, " must have ", numel, " elements, got ", t->numel());
    return static_cast<const T*>(t->data_ptr());
}

struct Prepared {
    b2s_sample_args a;
    Tensor tokens, processed, hist_out, steps_out, fin_out;
};

// Shared argument marshalling of the functional and in-place ops.
void fill_args(b2s_sample_args& a, const Tensor& logits, const optional<Tensor>& history, const optional<Tensor>& steps,
               const optional<Tensor>& seeds, const optional<Tensor>& requests, const optional<Tensor>& uniform_values,
               const optional<Tensor>& active, const optional<Tensor>& finished,
               const optional<Tensor>& row_temperature, const optional<Tensor>& row_top_p,
               const optional<Tensor>& row_top_k, const optional<Tensor>& alpha, const optional<Tensor>& status,
               double temperature, double top_p, int64_t top_k, int64_t min_keep, int64_t min_new, int64_t max_new,
               double presence, double frequency, int64_t eos, int64_t semantics, int64_t rng, int64_t max_top_k,
               int64_t flags, int64_t cluster, const optional<Tensor>& row_min_new = c10::nullopt,
               const optional<Tensor>& row_max_new = c10::nullopt) {
    TORCH_CHECK(logits.is_cuda(), "logits must be a CUDA tensor (this engine has no CPU path)");
    TORCH_CHECK(logits.dim() == 2, "logits must be [rows, vocab]");
    TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16,
                "logits must be float32 or bfloat16");
    TORCH_CHECK(logits.stride(1) == 1, "logits rows must be contiguous");
    const int64_t B = logits.size(0), V = logits.size(1);
    memset(&a, 0, sizeof(a));
    a.logits = logits.data_ptr();
    a.logits_dtype = logits.scalar_type() == at::kBFloat16 ? B2S_DTYPE_BF16 : B2S_DTYPE_F32;
    a.rows = (int32_t)B;
    a.vocab = (int32_t)V;
    a.cluster = (int32_t)cluster;
    a.logits_row_stride = B > 1 ? logits.stride(0) : V;
    if (history.has_value() && history->defined() && history->numel() > 0) {
        const Tensor& h = *history;
        TORCH_CHECK(h.is_cuda() && h.device() == logits.device(), "history must be on ", logits.device());
        TORCH_CHECK(h.scalar_type() == at::kLong && h.dim() == 2 && h.size(0) == B && h.stride(1) == 1,
                    "history must be int64 [rows, window] with contiguous rows");
        a.history = h.data_ptr<int64_t>();
        a.window = (int32_t)h.size(1);
        a.history_row_stride = B > 1 ? h.stride(0) : h.size(1);
    }
    a.steps = opt_ptr<int64_t>(steps, at::kLong, B, logits, "steps");
    a.seeds = opt_ptr<int64_t>(seeds, at::kLong, B, logits, "seeds");
    a.requests = opt_ptr<int64_t>(requests, at::kLong, B, logits, "requests");
    a.uniform_values = opt_ptr<float>(uniform_values, at::kFloat, B, logits, "uniform_values");
    a.active = opt_ptr<uint8_t>(active, at::kBool, B, logits, "active");
    a.finished = opt_ptr<uint8_t>(finished, at::kBool, B, logits, "finished");
    a.row_temperature = opt_ptr<float>(row_temperature, at::kFloat, B, logits, "row_temperature");
    a.row_top_p = opt_ptr<float>(row_top_p, at::kFloat, B, logits, "row_top_p");
    a.row_top_k = opt_ptr<int32_t>(row_top_k, at::kInt, B, logits, "row_top_k");
    a.row_min_new_tokens = opt_ptr<int64_t>(row_min_new, at::kLong, B, logits, "row_min_new");
    a.row_max_new_tokens = opt_ptr<int64_t>(row_max_new, at::kLong, B, logits, "row_max_new");
    if (alpha.has_value() && alpha->defined()) {
        const Tensor& al = *alpha;
        TORCH_CHECK(al.is_cuda() && al.device() == logits.device() && al.scalar_type() == at::kFloat && al.is_contiguous(),
                    "alpha must be a contiguous float32 CUDA tensor");
        TORCH_CHECK(al.dim() == 1 || (al.dim() == 2 && al.size(0) == B), "alpha must be [n] or [rows, n]");
        a.alpha = al.data_ptr<float>();
        a.alpha_len = (int32_t)al.size(-1);
        a.alpha_row_stride = al.dim() == 2 ? (int32_t)al.size(1) : 0;
    }
    if (status.has_value() && status->defined()) {
        TORCH_CHECK(status->is_cuda() && status->scalar_type() == at::kInt && status->numel() == 1,
                    "status must be a 1-element int32 CUDA tensor");
        a.status = reinterpret_cast<uint32_t*>(status->data_ptr<int32_t>());
    }
    a.temperature = (float)temperature;
    a.top_p = (float)top_p;
    a.top_k = (int32_t)top_k;
    a.min_keep = (int32_t)min_keep;
    a.min_new_tokens = min_new;
    a.max_new_tokens = max_new;
    a.presence_penalty = (float)presence;
    a.frequency_penalty = (float)frequency;
    a.eos = (int32_t)std::max<int64_t>(std::min<int64_t>(eos, INT32_MAX), -1);
    a.semantics = (int32_t)semantics;
    a.rng = (int32_t)rng;
    a.max_top_k = (int32_t)max_top_k;
    a.flags = (int32_t)flags;
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> sample_cuda(
    const Tensor& logits, const optional<Tensor>& history, const optional<Tensor>& steps, const optional<Tensor>& seeds,
    const optional<Tensor>& requests, const optional<Tensor>& uniform_values, const optional<Tensor>& active,
    const optional<Tensor>& finished, const optional<Tensor>& row_temperature, const optional<Tensor>& row_top_p,
    const optional<Tensor>& row_top_k, const optional<Tensor>& row_min_new, const optional<Tensor>& row_max_new,
    const optional<Tensor>& alpha, const optional<Tensor>& status,
    double temperature, double top_p, int64_t top_k, int64_t min_keep, int64_t min_new, int64_t max_new,
    double presence, double frequency, int64_t eos, int64_t semantics, int64_t rng, int64_t max_top_k, int64_t flags,
    bool want_tokens, bool want_processed, bool want_state, int64_t cluster) {
    c10::cuda::CUDAGuard guard(logits.device());
    b2s_sample_args a;
    fill_args(a, logits, history, steps, seeds, requests, uniform_values, active, finished, row_temperature, row_top_p,
              row_top_k, alpha, status, temperature, top_p, top_k, min_keep, min_new, max_new, presence, frequency, eos,
              semantics, rng, max_top_k, flags, cluster, row_min_new, row_max_new);
    const int64_t B = logits.size(0), V = logits.size(1);
    auto o64 = logits.options().dtype(at::kLong);
    Tensor tokens = want_tokens ? at::empty({B}, o64) : at::empty({0}, o64);
    Tensor processed = want_processed ? at::empty({B, V}, logits.options().dtype(at::kFloat))
                                      : at::empty({0}, logits.options().dtype(at::kFloat));
    Tensor hist_out, steps_out, fin_out;
    if (want_state) {
        TORCH_CHECK(history.has_value() && history->defined(), "want_state needs history");
        hist_out = at::empty_like(*history, at::MemoryFormat::Contiguous);
        steps_out = at::empty({B}, o64);
        fin_out = at::empty({B}, logits.options().dtype(at::kBool));
        a.history_out = hist_out.numel() ? hist_out.data_ptr<int64_t>() : nullptr;
        a.history_out_row_stride = hist_out.dim() == 2 ? hist_out.size(1) : 0;
        a.steps_out = steps_out.data_ptr<int64_t>();
        a.finished_out = reinterpret_cast<uint8_t*>(fin_out.data_ptr<bool>());
    } else {
        hist_out = at::empty({0}, o64);
        steps_out = at::empty({0}, o64);
        fin_out = at::empty({0}, logits.options().dtype(at::kBool));
    }
    if (want_tokens) a.tokens = tokens.data_ptr<int64_t>();
    if (want_processed) {
        a.processed = processed.data_ptr<float>();
        a.processed_row_stride = V;
    }
    check_rc(b2s_sample(&a, at::cuda::getCurrentCUDAStream().stream()), "b2s_sample");
    return {tokens, processed, hist_out, steps_out, fin_out};
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> sample_meta(
    const Tensor& logits, const optional<Tensor>& history, const optional<Tensor>&, const optional<Tensor>&,
    const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
    const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
    const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&, double, double, int64_t, int64_t,
    int64_t, int64_t, double, double, int64_t, int64_t, int64_t, int64_t, int64_t, bool want_tokens,
    bool want_processed, bool want_state, int64_t) {
    const int64_t B = logits.size(0), V = logits.size(1);
    auto o64 = logits.options().dtype(at::kLong);
    Tensor tokens = at::empty({want_tokens ? B : 0}, o64);
    Tensor processed = want_processed ? at::empty({B, V}, logits.options().dtype(at::kFloat))
                                      : at::empty({0}, logits.options().dtype(at::kFloat));
    Tensor h = want_state && history.has_value() ? at::empty_like(*history) : at::empty({0}, o64);
    Tensor s = at::empty({want_state ? B : 0}, o64);
    Tensor f = at::empty({want_state ? B : 0}, logits.options().dtype(at::kBool));
    return {tokens, processed, h, s, f};
}

// In-place step for captured graph bodies: history / steps / finished advance in place.
Tensor sample_state_cuda(const Tensor& logits, Tensor& history, Tensor& steps, Tensor& finished,
                         const optional<Tensor>& seeds, const optional<Tensor>& uniform_values,
                         const optional<Tensor>& active, const optional<Tensor>& alpha, const optional<Tensor>& status,
                         const optional<Tensor>& row_temperature, const optional<Tensor>& row_top_p,
                         const optional<Tensor>& row_top_k, double temperature, double top_p, int64_t top_k,
                         int64_t min_keep, int64_t min_new, int64_t max_new, int64_t eos, int64_t semantics, int64_t rng,
                         int64_t max_top_k, int64_t cluster, int64_t flags) {
    c10::cuda::CUDAGuard guard(logits.device());
    TORCH_CHECK(steps.is_contiguous() && finished.is_contiguous() && history.is_contiguous(),
                "state tensors must be contiguous");
    TORCH_CHECK(finished.scalar_type() == at::kBool, "finished must be bool");
    b2s_sample_args a;
    fill_args(a, logits, history, steps, seeds, c10::nullopt, uniform_values, active, finished, row_temperature,
              row_top_p, row_top_k, alpha, status, temperature, top_p, top_k, min_keep, min_new, max_new, 0.0,
              0.0, eos, semantics, rng, max_top_k, flags, cluster);
    Tensor tokens = at::empty({logits.size(0)}, logits.options().dtype(at::kLong));
    a.tokens = tokens.data_ptr<int64_t>();
    a.history_out = history.numel() ? history.data_ptr<int64_t>() : nullptr;
    a.history_out_row_stride = history.dim() == 2 ? history.size(1) : 0;
    a.steps_out = steps.data_ptr<int64_t>();
    a.finished_out = reinterpret_cast<uint8_t*>(finished.data_ptr<bool>());
    check_rc(b2s_sample(&a, at::cuda::getCurrentCUDAStream().stream()), "b2s_sample");
    return tokens;
}

// The Talker codec head and the step in one launch: logits = bf16(hidden @ head^T) written to `logits` (bf16
// [B, V], an output kept for inspection), then the step on them; history / steps / finished advance in place.
// `sync`: 4 int32 words, zero before the first call, one per stream.
Tensor head_sample_state_cuda(const Tensor& hidden, const Tensor& head, Tensor& logits, Tensor& sync, Tensor& history,
                              Tensor& steps, Tensor& finished, const optional<Tensor>& seeds,
                              const optional<Tensor>& uniform_values, const optional<Tensor>& active,
                              const optional<Tensor>& alpha, const optional<Tensor>& status,
                              const optional<Tensor>& row_temperature, const optional<Tensor>& row_top_p,
                              const optional<Tensor>& row_top_k, double temperature, double top_p, int64_t top_k,
                              int64_t min_keep, int64_t min_new, int64_t max_new, int64_t eos, int64_t semantics,
                              int64_t rng, int64_t max_top_k) {
    c10::cuda::CUDAGuard guard(logits.device());
    TORCH_CHECK(hidden.is_cuda() && head.is_cuda() && sync.is_cuda() && hidden.device() == logits.device() &&
                    head.device() == logits.device() && sync.device() == logits.device(),
                "hidden, head, logits and sync must be on one CUDA device");
    TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && head.scalar_type() == at::kBFloat16 &&
                    logits.scalar_type() == at::kBFloat16,
                "hidden, head and logits must be bfloat16");
    TORCH_CHECK(hidden.dim() == 2 && hidden.stride(1) == 1, "hidden must be [rows, hidden_dim] with contiguous rows");
    TORCH_CHECK(head.dim() == 2 && head.is_contiguous() && head.size(1) == hidden.size(1),
                "head must be contiguous [vocab, hidden_dim]");
    TORCH_CHECK(logits.dim() == 2 && logits.size(0) == hidden.size(0) && logits.size(1) == head.size(0),
                "logits must be [rows, vocab]");
    TORCH_CHECK(sync.scalar_type() == at::kInt && sync.numel() == 4 && sync.is_contiguous(),
                "sync must be 4 contiguous int32 words");
    TORCH_CHECK(steps.is_contiguous() && finished.is_contiguous() && history.is_contiguous(),
                "state tensors must be contiguous");
    TORCH_CHECK(finished.scalar_type() == at::kBool, "finished must be bool");
    b2s_sample_args a;
    fill_args(a, logits, history, steps, seeds, c10::nullopt, uniform_values, active, finished, row_temperature,
              row_top_p, row_top_k, alpha, status, temperature, top_p, top_k, min_keep, min_new, max_new, 0.0, 0.0, eos,
              semantics, rng, max_top_k, 0, 0);
    Tensor tokens = at::empty({logits.size(0)}, logits.options().dtype(at::kLong));
    a.tokens = tokens.data_ptr<int64_t>();
    a.history_out = history.numel() ? history.data_ptr<int64_t>() : nullptr;
    a.history_out_row_stride = history.dim() == 2 ? history.size(1) : 0;
    a.steps_out = steps.data_ptr<int64_t>();
    a.finished_out = reinterpret_cast<uint8_t*>(finished.data_ptr<bool>());
    b2s_head_args h;
    memset(&h, 0, sizeof(h));
    h.hidden = hidden.data_ptr();
    h.hidden_row_stride = hidden.size(0) > 1 ? hidden.stride(0) : hidden.size(1);
    h.head = head.data_ptr();
    h.hidden_dim = (int32_t)hidden.size(1);
    h.logits = logits.data_ptr();
    h.sync = reinterpret_cast<uint32_t*>(sync.data_ptr<int32_t>());
    check_rc(b2s_head_sample(&h, &a, at::cuda::getCurrentCUDAStream().stream()), "b2s_head_sample");
    return tokens;
}

// K frames in one launch: logits_k [K, B, V]; history / steps / finished advance in place over the frames.
Tensor sample_frames_cuda(const Tensor& logits_k, Tensor& history, Tensor& steps, Tensor& finished,
                          const optional<Tensor>& seeds, const optional<Tensor>& uniform_values,
                          const optional<Tensor>& active, const optional<Tensor>& alpha, const optional<Tensor>& status,
                          const optional<Tensor>& row_temperature, const optional<Tensor>& row_top_p,
                          const optional<Tensor>& row_top_k, double temperature, double top_p, int64_t top_k,
                          int64_t min_keep, int64_t min_new, int64_t max_new, int64_t eos, int64_t semantics,
                          int64_t rng, int64_t max_top_k) {
    c10::cuda::CUDAGuard guard(logits_k.device());
    TORCH_CHECK(logits_k.dim() == 3 && logits_k.stride(2) == 1, "logits_k must be [K, B, V] with contiguous rows");
    TORCH_CHECK(steps.is_contiguous() && finished.is_contiguous() && history.is_contiguous(),
                "state tensors must be contiguous");
    TORCH_CHECK(finished.scalar_type() == at::kBool, "finished must be bool");
    const int64_t K = logits_k.size(0), B = logits_k.size(1);
    optional<Tensor> u0 = c10::nullopt;
    if (uniform_values.has_value() && uniform_values->defined()) {
        TORCH_CHECK(uniform_values->numel() == K * B && uniform_values->is_contiguous() &&
                        uniform_values->scalar_type() == at::kFloat && uniform_values->is_cuda(),
                    "uniform_values must be contiguous float32 CUDA [K, B]");
        u0 = uniform_values->reshape({K * B}).narrow(0, 0, B);
    }
    b2s_sample_args a;
    fill_args(a, logits_k.select(0, 0), history, steps, seeds, c10::nullopt, u0, active, finished, row_temperature,
              row_top_p, row_top_k, alpha, status, temperature, top_p, top_k, min_keep, min_new, max_new, 0.0, 0.0, eos,
              semantics, rng, max_top_k, 0, 0);
    if (u0.has_value()) a.uniform_values = uniform_values->data_ptr<float>();
    Tensor tokens = at::empty({K, B}, logits_k.options().dtype(at::kLong));
    a.tokens = tokens.data_ptr<int64_t>();
    a.history_out = history.numel() ? history.data_ptr<int64_t>() : nullptr;
    a.history_out_row_stride = history.dim() == 2 ? history.size(1) : 0;
    a.steps_out = steps.data_ptr<int64_t>();
    a.finished_out = reinterpret_cast<uint8_t*>(finished.data_ptr<bool>());
    check_rc(b2s_sample_frames(&a, (int32_t)K, logits_k.stride(0), at::cuda::getCurrentCUDAStream().stream()),
             "b2s_sample_frames");
    return tokens;
}

Tensor sample_frames_meta(const Tensor& logits_k, Tensor&, Tensor&, Tensor&, const optional<Tensor>&,
                          const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                          const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                          const optional<Tensor>&, double, double, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                          int64_t, int64_t) {
    return at::empty({logits_k.size(0), logits_k.size(1)}, logits_k.options().dtype(at::kLong));
}

Tensor sample_state_meta(const Tensor& logits, Tensor&, Tensor&, Tensor&, const optional<Tensor>&,
                         const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                         const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                         const optional<Tensor>&, double, double, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                         int64_t, int64_t, int64_t, int64_t) {
    return at::empty({logits.size(0)}, logits.options().dtype(at::kLong));
}

// The Thinker's greedy step from its LM head: [B] int64 tokens; `keys` ([B] int64, zero between calls) is the
// reduction scratch the call leaves zero.
Tensor lmhead_argmax_cuda(const Tensor& hidden, const Tensor& head, Tensor& keys, const optional<Tensor>& status) {
    c10::cuda::CUDAGuard guard(hidden.device());
    TORCH_CHECK(hidden.is_cuda() && head.is_cuda() && keys.is_cuda() && head.device() == hidden.device() &&
                    keys.device() == hidden.device(),
                "hidden, head and keys must be on one CUDA device");
    TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && head.scalar_type() == at::kBFloat16,
                "hidden and head must be bfloat16");
    TORCH_CHECK(hidden.dim() == 2 && hidden.stride(1) == 1, "hidden must be [rows, hidden_dim] with contiguous rows");
    TORCH_CHECK(head.dim() == 2 && head.is_contiguous() && head.size(1) == hidden.size(1),
                "head must be contiguous [vocab, hidden_dim]");
    TORCH_CHECK(keys.scalar_type() == at::kLong && keys.is_contiguous() && keys.numel() == hidden.size(0),
                "keys must be [rows] int64");
    uint32_t* st = nullptr;
    if (status.has_value() && status->defined()) {
        TORCH_CHECK(status->is_cuda() && status->scalar_type() == at::kInt && status->numel() == 1,
                    "status must be a 1-element int32 CUDA tensor");
        st = reinterpret_cast<uint32_t*>(status->data_ptr<int32_t>());
    }
    Tensor tokens = at::empty({hidden.size(0)}, hidden.options().dtype(at::kLong));
    check_rc(b2s_lmhead_argmax(hidden.data_ptr(), hidden.size(0) > 1 ? hidden.stride(0) : hidden.size(1),
                               head.data_ptr(), (int32_t)hidden.size(1), (int32_t)head.size(0),
                               (int32_t)hidden.size(0), tokens.data_ptr<int64_t>(),
                               reinterpret_cast<uint64_t*>(keys.data_ptr<int64_t>()), st,
                               at::cuda::getCurrentCUDAStream().stream()),
             "b2s_lmhead_argmax");
    return tokens;
}

// One vocabulary shard of the same: [rows] int64 words whose max over the shards is the global argmax's key.
Tensor lmhead_argmax_keys_cuda(const Tensor& hidden, const Tensor& head, Tensor& keys, int64_t offset,
                               const optional<Tensor>& status) {
    c10::cuda::CUDAGuard guard(hidden.device());
    TORCH_CHECK(hidden.is_cuda() && head.is_cuda() && keys.is_cuda() && head.device() == hidden.device() &&
                    keys.device() == hidden.device(),
                "hidden, head and keys must be on one CUDA device");
    TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && head.scalar_type() == at::kBFloat16,
                "hidden and head must be bfloat16");
    TORCH_CHECK(hidden.dim() == 2 && hidden.stride(1) == 1, "hidden must be [rows, hidden_dim] with contiguous rows");
    TORCH_CHECK(head.dim() == 2 && head.is_contiguous() && head.size(1) == hidden.size(1),
                "head must be contiguous [vocab, hidden_dim]");
    TORCH_CHECK(keys.scalar_type() == at::kLong && keys.is_contiguous() && keys.numel() == hidden.size(0),
                "keys must be [rows] int64");
    uint32_t* st = nullptr;
    if (status.has_value() && status->defined()) {
        TORCH_CHECK(status->is_cuda() && status->scalar_type() == at::kInt && status->numel() == 1,
                    "status must be a 1-element int32 CUDA tensor");
        st = reinterpret_cast<uint32_t*>(status->data_ptr<int32_t>());
    }
    Tensor out = at::empty({hidden.size(0)}, hidden.options().dtype(at::kLong));
    check_rc(b2s_lmhead_argmax_keys(hidden.data_ptr(), hidden.size(0) > 1 ? hidden.stride(0) : hidden.size(1),
                                    head.data_ptr(), (int32_t)hidden.size(1), (int32_t)head.size(0), offset,
                                    (int32_t)hidden.size(0), out.data_ptr<int64_t>(),
                                    reinterpret_cast<uint64_t*>(keys.data_ptr<int64_t>()), st,
                                    at::cuda::getCurrentCUDAStream().stream()),
             "b2s_lmhead_argmax_keys");
    return out;
}

Tensor lmhead_argmax_keys_meta(const Tensor& hidden, const Tensor&, Tensor&, int64_t, const optional<Tensor>&) {
    return at::empty({hidden.size(0)}, hidden.options().dtype(at::kLong));
}

Tensor lmhead_argmax_meta(const Tensor& hidden, const Tensor&, Tensor&, const optional<Tensor>&) {
    return at::empty({hidden.size(0)}, hidden.options().dtype(at::kLong));
}

Tensor head_sample_state_meta(const Tensor& hidden, const Tensor&, Tensor&, Tensor&, Tensor&, Tensor&, Tensor&,
                              const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                              const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                              const optional<Tensor>&, const optional<Tensor>&, double, double, int64_t, int64_t,
                              int64_t, int64_t, int64_t, int64_t, int64_t, int64_t) {
    return at::empty({hidden.size(0)}, hidden.options().dtype(at::kLong));
}

Tensor argmax_cuda(const Tensor& logits) {
    c10::cuda::CUDAGuard guard(logits.device());
    TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "logits must be CUDA [rows, vocab]");
    TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16,
                "logits must be float32 or bfloat16");
    const int64_t B = logits.size(0), V = logits.size(1);
    Tensor out = at::empty({B}, logits.options().dtype(at::kLong));
    check_rc(b2s_argmax(logits.data_ptr(), logits.scalar_type() == at::kBFloat16 ? B2S_DTYPE_BF16 : B2S_DTYPE_F32,
                        (int32_t)B, (int32_t)V, B > 1 ? logits.stride(0) : V, out.data_ptr<int64_t>(),
                        at::cuda::getCurrentCUDAStream().stream()),
             "b2s_argmax");
    return out;
}

Tensor argmax_meta(const Tensor& logits) { return at::empty({logits.size(0)}, logits.options().dtype(at::kLong)); }

std::tuple<Tensor, Tensor, Tensor> shard_candidates_cuda(
    const Tensor& logits, const optional<Tensor>& history, const optional<Tensor>& steps, const optional<Tensor>& alpha,
    const optional<Tensor>& row_temperature, const optional<Tensor>& row_top_p, const optional<Tensor>& row_top_k,
    const optional<Tensor>& status, double temperature, double top_p, int64_t top_k, int64_t min_keep,
    double presence, double frequency, int64_t eos, int64_t max_top_k, int64_t offset, int64_t cap, int64_t cluster) {
    c10::cuda::CUDAGuard guard(logits.device());
    b2s_sample_args a;
    fill_args(a, logits, history, steps, c10::nullopt, c10::nullopt, c10::nullopt, c10::nullopt, c10::nullopt,
              row_temperature, row_top_p, row_top_k, alpha, status, temperature, top_p, top_k, min_keep, 0,
              (int64_t)1 << 62, presence, frequency, -1, B2S_SEM_OMNI, B2S_RNG_UNIFORM, max_top_k, 0, cluster);
    a.eos = (int32_t)std::max<int64_t>(std::min<int64_t>(eos, INT32_MAX), -1);
    const int64_t B = logits.size(0);
    Tensor v = at::empty({B, cap}, logits.options().dtype(at::kFloat));
    Tensor i = at::empty({B, cap}, logits.options().dtype(at::kInt));
    Tensor n = at::empty({B}, logits.options().dtype(at::kInt));
    check_rc(b2s_shard_candidates(&a, offset, (int32_t)cap, v.data_ptr<float>(), i.data_ptr<int32_t>(),
                                  n.data_ptr<int32_t>(), at::cuda::getCurrentCUDAStream().stream()),
             "b2s_shard_candidates");
    return {v, i, n};
}

std::tuple<Tensor, Tensor, Tensor> shard_candidates_meta(
    const Tensor& logits, const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
    const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&, double,
    double, int64_t, int64_t, double, double, int64_t, int64_t, int64_t, int64_t cap, int64_t) {
    const int64_t B = logits.size(0);
    return {at::empty({B, cap}, logits.options().dtype(at::kFloat)), at::empty({B, cap}, logits.options().dtype(at::kInt)),
            at::empty({B}, logits.options().dtype(at::kInt))};
}

// values / ids: [shards, rows, cap]; counts: [shards, rows]
std::tuple<Tensor, Tensor> shard_merge_cuda(const Tensor& values, const Tensor& ids, const Tensor& counts, int64_t vocab,
                        const optional<Tensor>& steps, const optional<Tensor>& seeds, const optional<Tensor>& requests,
                        const optional<Tensor>& uniform_values, const optional<Tensor>& row_top_p,
                        const optional<Tensor>& row_top_k, const optional<Tensor>& status, double top_p,
                        int64_t top_k, int64_t min_keep, int64_t rng, int64_t flags) {
    c10::cuda::CUDAGuard guard(values.device());
    TORCH_CHECK(values.is_cuda() && values.dim() == 3 && values.scalar_type() == at::kFloat && values.is_contiguous(),
                "values must be contiguous float32 CUDA [shards, rows, cap]");
    TORCH_CHECK(ids.sizes() == values.sizes() && ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.is_cuda(),
                "ids must be contiguous int32 CUDA [shards, rows, cap]");
    TORCH_CHECK(counts.dim() == 2 && counts.size(0) == values.size(0) && counts.size(1) == values.size(1) &&
                    counts.scalar_type() == at::kInt && counts.is_contiguous() && counts.is_cuda(),
                "counts must be contiguous int32 CUDA [shards, rows]");
    const int64_t S = values.size(0), B = values.size(1), cap = values.size(2);
    b2s_sample_args a;
    memset(&a, 0, sizeof(a));
    Tensor dummy = values.select(0, 0);
    a.steps = opt_ptr<int64_t>(steps, at::kLong, B, values, "steps");
    a.seeds = opt_ptr<int64_t>(seeds, at::kLong, B, values, "seeds");
    a.requests = opt_ptr<int64_t>(requests, at::kLong, B, values, "requests");
    a.uniform_values = opt_ptr<float>(uniform_values, at::kFloat, B, values, "uniform_values");
    a.row_top_p = opt_ptr<float>(row_top_p, at::kFloat, B, values, "row_top_p");
    a.row_top_k = opt_ptr<int32_t>(row_top_k, at::kInt, B, values, "row_top_k");
    if (status.has_value() && status->defined()) a.status = reinterpret_cast<uint32_t*>(status->data_ptr<int32_t>());
    a.top_p = (float)top_p;
    a.top_k = (int32_t)top_k;
    a.min_keep = (int32_t)min_keep;
    a.rng = (int32_t)rng;
    a.flags = (int32_t)flags;
    Tensor tokens = at::empty({B}, values.options().dtype(at::kLong));
    // one b2s_shard_pending record per row (32 bytes), kept opaque on the Python side
    static_assert(sizeof(b2s_shard_pending) == 32, "b2s_shard_pending is 32 bytes");
    Tensor pending = at::empty({B, 4}, values.options().dtype(at::kLong));
    a.tokens = tokens.data_ptr<int64_t>();
    check_rc(b2s_shard_merge(values.data_ptr<float>(), ids.data_ptr<int32_t>(), counts.data_ptr<int32_t>(), (int32_t)S,
                             (int32_t)B, (int32_t)cap, (int32_t)vocab, &a,
                             reinterpret_cast<b2s_shard_pending*>(pending.data_ptr<int64_t>()),
                             at::cuda::getCurrentCUDAStream().stream()),
             "b2s_shard_merge");
    return {tokens, pending};
}

std::tuple<Tensor, Tensor> shard_merge_meta(const Tensor& values, const Tensor&, const Tensor&, int64_t,
                                            const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                                            const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&,
                                            const optional<Tensor>&, double, int64_t, int64_t, int64_t, int64_t) {
    return {at::empty({values.size(1)}, values.options().dtype(at::kLong)),
            at::empty({values.size(1), 4}, values.options().dtype(at::kLong))};
}

// Stage 3 on this rank's shard: tokens for the rows pending on `shard`, the merged ones elsewhere, -1 for the rest.
Tensor shard_resolve_cuda(const Tensor& logits, const optional<Tensor>& history, const optional<Tensor>& steps,
                          const optional<Tensor>& alpha, const optional<Tensor>& row_temperature,
                          const optional<Tensor>& status, const Tensor& pending, const Tensor& merged,
                          double temperature, double presence, double frequency, int64_t eos, int64_t min_new,
                          int64_t offset, int64_t shard) {
    c10::cuda::CUDAGuard guard(logits.device());
    const int64_t B = logits.size(0);
    TORCH_CHECK(pending.is_cuda() && pending.dim() == 2 && pending.size(0) == B && pending.size(1) == 4 &&
                    pending.scalar_type() == at::kLong && pending.is_contiguous(),
                "pending must be the [rows, 4] int64 CUDA records of shard_merge");
    TORCH_CHECK(merged.is_cuda() && merged.numel() == B && merged.scalar_type() == at::kLong && merged.is_contiguous(),
                "merged must be the [rows] int64 CUDA tokens of shard_merge");
    b2s_sample_args a;
    fill_args(a, logits, history, steps, c10::nullopt, c10::nullopt, c10::nullopt, c10::nullopt, c10::nullopt,
              row_temperature, c10::nullopt, c10::nullopt, alpha, status, temperature, 1.0, 1, 1, min_new,
              (int64_t)1 << 62, presence, frequency, -1, B2S_SEM_OMNI, B2S_RNG_UNIFORM, 1, 0, 0);
    a.eos = (int32_t)std::max<int64_t>(std::min<int64_t>(eos, INT32_MAX), -1);
    Tensor out = at::empty({B}, logits.options().dtype(at::kLong));
    check_rc(b2s_shard_resolve(&a, offset, (int32_t)shard,
                               reinterpret_cast<const b2s_shard_pending*>(pending.data_ptr<int64_t>()),
                               merged.data_ptr<int64_t>(), out.data_ptr<int64_t>(),
                               at::cuda::getCurrentCUDAStream().stream()),
             "b2s_shard_resolve");
    return out;
}

Tensor shard_resolve_meta(const Tensor& logits, const optional<Tensor>&, const optional<Tensor>&,
                          const optional<Tensor>&, const optional<Tensor>&, const optional<Tensor>&, const Tensor&,
                          const Tensor&, double, double, double, int64_t, int64_t, int64_t, int64_t) {
    return at::empty({logits.size(0)}, logits.options().dtype(at::kLong));
}

Tensor penalty_cuda(const Tensor& x, const Tensor& history, const Tensor& alpha) {
    c10::cuda::CUDAGuard guard(x.device());
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "x must be CUDA [rows, vocab] with contiguous rows");
    TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16, "x must be float32 or bfloat16");
    TORCH_CHECK(history.is_cuda() && history.device() == x.device() && history.scalar_type() == at::kLong &&
                    history.dim() == 2 && history.size(0) == x.size(0) && history.stride(1) == 1,
                "history must be int64 CUDA [rows, window]");
    TORCH_CHECK(alpha.is_cuda() && alpha.scalar_type() == at::kFloat && alpha.is_contiguous() &&
                    (alpha.dim() == 1 || (alpha.dim() == 2 && alpha.size(0) == x.size(0))),
                "alpha must be float32 CUDA [n] or [rows, n]");
    const int64_t B = x.size(0), V = x.size(1);
    Tensor out = at::empty({B, V}, x.options().dtype(at::kFloat));
    check_rc(b2s_repetition_penalty(x.data_ptr(), x.scalar_type() == at::kBFloat16 ? B2S_DTYPE_BF16 : B2S_DTYPE_F32,
                                    (int32_t)B, (int32_t)V, B > 1 ? x.stride(0) : V, history.data_ptr<int64_t>(),
                                    (int32_t)history.size(1), B > 1 ? history.stride(0) : history.size(1),
                                    alpha.data_ptr<float>(), (int32_t)alpha.size(-1),
                                    alpha.dim() == 2 ? (int32_t)alpha.size(1) : 0, out.data_ptr<float>(), V, nullptr,
                                    at::cuda::getCurrentCUDAStream().stream()),
             "b2s_repetition_penalty");
    return out;
}

Tensor penalty_meta(const Tensor& x, const Tensor&, const Tensor&) {
    return at::empty({x.size(0), x.size(1)}, x.options().dtype(at::kFloat));
}

Tensor uniform_cuda(const Tensor& seeds, const Tensor& steps, const optional<Tensor>& requests, int64_t rng) {
    c10::cuda::CUDAGuard guard(seeds.device());
    TORCH_CHECK(seeds.is_cuda() && steps.is_cuda() && seeds.scalar_type() == at::kLong &&
                    steps.scalar_type() == at::kLong && seeds.is_contiguous() && steps.is_contiguous() &&
                    seeds.numel() == steps.numel(),
                "seeds / steps must be contiguous int64 CUDA tensors of one size");
    Tensor out = at::empty(seeds.sizes(), seeds.options().dtype(at::kFloat));
    const int64_t* rq = opt_ptr<int64_t>(requests, at::kLong, seeds.numel(), seeds, "requests");
    check_rc(b2s_uniform(seeds.data_ptr<int64_t>(), steps.data_ptr<int64_t>(), rq, seeds.numel(), (int32_t)rng,
                         out.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()),
             "b2s_uniform");
    return out;
}

Tensor uniform_meta(const Tensor& seeds, const Tensor&, const optional<Tensor>&, int64_t) {
    return at::empty(seeds.sizes(), seeds.options().dtype(at::kFloat));
}

}  // namespace

TORCH_LIBRARY(minicpmo_sampler, m) {
    m.def(
        "sample(Tensor logits, Tensor? history, Tensor? steps, Tensor? seeds, Tensor? requests, "
        "Tensor? uniform_values, Tensor? active, Tensor? finished, Tensor? row_temperature, Tensor? row_top_p, "
        "Tensor? row_top_k, Tensor? row_min_new, Tensor? row_max_new, Tensor? alpha, Tensor? status, "
        "float temperature, float top_p, int top_k, int min_keep, "
        "int min_new_tokens, int max_new_tokens, float presence_penalty, float frequency_penalty, int eos, "
        "int semantics, int rng, int max_top_k, int flags, bool want_tokens, bool want_processed, bool want_state, "
        "int cluster) -> (Tensor tokens, Tensor processed, Tensor history_out, Tensor steps_out, Tensor finished_out)");
    m.def(
        "sample_state_(Tensor logits, Tensor(a!) history, Tensor(b!) steps, Tensor(c!) finished, Tensor? seeds, "
        "Tensor? uniform_values, Tensor? active, Tensor? alpha, Tensor? status, Tensor? row_temperature, "
        "Tensor? row_top_p, Tensor? row_top_k, float temperature, float top_p, int top_k, int min_keep, "
        "int min_new_tokens, int max_new_tokens, int eos, int semantics, int rng, int max_top_k, int cluster, "
        "int flags=0) -> Tensor tokens");
    m.def(
        "sample_frames_(Tensor logits_k, Tensor(a!) history, Tensor(b!) steps, Tensor(c!) finished, Tensor? seeds, "
        "Tensor? uniform_values, Tensor? active, Tensor? alpha, Tensor? status, Tensor? row_temperature, "
        "Tensor? row_top_p, Tensor? row_top_k, float temperature, float top_p, int top_k, int min_keep, "
        "int min_new_tokens, int max_new_tokens, int eos, int semantics, int rng, int max_top_k) -> Tensor tokens");
    m.def(
        "head_sample_state_(Tensor hidden, Tensor head, Tensor(a!) logits, Tensor(b!) sync, Tensor(c!) history, "
        "Tensor(d!) steps, Tensor(e!) finished, Tensor? seeds, Tensor? uniform_values, Tensor? active, Tensor? alpha, "
        "Tensor? status, Tensor? row_temperature, Tensor? row_top_p, Tensor? row_top_k, float temperature, "
        "float top_p, int top_k, int min_keep, int min_new_tokens, int max_new_tokens, int eos, int semantics, "
        "int rng, int max_top_k) -> Tensor tokens");
    m.def("lmhead_argmax(Tensor hidden, Tensor head, Tensor(a!) keys, Tensor? status) -> Tensor tokens");
    m.def("lmhead_argmax_keys(Tensor hidden, Tensor head, Tensor(a!) keys, int offset, Tensor? status) -> Tensor");
    m.def("argmax(Tensor logits) -> Tensor");
    m.def("uniform(Tensor seeds, Tensor steps, Tensor? requests, int rng) -> Tensor");
    m.def("repetition_penalty(Tensor x, Tensor history, Tensor alpha) -> Tensor");
    m.def(
        "shard_candidates(Tensor logits, Tensor? history, Tensor? steps, Tensor? alpha, Tensor? row_temperature, "
        "Tensor? row_top_p, Tensor? row_top_k, Tensor? status, float temperature, float top_p, int top_k, "
        "int min_keep, float presence_penalty, float frequency_penalty, int eos, int max_top_k, int offset, int cap, "
        "int cluster) -> (Tensor values, Tensor ids, Tensor count)");
    m.def(
        "shard_merge(Tensor values, Tensor ids, Tensor counts, int vocab, Tensor? steps, Tensor? seeds, "
        "Tensor? requests, Tensor? uniform_values, Tensor? row_top_p, Tensor? row_top_k, Tensor? status, "
        "float top_p, int top_k, int min_keep, int rng, int flags) -> (Tensor tokens, Tensor pending)");
    m.def(
        "shard_resolve(Tensor logits, Tensor? history, Tensor? steps, Tensor? alpha, Tensor? row_temperature, "
        "Tensor? status, Tensor pending, Tensor merged, float temperature, float presence_penalty, "
        "float frequency_penalty, int eos, int min_new_tokens, int offset, int shard) -> Tensor");
}

TORCH_LIBRARY_IMPL(minicpmo_sampler, CUDA, m) {
    m.impl("sample", &sample_cuda);
    m.impl("sample_state_", &sample_state_cuda);
    m.impl("sample_frames_", &sample_frames_cuda);
    m.impl("head_sample_state_", &head_sample_state_cuda);
    m.impl("lmhead_argmax", &lmhead_argmax_cuda);
    m.impl("lmhead_argmax_keys", &lmhead_argmax_keys_cuda);
    m.impl("argmax", &argmax_cuda);
    m.impl("uniform", &uniform_cuda);
    m.impl("repetition_penalty", &penalty_cuda);
    m.impl("shard_candidates", &shard_candidates_cuda);
    m.impl("shard_merge", &shard_merge_cuda);
    m.impl("shard_resolve", &shard_resolve_cuda);
}

TORCH_LIBRARY_IMPL(minicpmo_sampler, Meta, m) {
    m.impl("sample", &sample_meta);
    m.impl("sample_state_", &sample_state_meta);
    m.impl("sample_frames_", &sample_frames_meta);
    m.impl("head_sample_state_", &head_sample_state_meta);
    m.impl("lmhead_argmax", &lmhead_argmax_meta);
    m.impl("lmhead_argmax_keys", &lmhead_argmax_keys_meta);
    m.impl("argmax", &argmax_meta);
    m.impl("uniform", &uniform_meta);
    m.impl("repetition_penalty", &penalty_meta);
    m.impl("shard_candidates", &shard_candidates_meta);
    m.impl("shard_merge", &shard_merge_meta);
    m.impl("shard_resolve", &shard_resolve_meta);
}
