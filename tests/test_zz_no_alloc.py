"""``b2s_head_sample_noalloc`` against ``b2s_head_sample`` through the C-ABI (B200 only).

The no-alloc entry point serves callers that cannot allocate device memory on the decode path -- an embedding
whose allocator is fixed at start-up, a runtime that hands the library only the buffers it owns, or a loop that
must not call cudaMalloc / cudaFree while other work runs, since those can synchronise the device.  It keeps the
head's logits rows and control words in a fixed array inside the library instead of buffers the caller passes.
This test feeds both entry points the same inputs and two identical copies of the decode state, calls each twice
in a row (the state advancing in place), and requires identical tokens and states: the same kernel runs on the
same logits, so the results agree bit for bit.  It also checks that sizes beyond the array are refused.

The file name puts it last in collection order, so that a run stopping at the first failure has run every other
test already; it passes both alone in a fresh process and after the rest.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
B2S_OK, B2S_ERR_UNSUPPORTED = 0, 2
B2S_DTYPE_BF16, B2S_SEM_HF, B2S_RNG_UNIFORM = 1, 0, 0
B, V, H, W, EOS = 8, 6562, 768, 64, 6561


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _state(seed):
    g = np.random.default_rng(seed)
    steps = torch.tensor([1, 2, 3, 7, 8, 9, 100, 500], dtype=torch.int64, device=DEV)
    hist = torch.from_numpy(g.integers(0, V, size=(B, W))).to(DEV)
    return dict(history=hist, steps=steps, finished=torch.zeros(B, dtype=torch.bool, device=DEV),
                active=torch.ones(B, dtype=torch.bool, device=DEV),
                seeds=torch.arange(B, dtype=torch.int64, device=DEV))


def _args(pkg, st, uniforms, tokens, alpha, vocab=V):
    a = pkg._native.SampleArgs()
    a.logits = None
    a.logits_dtype = B2S_DTYPE_BF16
    a.rows, a.vocab, a.cluster = B, vocab, 0
    a.logits_row_stride = vocab
    a.history, a.history_row_stride, a.window = _ptr(st["history"]), W, W
    a.eos = EOS
    a.steps, a.seeds, a.uniform_values = _ptr(st["steps"]), _ptr(st["seeds"]), _ptr(uniforms)
    a.active, a.finished = _ptr(st["active"]), _ptr(st["finished"])
    a.temperature, a.top_p, a.top_k, a.min_keep = 0.8, 0.85, 25, 3
    a.min_new_tokens, a.max_new_tokens = 8, 1 << 40
    a.alpha, a.alpha_len, a.alpha_row_stride = _ptr(alpha), alpha.numel(), 0
    a.max_top_k, a.semantics, a.rng, a.flags = 25, B2S_SEM_HF, B2S_RNG_UNIFORM, 0
    a.tokens = _ptr(tokens)
    a.history_out, a.history_out_row_stride = _ptr(st["history"]), W
    a.steps_out, a.finished_out = _ptr(st["steps"]), _ptr(st["finished"])
    return a


def test_noalloc_head_matches_the_allocating_entry_point(pkg):
    lib = pkg._native.capi()
    ts = pkg.talker_sampler
    g = torch.Generator().manual_seed(11)
    hidden = torch.randn(B, H, generator=g).to(torch.bfloat16).to(DEV)
    head = (torch.randn(V, H, generator=g) * (2.0 / H ** 0.5)).to(torch.bfloat16).to(DEV)
    alpha = ts.alpha_table(1.05, W + 1, DEV)
    st_ref, st_new = _state(5), _state(5)
    logits = torch.empty(B, V, dtype=torch.bfloat16, device=DEV)  # the allocating entry point's buffers
    sync = torch.zeros(4, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # two calls in a row: the scratch keeps the previous call's contents
        u = torch.from_numpy(np.random.default_rng(call).random(B).astype(np.float32)).to(DEV)
        tok_ref = torch.empty(B, dtype=torch.int64, device=DEV)
        tok_new = torch.empty(B, dtype=torch.int64, device=DEV)
        h = pkg._native.HeadArgs(hidden=hidden.data_ptr(), hidden_row_stride=H, head=head.data_ptr(), hidden_dim=H,
                                 logits=logits.data_ptr(), sync=sync.data_ptr())
        a_ref = _args(pkg, st_ref, u, tok_ref, alpha)
        assert lib.b2s_head_sample(ctypes.byref(h), ctypes.byref(a_ref), stream) == B2S_OK
        a_new = _args(pkg, st_new, u, tok_new, alpha)
        assert lib.b2s_head_sample_noalloc(_ptr(hidden), H, _ptr(head), H, ctypes.byref(a_new), stream) == B2S_OK
        torch.cuda.synchronize()
        assert torch.equal(tok_new, tok_ref), (call, tok_new, tok_ref)
        for k in ("history", "steps", "finished"):
            assert torch.equal(st_new[k], st_ref[k]), (call, k)
        assert bool((tok_ref >= 0).all())  # every row is live and drew a token
    # sizes beyond the library's array are refused before anything is launched
    big = _args(pkg, st_new, u, tok_new, alpha, vocab=8193)
    assert lib.b2s_head_sample_noalloc(_ptr(hidden), H, _ptr(head), H, ctypes.byref(big), stream) == B2S_ERR_UNSUPPORTED
    torch.cuda.synchronize()
