"""The Talker codec head fused with the decode step (``CodecHead`` / ``b2s_head_sample``) on the B200.

The head's logits are checked against a plain matmul of the same bf16 operands (float64 on the CPU): the launch
rounds its fp32 tensor-core sum to bf16, so each logit is the bf16 rounding of the exact dot product up to the
order of the fp32 accumulation -- equal to it for at least 99.5 % of the logits and never more than one bf16 ulp
away.  The tokens and the state are bit-exact against the oracle run on the launch's own logits, and equal to the
oracle run on the rounded exact logits in every row whose logits agree bit for bit.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests.golden import inputs as I

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
V_TALKER, EOS = 6562, 6561


def _operands(B, V, H, seed, hid_pad=0):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(B, H + hid_pad, generator=g).to(torch.bfloat16)
    head = (torch.randn(V, H, generator=g) * (2.0 / H ** 0.5)).to(torch.bfloat16)  # logits ~ N(0, 2)
    return hidden, head


def _exact(hidden, head):
    H = head.shape[1]
    return hidden[:, :H].double() @ head.double().T


def _check_logits(got_bf16, exact):
    got = got_bf16.float().cpu().double()
    want = exact.to(torch.bfloat16).double()
    same = (got == want).double().mean().item()
    assert same >= 0.995, same
    # one bf16 ulp at |exact|, plus 1e-4 for the fp32 accumulation of 768 products of magnitude <= ~4 (it only
    # matters for logits within ~1e-2 of zero)
    ulp = torch.clamp(exact.abs(), min=2.0 ** -100).log2().floor().sub(7).exp2()
    assert bool(((got - exact).abs() <= ulp + 1e-4).all())
    return (got == want).all(dim=1).numpy()


def _expect_state(hist, steps, fin, active, tok, eos):
    live = active & ~fin
    adv = live & (tok != I.PAD)
    h2 = hist.copy()
    if hist.shape[1]:
        h2[adv] = np.concatenate([hist[adv, 1:], tok[adv, None]], axis=1)
    return h2, steps + adv, fin | (adv & (tok == eos))


def _run_case(pkg, *, B, V, H, W, cfg_kw, eos, steps, seed, rng="uniform", per_row=None, hid_pad=0, calls=2):
    ts = pkg.talker_sampler
    hidden_h, head_h = _operands(B, V, H, seed, hid_pad)
    ch = ts.CodecHead(head_h.to(DEV), B)
    g = np.random.default_rng(seed)
    hist = np.full((B, W), I.PAD, np.int64)
    for r in range(B):
        n = int(min(steps[r], W))
        if n:
            hist[r, W - n:] = g.integers(0, V, size=n)
    cfg = ts.TalkerSampling(**cfg_kw, window=W, rng="counter")
    st = ts.DecodeState.new(list(range(100, 100 + B)), cfg, device=DEV)
    st.history.copy_(torch.from_numpy(hist))
    st.steps.copy_(torch.from_numpy(np.asarray(steps, np.int64)))
    rp, rowkw = None, {}
    if per_row:
        T, P, K = per_row
        rp = ts.RowParams(temperature=torch.tensor(T, dtype=torch.float32, device=DEV),
                          top_p=torch.tensor(P, dtype=torch.float32, device=DEV),
                          top_k=torch.tensor(K, dtype=torch.int32, device=DEV), max_top_k=max(K))
        rowkw = dict(row_temperature=np.asarray(T, np.float32), row_top_p=np.asarray(P, np.float32),
                     row_top_k=np.asarray(K, np.int32))
    ocfg = orc.Cfg(**cfg_kw, window=W)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for call in range(calls):
        hidden = (hidden_h if call == 0 else torch.roll(hidden_h, 1, dims=1)).to(DEV)
        hid = hidden[:, :H] if hid_pad else hidden
        h0, s0, f0 = st.history.cpu().numpy(), st.steps.cpu().numpy(), st.finished.cpu().numpy()
        act = st.active.cpu().numpy()
        u = np.random.default_rng(seed * 7 + call).random(B).astype(np.float32)
        if rng == "uniform":
            tok = ch.step_(st, hid, eos, cfg, uniform_values=torch.from_numpy(u).to(DEV), status=status,
                           row_params=rp)
            okw = dict(uniforms=u, rng=orc.RNG_COUNTER)
        else:
            tok = ch.step_(st, hid, eos, cfg, status=status, row_params=rp, rng=rng)
            okw = dict(rng=orc.RNG_PHILOX if rng == "philox" else orc.RNG_COUNTER,
                       requests=np.zeros(B, np.int64) if rng == "philox" else None)
        torch.cuda.synchronize()
        got = tok.cpu().numpy()
        lg = ch.logits.clone()
        rows_exact = _check_logits(lg, _exact(hidden.cpu(), head_h))
        bits = lg.cpu().view(torch.int16).numpy().view(np.uint16)
        _, want, _, _ = orc.sample(bits, h0, s0, np.arange(100, 100 + B, dtype=np.int64), eos, ocfg,
                                   want_processed=False, **okw, **rowkw)
        want = np.where(act & ~f0, want, I.PAD)
        assert np.array_equal(got, want), (call, got, want)
        # the oracle on the bf16 rounding of the exact logits: same tokens wherever the logits agree
        ebits = _exact(hidden.cpu(), head_h).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        _, want_e, _, _ = orc.sample(ebits, h0, s0, np.arange(100, 100 + B, dtype=np.int64), eos, ocfg,
                                     want_processed=False, **okw, **rowkw)
        want_e = np.where(act & ~f0, want_e, I.PAD)
        assert np.array_equal(got[rows_exact], want_e[rows_exact])
        h1, s1, f1 = _expect_state(h0, s0, f0, act, got, eos)
        assert np.array_equal(st.history.cpu().numpy(), h1)
        assert np.array_equal(st.steps.cpu().numpy(), s1)
        assert np.array_equal(st.finished.cpu().numpy(), f1)
        assert int(status.item()) == 0
        assert ch.sync.cpu().tolist() == [0, 0, 0, 0]  # every completed launch leaves the control words zero
    return ch


def test_head_talker_batched(pkg):
    """BASELINE config 2's batch from the codec head: 8 rows, per-row T / k / p, hf order, 64-token window,
    EOS masked for 8 steps, rows on frame 0 (full-row path) and past it; two launches in a row."""
    _run_case(pkg, B=8, V=V_TALKER, H=768, W=64,
              cfg_kw=dict(temperature=0.8, top_k=25, top_p=0.85, repetition_penalty=1.05, min_new_tokens=8,
                          max_new_tokens=1 << 40, min_keep=3, semantics="hf"),
              eos=EOS, steps=[0, 1, 3, 7, 8, 9, 100, 500], seed=1,
              per_row=([(0.6, 0.8, 1.0)[r % 3] for r in range(8)], [(0.7, 0.85, 0.95)[r % 3] for r in range(8)],
                       [(20, 25, 50)[r % 3] for r in range(8)]))


def test_head_single_stream_counter_rng(pkg):
    """BASELINE config 1's shape (one row, 16-token window) from the head, the reference's counter RNG."""
    _run_case(pkg, B=1, V=V_TALKER, H=768, W=16,
              cfg_kw=dict(temperature=0.8, top_k=25, top_p=0.85, repetition_penalty=1.05, min_new_tokens=0,
                          max_new_tokens=1 << 40, min_keep=3, semantics="hf"),
              eos=EOS, steps=[5], seed=2, rng="counter", calls=3)


def test_head_full_batch_omni_philox(pkg):
    """16 rows (the head's largest batch), a vocabulary that is not a multiple of the 128-id tile, hidden 512,
    omni order, Philox draws."""
    _run_case(pkg, B=16, V=1000, H=512, W=32,
              cfg_kw=dict(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.1, min_new_tokens=0,
                          max_new_tokens=1 << 40, min_keep=1, semantics="omni"),
              eos=-1, steps=list(range(3, 19)), seed=3, rng="philox")


def test_head_one_k_block_strided_hidden(pkg):
    """hidden 64 (one K block of the MMA chain), hidden rows taken from a wider tensor (row stride 128)."""
    _run_case(pkg, B=3, V=V_TALKER, H=64, W=8,
              cfg_kw=dict(temperature=1.0, top_k=50, top_p=0.95, repetition_penalty=1.05, min_new_tokens=0,
                          max_new_tokens=1 << 40, min_keep=3, semantics="hf"),
              eos=EOS, steps=[1, 2, 3], seed=4, hid_pad=64)


def test_head_is_one_launch(pkg):
    """The head and the step are one kernel: no GEMM library kernel, no separate sampling kernel."""
    from torch.profiler import ProfilerActivity, profile

    ts = pkg.talker_sampler
    hidden, head = _operands(8, V_TALKER, 768, 5)
    ch = ts.CodecHead(head.to(DEV), 8)
    cfg = ts.TalkerSampling(window=64, min_new_tokens=0, rng="counter")
    st = ts.DecodeState.new(list(range(8)), cfg, device=DEV)
    st.steps.fill_(1)
    h = hidden.to(DEV)
    ch.step_(st, h, EOS, cfg)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        ch.step_(st, h, EOS, cfg)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
    if not names:
        pytest.skip("the profiler recorded no CUDA kernels here")
    kernels = [n for n in names if "Memcpy" not in n and "Memset" not in n]
    assert any("head_kernel" in n for n in kernels), kernels
    assert not any("gemm" in n.lower() or "short_kernel" in n for n in kernels), kernels


def test_head_rejects_what_it_cannot_take(pkg):
    """Host-side checks, before any launch: more than 16 rows, hidden beyond 768, non-bf16 operands."""
    ts = pkg.talker_sampler
    cfg = ts.TalkerSampling(window=16, rng="counter")
    head = torch.zeros(V_TALKER, 768, dtype=torch.bfloat16, device=DEV)
    ch = ts.CodecHead(head, 17)
    st = ts.DecodeState.new(list(range(17)), cfg, device=DEV)
    with pytest.raises(RuntimeError, match="unsupported"):
        ch.step_(st, torch.zeros(17, 768, dtype=torch.bfloat16, device=DEV), EOS, cfg)
    ch = ts.CodecHead(torch.zeros(V_TALKER, 832, dtype=torch.bfloat16, device=DEV), 2)
    st = ts.DecodeState.new([0, 1], cfg, device=DEV)
    with pytest.raises(RuntimeError, match="unsupported"):
        ch.step_(st, torch.zeros(2, 832, dtype=torch.bfloat16, device=DEV), EOS, cfg)
    with pytest.raises(ValueError):
        ts.CodecHead(torch.zeros(V_TALKER, 768, dtype=torch.float32, device=DEV), 2)
    torch.cuda.synchronize()


def test_head_graph_replay_matches_eager(pkg):
    """CodecHead.step_ captured once in a CUDA graph and replayed frame by frame (new hidden rows copied into the
    captured buffer) == eager calls on a copy of the state: the same tokens, history, steps and finished flags,
    through EOS masking and forcing and an inactive row -- the form of the reference's graph bodies
    (engine/runtime/talker_post_graph.py:56-76)."""
    ts = pkg.talker_sampler
    B, Hd, F = 6, 768, 16
    cfg = ts.TalkerSampling(semantics="hf", rng="counter", min_new_tokens=3, max_new_tokens=12, window=16)
    hidden_h, head_h = _operands(B, V_TALKER, Hd, 21)
    head = head_h.to(DEV)
    g = torch.Generator().manual_seed(22)
    frames = torch.randn(F, B, Hd, generator=g).to(torch.bfloat16).to(DEV)
    eager_h, graph_h = ts.CodecHead(head, B), ts.CodecHead(head, B)
    eager = ts.DecodeState.new(list(range(40, 40 + B)), cfg, device=DEV)
    graphed = ts.DecodeState.new(list(range(40, 40 + B)), cfg, device=DEV)
    for st in (eager, graphed):
        st.active[4] = False
    static_h = frames[0].clone()
    warm = ts.DecodeState.new(list(range(40, 40 + B)), cfg, device=DEV)
    graph_h.step_(warm, static_h, EOS, cfg)  # builds the penalty table before capture
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=DEV)
    with torch.cuda.graph(gr, stream=s, capture_error_mode="thread_local"):
        static_tok = graph_h.step_(graphed, static_h, EOS, cfg)
    for f in range(F):
        static_h.copy_(frames[f])
        gr.replay()
        want = eager_h.step_(eager, frames[f], EOS, cfg)
        torch.cuda.synchronize()
        assert torch.equal(static_tok, want), f
        assert torch.equal(graph_h.logits, eager_h.logits), f
        assert torch.equal(graphed.history, eager.history) and torch.equal(graphed.steps, eager.steps)
        assert torch.equal(graphed.finished, eager.finished)
    assert int(eager.steps[4]) == 0 and bool(eager.finished.any())  # max_new_tokens forced EOS
    assert graph_h.sync.cpu().tolist() == [0, 0, 0, 0]
    del gr
