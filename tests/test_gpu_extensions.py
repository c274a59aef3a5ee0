"""GPU parity of the paths beyond the reference's own sampler: presence / frequency penalties, the public
Thinker entry (``thinker_sampler.sample`` in every RNG mode and its temperature-0 branch), per-row top-k
above the scalar one, the native-RNG draw on CUDA generators, and CUDA-graph replay of the in-place step.

Presence / frequency penalties and the non-greedy Thinker step have no reference implementation; their
oracle is the composition of the reference's functions that the CPU oracle restates (penalty, then
``- presence``, ``- frequency * count``, then ``/ T``, in the omni order).  Bar: bit-identical processed
values, kept set and token ids.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests import _harness as H
from tests.golden import inputs as I

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _bf16(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(I.to_bf16_bits(x).view(np.int16)).view(torch.bfloat16).to(DEV)


def _rows(kind: str, B: int, seed: int):
    """(logits fp32 values, device logits, history) of a thinker-shaped bf16 batch or a talker-shaped fp32
    one; every history repeats a few ids several times (counts 2..6)."""
    g = I.rng(seed)
    if kind == "thinker":
        logits, hist = I.zipf_rows(g, B, I.THINKER_V, 256)
        logits = I.bf16_bits_to_f32(I.to_bf16_bits(logits))
        x = _bf16(logits)
    else:
        logits = (g.standard_normal((B, I.TALKER_V)) * 2.0).astype(np.float32)
        hist = g.integers(0, I.TALKER_V, size=(B, 64))
        x = torch.from_numpy(logits).to(DEV)
    # top ids of each row repeated: the penalties then decide which of them stay
    top = np.argsort(-logits, axis=1)[:, :4]
    for r in range(B):
        for j, t in enumerate(top[r]):
            hist[r, 3 * j: 3 * j + 2 + j] = t
    hist[::3, -1] = -1
    return logits, x, hist.astype(np.int64)


@pytest.mark.parametrize("kind", ["thinker", "talker"])
@pytest.mark.parametrize("presence,frequency", [(0.5, 0.0), (0.0, 0.35), (0.75, 0.25), (-0.4, 0.1)])
def test_presence_frequency_penalties_match_oracle(pkg, kind, presence, frequency):
    ts = pkg.talker_sampler
    B = 8
    logits, x, hist = _rows(kind, B, 500 + int(presence * 100) + int(frequency * 1000))
    steps = np.full(B, 4, np.int64)
    seeds = np.arange(B, dtype=np.int64) * 977 + 3
    u = I.rng(9).random(B, dtype=np.float32)
    cfg = orc.Cfg(temperature=0.7, top_p=0.8, top_k=20, repetition_penalty=1.1, window=hist.shape[1], min_new_tokens=0,
                  max_new_tokens=1 << 40, min_keep=1, semantics="omni", presence_penalty=presence,
                  frequency_penalty=frequency)
    xin = I.to_bf16_bits(logits) if kind == "thinker" else logits
    want_p, want_t, _, _ = orc.sample(xin, hist, steps, seeds, -1, cfg, uniforms=u)
    tcfg = ts.TalkerSampling(temperature=0.7, top_p=0.8, top_k=20, repetition_penalty=1.1, window=hist.shape[1],
                             min_new_tokens=0, max_new_tokens=1 << 40, min_keep=1, semantics="omni")
    hd = torch.from_numpy(hist).to(DEV)
    kw = ts._cfg_kwargs(tcfg, hd, DEV)
    for processed in (True, False):
        tok, proc, _, _, _ = ts._run(x, history=hd, steps=torch.from_numpy(steps).to(DEV),
                                     uniform_values=torch.from_numpy(u).to(DEV), rng=ts.RNG_UNIFORM, presence=presence,
                                     frequency=frequency, processed=processed, **kw)
        assert np.array_equal(tok.cpu().numpy(), want_t), (processed, tok.cpu().numpy(), want_t)
        if processed:
            assert len(H.compare_processed(want_p, proc.cpu().numpy())) == 0
    # the same through the public Thinker entry (Philox RNG keyed by (seed, step, request))
    ths = pkg.thinker_sampler
    tcfg2 = ths.ThinkerSampling(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.1, presence_penalty=presence,
                                frequency_penalty=frequency, window=hist.shape[1], rng="philox")
    req = np.arange(B, dtype=np.int64) + 40
    got = ths.sample(x, hd, torch.from_numpy(seeds).to(DEV), torch.from_numpy(steps).to(DEV), tcfg2,
                     requests=torch.from_numpy(req).to(DEV)).cpu().numpy()
    _, want_ph, _, _ = orc.sample(xin, hist, steps, seeds, -1, cfg, rng=orc.RNG_PHILOX, requests=req)
    assert np.array_equal(got, want_ph)


@pytest.mark.parametrize("kind", ["thinker", "talker"])
def test_thinker_sample_entry_all_modes(pkg, kind):
    """thinker_sampler.sample: Philox, counter and injected uniforms against the oracle; temperature 0 is the
    first index of the penalised maximum (with penalties) or the plain argmax (without)."""
    ths = pkg.thinker_sampler
    B = 12
    logits, x, hist = _rows(kind, B, 61)
    W = hist.shape[1]
    xin = I.to_bf16_bits(logits) if kind == "thinker" else logits
    steps = np.arange(B, dtype=np.int64) + 1
    seeds = ((np.arange(B, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)) & np.uint64((1 << 63) - 1)).astype(np.int64)
    u = I.rng(3).random(B, dtype=np.float32)
    hd, sd, td = (torch.from_numpy(a).to(DEV) for a in (hist, seeds, steps))
    ocfg = orc.Cfg(temperature=0.9, top_p=0.9, top_k=32, repetition_penalty=1.05, window=W, min_new_tokens=0,
                   max_new_tokens=1 << 40, min_keep=1, semantics="omni")
    cfg = ths.ThinkerSampling(temperature=0.9, top_k=32, top_p=0.9, repetition_penalty=1.05, window=W)
    _, want, _, _ = orc.sample(xin, hist, steps, seeds, -1, ocfg, rng=orc.RNG_PHILOX)
    assert np.array_equal(ths.sample(x, hd, sd, td, cfg).cpu().numpy(), want)
    _, want, _, _ = orc.sample(xin, hist, steps, seeds, -1, ocfg, rng=orc.RNG_COUNTER)
    got = ths.sample(x, hd, sd.to(torch.int32) if kind == "talker" else sd, td.to(torch.int32),
                     ths.ThinkerSampling(**{**cfg.__dict__, "rng": "counter"}))
    if kind == "talker":  # int32 seeds: the low words only (the ints above were reduced to 63 bits)
        _, want, _, _ = orc.sample(xin, hist, steps, seeds.astype(np.int32).astype(np.int64), -1, ocfg,
                                   rng=orc.RNG_COUNTER)
    assert np.array_equal(got.cpu().numpy(), want)
    _, want, _, _ = orc.sample(xin, hist, steps, seeds, -1, ocfg, uniforms=u)
    assert np.array_equal(ths.sample(x, hd, sd, td, cfg, uniform_values=torch.from_numpy(u).to(DEV)).cpu().numpy(),
                          want)
    # temperature 0 with penalties: the first index of the penalised row's maximum
    g0 = ths.ThinkerSampling(temperature=0.0, repetition_penalty=1.3, presence_penalty=0.2, window=W)
    ocfg0 = orc.Cfg(temperature=1.0, top_p=1.0, top_k=1, repetition_penalty=1.3, window=W, min_new_tokens=0,
                    max_new_tokens=1 << 40, min_keep=1, semantics="omni", presence_penalty=0.2)
    want_p, want, _, _ = orc.sample(xin, hist, steps, seeds, -1, ocfg0, uniforms=np.zeros(B, np.float32))
    got = ths.sample(x, hd, sd, td, g0).cpu().numpy()
    assert np.array_equal(got, want)
    pen = orc.sample(xin, hist, steps, seeds, -1, orc.Cfg(**{**ocfg0.__dict__, "top_k": I.THINKER_V if kind ==
                     "thinker" else I.TALKER_V, "top_p": 1.0}), uniforms=np.zeros(B, np.float32))[0]
    assert np.array_equal(got, pen.argmax(axis=1))
    # temperature 0 without penalties: the plain argmax (first index on ties)
    plain = ths.sample(x, hd, sd, td, ths.ThinkerSampling(temperature=0.0, repetition_penalty=1.0, window=W))
    assert np.array_equal(plain.cpu().numpy(), orc.argmax(xin))


def test_per_row_top_k_above_the_scalar(pkg):
    """RowParams.top_k with rows above cfg.top_k (bound given by max_top_k): the oracle's tokens, no PAD."""
    ts = pkg.talker_sampler
    B = 9
    logits, x, hist = _rows("thinker", B, 88)
    xin = I.to_bf16_bits(logits)
    rk = np.array([1, 5, 20, 40, 64, 100, 128, 3, 77], np.int32)
    steps = np.full(B, 2, np.int64)
    u = I.rng(4).random(B, dtype=np.float32)
    ocfg = orc.Cfg(temperature=1.2, top_p=0.97, top_k=20, repetition_penalty=1.05, window=hist.shape[1],
                   min_new_tokens=0, max_new_tokens=1 << 40, min_keep=1, semantics="omni")
    want_p, want, _, _ = orc.sample(xin, hist, steps, None, -1, ocfg, uniforms=u, row_top_k=rk)
    cfg = ts.TalkerSampling(temperature=1.2, top_p=0.97, top_k=20, repetition_penalty=1.05, window=hist.shape[1],
                            min_new_tokens=0, max_new_tokens=1 << 40, min_keep=1, semantics="omni")
    rp = ts.RowParams(top_k=torch.from_numpy(rk).to(DEV), max_top_k=int(rk.max()))
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    hd = torch.from_numpy(hist).to(DEV)
    got = ts.sample(x, hd, torch.from_numpy(steps).to(DEV), None, -1, cfg, uniform_values=torch.from_numpy(u).to(DEV),
                    row_params=rp, status=status)
    assert int(status.item()) == 0
    assert np.array_equal(got.cpu().numpy(), want)
    proc = ts.processed_logits(x, hd, torch.from_numpy(steps).to(DEV), -1, cfg, row_params=rp)
    assert len(H.compare_processed(want_p, proc.cpu().numpy())) == 0


def test_draw_multinomial_on_cuda_generators(pkg):
    """draw_multinomial on CUDA generators == the reference's per-row formula (softmax, then one
    torch.multinomial per row with that row's generator) on generators cloned from the same seeds."""
    ts = pkg.talker_sampler
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(5, I.TALKER_V, device=DEV, generator=g) * 2.0
    ga = [torch.Generator(device=DEV).manual_seed(1000 + r) for r in range(5)]
    gb = [torch.Generator(device=DEV).manual_seed(1000 + r) for r in range(5)]
    for _ in range(3):
        got = ts.draw_multinomial(x, ga)
        probs = torch.softmax(x, dim=-1)
        want = torch.stack([torch.multinomial(probs[i], 1, generator=gb[i]).reshape(()) for i in range(5)])
        assert torch.equal(got, want)
    # and inside step() with the native RNG (omni + auto): PAD for inactive rows, state advanced for live ones
    cfg = ts.TalkerSampling(semantics="omni", rng="auto", min_new_tokens=0, window=8)
    st = ts.DecodeState.new([1, 2, 3, 4, 5], cfg, device=DEV)
    st.active[2] = False
    st.generators = [torch.Generator(device=DEV).manual_seed(7 + r) for r in range(5)]
    tok = ts.step(st, x, I.TALKER_EOS, cfg)
    assert tok[2].item() == ts.PAD and (tok[[0, 1, 3, 4]] >= 0).all()
    assert st.steps.tolist() == [1, 1, 0, 1, 1] and st.history[:, -1].tolist() == tok.tolist()


@pytest.mark.parametrize("sem", ["hf", "omni"])
def test_graph_replay_matches_eager(pkg, sem):
    """step_ captured in a CUDA graph and replayed frame by frame == eager step() on a copy of the state:
    the same tokens, history, steps and finished flags (the form the reference's graph bodies use,
    engine/runtime/talker_decode.py:120-128)."""
    ts = pkg.talker_sampler
    cfg = ts.TalkerSampling(semantics=sem, rng="counter", min_new_tokens=4, max_new_tokens=14, window=16)
    B, V, F = 6, I.TALKER_V, 18
    g = torch.Generator(device=DEV).manual_seed(5)
    frames = torch.randn(F, B, V, device=DEV, generator=g) * 2.0
    frames[9, 1, I.TALKER_EOS] = 40.0  # row 1 ends early
    eager = ts.DecodeState.new([11, 12, 13, 14, 15, 16], cfg, device=DEV)
    eager.active[3] = False
    graphed = ts.DecodeState.new([11, 12, 13, 14, 15, 16], cfg, device=DEV)
    graphed.active[3] = False
    static_x = frames[0].clone()
    ts.step_(graphed, static_x, I.TALKER_EOS, cfg)  # builds the penalty table before capture
    graphed = ts.DecodeState.new([11, 12, 13, 14, 15, 16], cfg, device=DEV)
    graphed.active[3] = False
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=DEV)
    with torch.cuda.graph(gr, stream=s, capture_error_mode="thread_local"):
        static_tok = ts.step_(graphed, static_x, I.TALKER_EOS, cfg)
    for f in range(F):
        static_x.copy_(frames[f])
        gr.replay()
        want = ts.step(eager, frames[f], I.TALKER_EOS, cfg)
        assert torch.equal(static_tok, want), f
        assert torch.equal(graphed.history, eager.history) and torch.equal(graphed.steps, eager.steps)
        assert torch.equal(graphed.finished, eager.finished)
    assert bool(eager.finished[1]) and int(eager.steps[3]) == 0
    del gr


@pytest.mark.parametrize("sem", ["hf", "omni"])
def test_k_frame_block_matches_step_loop(pkg, sem):
    """decode_k (one launch for K frames) and decode_k_ (in place) == K calls of step on a copy of the state: the
    same [K, B] tokens and final history / steps / finished, through frame 0 (hf: unfiltered), EOS masking and
    forcing, a row that draws EOS early and freezes, and an inactive row."""
    ts = pkg.talker_sampler
    cfg = ts.TalkerSampling(semantics=sem, rng="counter", min_new_tokens=3, max_new_tokens=20, window=16)
    B, V, K = 7, I.TALKER_V, 24
    g = torch.Generator(device=DEV).manual_seed(31)
    frames = torch.randn(K, B, V, device=DEV, generator=g) * 2.0
    frames[6:, 2, I.TALKER_EOS] = 40.0  # row 2 draws EOS once it is allowed
    for dt in (torch.float32, torch.bfloat16):
        x = frames.to(dt)
        a = ts.DecodeState.new([3, 4, 5, 6, 7, 8, 9], cfg, device=DEV)
        a.active[5] = False
        b = ts.DecodeState.new([3, 4, 5, 6, 7, 8, 9], cfg, device=DEV)
        b.active[5] = False
        c = ts.DecodeState.new([3, 4, 5, 6, 7, 8, 9], cfg, device=DEV)
        c.active[5] = False
        hist_c = c.history
        want = torch.stack([ts.step(a, x[f], I.TALKER_EOS, cfg) for f in range(K)])
        got = ts.decode_k(b, x, I.TALKER_EOS, cfg)
        got_ = ts.decode_k_(c, x, I.TALKER_EOS, cfg)
        for t, st in ((got, b), (got_, c)):
            assert torch.equal(t, want), (dt, t, want)
            assert torch.equal(st.history, a.history) and torch.equal(st.steps, a.steps)
            assert torch.equal(st.finished, a.finished)
        assert c.history is hist_c  # advanced in place
        assert bool(a.finished[2]) and int(a.steps[5]) == 0 and (want[:, 5] == ts.PAD).all()


def _expf_spec(pkg, x: torch.Tensor):
    N = pkg._native
    y, y2 = torch.empty_like(x), torch.empty_like(x)
    N.check(N.capi().b2s_expf_spec(x.data_ptr(), x.numel(), y.data_ptr(), y2.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream), "b2s_expf_spec")
    return y, y2


def test_device_exp_is_the_oracle_exp(pkg):
    """The kernels' fp32 exp (b2s_expf) equals the oracle's restatement bit for bit on a dense sweep of its whole
    range and the special values; the paired form of the normaliser equals it on every argument <= 0."""
    special = np.array([-0.0, 0.0, -np.inf, np.inf, np.nan, -1e-45, -1e-38, -87.33654, -87.33655, -87.3366,
                        -103.97208, -103.97209, -104.0, -150.0, 88.72283, 88.72284, 1e-30], np.float32)
    x = np.concatenate([np.linspace(-110.0, 90.0, 4_000_001, dtype=np.float32), special])
    y, y2 = _expf_spec(pkg, torch.from_numpy(x).to(DEV))
    want = orc.expf(x)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert np.array_equal(y2.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_paired_exp_equals_scalar_exp_exhaustively(pkg):
    """Every fp32 value in [-110, -0] (1.1e9 bit patterns, in chunks): the paired non-positive form == the scalar."""
    lo = 0x80000000  # -0.0; bit patterns grow toward -110 (0xC2DC0000)
    hi = int(np.array([-110.0], np.float32).view(np.uint32)[0])
    chunk = 1 << 26
    for start in range(lo, hi + 1, chunk):
        n = min(chunk, hi + 1 - start)
        bits = torch.arange(start - (1 << 32), start - (1 << 32) + n, dtype=torch.int64, device=DEV).to(torch.int32)
        y, y2 = _expf_spec(pkg, bits.view(torch.float32))
        assert torch.equal(y.view(torch.int32), y2.view(torch.int32)), hex(start)


def test_resident_history_edges_match_oracle(pkg):
    """Thinker-shaped omni rows on the row-resident kernel (its omni instantiation keeps the owned history ids in
    a hash table): the EOS id is every row's largest logit and repeats in some histories, censored on the rows
    before min_new and live on the others; top ids repeat up to five times, PAD entries are mixed in.  Tokens of
    the launcher's choice (two CTAs per row), of four and eight CTAs per row, and of the forced full-row path
    (which rebuilds the ranked structures) equal the oracle's."""
    ts = pkg.talker_sampler
    B = 6
    logits, _, hist = _rows("thinker", B, 77)
    eos = 4321
    logits[:, eos] = logits.max(axis=1) + 1.0
    logits = I.bf16_bits_to_f32(I.to_bf16_bits(logits))
    x = _bf16(logits)
    hist[0, 200:203] = eos
    hist[2, 100] = eos
    hist[4, 50:58] = eos
    steps = np.array([2, 9, 2, 9, 0, 20], np.int64)
    seeds = np.arange(B, dtype=np.int64) * 31 + 7
    u = I.rng(12).random(B, dtype=np.float32)
    ocfg = orc.Cfg(temperature=0.8, top_p=0.85, top_k=24, repetition_penalty=1.2, window=hist.shape[1],
                   min_new_tokens=8, max_new_tokens=1 << 40, min_keep=1, semantics="omni")
    _, want, _, _ = orc.sample(I.to_bf16_bits(logits), hist, steps, seeds, eos, ocfg, uniforms=u)
    tcfg = ts.TalkerSampling(temperature=0.8, top_p=0.85, top_k=24, repetition_penalty=1.2, window=hist.shape[1],
                             min_new_tokens=8, max_new_tokens=1 << 40, min_keep=1, semantics="omni")
    hd = torch.from_numpy(hist).to(DEV)
    kw = ts._cfg_kwargs(tcfg, hd, DEV)
    runs = [(0, 0), (4, 0), (8, 0), (2, ts.FLAG_FORCE_EXACT)]
    for cluster, flags in runs:
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        tok, _, _, _, _ = ts._run(x, history=hd, steps=torch.from_numpy(steps).to(DEV),
                                  uniform_values=torch.from_numpy(u).to(DEV), eos=eos, rng=ts.RNG_UNIFORM,
                                  status=status, flags=flags, cluster=cluster, tokens=True, processed=False, **kw)
        assert np.array_equal(tok.cpu().numpy(), want), (cluster, flags, tok.cpu().numpy(), want)
        assert int(status.item()) == 0
    assert want[0] != eos and want[2] != eos and want[4] != eos  # censored rows never draw the EOS
