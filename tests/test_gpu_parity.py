"""CUDA path against the CPU oracle and the reference's golden outputs (B200 only).

Parity bar: processed logits bit-identical (finite values and -inf pattern); kept set and token ids
identical -- no boundary exceptions against the oracle, which evaluates the same numerics spec.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests import _harness as H
from tests.golden import cases as C
from tests.golden import inputs as I

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GROUPS = {"talker": C.talker_cases, "thinker": C.thinker_cases, "edge": C.edge_cases}


def _cases():
    for group, make in GROUPS.items():
        for case in make():
            yield pytest.param(group, case, id=case.name)


def gpu_logits(case):
    if case.dtype == "bf16":
        return torch.from_numpy(case.bf16_bits().view(np.int16)).view(torch.bfloat16).to(DEV)
    return torch.from_numpy(case.logits).to(DEV)


def cfg_of(ts, case):
    c = case.cfgs[0]
    return ts.TalkerSampling(**{k: v for k, v in c.items() if k in ts.TalkerSampling.__dataclass_fields__})


def row_params(ts, case):
    if case.uniform_cfg():
        return None
    cs = case.cfgs
    return ts.RowParams(temperature=torch.tensor([c["temperature"] for c in cs], dtype=torch.float32, device=DEV),
                        top_p=torch.tensor([c["top_p"] for c in cs], dtype=torch.float32, device=DEV),
                        top_k=torch.tensor([c["top_k"] for c in cs], dtype=torch.int32, device=DEV),
                        repetition_penalty=[c["repetition_penalty"] for c in cs],
                        max_top_k=max(c["top_k"] for c in cs))


def run_gpu(ts, case, *, counter=False, exact=False, cluster=0, processed=True, flags=0):
    x = gpu_logits(case)
    hist = torch.from_numpy(case.history).to(DEV)
    steps = torch.from_numpy(case.steps).to(DEV)
    seeds = torch.from_numpy(case.seeds).to(DEV)
    u = None if counter else torch.from_numpy(case.uniforms).to(DEV)
    kw = ts._cfg_kwargs(cfg_of(ts, case), hist, DEV, row_params(ts, case))
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    tok, proc, _, _, _ = ts._run(x, history=hist, steps=steps, seeds=seeds, uniform_values=u, eos=case.eos,
                                 rng=ts.RNG_COUNTER if counter else ts.RNG_UNIFORM, status=status,
                                 flags=flags | (ts.FLAG_FORCE_EXACT if exact else 0), cluster=cluster, tokens=True,
                                 processed=processed, **kw)
    return (proc.cpu().numpy() if processed else None), tok.cpu().numpy(), int(status.item())


@pytest.mark.parametrize("group,case", list(_cases()))
def test_sample_matches_oracle_and_reference(pkg, group, case):
    ts = pkg.talker_sampler
    fx = H.fixture(group)
    assert str(fx[f"{case.name}.digest"]) == case.digest()
    want_p, want_t, meta, _ = H.run_oracle(case)
    got_p, got_t, status = run_gpu(ts, case)
    assert status == 0
    assert len(H.compare_processed(want_p, got_p)) == 0
    assert np.array_equal(got_t, want_t), (got_t, want_t, meta)
    # and the reference's own outputs (identical on every fixture so far)
    assert len(H.compare_processed(fx[f"{case.name}.processed"], got_p)) == 0
    mism = np.nonzero(fx[f"{case.name}.tok_u"] != got_t)[0]
    assert all(H.boundary_rows(meta)[r] for r in mism)
    # counter RNG (the reference's uniform(seed, step))
    _, got_c, _ = run_gpu(ts, case, counter=True, processed=False)
    assert np.array_equal(got_c, fx[f"{case.name}.tok_c"])


@pytest.mark.parametrize("group,case", [p for p in _cases() if p.values[1].name in (
    "hf_t5", "hf_t60", "omni_t7", "cfg2_talker_batched", "cfg3_thinker", "cfg4_large", "cfg5_ties",
    "edge_quantised_hf", "edge_quantised_omni", "edge_temperature_3.0_omni", "edge_penalty_big_hf",
    "edge_min_new_boundary_hf", "edge_bf16_hf", "edge_small_vocab_omni")])
def test_every_kernel_path_agrees(pkg, group, case):
    """The streaming kernel (candidate path and forced exact path, with and without processed output), the
    launcher's own pick for a decode step (the short-row kernel for rows it holds in registers), and the
    row-resident kernel at every cluster size it accepts for the case (1, 2, 4 or 8 CTAs per row; candidate
    and forced exact path) give the oracle's bits."""
    ts = pkg.talker_sampler
    want_p, want_t, _, _ = H.run_oracle(case)
    for exact in (False, True):
        got_p, got_t, _ = run_gpu(ts, case, exact=exact)
        assert len(H.compare_processed(want_p, got_p)) == 0, exact
        assert np.array_equal(got_t, want_t), (exact, got_t, want_t)
        _, got_t, _ = run_gpu(ts, case, exact=exact, processed=False, flags=ts.FLAG_STREAM)
        assert np.array_equal(got_t, want_t), ("stream", exact, got_t, want_t)
        _, got_t, _ = run_gpu(ts, case, exact=exact, processed=False)
        assert np.array_equal(got_t, want_t), ("auto", exact, got_t, want_t)
    ran = []
    k = max(max(c["top_k"] for c in case.cfgs), 1)
    for cluster in (1, 2, 4, 8):
        for exact in (False, True):
            try:
                _, got_t, _ = run_gpu(ts, case, exact=exact, processed=False, cluster=cluster)
            except RuntimeError as e:
                # the launcher refuses: hf with more than one CTA per row, top_k beyond the list stage, a slice
                # too large for one CTA's shared memory
                assert "unsupported" in str(e), e
                row_bytes = case.vocab * (2 if case.dtype == "bf16" else 4)
                must_run = k <= 128 and ((cluster == 1 and row_bytes <= 64 * 1024) or (
                    cluster == 2 and case.cfgs[0]["semantics"] == "omni" and row_bytes <= 320 * 1024))
                assert not must_run, (cluster, e)
                continue
            assert np.array_equal(got_t, want_t), ("resident", cluster, exact, got_t, want_t)
            ran.append(cluster)
    assert ran or k > 128


@pytest.mark.parametrize("group,case", list(_cases()))
def test_decode_step_matches_oracle(pkg, group, case):
    """The launcher's pick for a decode step (tokens only: the short-row kernel on Talker rows, the row-resident
    kernel on Thinker rows) against the oracle, with injected uniforms and with the Philox RNG."""
    ts = pkg.talker_sampler
    _, want_t, _, _ = H.run_oracle(case)
    _, got_t, status = run_gpu(ts, case, processed=False)
    assert np.array_equal(got_t, want_t), (got_t, want_t)
    assert status == 0


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type.name == "CUDA"}


def test_short_rows_take_the_short_kernel(pkg):
    """Talker-shaped decode steps (fp32 and bf16, hf and omni) launch the short-row kernel; Thinker rows the
    row-resident kernel; a cluster size asks for the row-resident kernel."""
    ts = pkg.talker_sampler
    case = C.talker_batched_cfg2()
    names = _kernel_names(lambda: run_gpu(ts, case, processed=False))
    if not names:
        pytest.skip("the profiler recorded no CUDA kernels here")
    assert any("short_kernel" in n for n in names), names
    assert any("short_kernel" in n for n in _kernel_names(lambda: run_gpu(ts, C.talker_order(5, "omni"), processed=False)))
    names = _kernel_names(lambda: run_gpu(ts, case, processed=False, cluster=1))
    assert any("resident_kernel" in n for n in names) and not any("short_kernel" in n for n in names), names
    names = _kernel_names(lambda: run_gpu(ts, C.thinker_cfg3(), processed=False))
    assert any("resident_kernel" in n for n in names), names


def test_draw_matches_reference(pkg):
    ts = pkg.talker_sampler
    fx = H.fixture("talker")
    for case in C.talker_cases():
        proc = torch.from_numpy(fx[f"{case.name}.processed"]).to(DEV)
        tok = ts.draw(proc, torch.from_numpy(case.seeds).to(DEV), torch.from_numpy(case.steps).to(DEV),
                      uniform_values=torch.from_numpy(case.uniforms).to(DEV))
        want, _ = orc.draw(fx[f"{case.name}.processed"], case.uniforms)
        assert np.array_equal(tok.cpu().numpy(), want), case.name
        assert np.array_equal(tok.cpu().numpy(), fx[f"{case.name}.tok_u"]), case.name


def test_uniform_counter_and_philox(pkg):
    ts = pkg.talker_sampler
    fx = H.fixture("rng")
    seeds = torch.from_numpy(fx["seeds"]).to(DEV)
    steps = torch.arange(1024, dtype=torch.int64, device=DEV)[:, None]
    got = ts.uniform(seeds[None, :], steps).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), fx["uniform"].view(np.uint32))
    s = np.repeat(fx["seeds"], 64)
    t = np.tile(np.arange(64, dtype=np.int64), len(fx["seeds"]))
    q = np.arange(s.size, dtype=np.int64) * 3
    want = orc.uniform(s, t, rng=orc.RNG_PHILOX, requests=q)
    got = ts.philox_uniform(torch.from_numpy(s).to(DEV), torch.from_numpy(t).to(DEV), torch.from_numpy(q).to(DEV))
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_argmax_matches_reference(pkg):
    fx = H.fixture("rng")
    g = I.rng(9)
    am_f32 = I.quantised_rows(g, 6, I.THINKER_V, q=4)
    am_f32[3, 1000:1010] = am_f32[3].max() + 1.0
    bits = I.to_bf16_bits(I.quantised_rows(g, 6, I.THINKER_V, q=16))
    am = pkg.thinker_sampler.argmax
    assert np.array_equal(am(torch.from_numpy(am_f32).to(DEV)).cpu().numpy(), fx["argmax_f32"])
    x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(DEV)
    assert np.array_equal(am(x).cpu().numpy(), fx["argmax_bf16"])
    # odd vocabularies / misaligned rows / NaN
    for V in (1, 7, 6562, 151_748):
        y = torch.randn(5, V + 3, device=DEV)[:, 3:]
        assert torch.equal(am(y), y.float().argmax(-1))
        yb = y.to(torch.bfloat16)
        assert torch.equal(am(yb), yb.float().cpu().argmax(-1).to(DEV))
    z = torch.randn(2, 1000, device=DEV)
    z[1, 17] = float("nan")
    assert am(z)[1].item() == 17
    # NaN in several threads' shares, rows of -inf, signed zeros, one value everywhere: first index wins
    w = torch.randn(6, I.THINKER_V)
    w[0, [90_001, 40_000, 151_000]] = float("nan")
    w[1] = float("-inf")
    w[2] = 0.0
    w[2, ::3] = -0.0
    w[3] = 2.5
    w[4, 5000:] = 7.0
    w[5, [151_935, 70_000]] = 1e30
    for dt in (torch.float32, torch.bfloat16):
        wd = w.to(dt)
        assert torch.equal(am(wd.to(DEV)).cpu(), wd.float().argmax(-1))


def test_sequences_match_reference(pkg):
    ts = pkg.talker_sampler
    fx = H.fixture("seq")
    for name in C.SEQUENCES:
        x, cfgd, seeds, inactive = C.sequence_inputs(name)
        assert str(fx[f"{name}.digest"]) == I.digest(x)
        cfg = ts.TalkerSampling(**cfgd)
        st = ts.DecodeState.new(seeds, cfg, device=DEV)
        for r in inactive:
            st.active[r] = False
        toks = ts.decode_k(st, torch.from_numpy(x).to(DEV), I.TALKER_EOS, cfg)
        assert np.array_equal(toks.cpu().numpy(), fx[f"{name}.tokens"]), name
        assert np.array_equal(st.steps.cpu().numpy(), fx[f"{name}.steps"])
        assert np.array_equal(st.history.cpu().numpy(), fx[f"{name}.history"])
        assert np.array_equal(st.finished.cpu().numpy(), fx[f"{name}.finished"])


def _full_size(ts, kind, B, seed):
    g = I.rng(seed)
    if kind == "cfg3":
        logits, hist = I.zipf_rows(g, B, I.THINKER_V, 512)
        logits = I.bf16_bits_to_f32(I.to_bf16_bits(logits))
        cfg = dict(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.05)
        dtype = "bf16"
    elif kind == "cfg4":
        logits = (g.standard_normal((B, I.THINKER_V)) * 3).astype(np.float32)
        hist = g.integers(0, I.THINKER_V, size=(B, 2048))
        cfg = dict(temperature=1.0, top_k=50, top_p=0.95, repetition_penalty=1.1)
        dtype = "f32"
    else:
        logits = I.quantised_rows(g, B, I.THINKER_V)
        hist = np.full((B, 4), -1, np.int64)
        cfg = dict(temperature=0.8, top_k=64, top_p=0.9, repetition_penalty=1.0)
        dtype = "bf16"
    case = C.Case(kind, logits, dtype, hist, np.full(B, 11, np.int64), g.integers(0, 1 << 62, size=B, dtype=np.int64),
                  g.random(B, dtype=np.float32), -1,
                  [C._cfg(window=hist.shape[1], min_new_tokens=0, max_new_tokens=C.BIG, min_keep=1, semantics="omni",
                          **cfg)] * B)
    return case


@pytest.mark.parametrize("kind,B", [("cfg3", 64), ("cfg4", 24), ("cfg5", 64)])
def test_benchmark_shapes_match_oracle(pkg, kind, B):
    """The benchmark workloads at (or near) full size: bit-identical processed rows and tokens."""
    ts = pkg.talker_sampler
    case = _full_size(ts, kind, B, 100 + B)
    want_p, want_t, _, _ = H.run_oracle(case)
    got_p, got_t, status = run_gpu(ts, case)
    assert status == 0
    assert len(H.compare_processed(want_p, got_p)) == 0
    assert np.array_equal(got_t, want_t)
    _, got_c, _ = run_gpu(ts, case, counter=True, processed=False)
    _, want_c, _, _ = H.run_oracle(case, counter=True)
    assert np.array_equal(got_c, want_c)


@pytest.mark.parametrize("sem", ["omni", "hf"])
def test_paired_cta_rows_with_eos_rules(pkg, sem):
    """Thinker-size rows at a batch small enough for two CTAs per row (no processed output asked), with the
    EOS masked (omni: censored to -inf first; hf: dropped from the draw) and the EOS id inside several
    histories: the same tokens as the oracle, and as the one-CTA path (the launch with processed output)."""
    ts = pkg.talker_sampler
    g = I.rng(211)
    B, V, W, eos = 12, I.THINKER_V, 96, 151_000
    logits, hist = I.zipf_rows(g, B, V, W)
    logits = I.bf16_bits_to_f32(I.to_bf16_bits(logits))
    logits[::2, eos] = logits[::2].max(axis=1) + 1.0  # EOS would win if it were not masked
    hist[1::3, :5] = eos
    hist[2::5, 7] = -1
    steps = np.full(B, 3, np.int64)
    cfg = C._cfg(semantics=sem, temperature=0.9, top_k=32, top_p=0.9, repetition_penalty=1.2, window=W,
                 min_new_tokens=10, max_new_tokens=C.BIG, min_keep=1 if sem == "omni" else 3)
    case = C._case(f"paired_{sem}", logits, "bf16", hist, steps, eos, cfg, 212)
    _, want_c, _, _ = H.run_oracle(case, counter=True)
    _, got_split, st1 = run_gpu(ts, case, counter=True, processed=False)
    _, got_one, st2 = run_gpu(ts, case, counter=True, processed=True)
    assert st1 == 0 and st2 == 0
    assert np.array_equal(got_split, want_c), (got_split, want_c)
    assert np.array_equal(got_one, want_c)
    assert not np.any(got_split == eos)


def test_step_state_matches_oracle_sequence(pkg):
    """step() over 40 frames (hf, EOS rules, penalties) equals the oracle driven frame by frame."""
    ts = pkg.talker_sampler
    cfg = ts.TalkerSampling(min_new_tokens=10, max_new_tokens=30)
    B, V = 6, I.TALKER_V
    g = I.rng(77)
    st = ts.DecodeState.new([int(s) for s in g.integers(0, 1 << 62, size=B)], cfg, device=DEV)
    st.active[4] = False
    hist = np.full((B, 16), -1, np.int64)
    steps = np.zeros(B, np.int64)
    fin = np.zeros(B, bool)
    act = np.ones(B, bool)
    act[4] = False
    seeds = st.seeds.cpu().numpy()
    ocfg = orc.Cfg(min_new_tokens=10, max_new_tokens=30)
    for f in range(40):
        x = (g.standard_normal((B, V)) * 2).astype(np.float32)
        if f == 12:
            x[1, I.TALKER_EOS] = 50.0
        tok = ts.step(st, torch.from_numpy(x).to(DEV), I.TALKER_EOS, cfg).cpu().numpy()
        _, want, _, _ = orc.sample(x, hist, steps, seeds, I.TALKER_EOS, ocfg, rng=orc.RNG_COUNTER)
        live = act & ~fin
        want = np.where(live, want, -1)
        assert np.array_equal(tok, want), f
        hist = np.where(live[:, None], np.concatenate([hist[:, 1:], want[:, None]], 1), hist)
        steps = steps + live
        fin = fin | (live & (want == I.TALKER_EOS))
        assert np.array_equal(st.history.cpu().numpy(), hist)
        assert np.array_equal(st.steps.cpu().numpy(), steps)
        assert np.array_equal(st.finished.cpu().numpy(), fin)
    assert fin[1] and steps[4] == 0


def test_step_inplace_matches_step(pkg):
    ts = pkg.talker_sampler
    cfg = ts.TalkerSampling(semantics="omni", rng="counter", min_new_tokens=3)
    a = ts.DecodeState.new([5, 6, 7], cfg, device=DEV)
    b = ts.DecodeState.new([5, 6, 7], cfg, device=DEV)
    hist_view = b.history
    for f in range(12):
        x = torch.randn(3, I.TALKER_V, device=DEV) * 2
        t1 = ts.step(a, x, I.TALKER_EOS, cfg)
        t2 = ts.step_(b, x, I.TALKER_EOS, cfg)
        assert torch.equal(t1, t2)
        assert torch.equal(a.history, b.history) and torch.equal(a.steps, b.steps)
        assert torch.equal(a.finished, b.finished)
    assert b.history is hist_view  # advanced in place


def test_repetition_penalty_matches_reference_formula(pkg):
    ts = pkg.talker_sampler
    g = torch.Generator().manual_seed(5)
    x = torch.randn(5, 1000, generator=g) * 3
    hist = torch.randint(0, 40, (5, 64), generator=g)
    hist[:, ::5] = -1
    for pen in (1.05, 0.7, 3.0):
        got = ts.repetition_penalty(x.to(DEV), hist.to(DEV), pen).cpu()
        valid = hist >= 0
        freq = torch.zeros_like(x).scatter_add_(1, hist.clamp(min=0), valid.to(x.dtype))
        alpha = torch.pow(torch.full_like(x, pen), freq)
        want = torch.where(x < 0, x * alpha, x / alpha)
        assert torch.equal(got, want)
    xb = x.to(torch.bfloat16)
    got = ts.repetition_penalty(xb.to(DEV), hist.to(DEV), 1.2).cpu()
    freq = torch.zeros(5, 1000).scatter_add_(1, hist.clamp(min=0), (hist >= 0).float())
    alpha = torch.pow(torch.full((5, 1000), 1.2), freq)
    xf = xb.float()
    assert torch.equal(got, torch.where(xf < 0, xf * alpha, xf / alpha))


def test_filters_match_oracle_forms(pkg):
    ts = pkg.talker_sampler
    g = torch.Generator().manual_seed(0)
    for scale in (0.3, 1.0, 3.0, 8.0):
        x = torch.randn(64, I.TALKER_V, generator=g) * scale
        xd = x.to(DEV)
        # top_k_filter: pure selection
        kth = torch.topk(x, 25, dim=-1).values[:, -1:]
        assert torch.equal(ts.top_k_filter(xd, 25, 3).cpu(), x.masked_fill(x < kth, float("-inf")))
        # fused hf / omni filters == the oracle on T=1, no history, step 1, no EOS column
        for sem, fn in (("hf", lambda: ts.top_p_top_k_filter(xd, 0.85, 25, 3)),
                        ("omni", lambda: ts.top_k_top_p_filter(xd, 25, 0.85, 1))):
            want, _, _, _ = orc.sample(x.numpy(), np.full((64, 1), -1), np.ones(64, np.int64), None, -1,
                                       orc.Cfg(temperature=1.0, top_p=0.85, top_k=25, min_new_tokens=0,
                                               max_new_tokens=1 << 40, min_keep=3, semantics=sem),
                                       uniforms=np.zeros(64, np.float32))
            got = fn().cpu().numpy()
            assert len(H.compare_processed(want, got)) == 0, sem


def test_two_pass_top_p_filter_is_the_reference_form(pkg):
    """top_p_filter (the reference's full-sort form, talker_sampler.py:87-92) on the device == the same
    formula on CPU torch, except where a cumulative mass sits within float rounding of the cut."""
    ts = pkg.talker_sampler
    g = torch.Generator().manual_seed(19)
    for scale in (0.3, 1.0, 3.0, 8.0):
        x = torch.randn(64, I.TALKER_V, generator=g) * scale
        s, idx = torch.sort(x, descending=False, dim=-1)
        cum = s.softmax(dim=-1).cumsum(dim=-1)
        remove = cum <= (1 - 0.85)
        remove[..., -3:] = False
        want = x.masked_fill(remove.scatter(1, idx, remove), float("-inf"))
        got = ts.top_p_filter(x.to(DEV), 0.85, 3).cpu()
        # rows whose cumulative mass sits within rounding of the cut may differ by that one element
        near = ((cum - (1 - 0.85)).abs() < 1e-5).any(dim=-1)
        same = (torch.isinf(want) == torch.isinf(got)).all(dim=-1)
        assert bool((same | near).all())


@pytest.mark.parametrize("sem", ["hf", "omni"])
def test_per_row_min_max_new_tokens(pkg, sem):
    """Per-row EOS rules (RowParams.min_new_tokens / max_new_tokens) == the oracle with the same per-row
    values: rows before min_new have EOS masked, rows at max_new - 1 are forced to EOS."""
    ts = pkg.talker_sampler
    g = np.random.default_rng(21)
    B, V, W, eos = 6, I.TALKER_V, 16, I.TALKER_V - 1
    x = (g.standard_normal((B, V)) * 2.0).astype(np.float32)
    x[:, eos] = 6.0  # EOS is likely whenever it is allowed
    hist = g.integers(0, V, size=(B, W)).astype(np.int64)
    steps = np.array([0, 3, 7, 10, 2040, 2046], np.int64)
    rmin = np.array([8, 2, 8, 50, 0, 0], np.int64)
    rmax = np.array([2048, 2048, 8, 12, 2048, 2047], np.int64)
    u = g.random(B).astype(np.float32)
    cfg = ts.TalkerSampling(semantics=sem, rng="counter", min_new_tokens=1, max_new_tokens=4096)
    want_p, want_t, _, _ = orc.sample(x, hist, steps, np.arange(B), eos,
                                      orc.Cfg(temperature=cfg.temperature, top_p=cfg.top_p, top_k=cfg.top_k,
                                              repetition_penalty=cfg.repetition_penalty, window=W,
                                              min_new_tokens=1, max_new_tokens=4096, min_keep=cfg.min_keep,
                                              semantics=sem),
                                      uniforms=u, row_min_new=rmin, row_max_new=rmax)
    rp = ts.RowParams(min_new_tokens=torch.from_numpy(rmin).to(DEV), max_new_tokens=torch.from_numpy(rmax).to(DEV))
    kw = ts._cfg_kwargs(cfg, torch.from_numpy(hist).to(DEV), DEV, rp)
    got_t, got_p = ts._run(torch.from_numpy(x).to(DEV), history=torch.from_numpy(hist).to(DEV),
                           steps=torch.from_numpy(steps).to(DEV), uniform_values=torch.from_numpy(u).to(DEV),
                           eos=eos, rng=ts.RNG_UNIFORM, processed=True, **kw)[:2]
    assert np.array_equal(got_t.cpu().numpy(), want_t)
    assert len(H.compare_processed(want_p, got_p.cpu().numpy())) == 0
    # the rules did apply: rows 2, 5 are forced to EOS, rows 0, 3 have EOS masked
    assert want_t[2] == eos and want_t[5] == eos and want_t[0] != eos and want_t[3] != eos


@pytest.mark.parametrize("sem", ["hf", "omni"])
def test_short_rows_head_and_tail_elements(pkg, sem):
    """Rows of 9..40 bf16 elements stored back to back, so that they start at every 2-byte offset: rows
    with no 16-byte interior vector at all, and rows with a ragged head and tail around one or two."""
    ts = pkg.talker_sampler
    g = I.rng(77)
    for V in (9, 13, 15, 20, 33, 40):
        for top_k in (1, 3):
            B = 16
            logits = (g.standard_normal((B, V)) * 2).astype(np.float32)
            hist = g.integers(0, V, size=(B, 6))
            cfg = C._cfg(semantics=sem, top_k=top_k, top_p=0.9, window=6, min_new_tokens=0, min_keep=1)
            case = C._case(f"short_{V}_{top_k}", logits, "bf16", hist, np.full(B, 3), -1, cfg, 90 + V)
            want_p, want_t, _, _ = H.run_oracle(case)
            got_p, got_t, status = run_gpu(ts, case)
            assert status == 0
            assert len(H.compare_processed(want_p, got_p)) == 0, (V, top_k)
            assert np.array_equal(got_t, want_t), (V, top_k, got_t, want_t)


def test_status_flags_and_pad_rows(pkg):
    ts = pkg.talker_sampler
    cfg = ts.TalkerSampling(semantics="omni", rng="counter", min_new_tokens=0)
    x = torch.randn(4, 100, device=DEV)
    hist = torch.tensor([[1, 2, 3, 500]] * 4, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    tok = ts.sample(x, hist, torch.ones(4, dtype=torch.int64, device=DEV), torch.arange(4, device=DEV), 99, cfg,
                    active=torch.tensor([True, False, True, True], device=DEV), status=status)
    assert int(status.item()) & 1  # B2S_STATUS_HISTORY_RANGE
    assert tok[1].item() == -1 and (tok[[0, 2, 3]] >= 0).all()
    with pytest.raises(ValueError):
        ts.sample(x.cpu(), hist.cpu(), torch.ones(4, dtype=torch.int64), torch.arange(4), 99, cfg)
    with pytest.raises(ValueError):
        ts.processed_logits(x, hist, torch.ones(4, dtype=torch.int64, device=DEV), 99,
                            ts.TalkerSampling(semantics="bogus"))
    with pytest.raises(ValueError):
        ts.processed_logits(x, hist, torch.ones(4, dtype=torch.int64, device=DEV), 99,
                            ts.TalkerSampling(temperature=0.0))


@pytest.mark.parametrize("rng", ["uniform", "philox"])
def test_shard_candidates_merge_equal_unsharded(pkg, rng):
    """Vocabulary-sharded sampling on one GPU (8 shards run one after the other: stage 1 per shard, the merge, the
    resolve per shard, the max over shards) == the unsharded kernel, with lists capped at k: the tie-heavy rows
    leave ties unsent, and rows whose draw falls among them are finished by their shard (stage 3)."""
    vs = pkg.vocab_shard
    ts = pkg.talker_sampler
    pending_seen = 0
    for kind, B in (("cfg5", 64), ("cfg3", 16), ("cfg4", 8)):
        case = _full_size(ts, kind, B, 7 + B)
        if kind == "cfg5":
            # rows whose largest values are one block of ties inside one shard: more of them than a shard sends, all
            # kept, so the draw falls among unsent ties -- stage 3 finishes those rows
            g = I.rng(55)
            Vs = I.THINKER_V // 8
            for r in range(0, B, 3):
                s = int(g.integers(0, 8))
                n_tie = int(g.integers(80, 400))
                case.logits[r, s * Vs + g.choice(Vs, n_tie, replace=False)] = 12.0
        x = gpu_logits(case)
        hist = torch.from_numpy(case.history).to(DEV)
        steps = torch.from_numpy(case.steps).to(DEV)
        seeds = torch.from_numpy(case.seeds).to(DEV)
        u = torch.from_numpy(case.uniforms).to(DEV)
        cfg = cfg_of(ts, case)
        uv = u if rng == "uniform" else None
        want = ts.sample(x, hist, steps, seeds, -1, cfg, uniform_values=uv, rng="philox").cpu().numpy()
        if rng == "uniform":
            _, want_o, _, _ = H.run_oracle(case)
            assert np.array_equal(want, want_o)
        shards = 8
        Vs = I.THINKER_V // shards
        xs = [x[:, s * Vs:(s + 1) * Vs].contiguous() for s in range(shards)]
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        cand = [vs.shard_candidates(xs[s], s * Vs, hist, steps, cfg, status=status) for s in range(shards)]
        assert cand[0][0].shape[1] == max(cfg.top_k, 1)  # cap = k
        tok, pend = vs.merge([c[0] for c in cand], [c[1] for c in cand], [c[2] for c in cand], I.THINKER_V, steps,
                             seeds, cfg, uniform_values=uv, rng="philox", status=status)
        pending_seen += int((tok == -2).sum())
        got = vs.merge_candidates([c[0] for c in cand], [c[1] for c in cand], [c[2] for c in cand], I.THINKER_V,
                                  steps, seeds, cfg, shard_logits=xs, offsets=[s * Vs for s in range(shards)],
                                  history=hist, uniform_values=uv, rng="philox", status=status).cpu().numpy()
        assert int(status.item()) == 0
        assert np.array_equal(got, want), (kind, got, want)
    assert pending_seen > 0  # some draws fell among unsent ties and were resolved by their shard


@pytest.mark.parametrize("sem", ["omni", "hf"])
def test_flat_and_tied_thinker_rows(pkg, sem):
    """Thinker-size rows where most (chunk, thread) shares clear the first threshold: a flat row, a row whose
    upper half ties at its maximum, and a plain row beside them.  A warp then holds more hit shares than its
    pass-2 list has room for, and the row must finish on the full-row path with the oracle's bits, with and
    without the processed-logits output."""
    ts = pkg.talker_sampler
    g = I.rng(123)
    V, B = 151_936, 4
    logits = np.zeros((B, V), np.float32)
    logits[1] = np.where(g.random(V) < 0.5, 1.0, np.round(g.standard_normal(V) * 16) / 16 - 2.0)
    logits[2] = np.round(g.standard_normal(V) * 4) / 4
    logits[3] = g.standard_normal(V) * 2
    hist = g.integers(0, V, size=(B, 64))
    cfg = C._cfg(semantics=sem, top_k=20, top_p=0.8, window=64, min_new_tokens=0, min_keep=1)
    case = C._case(f"flat_{sem}", logits, "bf16", hist, np.full(B, 5), -1, cfg, 321)
    want_p, want_t, _, _ = H.run_oracle(case)
    got_p, got_t, status = run_gpu(ts, case)
    assert status == 0
    assert len(H.compare_processed(want_p, got_p)) == 0
    assert np.array_equal(got_t, want_t), (got_t, want_t)
    _, got_lean, status = run_gpu(ts, case, processed=False)
    assert status == 0
    assert np.array_equal(got_lean, want_t), (got_lean, want_t)
