"""Host-side pieces of the drop-in module that need no GPU: argument checks of the per-row parameter form, and
the native-RNG block (``draw_multinomial`` + ``restore_multinomial_states_after_block``), which the engine
keeps as the reference's per-row torch calls (``engine/talker_sampler.py:175-212``) and which therefore runs
on CPU tensors and CPU generators as well."""

import numpy as np
import pytest
import torch

from tests.golden import make_golden


def test_row_top_k_requires_a_host_bound(pkg):
    """A per-row top_k tensor without RowParams.max_top_k is refused before any launch (rows above a
    guessed bound would otherwise come back as PAD with only a status bit)."""
    ts = pkg.talker_sampler
    cfg = ts.TalkerSampling(semantics="omni", top_k=20)
    rp = ts.RowParams(top_k=torch.tensor([5, 40], dtype=torch.int32))
    with pytest.raises(ValueError, match="max_top_k"):
        ts._cfg_kwargs(cfg, None, "cpu", rp)
    kw = ts._cfg_kwargs(cfg, None, "cpu", ts.RowParams(top_k=torch.tensor([5, 40], dtype=torch.int32), max_top_k=40))
    assert kw["max_top_k"] == 40
    # the scalar form and per-row temperatures alone need no bound
    assert ts._cfg_kwargs(cfg, None, "cpu", ts.RowParams(temperature=torch.ones(2)))["max_top_k"] == 20


def test_multinomial_block_matches_reference(pkg):
    """The reference's native-RNG block replayed through this module on CPU generators: the same K draws,
    and after the rewind to each row's last non-PAD draw, the same next draw (fixture made by running the
    reference, ``tests/golden/make_golden.py multinomial``)."""
    fx = np.load(make_golden.HERE / "multinomial.npz")
    got = make_golden.multinomial_scenario(pkg.talker_sampler)
    for k in ("block_tokens", "host_tokens", "after_restore"):
        assert np.array_equal(got[k], fx[k]), k


def test_restore_rewinds_to_last_draw_before_pad(pkg):
    """restore_multinomial_states_after_block on its own: a row whose first PAD is at block position d
    (0 < d < K) continues from its state after draw d - 1; rows with no PAD or a PAD at 0 keep their
    generator as it is; an empty state list is a no-op; a generator count that differs is an error."""
    ts = pkg.talker_sampler
    K, B = 5, 4
    gens = [torch.Generator().manual_seed(7 + r) for r in range(B)]
    states = []
    for _ in range(K):
        for gen in gens:
            torch.rand(3, generator=gen)
        states.append([gen.get_state() for gen in gens])
    end = [gen.get_state() for gen in gens]
    host = torch.zeros(K, B, dtype=torch.int64)
    host[2:, 1] = ts.PAD  # first PAD at 2 -> state after draw 1
    host[0:, 2] = ts.PAD  # PAD at 0 -> untouched
    host[4, 3] = ts.PAD   # PAD at 4 -> state after draw 3
    ts.restore_multinomial_states_after_block(gens, states, host)
    assert torch.equal(gens[0].get_state(), end[0])
    assert torch.equal(gens[1].get_state(), states[1][1])
    assert torch.equal(gens[2].get_state(), end[2])
    assert torch.equal(gens[3].get_state(), states[3][3])
    ts.restore_multinomial_states_after_block(gens, [], host)
    with pytest.raises(ValueError):
        ts.restore_multinomial_states_after_block(gens[:3], states, host)
    with pytest.raises(ValueError):
        ts.draw_multinomial(torch.zeros(3, 10), gens)


def test_request_seed_matches_reference(pkg):
    """Request seeds (explicit seed to 63 bits, else SHA-256 of the request id) == the reference's
    ``request_seed`` on the same requests (fixture made by running it, ``make_golden.py request_seed``)."""
    from types import SimpleNamespace

    fx = np.load(make_golden.HERE / "request_seed.npz")
    sd = pkg.seeds
    got = [sd.request_seed(SimpleNamespace(request_id=str(i), seed=None)) for i in fx["ids"]]
    assert got == [int(x) for x in fx["by_id"]]
    got = [sd.seed_of("r", int(e)) for e in fx["explicit"]]
    assert got == [int(x) for x in fx["by_seed"]]
    t = sd.request_seeds([SimpleNamespace(request_id="a", seed=None), SimpleNamespace(request_id="b", seed=9)])
    assert t.dtype == torch.int64 and t.tolist() == [sd.seed_of("a"), 9]
