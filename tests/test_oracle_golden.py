"""The CPU oracle against the reference's own outputs (golden fixtures made by tests/golden/make_golden.py)
and against published known-answer vectors.  CPU only."""

import numpy as np
import pytest

from oracle import oracle as orc
from tests import _harness as H
from tests.golden import cases as C
from tests.golden import inputs as I

GROUPS = {"talker": C.talker_cases, "thinker": C.thinker_cases, "edge": C.edge_cases}


def _cases():
    for group, make in GROUPS.items():
        for case in make():
            yield pytest.param(group, case, id=case.name)


@pytest.mark.parametrize("group,case", list(_cases()))
def test_oracle_matches_reference(group, case):
    fx = H.fixture(group)
    assert str(fx[f"{case.name}.digest"]) == case.digest(), "regenerated inputs differ from the fixture's"
    proc, tok_u, meta, bad = H.run_oracle(case)
    assert not bad
    bad_rows = H.compare_processed(fx[f"{case.name}.processed"], proc)
    # a processed-row difference is only acceptable as a top-p boundary case
    assert all(meta["topp_margin"][r] < H.TOPP_TOL for r in bad_rows), (bad_rows, meta[bad_rows])
    mism = np.nonzero(fx[f"{case.name}.tok_u"] != tok_u)[0]
    assert all(H.boundary_rows(meta)[r] for r in mism), (mism, meta[mism])
    assert len(bad_rows) == 0 and len(mism) == 0  # none observed on these fixtures
    _, tok_c, meta_c, _ = H.run_oracle(case, counter=True)
    mism_c = np.nonzero(fx[f"{case.name}.tok_c"] != tok_c)[0]
    assert len(mism_c) == 0, (mism_c, meta_c[mism_c])


def test_counter_uniform_matches_reference():
    fx = H.fixture("rng")
    seeds = fx["seeds"]
    steps = np.arange(1024, dtype=np.int64)
    got = orc.uniform(np.tile(seeds, 1024), np.repeat(steps, len(seeds))).reshape(1024, len(seeds))
    assert np.array_equal(got.view(np.uint32), fx["uniform"].view(np.uint32))


def test_philox_known_answers():
    """Random123 known-answer vectors for Philox4x32-10 (counter, key -> output)."""
    kat = [
        ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
        ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
        ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
         [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
    ]
    for ctr, key, want in kat:
        assert orc.philox4x32_10(ctr, key).tolist() == want


def test_philox_uniform_stats():
    u = orc.uniform(np.zeros(200_000, np.int64), np.arange(200_000), rng=orc.RNG_PHILOX,
                    requests=np.arange(200_000) % 7)
    assert u.min() >= 0 and u.max() < 1 and abs(u.mean() - 0.5) < 0.005
    assert len(np.unique(u)) > 190_000


def test_expf_accuracy():
    x = np.linspace(-104, 88.72, 3_000_001, dtype=np.float32)
    e = orc.expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    normal = ref > 1.2e-38
    ulp = np.spacing(ref[normal].astype(np.float32)).astype(np.float64)
    assert (np.abs(e[normal] - ref[normal]) / ulp).max() < 1.0
    assert np.isinf(orc.expf(np.array([89.0], np.float32)))[0]
    assert orc.expf(np.array([-200.0, -np.inf], np.float32)).tolist() == [0.0, 0.0]
    assert np.isnan(orc.expf(np.array([np.nan], np.float32)))[0]


def test_argmax_matches_reference():
    fx = H.fixture("rng")
    g = I.rng(9)
    am_f32 = I.quantised_rows(g, 6, I.THINKER_V, q=4)
    am_f32[3, 1000:1010] = am_f32[3].max() + 1.0
    bits = I.to_bf16_bits(I.quantised_rows(g, 6, I.THINKER_V, q=16))
    assert str(fx["argmax_f32_digest"]) == I.digest(am_f32)
    assert str(fx["argmax_bf16_digest"]) == I.digest(bits)
    assert np.array_equal(orc.argmax(am_f32), fx["argmax_f32"])
    assert orc.argmax(am_f32)[3] == 1000
    assert np.array_equal(orc.argmax(bits), fx["argmax_bf16"])


def test_bf16_rounding_matches_torch():
    import torch

    x = (np.random.default_rng(0).standard_normal(100_000) * 50).astype(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(I.to_bf16_bits(x), want)


def test_history_out_of_range_is_flagged():
    case = C.talker_order(5)
    hist = case.history.copy()
    hist[0, -1] = C.I.TALKER_V + 3
    _, _, _, bad = orc.sample(case.logits, hist, case.steps, case.seeds, case.eos, H.oracle_cfg(case),
                              uniforms=case.uniforms)
    assert bad


def test_per_row_min_max_new_equals_per_row_calls():
    """The oracle's per-row min_new / max_new arrays == calling it row by row with scalar values."""
    g = np.random.default_rng(4)
    B, V, W, eos = 5, 300, 8, 299
    x = (g.standard_normal((B, V)) * 2).astype(np.float32)
    x[:, eos] = 5.0
    hist = g.integers(0, V, size=(B, W)).astype(np.int64)
    steps = np.array([0, 2, 5, 9, 14], np.int64)
    rmin, rmax = np.array([3, 3, 0, 20, 0], np.int64), np.array([100, 3, 100, 100, 15], np.int64)
    u = g.random(B).astype(np.float32)
    for sem in ("hf", "omni"):
        base = dict(temperature=0.9, top_p=0.9, top_k=40, repetition_penalty=1.1, window=W, min_keep=2, semantics=sem)
        p_all, t_all, _, _ = orc.sample(x, hist, steps, None, eos, orc.Cfg(min_new_tokens=0, max_new_tokens=1, **base),
                                        uniforms=u, row_min_new=rmin, row_max_new=rmax)
        for r in range(B):
            p_r, t_r, _, _ = orc.sample(x[r:r + 1], hist[r:r + 1], steps[r:r + 1], None, eos,
                                        orc.Cfg(min_new_tokens=int(rmin[r]), max_new_tokens=int(rmax[r]), **base),
                                        uniforms=u[r:r + 1])
            assert t_r[0] == t_all[r]
            assert np.array_equal(p_r[0].view(np.uint32), p_all[r].view(np.uint32))
