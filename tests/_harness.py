"""Helpers shared by the parity tests: run the oracle on a golden case and compare results.

Parity rule (written here once, used by every test):
  * processed logits: identical -inf pattern and bit-identical finite values;
  * tokens: identical, except where the deciding quantity lies within float rounding of a
    boundary -- the top-p mass within ``TOPP_TOL`` of ``top_p`` or the scaled uniform within
    ``DRAW_TOL`` (relative to the total mass) of a cumulative-sum boundary.  Such rows are returned
    so that each test can assert how many there may be (none, for the oracle-vs-CUDA comparison).
"""

from __future__ import annotations

import numpy as np

from oracle import oracle as orc
from tests.golden import cases as C

TOPP_TOL = 1e-5  # absolute, on probabilities in [0, 1]
DRAW_TOL = 1e-5  # relative to the total mass cdf[-1]
FIXTURES = {}


def fixture(group: str):
    from pathlib import Path

    if group not in FIXTURES:
        FIXTURES[group] = dict(np.load(Path(__file__).resolve().parent / "golden" / f"{group}.npz"))
    return FIXTURES[group]


def oracle_cfg(case: C.Case) -> orc.Cfg:
    c = case.cfgs[0]
    return orc.Cfg(**{k: v for k, v in c.items() if k in orc.Cfg.__dataclass_fields__})


def per_row(case: C.Case):
    if case.uniform_cfg():
        return {}
    return dict(row_temperature=np.array([c["temperature"] for c in case.cfgs], np.float32),
                row_top_p=np.array([c["top_p"] for c in case.cfgs], np.float32),
                row_top_k=np.array([c["top_k"] for c in case.cfgs], np.int32),
                penalties=np.array([c["repetition_penalty"] for c in case.cfgs], np.float64))


def logits_input(case: C.Case):
    """The logits as the caller hands them over: fp32 values or bf16 bit patterns."""
    return case.bf16_bits() if case.dtype == "bf16" else case.logits


def run_oracle(case: C.Case, *, counter: bool = False):
    return orc.sample(logits_input(case), case.history, case.steps, case.seeds, case.eos, oracle_cfg(case),
                      uniforms=None if counter else case.uniforms, rng=orc.RNG_COUNTER, **per_row(case))


def compare_processed(want: np.ndarray, got: np.ndarray) -> np.ndarray:
    """Rows whose -inf pattern or finite values differ (bitwise)."""
    inf_eq = (np.isneginf(want) == np.isneginf(got)).all(axis=1)
    fin = ~np.isneginf(want)
    same = want.view(np.uint32) == got.view(np.uint32)
    val_eq = np.where(fin, same, True).all(axis=1)
    return np.nonzero(~(inf_eq & val_eq))[0]


def boundary_rows(meta) -> np.ndarray:
    return (meta["topp_margin"] < TOPP_TOL) | (meta["draw_margin"] < DRAW_TOL)
