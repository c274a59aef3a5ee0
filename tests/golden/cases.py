"""Parity cases for the sampler: inputs (regenerated from seeds) + the configuration per row.

``make_golden.py`` runs the reference module on each case and stores its outputs under
``tests/golden/*.npz``; the CPU tests check the oracle against those outputs and the GPU tests
check the CUDA path against both.  Configuration dicts use the reference ``TalkerSampling`` field
names (``engine/talker_sampler.py:34-51``); ``presence_penalty``/``frequency_penalty`` are the
Thinker extensions and are only ever 0 in cases that the reference is run on.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import inputs as I

BIG = 1 << 40  # max_new_tokens for Thinker rows: never forced


@dataclass
class Case:
    name: str
    logits: np.ndarray            # [B, V] fp32 values (bf16 cases: already bf16-rounded)
    dtype: str                    # "f32" or "bf16"
    history: np.ndarray           # [B, W] int64, PAD = -1
    steps: np.ndarray             # [B] int64
    seeds: np.ndarray             # [B] int64
    uniforms: np.ndarray          # [B] fp32, injected through draw(uniform_values=...)
    eos: int
    cfgs: list = field(default_factory=list)  # one dict per row

    @property
    def rows(self) -> int:
        return self.logits.shape[0]

    @property
    def vocab(self) -> int:
        return self.logits.shape[1]

    def bf16_bits(self) -> np.ndarray:
        return I.to_bf16_bits(self.logits)

    def digest(self) -> str:
        return I.digest(self.logits, self.history, self.steps, self.seeds, self.uniforms)

    def uniform_cfg(self) -> bool:
        return all(c == self.cfgs[0] for c in self.cfgs)


TALKER_DEFAULT = dict(temperature=0.8, top_p=0.85, top_k=25, repetition_penalty=1.05, window=16, min_new_tokens=50,
                      max_new_tokens=2048, min_keep=3, semantics="hf")


def _cfg(**kw) -> dict:
    c = dict(TALKER_DEFAULT)
    c.update(kw)
    return c


def _bf16(x: np.ndarray) -> np.ndarray:
    return I.bf16_bits_to_f32(I.to_bf16_bits(x))


def _case(name, logits, dtype, history, steps, eos, cfgs, seed):
    g = I.rng(seed + 7919)
    B = logits.shape[0]
    if dtype == "bf16":
        logits = _bf16(logits)
    seeds = g.integers(0, 1 << 62, size=B, dtype=np.int64)
    uniforms = g.random(B, dtype=np.float32)
    if not isinstance(cfgs, list):
        cfgs = [cfgs] * B
    return Case(name, np.ascontiguousarray(logits, np.float32), dtype, np.ascontiguousarray(history, np.int64),
                np.asarray(steps, np.int64).reshape(B), seeds, uniforms, int(eos), cfgs)


def talker_order(t: int, semantics: str = "hf", rows: int = 8) -> Case:
    """The reference's test_hf_order shape: randn*3 logits, small-alphabet history, step t."""
    g = I.rng(1000 + t + (500 if semantics == "omni" else 0))
    logits = (g.standard_normal((rows, I.TALKER_V)) * 3).astype(np.float32)
    hist = I.small_alphabet_history(g, rows, 16, t)
    return _case(f"{semantics}_t{t}", logits, "f32", hist, np.full(rows, t), I.TALKER_EOS, _cfg(semantics=semantics),
                 2000 + t)


def talker_batched_cfg2() -> Case:
    """Batched Talker at streaming concurrency: per-row temperature/top-k/top-p (row i takes index i mod 3),
    bf16 logits N(0,2) with a per-row shift U(-1,1), 64-token penalty history, EOS masked for 8 steps."""
    g = I.rng(2)
    B = 8
    logits = (g.standard_normal((B, I.TALKER_V)) * 2.0 + g.uniform(-1, 1, size=(B, 1))).astype(np.float32)
    steps = np.array([0, 1, 3, 7, 8, 9, 100, 500])
    hist = np.full((B, 64), I.PAD, np.int64)
    for r in range(B):
        n = int(min(steps[r], 64))
        if n:
            hist[r, 64 - n:] = g.integers(0, I.TALKER_V, size=n)
    temps, ks, ps = (0.6, 0.8, 1.0), (20, 25, 50), (0.7, 0.85, 0.95)
    cfgs = [_cfg(temperature=temps[r % 3], top_k=ks[r % 3], top_p=ps[r % 3], window=64, min_new_tokens=8) for r in range(B)]
    return _case("cfg2_talker_batched", logits, "bf16", hist, steps, I.TALKER_EOS, cfgs, 22)


def thinker_cfg3(rows: int = 2) -> Case:
    """Thinker text sampling on a Qwen3-8B-sized head: Zipf(1.1) profile + N(0,1), permuted per row; 512-token
    Zipf history; omni order (top-k -> top-p, min_keep 1), no EOS rules."""
    g = I.rng(3)
    logits, hist = I.zipf_rows(g, rows, I.THINKER_V, 512)
    cfg = _cfg(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.05, window=512, min_new_tokens=0,
               max_new_tokens=BIG, min_keep=1, semantics="omni")
    return _case("cfg3_thinker", logits, "bf16", hist, np.full(rows, 100), -1, cfg, 33)


def large_cfg4(rows: int = 1) -> Case:
    g = I.rng(4)
    logits = (g.standard_normal((rows, I.THINKER_V)) * 3.0).astype(np.float32)
    hist = g.integers(0, I.THINKER_V, size=(rows, 2048))
    cfg = _cfg(temperature=1.0, top_k=50, top_p=0.95, repetition_penalty=1.1, window=2048, min_new_tokens=0,
               max_new_tokens=BIG, min_keep=1, semantics="omni")
    return _case("cfg4_large", logits, "f32", hist, np.full(rows, 7), -1, cfg, 44)


def ties_cfg5(rows: int = 2) -> Case:
    g = I.rng(5)
    logits = I.quantised_rows(g, rows, I.THINKER_V)
    hist = np.full((rows, 4), I.PAD, np.int64)
    cfg = _cfg(temperature=0.8, top_k=64, top_p=0.9, repetition_penalty=1.0, window=4, min_new_tokens=0,
               max_new_tokens=BIG, min_keep=1, semantics="omni")
    return _case("cfg5_ties", logits, "bf16", hist, np.full(rows, 3), -1, cfg, 55)


def edge_cases() -> list[Case]:
    V, EOS = I.TALKER_V, I.TALKER_EOS
    out = []
    g = I.rng(6)
    B = 4
    base = (g.standard_normal((B, V)) * 3).astype(np.float32)
    hist = I.small_alphabet_history(g, B, 16, 12)
    for sem in ("hf", "omni"):
        out.append(_case(f"edge_all_equal_{sem}", np.zeros((B, V), np.float32), "f32", hist, np.full(B, 3), EOS,
                         _cfg(semantics=sem), 60))
        q = (np.round(g.standard_normal((B, V)) * 4) / 4).astype(np.float32)
        out.append(_case(f"edge_quantised_{sem}", q, "f32", hist, np.full(B, 9), EOS, _cfg(semantics=sem), 61))
        out.append(_case(f"edge_topk_gt_vocab_{sem}", base, "f32", hist, np.full(B, 5), EOS,
                         _cfg(semantics=sem, top_k=10000), 62))
        out.append(_case(f"edge_topk_1000_{sem}", base, "f32", hist, np.full(B, 5), EOS,
                         _cfg(semantics=sem, top_k=1000, top_p=0.999), 63))
        out.append(_case(f"edge_topp_one_{sem}", base, "f32", hist, np.full(B, 5), EOS,
                         _cfg(semantics=sem, top_p=1.0), 64))
        out.append(_case(f"edge_topp_zero_{sem}", base, "f32", hist, np.full(B, 5), EOS,
                         _cfg(semantics=sem, top_p=0.0), 65))
        ninf = base.copy()
        ninf[g.random((B, V)) < 0.3] = -np.inf
        out.append(_case(f"edge_neg_inf_{sem}", ninf, "f32", hist, np.full(B, 5), EOS, _cfg(semantics=sem), 66))
        out.append(_case(f"edge_forced_eos_{sem}", base, "f32", hist, np.array([2046, 2047, 3000, 2045]), EOS,
                         _cfg(semantics=sem), 67))
        out.append(_case(f"edge_min_new_boundary_{sem}", base, "f32", hist, np.array([49, 50, 0, 1]), EOS,
                         _cfg(semantics=sem), 68))
        mixed = I.small_alphabet_history(g, B, 16, 16, alphabet=20)
        mixed[:, ::3] = I.PAD
        out.append(_case(f"edge_history_pad_mixed_{sem}", base, "f32", mixed, np.full(B, 30), EOS,
                         _cfg(semantics=sem), 69))
        out.append(_case(f"edge_small_vocab_{sem}", (g.standard_normal((B, 8)) * 2).astype(np.float32), "f32",
                         g.integers(0, 8, size=(B, 16)), np.full(B, 4), 7, _cfg(semantics=sem), 70))
        heavy = I.small_alphabet_history(g, B, 16, 16, alphabet=3)
        out.append(_case(f"edge_penalty_lt_one_{sem}", base, "f32", heavy, np.full(B, 16), EOS,
                         _cfg(semantics=sem, repetition_penalty=0.7), 71))
        out.append(_case(f"edge_penalty_big_{sem}", base, "f32", heavy, np.full(B, 16), EOS,
                         _cfg(semantics=sem, repetition_penalty=4.0), 72))
        for T in (3.0, 1.7, 0.1):
            out.append(_case(f"edge_temperature_{T}_{sem}", base, "f32", hist, np.full(B, 5), EOS,
                             _cfg(semantics=sem, temperature=T), 73))
        bfl = (g.standard_normal((B, V)) * 2).astype(np.float32)
        out.append(_case(f"edge_bf16_{sem}", bfl, "bf16", hist, np.array([0, 1, 2, 60]), EOS, _cfg(semantics=sem), 74))
        out.append(_case(f"edge_eos_none_{sem}", base, "f32", hist, np.full(B, 5), -1, _cfg(semantics=sem), 75))
        out.append(_case(f"edge_min_keep_5_{sem}", base * 3, "f32", hist, np.full(B, 5), EOS,
                         _cfg(semantics=sem, min_keep=5, top_p=0.05), 76))
    return out


def talker_cases() -> list[Case]:
    cs = [talker_order(t, "hf") for t in (0, 1, 5, 16, 40, 49, 50, 60, 2047)]
    cs += [talker_order(t, "omni") for t in (0, 1, 7, 60, 2047)]
    g = I.rng(8)
    flat = (g.standard_normal((8, I.TALKER_V)) * 0.5).astype(np.float32)
    peaked = (g.standard_normal((8, I.TALKER_V)) * 8).astype(np.float32)
    h = I.small_alphabet_history(g, 8, 16, 20)
    cs.append(_case("hf_flat", flat, "f32", h, np.full(8, 20), I.TALKER_EOS, _cfg(), 80))
    cs.append(_case("hf_peaked", peaked, "f32", h, np.full(8, 20), I.TALKER_EOS, _cfg(), 81))
    cs.append(talker_batched_cfg2())
    return cs


def thinker_cases() -> list[Case]:
    return [thinker_cfg3(), large_cfg4(), ties_cfg5()]


def all_cases() -> list[Case]:
    return talker_cases() + thinker_cases() + edge_cases()


# ---------------------------------------------------------------- sequences (step / decode_k)

SEQ_SEEDS = [0, 42, (1 << 63) - 1, (1 << 60) + 1234567, 1 << 32, 1, 2035223770, (1 << 32) - 1]


def seq_logits(name: str, frames: int, rows: int, vocab: int = I.TALKER_V) -> np.ndarray:
    g = I.rng(abs(hash_name(name)) % (1 << 31))
    x = g.standard_normal((frames, rows, vocab)).astype(np.float32)
    return x


def hash_name(name: str) -> int:
    h = 0
    for ch in name.encode():
        h = (h * 131 + ch) & 0x7FFFFFFF
    return h


SEQUENCES = {
    # name: (frames, rows, cfg, eos spike (frame,row) or None, inactive rows)
    "seq_hf_counter": (12, 4, _cfg(min_new_tokens=4), (8, 1), (2,)),
    "seq_omni_counter": (10, 3, _cfg(semantics="omni", rng="counter", min_new_tokens=2), (5, 0), ()),
}


def sequence_inputs(name: str):
    frames, rows, cfg, spike, inactive = SEQUENCES[name]
    x = seq_logits(name, frames, rows)
    if spike is not None:
        x[spike[0], spike[1], I.TALKER_EOS] = 1e4
    return x, cfg, list(SEQ_SEEDS[:rows]), list(inactive)
