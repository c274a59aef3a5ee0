"""Seeded synthetic inputs for the sampler parity cases (shared by the fixture generator and the tests).

Every array is a pure function of its case name and numpy's PCG64 stream, so fixtures only store
the reference's outputs plus a sha256 of the inputs they were computed from; a test regenerates
the inputs and checks the digest before comparing.  The shapes and distributions follow the five
workloads of the benchmark plan (Talker V=6562 with EOS=6561; Thinker V=151,936), cut to sizes that
the CPU oracle finishes in seconds.
"""

from __future__ import annotations

import hashlib

import numpy as np

TALKER_V, TALKER_EOS = 6562, 6561
THINKER_V = 151_936
PAD = -1


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (torch's ``.to(torch.bfloat16)``)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    lsb = (b >> 16) & 1
    r = ((b + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def small_alphabet_history(g: np.random.Generator, rows: int, window: int, t: int, alphabet: int = 300) -> np.ndarray:
    """Last ``window`` of ``t`` previous frames drawn from a small alphabet, PAD-filled on the left
    (mirrors the reference test's ``_state_rows``: repeats make the penalty counts > 1)."""
    h = np.full((rows, window), PAD, np.int64)
    n = min(t, window)
    if n:
        h[:, window - n:] = g.integers(0, alphabet, size=(rows, n))
    return h


def zipf_rows(g: np.random.Generator, rows: int, vocab: int, window: int, s: float = 1.1):
    """Thinker workload: logit_r = -s*ln(rank) + N(0,1), randomly permuted per row; history ids drawn
    Zipf(s) over ranks and mapped through the row's permutation."""
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    base = -s * np.log(ranks)
    w = ranks ** (-s)
    w /= w.sum()
    logits = np.empty((rows, vocab), np.float32)
    hist = np.empty((rows, window), np.int64)
    for r in range(rows):
        perm = g.permutation(vocab)
        row = (base + g.standard_normal(vocab)).astype(np.float32)
        logits[r, perm] = row
        hist[r] = perm[g.choice(vocab, size=window, p=w)]
    return logits, hist


def quantised_rows(g: np.random.Generator, rows: int, vocab: int, sigma: float = 2.0, q: int = 16) -> np.ndarray:
    """Tie-heavy logits: N(0, sigma) rounded to multiples of 1/q (exact in bf16 for |x| < 16)."""
    return (np.round(g.standard_normal((rows, vocab)) * sigma * q) / q).astype(np.float32)
