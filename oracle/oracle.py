"""CPU oracle for the token-sampling path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` import this
module; the product package never does.  It wraps ``oracle/sampler_oracle.c`` (a C restatement of
``engine/talker_sampler.py:60-172`` of the reference, built by ``oracle/Makefile``) with numpy
in/out arrays.

The repetition-penalty factors are the reference's own ``torch.pow(torch.full_like(x, penalty),
freq)`` (``engine/talker_sampler.py:83``) evaluated on the CPU for every count ``0..window``: CPU
``torch.pow`` in fp32 is not correctly rounded, so the table is taken from it rather than
recomputed (the CUDA path receives the same table through its C-ABI).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

HF, OMNI = 0, 1
RNG_UNIFORM, RNG_COUNTER, RNG_PHILOX = 0, 1, 2


class OrcCfg(ctypes.Structure):
    _fields_ = [
        ("vocab", ctypes.c_int32), ("window", ctypes.c_int32), ("eos", ctypes.c_int32),
        ("semantics", ctypes.c_int32), ("top_k", ctypes.c_int32), ("min_keep", ctypes.c_int32),
        ("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("presence", ctypes.c_float),
        ("frequency", ctypes.c_float), ("min_new", ctypes.c_int64), ("max_new", ctypes.c_int64),
        ("apply_filter_at_step0", ctypes.c_int32), ("pad_", ctypes.c_int32),
    ]


class OrcMeta(ctypes.Structure):
    _fields_ = [
        ("kept", ctypes.c_int32), ("mode", ctypes.c_int32), ("thr", ctypes.c_float), ("lse", ctypes.c_float),
        ("topp_margin", ctypes.c_double), ("draw_margin", ctypes.c_double), ("target", ctypes.c_float),
        ("cdf_last", ctypes.c_float), ("token", ctypes.c_int64),
    ]


META_DTYPE = np.dtype([("kept", np.int32), ("mode", np.int32), ("thr", np.float32), ("lse", np.float32),
                       ("topp_margin", np.float64), ("draw_margin", np.float64), ("target", np.float32),
                       ("cdf_last", np.float32), ("token", np.int64)], align=True)
assert META_DTYPE.itemsize == ctypes.sizeof(OrcMeta)


class OrcBatch(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p), ("logits_dtype", ctypes.c_int32), ("rows", ctypes.c_int32),
        ("logits_row_stride", ctypes.c_int64), ("history", ctypes.c_void_p), ("history_row_stride", ctypes.c_int64),
        ("steps", ctypes.c_void_p), ("seeds", ctypes.c_void_p), ("requests", ctypes.c_void_p),
        ("uniforms", ctypes.c_void_p), ("alpha", ctypes.c_void_p), ("alpha_len", ctypes.c_int32),
        ("alpha_row_stride", ctypes.c_int32), ("row_temperature", ctypes.c_void_p), ("row_top_p", ctypes.c_void_p),
        ("row_top_k", ctypes.c_void_p), ("rng", ctypes.c_int32), ("threads", ctypes.c_int32),
        ("processed", ctypes.c_void_p), ("tokens", ctypes.c_void_p), ("meta", ctypes.c_void_p),
        ("bad_history", ctypes.c_void_p), ("row_min_new", ctypes.c_void_p), ("row_max_new", ctypes.c_void_p),
    ]


_LIB = None


def build(force: bool = False) -> Path:
    """Compile the C restatement with ``oracle/Makefile`` (gcc, OpenMP)."""
    src = HERE / "sampler_oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        env = dict(os.environ)
        env.pop("CC", None)
        subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True, env=env)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.orc_sample_batch.argtypes = [ctypes.POINTER(OrcBatch), ctypes.POINTER(OrcCfg)]
        L.orc_draw_batch.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]
        L.orc_argmax_batch.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                       ctypes.c_void_p]
        L.orc_expf_batch.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.orc_uniform_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.c_int32, ctypes.c_void_p]
        L.orc_philox4x32_10.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.b2s_expf.argtypes = [ctypes.c_float]
        L.b2s_expf.restype = ctypes.c_float
        _LIB = L
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data


def alpha_table(penalty: float, length: int) -> np.ndarray:
    """``penalty ** n`` for n in [0, length) exactly as the reference evaluates it (CPU torch.pow, fp32)."""
    import torch

    n = torch.arange(length, dtype=torch.float32)
    return torch.pow(torch.full_like(n, float(penalty)), n).numpy()


@dataclass(frozen=True)
class Cfg:
    """Sampling configuration in the field names of the reference ``TalkerSampling``
    (``engine/talker_sampler.py:34-51``) plus the Thinker extensions."""

    temperature: float = 0.8
    top_p: float = 0.85
    top_k: int = 25
    repetition_penalty: float = 1.05
    window: int = 16
    min_new_tokens: int = 50
    max_new_tokens: int = 2048
    min_keep: int = 3
    semantics: str = "hf"
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0


def _cfg_struct(cfg, vocab: int, window: int, eos: int) -> OrcCfg:
    sem = {"hf": HF, "omni": OMNI}[cfg.semantics]
    return OrcCfg(vocab=vocab, window=window, eos=int(eos), semantics=sem, top_k=int(cfg.top_k),
                  min_keep=int(cfg.min_keep), temperature=float(np.float32(cfg.temperature)),
                  top_p=float(np.float32(cfg.top_p)), presence=float(getattr(cfg, "presence_penalty", 0.0)),
                  frequency=float(getattr(cfg, "frequency_penalty", 0.0)), min_new=int(cfg.min_new_tokens),
                  max_new=int(cfg.max_new_tokens), apply_filter_at_step0=0, pad_=0)


def _as_np(t, dtype=None):
    try:
        import torch

        if isinstance(t, torch.Tensor):
            t = t.detach().cpu()
            if t.dtype == torch.bfloat16:
                return np.ascontiguousarray(t.view(torch.int16).numpy().view(np.uint16))
            t = t.numpy()
    except ImportError:
        pass
    a = np.ascontiguousarray(t)
    return a if dtype is None else np.ascontiguousarray(a, dtype=dtype)


def sample(logits, history, steps, seeds, eos: int, cfg, *, uniforms=None, rng: int = RNG_COUNTER, requests=None,
           penalties=None, row_temperature=None, row_top_p=None, row_top_k=None, row_min_new=None, row_max_new=None,
           want_processed: bool = True, threads: int = 0):
    """processed_logits + draw for a batch.  ``logits``: [B, V] fp32 array, or bf16 given as a torch
    tensor / uint16 bit array.  ``penalties``: optional per-row repetition penalties.  Returns
    ``(processed [B,V] fp32 or None, tokens [B] int64, meta [B] structured, bad_history flag)``."""
    is_bf16 = False
    try:
        import torch

        is_bf16 = isinstance(logits, torch.Tensor) and logits.dtype == torch.bfloat16
    except ImportError:
        pass
    x = _as_np(logits)
    if x.dtype == np.uint16:
        is_bf16 = True
    elif x.dtype != np.float32:
        x = x.astype(np.float32)
    B, V = x.shape
    hist = _as_np(history, np.int64).reshape(B, -1)
    W = hist.shape[1]
    steps_a = _as_np(steps, np.int64).reshape(B)
    seeds_a = _as_np(seeds, np.int64).reshape(B) if seeds is not None else np.zeros(B, np.int64)
    req = _as_np(requests, np.int64).reshape(B) if requests is not None else None
    if uniforms is not None:
        uni = _as_np(uniforms, np.float32).reshape(B)
        rng = RNG_UNIFORM
    else:
        uni = None
    alen = max(W, 1) + 1
    if penalties is None:
        alpha = alpha_table(cfg.repetition_penalty, alen)
        astride = 0
    else:
        pens = _as_np(penalties, np.float64).reshape(B)
        alpha = np.stack([alpha_table(float(p), alen) for p in pens])
        astride = alen
    alpha = np.ascontiguousarray(alpha, np.float32)
    rt = _as_np(row_temperature, np.float32).reshape(B) if row_temperature is not None else None
    rp = _as_np(row_top_p, np.float32).reshape(B) if row_top_p is not None else None
    rk = _as_np(row_top_k, np.int32).reshape(B) if row_top_k is not None else None
    rmin = _as_np(row_min_new, np.int64).reshape(B) if row_min_new is not None else None
    rmax = _as_np(row_max_new, np.int64).reshape(B) if row_max_new is not None else None
    processed = np.empty((B, V), np.float32) if want_processed else None
    tokens = np.empty(B, np.int64)
    meta = np.zeros(B, META_DTYPE)
    bad = np.zeros(1, np.int32)
    b = OrcBatch(logits=_ptr(x), logits_dtype=1 if is_bf16 else 0, rows=B, logits_row_stride=V, history=_ptr(hist),
                 history_row_stride=W, steps=_ptr(steps_a), seeds=_ptr(seeds_a), requests=_ptr(req), uniforms=_ptr(uni),
                 alpha=_ptr(alpha), alpha_len=alen, alpha_row_stride=astride, row_temperature=_ptr(rt),
                 row_top_p=_ptr(rp), row_top_k=_ptr(rk), rng=rng, threads=threads, processed=_ptr(processed),
                 tokens=_ptr(tokens), meta=_ptr(meta), bad_history=_ptr(bad), row_min_new=_ptr(rmin),
                 row_max_new=_ptr(rmax))
    c = _cfg_struct(cfg, V, W, eos)
    lib().orc_sample_batch(ctypes.byref(b), ctypes.byref(c))
    return processed, tokens, meta, bool(bad[0])


def draw(x, uniforms, threads: int = 0):
    """draw() on fp32 rows with the given uniforms -> (tokens, meta)."""
    xa = _as_np(x, np.float32)
    B, V = xa.shape
    u = _as_np(uniforms, np.float32).reshape(B)
    tokens = np.empty(B, np.int64)
    meta = np.zeros(B, META_DTYPE)
    lib().orc_draw_batch(_ptr(xa), B, V, V, _ptr(u), _ptr(tokens), _ptr(meta), threads)
    return tokens, meta


def argmax(logits):
    x = _as_np(logits)
    dt = 1 if x.dtype == np.uint16 else 0
    if dt == 0 and x.dtype != np.float32:
        x = x.astype(np.float32)
    B, V = x.shape
    out = np.empty(B, np.int64)
    lib().orc_argmax_batch(_ptr(x), dt, B, V, V, _ptr(out))
    return out


def uniform(seeds, steps, rng: int = RNG_COUNTER, requests=None):
    s = _as_np(seeds, np.int64).reshape(-1)
    t = _as_np(steps, np.int64).reshape(-1)
    r = _as_np(requests, np.int64).reshape(-1) if requests is not None else None
    out = np.empty(s.shape[0], np.float32)
    lib().orc_uniform_batch(_ptr(s), _ptr(t), _ptr(r), s.shape[0], rng, _ptr(out))
    return out


def philox4x32_10(counter, key):
    c = np.ascontiguousarray(counter, np.uint32)
    k = np.ascontiguousarray(key, np.uint32)
    out = np.empty(4, np.uint32)
    lib().orc_philox4x32_10(_ptr(c), _ptr(k), _ptr(out))
    return out


def expf(x):
    xa = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(xa)
    lib().orc_expf_batch(_ptr(xa), xa.size, _ptr(out))
    return out
