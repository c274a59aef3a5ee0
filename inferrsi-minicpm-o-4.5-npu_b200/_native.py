"""Loading of the native pieces: ``libb2s.so`` (C-ABI, ctypes view) and the torch op library.

There is no fallback: if the CUDA library is missing or cannot be loaded, every sampling entry point
raises.  Build with ``build.py`` (or ``__graft_entry__.build()``); the built files live in-tree.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB = PKG / "libb2s.so"
OPS = PKG / "_build" / "b2s_torch_ops.so"

_lock = threading.Lock()
_capi = None
_ops_loaded = False


class SampleArgs(ctypes.Structure):
    """ctypes mirror of ``b2s_sample_args`` (include/b2s_sampler.h)."""

    _fields_ = [
        ("logits", ctypes.c_void_p), ("logits_dtype", ctypes.c_int32), ("rows", ctypes.c_int32),
        ("vocab", ctypes.c_int32), ("cluster", ctypes.c_int32), ("logits_row_stride", ctypes.c_int64),
        ("history", ctypes.c_void_p), ("history_row_stride", ctypes.c_int64), ("window", ctypes.c_int32),
        ("eos", ctypes.c_int32), ("steps", ctypes.c_void_p), ("seeds", ctypes.c_void_p),
        ("requests", ctypes.c_void_p), ("uniform_values", ctypes.c_void_p), ("active", ctypes.c_void_p),
        ("finished", ctypes.c_void_p), ("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
        ("presence_penalty", ctypes.c_float), ("frequency_penalty", ctypes.c_float), ("top_k", ctypes.c_int32),
        ("min_keep", ctypes.c_int32), ("min_new_tokens", ctypes.c_int64), ("max_new_tokens", ctypes.c_int64),
        ("row_temperature", ctypes.c_void_p), ("row_top_p", ctypes.c_void_p), ("row_top_k", ctypes.c_void_p),
        ("alpha", ctypes.c_void_p), ("alpha_len", ctypes.c_int32), ("alpha_row_stride", ctypes.c_int32),
        ("max_top_k", ctypes.c_int32), ("semantics", ctypes.c_int32), ("rng", ctypes.c_int32),
        ("flags", ctypes.c_int32), ("tokens", ctypes.c_void_p), ("processed", ctypes.c_void_p),
        ("processed_row_stride", ctypes.c_int64), ("history_out", ctypes.c_void_p),
        ("history_out_row_stride", ctypes.c_int64), ("steps_out", ctypes.c_void_p),
        ("finished_out", ctypes.c_void_p), ("status", ctypes.c_void_p),
        ("row_min_new_tokens", ctypes.c_void_p), ("row_max_new_tokens", ctypes.c_void_p),
    ]


class HeadArgs(ctypes.Structure):
    """b2s_head_args of include/b2s_sampler.h."""
    _fields_ = [
        ("hidden", ctypes.c_void_p), ("hidden_row_stride", ctypes.c_int64), ("head", ctypes.c_void_p),
        ("hidden_dim", ctypes.c_int32), ("logits", ctypes.c_void_p), ("sync", ctypes.c_void_p),
    ]


# every entry point of include/b2s_sampler.h with its ctypes signature
CAPI_SIGNATURES = {
    "b2s_sample": (ctypes.c_int, [ctypes.POINTER(SampleArgs), ctypes.c_void_p]),
    "b2s_head_sample": (ctypes.c_int, [ctypes.POINTER(HeadArgs), ctypes.POINTER(SampleArgs), ctypes.c_void_p]),
    "b2s_lmhead_argmax": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_lmhead_argmax_keys": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_head_sample_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32,
                                               ctypes.POINTER(SampleArgs), ctypes.c_void_p]),
    "b2s_sample_frames": (ctypes.c_int, [ctypes.POINTER(SampleArgs), ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p]),
    "b2s_argmax": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_uniform": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                                   ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_shard_candidates": (ctypes.c_int, [ctypes.POINTER(SampleArgs), ctypes.c_int64, ctypes.c_int32,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_shard_merge": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(SampleArgs),
                                       ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_shard_resolve": (ctypes.c_int, [ctypes.POINTER(SampleArgs), ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_repetition_penalty": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                              ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_expf_spec": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "b2s_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "b2s_last_cuda_error": (ctypes.c_char_p, []),
    "b2s_abi_version": (ctypes.c_int, []),
}


def capi() -> ctypes.CDLL:
    """The C-ABI library through ctypes (loading needs no GPU)."""
    global _capi
    with _lock:
        if _capi is None:
            if not LIB.exists():
                raise RuntimeError(f"{LIB} is missing: build the CUDA library first (build.py)")
            lib = ctypes.CDLL(str(LIB), mode=ctypes.RTLD_GLOBAL)
            for name, (res, args) in CAPI_SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _capi = lib
    return _capi


def ops():
    """``torch.ops.minicpmo_sampler`` with its CUDA kernels registered."""
    global _ops_loaded
    import torch

    capi()  # libb2s.so first (RTLD_GLOBAL): the op library links against it by soname
    with _lock:
        if not _ops_loaded:
            if not OPS.exists():
                raise RuntimeError(f"{OPS} is missing: build the torch op layer first (build.py)")
            torch.ops.load_library(str(OPS))
            _ops_loaded = True
    return torch.ops.minicpmo_sampler


def check(rc: int, what: str) -> None:
    if rc != 0:
        lib = capi()
        msg = lib.b2s_error_string(rc).decode()
        if rc == 3:
            msg += f" ({lib.b2s_last_cuda_error().decode()})"
        raise RuntimeError(f"{what} failed: {msg}")
