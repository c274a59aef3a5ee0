"""Per-request RNG seeds for the sampling state (``engine/runtime/backend.py:51-54``).

A request's seed is its explicit ``seed`` reduced to 63 bits, or -- when it has none -- the first 15 hex digits
of the SHA-256 of its ``request_id`` (60 bits).  The reference passes it to ``DecodeState.new`` for the Talker
(``backend.py:271``, ``backend_s.py:1001``) and to the native generators of the omni order
(``backend_npu.py:999``).  The sampling kernels take it as the ``seeds`` input of the counter hash and as the
Philox key, so every request keeps the same random stream whichever batch row it lands in.
"""

from __future__ import annotations

import hashlib
from typing import Iterable, Optional

import torch

M63 = (1 << 63) - 1


def request_seed(req) -> int:
    """The seed of a request object with ``seed`` (int or None) and ``request_id`` (str) attributes."""
    return seed_of(getattr(req, "request_id"), getattr(req, "seed", None))


def seed_of(request_id: str, seed: Optional[int] = None) -> int:
    """``request_seed`` from the two fields directly."""
    if seed is not None:
        return int(seed) & M63
    return int(hashlib.sha256(request_id.encode()).hexdigest()[:15], 16)


def request_seeds(reqs: Iterable, device=None) -> torch.Tensor:
    """[B] int64 seeds of a batch of requests, in row order (the ``seeds`` input of the sampling kernels)."""
    return torch.tensor([request_seed(r) for r in reqs], dtype=torch.int64, device=device)
