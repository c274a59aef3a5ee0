"""Thinker text-token sampling step on B200 kernels.

The reference Thinker samples greedily at every call site -- ``F.linear(h, lm_head).float().argmax(-1)``
(``engine/runtime/thinker_decode.py:83,107``, ``engine/runtime/backend_s.py:893``,
``engine/runtime/backend.py:238``, ``engine/runtime/backend_npu.py:890``, ``engine/runtime/track_s.py:60``).
``argmax`` replaces the ``.float().argmax(-1)`` tail: it reads bf16 or fp32 logits directly (no fp32 copy)
and keeps torch's first-index tie-break.

``sample`` is the non-greedy Thinker step (temperature, top-k, top-p, count-based repetition penalty,
optional presence / frequency penalties) in the vLLM-Omni order of the reference's ``omni`` semantics
(``engine/talker_sampler.py:142-147``: penalty -> /T -> top-k -> top-p with min_keep 1), with no EOS rules.
Temperature 0 means greedy: the argmax of the penalised logits, first index among ties.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _native
from . import talker_sampler as ts


@dataclass(frozen=True)
class ThinkerSampling:
    temperature: float = 0.7
    top_k: int = 20
    top_p: float = 0.8
    repetition_penalty: float = 1.05
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    window: int = 512
    rng: str = "philox"  # "philox" (Philox4x32-10 keyed by (seed, step, request)) or "counter"


def argmax(logits: torch.Tensor) -> torch.Tensor:
    """[B] int64 argmax of [B, V] bf16/fp32 logits; first index among equal maxima, NaN is the maximum."""
    ts._need_cuda(logits)
    return _native.ops().argmax(logits)


class LMHeadArgmax:
    """The Thinker's greedy step straight from its LM head: ``F.linear(hidden, lm_head).float().argmax(-1)``
    (``engine/runtime/thinker_decode.py:83,107``, ``engine/runtime/backend_s.py:893``) as one tensor-core GEMM whose
    epilogue keeps each row's maximum, so the [B, V] logits are never written.  Holds the head ([V, H] bf16) and
    ``rows`` 64-bit reduction words (zero between calls); one instance per stream.  Up to 64 rows, H a multiple of
    64.  Each logit is the bf16 rounding of an fp32 tensor-core sum, as F.linear's bf16 output is; ties keep the
    first index and NaN wins, as torch's argmax."""

    def __init__(self, head: torch.Tensor, rows: int):
        ts._need_cuda(head)
        if head.dtype != torch.bfloat16 or head.dim() != 2:
            raise ValueError("head must be a bf16 [vocab, hidden] tensor")
        self.head = head.contiguous()
        self.rows = int(rows)
        self.keys = torch.zeros(self.rows, dtype=torch.int64, device=head.device)

    def __call__(self, hidden: torch.Tensor, status: Optional[torch.Tensor] = None) -> torch.Tensor:
        ts._need_cuda(hidden)
        if hidden.dim() != 2 or hidden.shape[0] != self.rows or hidden.dtype != torch.bfloat16:
            raise ValueError(f"hidden must be bf16 [{self.rows}, hidden]")
        return _native.ops().lmhead_argmax(hidden, self.head, self.keys, status)


def sample(logits: torch.Tensor, history: Optional[torch.Tensor], seeds: torch.Tensor, steps: torch.Tensor,
           cfg: ThinkerSampling = ThinkerSampling(), *, uniform_values: Optional[torch.Tensor] = None,
           requests: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None,
           cluster: int = 0) -> torch.Tensor:
    """One sampled Thinker token per row ([B] int64)."""
    ts._need_cuda(logits, history, seeds, steps, uniform_values, requests)
    seeds, steps, requests = ts._i64(seeds), ts._i64(steps), ts._i64(requests)
    W = 0 if history is None else history.shape[-1]
    no_pen = cfg.repetition_penalty == 1.0 and cfg.presence_penalty == 0.0 and cfg.frequency_penalty == 0.0
    if cfg.temperature == 0.0 and (no_pen or W == 0):
        return argmax(logits)
    alpha = ts.alpha_table(cfg.repetition_penalty, W + 1, logits.device) if W > 0 else None
    if cfg.temperature == 0.0:
        # greedy over the penalised logits: keep the maximum value only and take the first kept index (u = 0)
        u = torch.zeros(logits.shape[0], dtype=torch.float32, device=logits.device)
        return ts._run(logits, history=history, steps=steps, uniform_values=u, alpha=alpha, status=status,
                       temperature=1.0, top_p=1.0, top_k=1, min_keep=1, presence=cfg.presence_penalty,
                       frequency=cfg.frequency_penalty, semantics=ts.SEM_OMNI, rng=ts.RNG_UNIFORM, max_top_k=1,
                       flags=ts.FLAG_TOPK_ONLY, cluster=cluster)[0]
    if uniform_values is not None:
        rng = ts.RNG_UNIFORM
        uniform_values = uniform_values.to(torch.float32).contiguous()
    else:
        rng = {"philox": ts.RNG_PHILOX, "counter": ts.RNG_COUNTER}[cfg.rng]
    return ts._run(logits, history=history, steps=steps, seeds=seeds, requests=requests,
                   uniform_values=uniform_values, alpha=alpha, status=status,
                   temperature=ts._temperature(cfg.temperature), top_p=cfg.top_p, top_k=cfg.top_k, min_keep=1,
                   presence=cfg.presence_penalty, frequency=cfg.frequency_penalty, semantics=ts.SEM_OMNI, rng=rng,
                   max_top_k=max(cfg.top_k, 1), cluster=cluster)[0]
