"""Vocabulary-sharded Thinker sampling across the GPUs of one node (no counterpart in the reference, which runs on a
single device).

Rank s holds logits for the contiguous columns [offset_s, offset_s + V_s) of the LM head.  One step:

1. ``shard_candidates`` (kernel): the shard's processed values (omni order: penalty -> /T) -- every element above
   the shard's k-th largest value, then elements equal to it up to ``cap`` >= k, as (value, global id) pairs, and the
   count of every element >= the shard's k-th value.  With ``cap = k`` a row costs 8k + 4 bytes.
2. one ``all_gather_into_tensor`` over NCCL of the packed [rows, 2*cap+1] int32 buffer (values as bits, ids, count).
3. ``merge`` (kernel, on every rank): the row's top-k values (the sent ones and, by value and count, the ties a shard
   did not send), the top-p cut, the value threshold, and the shard whose range holds the draw; the token when that
   shard sent all its kept elements, else a pending record naming it.
4. ``resolve`` (kernel, on every rank): the pending shard's rank scans its row in vocabulary order for the token;
   one max-all-reduce of [rows] int64 gives every rank the same tokens.

The tokens equal the unsharded kernel's on the concatenated row, however many elements tie at the threshold.
"""

from __future__ import annotations

from datetime import timedelta
from typing import Optional, Sequence

import torch

from . import _native
from . import talker_sampler as ts


class ShardExchangeError(RuntimeError):
    """A collective of the sharded step failed or did not finish within the caller's timeout (a rank left, or
    stopped answering).  The step's tokens are not valid; the caller fails the rows of the step, as the reference
    fails the requests of a tick that raised (``engine/runtime/backend.py:197-203``), and rebuilds the group."""


def _wait(work, what: str, timeout: Optional[float]) -> None:
    try:
        if timeout is None:
            work.wait()
        elif not work.wait(timedelta(seconds=float(timeout))):
            raise ShardExchangeError(f"{what} did not finish within {timeout} s")
    except ShardExchangeError:
        raise
    except Exception as e:  # the backend's own error (a peer that left, a timeout of its own)
        raise ShardExchangeError(f"{what} failed: {type(e).__name__}: {e}") from e


def _k(cfg) -> int:
    return max(int(cfg.top_k), 1)


def default_cap(cfg) -> int:
    """The list capacity per shard and row: k (every element above the shard's k-th value fits)."""
    return _k(cfg)


def _alpha(cfg, history, device):
    W = 0 if history is None else history.shape[-1]
    return ts.alpha_table(cfg.repetition_penalty, W + 1, device) if W > 0 else None


def shard_candidates(logits: torch.Tensor, offset: int, history: Optional[torch.Tensor], steps: torch.Tensor, cfg, *,
                     cap: Optional[int] = None, eos: int = -1, status: Optional[torch.Tensor] = None,
                     cluster: int = 0):
    """Stage 1 on this rank's shard ``logits`` [B, V_s] (columns start at global id ``offset``; history ids are
    global).  Returns (values [B, cap] fp32, ids [B, cap] int32 global, count [B] int32)."""
    ts._need_cuda(logits, history, steps)
    cap = cap or default_cap(cfg)
    if cap < _k(cfg):
        raise ValueError(f"cap ({cap}) must be >= top_k ({_k(cfg)})")
    return _native.ops().shard_candidates(
        logits, history, steps.to(torch.int64), _alpha(cfg, history, logits.device), None, None, None, status,
        ts._temperature(cfg.temperature), float(cfg.top_p), int(cfg.top_k), 1,
        float(getattr(cfg, "presence_penalty", 0.0)), float(getattr(cfg, "frequency_penalty", 0.0)), int(eos), _k(cfg),
        int(offset), int(cap), int(cluster))


def merge(values, ids, counts, vocab: int, steps: torch.Tensor, seeds: Optional[torch.Tensor], cfg, *,
          uniform_values: Optional[torch.Tensor] = None, requests: Optional[torch.Tensor] = None,
          rng: str = "philox", status: Optional[torch.Tensor] = None):
    """Stage 2 over all shards' candidates (lists of per-shard tensors, or stacked [S, B, cap] / [S, B]).
    Returns (tokens [B] int64 -- -2 where the row is pending --, pending [B, 4] int64 records)."""
    if isinstance(values, (list, tuple)):
        values, ids, counts = torch.stack(list(values)), torch.stack(list(ids)), torch.stack(list(counts))
    ts._need_cuda(values, ids, counts, steps, seeds, uniform_values, requests)
    if _k(cfg) > 128:
        raise ValueError("vocabulary-sharded sampling supports top_k <= 128")
    if uniform_values is not None:
        r = ts.RNG_UNIFORM
        uniform_values = uniform_values.to(torch.float32).contiguous()
    else:
        r = {"philox": ts.RNG_PHILOX, "counter": ts.RNG_COUNTER}[rng]
    return _native.ops().shard_merge(values.contiguous(), ids.contiguous(), counts.contiguous(), int(vocab),
                                     steps.to(torch.int64), ts._i64(seeds), ts._i64(requests), uniform_values, None,
                                     None, status, float(cfg.top_p), int(cfg.top_k), 1, r, 0)


def resolve(logits: torch.Tensor, offset: int, shard: int, history: Optional[torch.Tensor], steps: torch.Tensor, cfg,
            tokens: torch.Tensor, pending: torch.Tensor, *, eos: int = -1,
            status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Stage 3 on shard ``shard``: [B] int64 -- the tokens of the rows pending on this shard, the merged tokens of
    resolved rows, -1 for rows pending on other shards (the max over all shards is the result)."""
    ts._need_cuda(logits, history, steps, tokens, pending)
    return _native.ops().shard_resolve(
        logits, history, steps.to(torch.int64), _alpha(cfg, history, logits.device), None, status, pending, tokens,
        ts._temperature(cfg.temperature), float(getattr(cfg, "presence_penalty", 0.0)),
        float(getattr(cfg, "frequency_penalty", 0.0)), int(eos), 0, int(offset), int(shard))


def merge_candidates(values, ids, counts, vocab: int, steps, seeds, cfg, *, shard_logits: Sequence[torch.Tensor],
                     offsets: Sequence[int], history=None, uniform_values=None, requests=None, rng: str = "philox",
                     status=None) -> torch.Tensor:
    """Stages 2 and 3 with every shard's logits on this device (one process holding all shards): the tokens."""
    tok, pend = merge(values, ids, counts, vocab, steps, seeds, cfg, uniform_values=uniform_values,
                      requests=requests, rng=rng, status=status)
    out = None
    for s, (x, off) in enumerate(zip(shard_logits, offsets)):
        t = resolve(x, off, s, history, steps, cfg, tok, pend, status=status)
        out = t if out is None else torch.maximum(out, t)
    return out


def pack(values: torch.Tensor, ids: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """[B, 2*cap+1] int32: value bits | ids | count (one buffer -> one collective)."""
    return torch.cat([values.view(torch.int32), ids, counts[:, None]], dim=1).contiguous()


def unpack(buf: torch.Tensor, shards: int, rows: int, cap: int):
    b = buf.view(shards, rows, 2 * cap + 1)
    return (b[:, :, :cap].contiguous().view(torch.float32), b[:, :, cap:2 * cap].contiguous(),
            b[:, :, 2 * cap].contiguous())


def exchange(values: torch.Tensor, ids: torch.Tensor, counts: torch.Tensor, *, group=None,
             timeout: Optional[float] = None):
    """Every shard's candidate lists on every rank: one ``all_gather_into_tensor`` of the packed buffer.
    Returns (values [S, B, cap], ids [S, B, cap], counts [S, B]) in rank order.  Works on any backend that
    gathers into one tensor (NCCL on the GPUs; gloo on the CPU for the host-side tests).  ``timeout`` (seconds):
    raise ShardExchangeError when the gather has not finished by then (None: the process group's own timeout)."""
    import torch.distributed as dist

    mine = pack(values, ids, counts)
    world = dist.get_world_size(group)
    allb = torch.empty((world * mine.shape[0], mine.shape[1]), dtype=torch.int32, device=mine.device)
    try:
        work = dist.all_gather_into_tensor(allb, mine, group=group, async_op=True)
    except Exception as e:
        raise ShardExchangeError(f"candidate all-gather failed: {type(e).__name__}: {e}") from e
    _wait(work, "candidate all-gather", timeout)
    return unpack(allb, world, mine.shape[0], values.shape[1])


def publish(tokens: torch.Tensor, *, group=None, timeout: Optional[float] = None) -> torch.Tensor:
    """The max over the shards' stage-3 tokens, in place (a max-all-reduce of [B] int64)."""
    import torch.distributed as dist

    try:
        work = dist.all_reduce(tokens, op=dist.ReduceOp.MAX, group=group, async_op=True)
    except Exception as e:
        raise ShardExchangeError(f"token all-reduce failed: {type(e).__name__}: {e}") from e
    _wait(work, "token all-reduce", timeout)
    return tokens


def lmhead_keys(hidden: torch.Tensor, head_shard: torch.Tensor, offset: int, keys: torch.Tensor,
                status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The greedy step's per-shard words from this rank's slice of the Thinker LM head (``b2s_lmhead_argmax_keys``):
    [B] int64 whose max over the shards is the global argmax's key.  ``keys``: [B] int64 scratch, zero between
    calls (``thinker_sampler.LMHeadArgmax(head_shard, B).keys`` serves)."""
    ts._need_cuda(hidden, head_shard, keys)
    return _native.ops().lmhead_argmax_keys(hidden, head_shard, keys, int(offset), status)


def decode_keys(words: torch.Tensor) -> torch.Tensor:
    """Global argmax ids from the max-reduced words of ``lmhead_keys`` (PAD where no shard had a candidate)."""
    k = torch.bitwise_xor(words, torch.tensor(-(1 << 63), dtype=torch.int64, device=words.device))
    ids = 0xFFFFFFFF - torch.bitwise_and(k, 0xFFFFFFFF)
    return torch.where(words == -(1 << 63), torch.full_like(ids, ts.PAD), ids)


def lmhead_argmax_sharded(hidden: torch.Tensor, head_shard: torch.Tensor, offset: int, keys: torch.Tensor, *,
                          group=None, timeout: Optional[float] = None) -> torch.Tensor:
    """The vocabulary-sharded Thinker head for the greedy step: this rank's LM-head slice (ids ``offset`` ..)
    on the tensor cores with the argmax in its epilogue, one max-all-reduce of [B] int64 words, the global
    argmax ids on every rank (first id among equal maxima, as torch's argmax over the whole row).  The logits are
    never written.  ``timeout`` as for ``exchange``."""
    return merge_keys(lmhead_keys(hidden, head_shard, offset, keys), group=group, timeout=timeout)


def merge_keys(words: torch.Tensor, *, group=None, timeout: Optional[float] = None) -> torch.Tensor:
    """The shards' [B] int64 words max-all-reduced in place (NCCL on the GPUs, gloo on the CPU), decoded to the
    global argmax ids.  ``timeout`` as for ``exchange``."""
    import torch.distributed as dist

    try:
        work = dist.all_reduce(words, op=dist.ReduceOp.MAX, group=group, async_op=True)
    except Exception as e:
        raise ShardExchangeError(f"argmax all-reduce failed: {type(e).__name__}: {e}") from e
    _wait(work, "argmax all-reduce", timeout)
    return decode_keys(words)


def sample_sharded(logits: torch.Tensor, offset: int, vocab: int, history: Optional[torch.Tensor],
                   steps: torch.Tensor, seeds: Optional[torch.Tensor], cfg, *, group=None, cap: Optional[int] = None,
                   uniform_values: Optional[torch.Tensor] = None, requests: Optional[torch.Tensor] = None,
                   rng: str = "philox", status: Optional[torch.Tensor] = None,
                   timeout: Optional[float] = None) -> torch.Tensor:
    """One sampled token per row of the full vocabulary, from this rank's shard; every rank returns the same
    tokens.  ``group``: the torch.distributed process group of the shards (rank order = shard order).  Two
    collectives: the all-gather of the candidate lists and a max-all-reduce of [B] int64 tokens.  ``timeout``
    (seconds) bounds each of them: a rank that left or hangs turns into ShardExchangeError, not a hang."""
    import torch.distributed as dist

    cap = cap or default_cap(cfg)
    v, i, n = shard_candidates(logits, offset, history, steps, cfg, cap=cap, status=status)
    vv, ii, nn = exchange(v, i, n, group=group, timeout=timeout)
    tok, pend = merge(vv, ii, nn, vocab, steps, seeds, cfg, uniform_values=uniform_values, requests=requests, rng=rng,
                      status=status)
    out = resolve(logits, offset, dist.get_rank(group), history, steps, cfg, tok, pend, status=status)
    return publish(out, group=group, timeout=timeout)


def shard_bounds(vocab: int, shards: int) -> Sequence[int]:
    """Contiguous shard offsets (the last shard takes the remainder)."""
    per = -(-vocab // shards)
    return [min(vocab, s * per) for s in range(shards + 1)]
