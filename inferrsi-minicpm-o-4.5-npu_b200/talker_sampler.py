"""Drop-in replacement of the reference module ``engine/talker_sampler.py`` running on B200 kernels.

Same public names and call signatures as the reference (``engine/talker_sampler.py:30-254``):
``PAD``, ``M32``, ``TalkerSampling``, ``uniform``, ``repetition_penalty``, ``top_k_filter``,
``top_p_top_k_filter``, ``top_k_top_p_filter``, ``processed_logits``, ``draw``, ``draw_multinomial``,
``restore_multinomial_states_after_block``, ``DecodeState``, ``step`` and ``decode_k``; plus the fused
``sample`` / ``step_`` entry points used by captured graph bodies and the per-row parameter form
(``RowParams``) for batches whose rows carry different temperature / top-k / top-p / penalty.

Every tensor argument must live on a CUDA device: this engine has no CPU path, and calls with CPU
tensors raise ``ValueError``.  All entry points are asynchronous (no host synchronisation) and can be
captured in a CUDA graph once the per-penalty factor table has been built by a first call.

Numerics (identical to the CPU oracle of this repository, bit for bit): every element-wise fp32 op of
the reference is one IEEE op; ``penalty ** n`` comes from the reference's own ``torch.pow`` on the CPU;
sums accumulate in fp64 and round once; exp is a fixed FMA sequence.  Against the reference's CPU torch
the kept set and token agree except within float rounding of a top-p or inverse-CDF boundary.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _native

PAD = -1
M32 = 0xFFFFFFFF

SEM_HF, SEM_OMNI, SEM_IDENTITY = 0, 1, 2
RNG_UNIFORM, RNG_COUNTER, RNG_PHILOX = 0, 1, 2
FLAG_FORCE_EXACT = 1
FLAG_STREAM = 4  # the streaming kernel even where the row-resident one applies (include/b2s_sampler.h)
NEVER = 1 << 62  # max_new_tokens that never forces EOS


@dataclass(frozen=True)
class TalkerSampling:
    """Per-call sampling configuration; fields and defaults of ``engine/talker_sampler.py:34-51``."""

    temperature: float = 0.8
    top_p: float = 0.85
    top_k: int = 25
    repetition_penalty: float = 1.05
    window: int = 16
    min_new_tokens: int = 50
    max_new_tokens: int = 2048
    min_keep: int = 3
    # ``hf``: MiniCPM-o's transformers order; ``omni``: vLLM-Omni order (top-k before top-p, keep >= 1,
    # filters on frame zero too)
    semantics: str = "hf"
    # ``auto``: native per-request generators for omni, counter RNG for hf; ``counter`` batches the omni draw
    rng: str = "auto"

    @property
    def uses_native_rng(self) -> bool:
        if self.rng not in ("auto", "native", "counter"):
            raise ValueError(f"unknown Talker RNG mode: {self.rng!r}")
        return self.rng == "native" or (self.rng == "auto" and self.semantics == "omni")


@dataclass(frozen=True)
class RowParams:
    """Per-row parameters for a batch whose rows differ (CUDA tensors of length B; None = use the cfg).
    ``repetition_penalty`` is a host sequence (the factor table is built from it on the CPU)."""

    temperature: Optional[torch.Tensor] = None  # float32
    top_p: Optional[torch.Tensor] = None        # float32
    top_k: Optional[torch.Tensor] = None        # int32
    repetition_penalty: Optional[Sequence[float]] = None
    max_top_k: int = 0                          # host bound on every row's top_k; required with ``top_k``
    min_new_tokens: Optional[torch.Tensor] = None  # int64: EOS masked while steps < min_new_tokens
    max_new_tokens: Optional[torch.Tensor] = None  # int64: EOS forced once steps >= max_new_tokens - 1


# ---------------------------------------------------------------- helpers

def _need_cuda(*ts) -> None:
    for t in ts:
        if isinstance(t, torch.Tensor) and not t.is_cuda:
            raise ValueError("b2s sampler tensors must be CUDA tensors (this engine has no CPU path)")


def _sem(cfg) -> int:
    if cfg.semantics not in ("hf", "omni"):
        raise ValueError(f"unknown Talker sampling semantics: {cfg.semantics!r}")
    return SEM_HF if cfg.semantics == "hf" else SEM_OMNI


def _temperature(t: float) -> float:
    if not (t > 0.0):
        raise ValueError(f"temperature must be > 0 for sampling, got {t!r}")
    return float(t)


_alpha_cache: dict = {}


def alpha_table(penalty, length: int, device) -> torch.Tensor:
    """``penalty ** n`` for n in [0, length) as the reference computes it (``talker_sampler.py:83``: CPU
    ``torch.pow`` in fp32, which is not correctly rounded, hence taken from torch itself), cached per device.
    ``penalty`` may be a float or a per-row sequence (-> [rows, length])."""
    device = torch.device(device)
    if isinstance(penalty, (list, tuple)):
        key = (tuple(float(p) for p in penalty), int(length), device)
    else:
        key = (float(penalty), int(length), device)
    t = _alpha_cache.get(key)
    if t is None:
        n = torch.arange(length, dtype=torch.float32)
        if isinstance(penalty, (list, tuple)):
            cpu = torch.stack([torch.pow(torch.full_like(n, float(p)), n) for p in penalty])
        else:
            cpu = torch.pow(torch.full_like(n, float(penalty)), n)
        t = cpu.to(device)
        _alpha_cache[key] = t
    return t


def _k_bound(cfg_top_k: int, min_keep: int, rp: Optional[RowParams]) -> int:
    """The launch's bound on k = max(top_k, min_keep) over its rows (it sizes the kernel's on-chip lists).
    A per-row ``top_k`` tensor needs ``RowParams.max_top_k``: reading the bound off the tensor would
    synchronise with the device, and a row above the bound would only come back as PAD."""
    kb = max(int(cfg_top_k), int(min_keep), 1)
    if rp is not None and rp.top_k is not None and not rp.max_top_k:
        raise ValueError("RowParams.top_k needs RowParams.max_top_k, a host bound on every row's top_k")
    if rp is not None and rp.max_top_k:
        kb = max(kb, int(rp.max_top_k), int(min_keep))
    return kb


def _run(logits, *, history=None, steps=None, seeds=None, requests=None, uniform_values=None, active=None,
         finished=None, rp: Optional[RowParams] = None, alpha=None, status=None, temperature=1.0, top_p=1.0, top_k=1,
         min_keep=1, min_new=0, max_new=NEVER, presence=0.0, frequency=0.0, eos=-1, semantics=SEM_OMNI,
         rng=RNG_COUNTER, max_top_k=0, flags=0, tokens=True, processed=False, state=False, cluster=0):
    return _native.ops().sample(
        logits, history, steps, seeds, requests, uniform_values, active, finished,
        None if rp is None else rp.temperature, None if rp is None else rp.top_p, None if rp is None else rp.top_k,
        None if rp is None else _i64(rp.min_new_tokens), None if rp is None else _i64(rp.max_new_tokens),
        alpha, status, float(temperature), float(top_p), int(top_k), int(min_keep), int(min_new), int(max_new),
        float(presence), float(frequency), int(eos), int(semantics), int(rng), int(max_top_k), int(flags),
        bool(tokens), bool(processed), bool(state), int(cluster))


def _i64(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if t is None else t.to(torch.int64)


def _cfg_kwargs(cfg: TalkerSampling, history: Optional[torch.Tensor], device, rp: Optional[RowParams] = None) -> dict:
    sem = _sem(cfg)
    min_keep = cfg.min_keep if sem == SEM_HF else 1
    W = 0 if history is None else history.shape[-1]
    pens = rp.repetition_penalty if rp is not None and rp.repetition_penalty is not None else None
    alpha = alpha_table(list(pens) if pens is not None else cfg.repetition_penalty, W + 1, device) if W > 0 else None
    return dict(alpha=alpha, temperature=_temperature(cfg.temperature), top_p=cfg.top_p, top_k=cfg.top_k,
                min_keep=min_keep, min_new=cfg.min_new_tokens, max_new=cfg.max_new_tokens, semantics=sem,
                max_top_k=_k_bound(cfg.top_k, min_keep, rp), rp=rp)


# ---------------------------------------------------------------- reference-named API

def uniform(seeds: torch.Tensor, steps: torch.Tensor) -> torch.Tensor:
    """U[0, 1) per row from (seed, frame index): the reference counter hash (``talker_sampler.py:60-76``).
    Broadcasts like the reference (e.g. ``seeds[None, :]`` with ``steps[:, None]``)."""
    _need_cuda(seeds, steps)
    s, t = torch.broadcast_tensors(seeds.to(torch.int64), steps.to(torch.int64))
    out = _native.ops().uniform(s.contiguous().reshape(-1), t.contiguous().reshape(-1), None, RNG_COUNTER)
    return out.reshape(s.shape)


def philox_uniform(seeds: torch.Tensor, steps: torch.Tensor, requests: Optional[torch.Tensor] = None) -> torch.Tensor:
    """U[0, 1) from Philox4x32-10 keyed by the seed, counter (step, request)."""
    _need_cuda(seeds, steps, requests)
    if requests is None:
        s, t = torch.broadcast_tensors(seeds.to(torch.int64), steps.to(torch.int64))
        q = None
    else:
        s, t, q = torch.broadcast_tensors(seeds.to(torch.int64), steps.to(torch.int64), requests.to(torch.int64))
        q = q.contiguous().reshape(-1)
    out = _native.ops().uniform(s.contiguous().reshape(-1), t.contiguous().reshape(-1), q, RNG_PHILOX)
    return out.reshape(s.shape)


def repetition_penalty(x: torch.Tensor, history: torch.Tensor, penalty: float) -> torch.Tensor:
    """``history``: [B, W] previous frames (most recent last), ``PAD`` where empty; a token seen n times is
    multiplied by ``penalty**n`` when negative and divided by it otherwise (``talker_sampler.py:79-84``)."""
    _need_cuda(x, history)
    return _native.ops().repetition_penalty(x, history, alpha_table(float(penalty), history.shape[-1] + 1, x.device))


def top_p_filter(x: torch.Tensor, top_p: float, min_keep: int) -> torch.Tensor:
    """The two-pass nucleus filter over the fully sorted row (``talker_sampler.py:87-92``): drop the
    ascending prefix whose cumulative softmax mass is <= 1 - top_p, never the last ``min_keep``.

    The reference keeps this form only as the test oracle of the fused filters; it is kept here as the
    same device torch ops (sort, softmax, cumsum, scatter) and is not on the sampling path, which uses the
    fused kernels.  Where values tie across the cut, which copies survive follows the sort's order."""
    _need_cuda(x)
    s, idx = torch.sort(x, descending=False, dim=-1)
    cum = s.softmax(dim=-1).cumsum(dim=-1)
    remove = cum <= (1 - top_p)
    remove[..., -min_keep:] = False
    return x.masked_fill(remove.scatter(1, idx, remove), float("-inf"))


def top_k_filter(x: torch.Tensor, top_k: int, min_keep: int) -> torch.Tensor:
    """Keep values >= the k-th largest, k = min(max(top_k, min_keep), V) (``talker_sampler.py:95-98``)."""
    _need_cuda(x)
    k = max(int(top_k), int(min_keep))
    out = _run(x, steps=torch.ones(x.shape[0], dtype=torch.int64, device=x.device), top_k=k, min_keep=k,
               semantics=SEM_OMNI, max_top_k=k, flags=FLAG_TOPK_ONLY, tokens=False, processed=True)
    return out[1]


def top_p_top_k_filter(x: torch.Tensor, top_p: float, top_k: int, min_keep: int) -> torch.Tensor:
    """HF order on already-scaled logits: top-p over the full-row normaliser (min_keep), then top-k
    (``talker_sampler.py:101-116``)."""
    _need_cuda(x)
    out = _run(x, steps=torch.ones(x.shape[0], dtype=torch.int64, device=x.device), top_p=top_p, top_k=top_k,
               min_keep=min_keep, semantics=SEM_HF, max_top_k=max(int(top_k), int(min_keep)), tokens=False,
               processed=True)
    return out[1]


def top_k_top_p_filter(x: torch.Tensor, top_k: int, top_p: float, min_keep: int = 1) -> torch.Tensor:
    """vLLM order: top-k, then top-p over the top-k softmax (``talker_sampler.py:119-133``)."""
    _need_cuda(x)
    out = _run(x, steps=torch.ones(x.shape[0], dtype=torch.int64, device=x.device), top_p=top_p, top_k=top_k,
               min_keep=min_keep, semantics=SEM_OMNI, max_top_k=max(int(top_k), int(min_keep)), tokens=False,
               processed=True)
    return out[1]


def processed_logits(logits: torch.Tensor, history: torch.Tensor, steps: torch.Tensor, eos: int,
                     cfg: TalkerSampling, *, row_params: Optional[RowParams] = None) -> torch.Tensor:
    """The [B, V] fp32 logits after the HF or vLLM-Omni contract (``talker_sampler.py:136-158``)."""
    _need_cuda(logits, history, steps)
    kw = _cfg_kwargs(cfg, history, logits.device, row_params)
    return _run(logits, history=history, steps=steps.to(torch.int64), eos=eos, tokens=False, processed=True, **kw)[1]


def draw(x: torch.Tensor, seeds: torch.Tensor, steps: torch.Tensor, *,
         uniform_values: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax -> cumsum in vocabulary order -> first index whose cdf exceeds ``u * cdf[-1]``, clamped to
    V - 1 (``talker_sampler.py:161-172``); ``u`` from the counter hash or ``uniform_values``."""
    _need_cuda(x, seeds, steps, uniform_values)
    if uniform_values is not None:
        return _run(x, steps=steps.to(torch.int64), uniform_values=uniform_values.to(torch.float32).contiguous(),
                    semantics=SEM_IDENTITY, rng=RNG_UNIFORM)[0]
    return _run(x, steps=steps.to(torch.int64), seeds=seeds.to(torch.int64), semantics=SEM_IDENTITY,
                rng=RNG_COUNTER)[0]


def draw_multinomial(x: torch.Tensor, generators: list) -> torch.Tensor:
    """One native ``torch.multinomial`` draw from each row's generator (``talker_sampler.py:175-188``).

    This is the vLLM-Omni RNG contract: one independently seeded generator per request, so it stays a
    per-row torch call on the device (a batched kernel cannot reproduce torch's generator streams)."""
    if len(generators) != x.size(0):
        raise ValueError(f"expected {x.size(0)} generators, got {len(generators)}")
    probs = torch.softmax(x, dim=-1)
    return torch.stack([torch.multinomial(probs[i], 1, generator=generators[i]).reshape(()) for i in range(x.size(0))])


def restore_multinomial_states_after_block(generators: list, states_after_step: list, host_tokens: torch.Tensor) -> None:
    """Rewind each row's generator to its state after the row's last non-PAD draw of a K block
    (``talker_sampler.py:191-212``): rows keep decoding masked after EOS, but a native generator may only
    advance through the EOS draw."""
    if not states_after_step:
        return
    if len(generators) != host_tokens.size(1):
        raise ValueError("generator/token row mismatch")
    steps_in_block = len(states_after_step)
    for row, gen in enumerate(generators):
        col = host_tokens[:, row]
        pad_at = (col == PAD).nonzero()
        draws = int(pad_at[0]) if pad_at.numel() else host_tokens.size(0)
        if 0 < draws < steps_in_block:
            gen.set_state(states_after_step[draws - 1][row])


@dataclass
class DecodeState:
    """Per-row Talker sampling state (``talker_sampler.py:215-231``): frame index, last ``window`` frames,
    finished flag, active flag, optional native generators."""

    seeds: torch.Tensor  # [B] int64
    steps: torch.Tensor  # [B] int64, next frame index
    history: torch.Tensor  # [B, W] int64, PAD where empty
    finished: torch.Tensor  # [B] bool
    active: torch.Tensor  # [B] bool
    generators: Optional[list] = None

    @classmethod
    def new(cls, seeds: list, cfg: TalkerSampling = TalkerSampling(), device="cpu") -> "DecodeState":
        """The reference's constructor and default device (``talker_sampler.py:226-231``); the sampling
        entry points of this engine need the state on a CUDA device, so callers pass ``device``."""
        b = len(seeds)
        return cls(seeds=torch.tensor(seeds, dtype=torch.int64, device=device),
                   steps=torch.zeros(b, dtype=torch.int64, device=device),
                   history=torch.full((b, cfg.window), PAD, dtype=torch.int64, device=device),
                   finished=torch.zeros(b, dtype=torch.bool, device=device),
                   active=torch.ones(b, dtype=torch.bool, device=device))


def step(state: DecodeState, logits: torch.Tensor, eos: int, cfg: TalkerSampling = TalkerSampling()) -> torch.Tensor:
    """Sample one frame per row and advance the state (``talker_sampler.py:234-249``): inactive or finished
    rows return ``PAD`` and keep their state.  Like the reference, the new history / steps / finished are
    fresh tensors bound to ``state`` (callers may hold views of the old ones)."""
    _need_cuda(logits, state.history, state.steps, state.seeds)
    if cfg.uses_native_rng:
        if state.generators is None:
            raise ValueError("native Talker RNG requires one generator per row")
        live = state.active & ~state.finished
        tok = draw_multinomial(processed_logits(logits, state.history, state.steps, eos, cfg), state.generators)
        tok = torch.where(live, tok, torch.full_like(tok, PAD))
        shifted = torch.cat([state.history[:, 1:], tok[:, None]], dim=1)
        state.history = torch.where(live[:, None], shifted, state.history)
        state.steps = state.steps + live.to(torch.int64)
        state.finished = state.finished | (live & (tok == eos))
        return tok
    kw = _cfg_kwargs(cfg, state.history, logits.device)
    tok, _, hist, steps, fin = _run(logits, history=state.history, steps=state.steps, seeds=state.seeds,
                                    active=state.active, finished=state.finished, eos=eos, rng=RNG_COUNTER,
                                    tokens=True, state=True, **kw)
    if state.history.shape[-1] > 0:
        state.history = hist
    state.steps, state.finished = steps, fin
    return tok


def decode_k(state: DecodeState, logits_k: torch.Tensor, eos: int, cfg: TalkerSampling = TalkerSampling()) -> torch.Tensor:
    """K frames from precomputed per-frame logits [K, B, V]: identical to K calls of ``step``
    (``talker_sampler.py:252-254``); an EOS freezes its row.  One launch runs all K frames (each row's frames in
    order on one CTA, the next frame's logits in flight under the current draw); the new history / steps /
    finished are fresh tensors bound to ``state``, as K ``step`` calls would leave them.  The native-generator
    mode keeps the reference's per-frame torch calls."""
    if cfg.uses_native_rng:
        return torch.stack([step(state, logits_k[i], eos, cfg) for i in range(logits_k.size(0))])
    hist, steps, fin = state.history.clone(), state.steps.clone(), state.finished.clone()
    tok = _frames(logits_k, hist, steps, fin, state.seeds, state.active, eos, cfg, None, None)
    if state.history.shape[-1] > 0:
        state.history = hist
    state.steps, state.finished = steps, fin
    return tok


def decode_k_(state: DecodeState, logits_k: torch.Tensor, eos: int, cfg: TalkerSampling = TalkerSampling(), *,
              uniform_values: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``decode_k`` advancing ``state.history`` / ``steps`` / ``finished`` IN PLACE (the K-frame graph body of
    ``engine/runtime/talker_decode.py:120-128``, ``talker_block_graph.py:70-89``); returns the [K, B] tokens.
    ``uniform_values``: [K, B] injected uniforms instead of the counter RNG."""
    if cfg.uses_native_rng:
        raise ValueError("decode_k_ needs the counter RNG or injected uniforms")
    return _frames(logits_k, state.history, state.steps, state.finished, state.seeds, state.active, eos, cfg,
                   uniform_values, status)


def _frames(logits_k, hist, steps, fin, seeds, active, eos, cfg, uniform_values, status) -> torch.Tensor:
    _need_cuda(logits_k, hist, steps, fin, seeds, active, uniform_values)
    kw = _cfg_kwargs(cfg, hist, logits_k.device)
    r = RNG_UNIFORM if uniform_values is not None else RNG_COUNTER
    u = None if uniform_values is None else uniform_values.to(torch.float32).contiguous()
    return _native.ops().sample_frames_(
        logits_k, hist, steps, fin, seeds, u, active, kw["alpha"], status, None, None, None, kw["temperature"],
        float(cfg.top_p), int(cfg.top_k), int(kw["min_keep"]), int(cfg.min_new_tokens), int(cfg.max_new_tokens),
        int(eos), int(kw["semantics"]), r, int(kw["max_top_k"]))


# ---------------------------------------------------------------- fused / in-place entry points

def sample(logits: torch.Tensor, history: Optional[torch.Tensor], steps: torch.Tensor, seeds: Optional[torch.Tensor],
           eos: int, cfg: TalkerSampling, *, uniform_values: Optional[torch.Tensor] = None, rng: str = "counter",
           requests: Optional[torch.Tensor] = None, active: Optional[torch.Tensor] = None,
           finished: Optional[torch.Tensor] = None, row_params: Optional[RowParams] = None,
           status: Optional[torch.Tensor] = None, cluster: int = 0) -> torch.Tensor:
    """``draw(processed_logits(...))`` in one kernel: [B] int64 tokens (PAD for rows that are not live).
    ``rng``: ``counter`` (reference hash), ``philox`` (Philox4x32-10 keyed by (seed, step, request)); ignored
    when ``uniform_values`` is given."""
    _need_cuda(logits, history, steps, seeds, uniform_values, requests, active, finished)
    kw = _cfg_kwargs(cfg, history, logits.device, row_params)
    if uniform_values is not None:
        r = RNG_UNIFORM
        uniform_values = uniform_values.to(torch.float32).contiguous()
    else:
        r = {"counter": RNG_COUNTER, "philox": RNG_PHILOX}[rng]
    return _run(logits, history=history, steps=_i64(steps), seeds=_i64(seeds), requests=_i64(requests),
                uniform_values=uniform_values, active=active, finished=finished, status=status, eos=eos, rng=r,
                cluster=cluster, **kw)[0]


def step_(state: DecodeState, logits: torch.Tensor, eos: int, cfg: TalkerSampling = TalkerSampling(), *,
          uniform_values: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``step`` that advances ``state.history`` / ``steps`` / ``finished`` IN PLACE (the form captured graph
    bodies use, ``engine/runtime/talker_post_graph.py:56-76``); returns the [B] tokens."""
    _need_cuda(logits, state.history, state.steps)
    if cfg.uses_native_rng:
        raise ValueError("step_ needs the counter RNG or injected uniforms")
    kw = _cfg_kwargs(cfg, state.history, logits.device)
    r = RNG_UNIFORM if uniform_values is not None else RNG_COUNTER
    return _native.ops().sample_state_(
        logits, state.history, state.steps, state.finished, state.seeds,
        None if uniform_values is None else uniform_values.to(torch.float32).contiguous(), state.active, kw["alpha"],
        status, None, None, None, kw["temperature"], float(cfg.top_p), int(cfg.top_k), int(kw["min_keep"]),
        int(cfg.min_new_tokens), int(cfg.max_new_tokens), int(eos), int(kw["semantics"]), r, int(kw["max_top_k"]), 0)


class CodecHead:
    """The Talker's codec head and the decode step in ONE launch: ``F.linear(hidden, head)`` on the tensor cores
    (bf16 operands, fp32 accumulation, logits rounded to bf16 like F.linear's bf16 output), then ``step_`` on
    those logits -- the graph body of ``engine/runtime/talker_post_graph.py:56-76`` (``F.linear(st["hidden"],
    self.head).float()``, ``processed_logits``, ``draw``, the state update) and the head + sampler of
    ``engine/runtime/talker_decode.py:120-128``.

    Holds the head (``[vocab, hidden]`` bf16, as ``engine/models/talker.py:106-109`` builds it), the ``[rows,
    vocab]`` bf16 logits buffer the launch writes (kept for inspection: ``self.logits``) and 4 int32 control words
    (``self.sync``).  One instance per stream: launches that share the control words must not overlap.  The head
    is read while the stream's previous kernel may still run, so that kernel must not write it.  Limits: rows <= 16,
    hidden a multiple of 64 up to 768."""

    def __init__(self, head: torch.Tensor, rows: int):
        _need_cuda(head)
        if head.dtype != torch.bfloat16 or head.dim() != 2:
            raise ValueError("head must be a bf16 [vocab, hidden] tensor")
        self.head = head.contiguous()
        self.rows = int(rows)
        self.logits = torch.empty(self.rows, head.shape[0], dtype=torch.bfloat16, device=head.device)
        self.sync = torch.zeros(4, dtype=torch.int32, device=head.device)

    def step_(self, state: DecodeState, hidden: torch.Tensor, eos: int, cfg: TalkerSampling = TalkerSampling(), *,
              uniform_values: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None,
              row_params: Optional[RowParams] = None, rng: str = "counter") -> torch.Tensor:
        """One frame per row from ``hidden`` ([rows, hidden] bf16): advances ``state`` IN PLACE like ``step_``
        and returns the [rows] tokens (PAD for rows that are not live).  ``rng``: ``counter`` (reference hash)
        or ``philox``; ignored when ``uniform_values`` is given."""
        _need_cuda(hidden, state.history, state.steps)
        if hidden.dim() != 2 or hidden.shape[0] != self.rows or hidden.dtype != torch.bfloat16:
            raise ValueError(f"hidden must be bf16 [{self.rows}, hidden]")
        if cfg.uses_native_rng:
            raise ValueError("CodecHead.step_ needs the counter / Philox RNG or injected uniforms")
        rp = row_params
        if rp is not None and (rp.min_new_tokens is not None or rp.max_new_tokens is not None):
            raise ValueError("CodecHead.step_ takes per-row temperature / top_p / top_k / penalty only")
        kw = _cfg_kwargs(cfg, state.history, hidden.device, rp)
        if uniform_values is not None:
            r = RNG_UNIFORM
            uniform_values = uniform_values.to(torch.float32).contiguous()
        else:
            r = {"counter": RNG_COUNTER, "philox": RNG_PHILOX}[rng]
        return _native.ops().head_sample_state_(
            hidden, self.head, self.logits, self.sync, state.history, state.steps, state.finished, state.seeds,
            uniform_values, state.active, kw["alpha"], status, None if rp is None else rp.temperature,
            None if rp is None else rp.top_p, None if rp is None else rp.top_k, kw["temperature"], float(cfg.top_p),
            int(cfg.top_k), int(kw["min_keep"]), int(cfg.min_new_tokens), int(cfg.max_new_tokens), int(eos),
            int(kw["semantics"]), r, int(kw["max_top_k"]))


FLAG_TOPK_ONLY = 2


# the name the reference's captured graph bodies call (engine/runtime/talker_decode.py:29-31)
processed_logits_static = processed_logits
