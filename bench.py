"""Benchmark of the fused sampling step (sampled rows/s; % of the HBM roofline; CPU baseline beside it).

Workload (default ``thinker``): Thinker text sampling on a Qwen3-8B-sized head, the configuration the
north-star target is quoted on (B >= 64, V = 151,936 on one B200): per GPU B = 64 rows of bf16 logits
(Zipf(1.1) rank profile + N(0,1), permuted per row), temperature 0.7, top-k 20, top-p 0.8, count-based
repetition penalty 1.05 over a 512-token history, omni order, Philox4x32-10 uniforms keyed by
(seed = row, step).  One step = one launch of the fused kernel over the batch: penalties, temperature,
top-k, top-p, draw, and the in-place history / step update.  Synthetic data, generated on the host.

``--gpus N`` (under torchrun): every rank runs its own B rows (row sharding, no collective on the data
path; ``scaling`` = weak); timing is the max over ranks, and ``value`` is the whole job's rows/s
(``value_per_gpu`` beside it).  ``--impl reference`` times the reference's own sampler
(``engine/talker_sampler.py``: ``processed_logits`` + ``draw`` under CPU torch on every host core, loaded
from the bytecode that ``oracle/ref_build.py`` compiles into ``oracle/_ref``) on the same workload; the C
restatement of the oracle is timed beside it as a second CPU figure.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # name: rows per GPU, vocab, dtype, window, temperature, top_k, top_p, penalty
    "thinker": dict(rows=64, vocab=151_936, dtype="bf16", window=512, temperature=0.7, top_k=20, top_p=0.8,
                    penalty=1.05),
    "large": dict(rows=1024, vocab=151_936, dtype="f32", window=2048, temperature=1.0, top_k=50, top_p=0.95,
                  penalty=1.1),
    # batched Talker at streaming concurrency -- per-row T / k / p (row i takes index i mod 3),
    # EOS (the last column) masked for the first 8 steps, rows shifted by U(-1, 1)
    "talker": dict(rows=8, vocab=6562, dtype="bf16", window=64, temperature=0.8, top_k=25, top_p=0.85, penalty=1.05,
                   order="hf", min_keep=3, eos=6561, min_new=8, row_temperature=(0.6, 0.8, 1.0),
                   row_top_k=(20, 25, 50), row_top_p=(0.7, 0.85, 0.95)),
    # BASELINE config 2 decoded K = 16 frames per launch (the K-frame device block of decode_k): a step is 16 frames
    "talker_k": dict(rows=8, vocab=6562, dtype="bf16", window=64, temperature=0.8, top_k=25, top_p=0.85, penalty=1.05,
                     order="hf", min_keep=3, eos=6561, min_new=8, row_temperature=(0.6, 0.8, 1.0),
                     row_top_k=(20, 25, 50), row_top_p=(0.7, 0.85, 0.95), frames=16),
    # BASELINE config 2's batch from the Talker's codec head (hidden 768): the bf16 head GEMM and the step in one
    # launch (talker_post_graph.py:58-63); a step reads the whole 6562 x 768 head
    "talker_head": dict(rows=8, vocab=6562, dtype="bf16", window=64, temperature=0.8, top_k=25, top_p=0.85,
                        penalty=1.05, order="hf", min_keep=3, eos=6561, min_new=8, row_temperature=(0.6, 0.8, 1.0),
                        row_top_k=(20, 25, 50), row_top_p=(0.7, 0.85, 0.95), hidden=768, op="head"),
    # the single-stream Talker (one row, fp32, hf order, 16-token history)
    "talker1": dict(rows=1, vocab=6562, dtype="f32", window=16, temperature=0.8, top_k=25, top_p=0.85, penalty=1.05,
                    order="hf", min_keep=3, eos=6561, min_new=0),
    # vocabulary-sharded Thinker head -- each rank holds V / N contiguous columns; per-shard
    # candidates, one NCCL all-gather, the merged draw on every rank.  Tie-heavy bf16 logits (multiples of 1/16)
    "vocab_shard": dict(rows=256, vocab=151_936, dtype="bf16", window=0, temperature=0.8, top_k=64, top_p=0.9,
                        penalty=1.0, op="vocab_shard"),
    # the Thinker greedy step from its LM head (hidden 4096, a 151,936 x 4096 bf16 head): the GEMM and the argmax in
    # one launch, the logits never written (thinker_decode.py:83,107)
    "greedy_head": dict(rows=64, vocab=151_936, dtype="bf16", window=0, temperature=0.0, top_k=1, top_p=1.0,
                        penalty=1.0, hidden=4096, op="lmhead"),
    # the Thinker greedy step (argmax over the head's logits, first index on ties) on the thinker shape
    "greedy": dict(rows=64, vocab=151_936, dtype="bf16", window=0, temperature=0.0, top_k=1, top_p=1.0, penalty=1.0,
                   op="argmax"),
}
L2_BYTES = 126 * 1024 * 1024


def bytes_per_row(w) -> float:
    """Algorithmic bytes of one sampled row: logits read once, history ids as int32, 40 B params/state/token.
    From the codec head: the head read once per step (its share per row), the row's hidden instead of logits
    (which stay on chip and in L2)."""
    if w.get("op") == "head":
        return w["vocab"] * w["hidden"] * 2 / w["rows"] + 2 * w["hidden"] + 4 * w["window"] + 40
    if w.get("op") == "lmhead":
        return w["vocab"] * w["hidden"] * 2 / w["rows"] + 2 * w["hidden"] + 8
    e = 2 if w["dtype"] == "bf16" else 4
    return w["vocab"] * e + 4 * w["window"] + 40


def head_operands(w, rows: int, seed: int):
    """Hidden rows [rows, H] and a head [V, H] (fp32 arrays holding bf16 values): logits ~ N(0, 2); hidden
    column 0 is 8 and the EOS row's entry there -4, so that EOS stays far below the rest and rows stay live."""
    from tests.golden import inputs as I

    g = I.rng(seed)
    H, V = w["hidden"], w["vocab"]
    hid = g.standard_normal((rows, H)).astype(np.float32)
    hid[:, 0] = 8.0
    head = (g.standard_normal((V, H)) * (2.0 / H ** 0.5)).astype(np.float32)
    if w.get("eos", -1) >= 0:
        head[w["eos"], 0] = -4.0
    bf = lambda a: I.bf16_bits_to_f32(I.to_bf16_bits(a))
    return bf(hid), bf(head)


def make_inputs(w, rows: int, seed: int):
    """Host arrays of one batch: logits (fp32 values, bf16-rounded for bf16), history, seeds."""
    from tests.golden import inputs as I

    g = I.rng(seed)
    if w.get("op") == "vocab_shard":
        return I.quantised_rows(g, rows, w["vocab"], sigma=2.0, q=16), np.zeros((rows, 0), np.int64)
    if w["vocab"] == 151_936 and w["dtype"] == "bf16":
        logits, hist = I.zipf_rows(g, rows, w["vocab"], w["window"])
    elif w.get("order") == "hf":  # Talker: N(0, 2); several rows also get a per-row shift U(-1, 1)
        logits = (g.standard_normal((rows, w["vocab"])) * 2.0).astype(np.float32)
        if rows > 1:
            logits += g.uniform(-1.0, 1.0, size=(rows, 1)).astype(np.float32)
        hist = g.integers(0, w["vocab"], size=(rows, w["window"]))
    else:
        logits = (g.standard_normal((rows, w["vocab"])) * 3.0).astype(np.float32)
        hist = g.integers(0, w["vocab"], size=(rows, w["window"]))
    if w.get("eos", -1) >= 0:
        # the EOS column stays far below the rest, so that rows stay live over any number of steps (its masking
        # and forcing rules still run every step)
        logits[:, w["eos"]] = -30.0
    if w["dtype"] == "bf16":
        logits = I.bf16_bits_to_f32(I.to_bf16_bits(logits))
    return logits, hist.astype(np.int64)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_gbs():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def profiled_traffic(workload: str, w, path: str = "auto") -> float | None:
    """DRAM bytes per launch of the workload's kernel from the committed ncu summary, or None (the summary of the
    kernel the launcher picks for the workload first: short-row, row-resident, then streaming)."""
    kernels = ["argmax_kernel"] if w.get("op") == "argmax" else ["head_kernel"] if w.get("op") == "head" else \
        ["lmhead_argmax_kernel"] if w.get("op") == "lmhead" else (
        ["sample_kernel"] if path == "stream" else ["resident_kernel"] if path == "resident" else
        ["short_kernel", "resident_kernel", "sample_kernel"])
    for kernel in kernels:
        f = ROOT / "profiles" / f"{kernel}_{workload}.md"
        if f.exists():
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
            return float(m.group(1)) if m else None
    return None


def cpu_baseline(w, seconds: float = 10.0, threads: int = 0) -> dict:
    """The CPU oracle (reference algorithm in C, OpenMP over rows) on rows of the same workload."""
    from oracle import oracle as orc
    from tests.golden import inputs as I

    threads = threads or len(os.sched_getaffinity(0))
    rows = min(w["rows"], 64)
    logits, hist = make_inputs(w, rows, 1234)
    x = I.to_bf16_bits(logits) if w["dtype"] == "bf16" else logits
    cfg = orc.Cfg(temperature=w["temperature"], top_p=w["top_p"], top_k=w["top_k"], repetition_penalty=w["penalty"],
                  window=w["window"], min_new_tokens=w.get("min_new", 0), max_new_tokens=1 << 40,
                  min_keep=w.get("min_keep", 1), semantics=w.get("order", "omni"))
    rowkw = {}
    if "row_temperature" in w:
        rowkw = dict(row_temperature=np.array([w["row_temperature"][i % 3] for i in range(rows)], np.float32),
                     row_top_p=np.array([w["row_top_p"][i % 3] for i in range(rows)], np.float32),
                     row_top_k=np.array([w["row_top_k"][i % 3] for i in range(rows)], np.int32))
    seeds = np.arange(rows, dtype=np.int64)
    head = w.get("op") == "head"
    if head:  # the head's matmul in fp32 (numpy), rounded to bf16, inside every step
        hid, hw = head_operands(w, rows, 1234)
        logits_of = lambda: I.to_bf16_bits(hid @ hw.T)
        x = logits_of()
    if w.get("op") == "argmax":
        orc.argmax(x)
        done, t0, step = 0, time.perf_counter(), 0
        while True:
            orc.argmax(x)
            done += rows
            step += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        return {"value": done / el, "unit": "rows/s", "cores": 1, "kind": "port",
                "sample": f"{step} x {rows} rows argmax (oracle/sampler_oracle.c, one thread)"}
    # one untimed call: loads the library and builds the penalty table
    eos = w.get("eos", -1)
    orc.sample(x, hist, np.ones(rows, np.int64), seeds, eos, cfg, rng=orc.RNG_PHILOX, requests=np.zeros(rows, np.int64),
               want_processed=False, threads=threads, **rowkw)
    done = 0
    t0 = time.perf_counter()
    step = 0
    while True:
        if head:
            x = logits_of()
        orc.sample(x, hist, np.full(rows, step + 1, np.int64), seeds, eos, cfg, rng=orc.RNG_PHILOX,
                   requests=np.zeros(rows, np.int64), want_processed=False, threads=threads, **rowkw)
        done += rows
        step += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": done / el, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{step} steps x {rows} rows of the {w['vocab']}-vocab workload in {el:.1f} s "
                      f"({'numpy fp32 head matmul + ' if head else ''}oracle/sampler_oracle.c, OpenMP)"}


def reference_cpu(w, *, steps: int = 0, warmup: int = 1, seconds: float = 10.0, threads: int = 0) -> dict:
    """The reference's own sampler on the host cores: ``engine/talker_sampler.py`` imported unchanged from
    its bytecode in ``oracle/_ref`` (``oracle/ref_build.py``), ``processed_logits`` + ``draw`` (counter RNG)
    under CPU torch with every host thread; the greedy workload times the reference's
    ``logits.float().argmax(-1)`` tail (``engine/runtime/thinker_decode.py:107``).  Each step is one batch
    of at most 64 rows of the workload; ``steps`` > 0 times exactly that many steps, else as many as fit
    in ``seconds``.  Rows whose configs differ (the batched Talker) run as one call per distinct config,
    as a reference caller would."""
    import torch

    from oracle import ref_build

    ref = ref_build.load()
    threads = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    rows = min(w["rows"], 64)
    logits, hist = make_inputs(w, rows, 1234)
    x = torch.from_numpy(logits)
    if w["dtype"] == "bf16":
        x = x.to(torch.bfloat16)
    h = torch.from_numpy(hist)
    head = w.get("op") == "head"
    if head:  # the reference graph body: F.linear(hidden, head).float() (bf16 operands) before the sampler
        hid, hw = head_operands(w, rows, 1234)
        hid_t, hw_t = torch.from_numpy(hid).to(torch.bfloat16), torch.from_numpy(hw).to(torch.bfloat16)
    seeds = torch.arange(rows, dtype=torch.int64)
    eos = w.get("eos", -1)
    groups = [(list(range(rows)), w["temperature"], w["top_k"], w["top_p"])]
    if "row_temperature" in w:
        groups = [([r for r in range(rows) if r % 3 == j], w["row_temperature"][j], w["row_top_k"][j],
                   w["row_top_p"][j]) for j in range(3)]
    cfgs = [(torch.tensor(idx), ref.TalkerSampling(temperature=T, top_p=p, top_k=k, repetition_penalty=w["penalty"],
                                                   window=w["window"], min_new_tokens=w.get("min_new", 0),
                                                   max_new_tokens=1 << 40, min_keep=w.get("min_keep", 1),
                                                   semantics=w.get("order", "omni"), rng="counter"))
            for idx, T, k, p in groups if idx]

    def one(step: int):
        st = torch.full((rows,), step + 1, dtype=torch.int64)
        if w.get("op") == "argmax":
            return x.float().argmax(-1)
        out = []
        xx = torch.nn.functional.linear(hid_t, hw_t).float() if head else x
        for idx, cfg in cfgs:
            xs, hs, ss = (xx, h, st) if len(cfgs) == 1 else (xx[idx], h[idx], st[idx])
            proc = ref.processed_logits(xs, hs, ss, eos, cfg)
            out.append(ref.draw(proc, seeds[idx], ss))
        return out

    for i in range(max(1, warmup)):
        one(i)
    done, n, t0 = 0, 0, time.perf_counter()
    while True:
        one(n)
        n += 1
        done += rows
        el = time.perf_counter() - t0
        if (steps > 0 and n >= steps) or (steps <= 0 and el >= seconds):
            break
    what = ("logits.float().argmax(-1)" if w.get("op") == "argmax" else
            "F.linear(hidden, head).float() + processed_logits + draw" if head else "processed_logits + draw")
    return {"value": done / el, "unit": "rows/s", "cores": threads, "kind": "reference",
            "sample": f"{n} steps x {rows} rows of the {w['vocab']}-vocab workload in {el:.1f} s "
                      f"(reference engine/talker_sampler.py {what}, CPU torch {torch.__version__}, "
                      f"{threads} threads)"}


def metric_of(w) -> str:
    if w.get("op") == "vocab_shard":
        return (f"sampled rows/s at B={w['rows']} x V={w['vocab']} over the job's vocabulary shards "
                "(per-shard candidates + NCCL all-gather + merged draw)")
    if w.get("op") == "lmhead":
        return (f"greedy rows/s from the LM head, whole job (n_gpus x B={w['rows']} rows per GPU) at V={w['vocab']}, "
                f"hidden {w['hidden']}; per GPU = value_per_gpu (bf16 LM-head GEMM on the tensor cores + argmax, one "
                "launch and a finishing block, logits never written)")
    if w.get("op") == "head":
        return (f"sampled rows/s from the codec head, whole job (n_gpus x B={w['rows']} rows per GPU) at "
                f"V={w['vocab']}, hidden {w['hidden']}; per GPU = value_per_gpu (bf16 head GEMM on the tensor cores "
                "+ fused penalty+temperature+top-k+top-p+draw, one launch)")
    if w.get("op") == "argmax":
        return (f"greedy rows/s, whole job (n_gpus x B={w['rows']} rows per GPU) at V={w['vocab']}; per GPU = "
                "value_per_gpu (argmax, first index on ties)")
    return (f"sampled rows/s, whole job (n_gpus x B={w['rows']} rows per GPU) at V={w['vocab']}; per GPU = "
            "value_per_gpu (fused penalty+temperature+top-k+top-p+draw)")


def dtype_of(w) -> str:
    return "bf16->f32" if w["dtype"] == "bf16" else "f32"


def rotating_buffers(w) -> int:
    """Distinct logits buffers (heads, for the codec head): one sweep exceeds twice the L2 and 640 MiB, at most
    8192 buffers (the single-row Talker's 26 KB rows: 215 MB, still larger than the L2)."""
    if w.get("op") == "lmhead":
        return 1  # one head already exceeds the L2
    buf = (w["vocab"] * w["hidden"] * 2 if w.get("op") == "head" else
           w["rows"] * w["vocab"] * (2 if w["dtype"] == "bf16" else 4))
    return max(2, min(8192, math.ceil(max(2 * L2_BYTES, 640 * 2**20) / buf)))


def config_of(args, w, world: int) -> dict:
    """The workload as both arms report it."""
    B, V = w["rows"], w["vocab"]
    nbuf = rotating_buffers(w)
    if getattr(args, "strong", False):
        B //= world
    return {"workload": args.workload, "rows_per_gpu": B, "global_batch": B * world, "vocab": V,
            "logits_dtype": w["dtype"], "window": w["window"], "temperature": w["temperature"], "top_k": w["top_k"],
            "top_p": w["top_p"], "repetition_penalty": w["penalty"], "order": w.get("order", "omni"), "rng": "philox",
            "min_keep": w.get("min_keep", 1), "eos": w.get("eos", -1), "min_new_tokens": w.get("min_new", 0),
            "per_row": {k: list(w[k]) for k in ("row_temperature", "row_top_k", "row_top_p") if k in w} or None,
            "parallelism": f"rows x{world}",
            "l2": (f"{nbuf} rotating heads ({nbuf * V * w['hidden'] * 2 / 2**20:.0f} MiB > L2)"
                   if w.get("op") in ("head", "lmhead")
                   else f"{nbuf} rotating logits buffers "
                        f"({nbuf * B * V * (2 if w['dtype'] == 'bf16' else 4) / 2**20:.0f} MiB > L2)"),
            "hidden": w.get("hidden"),
            "cuda_graph_steps": 0 if args.eager else min(args.steps, 1000), "kernel_path": args.path,
            "cluster": args.cluster, "frames_per_step": w.get("frames", 1)}


def run_vocab_shard(args, w, rank: int, world: int, local: int):
    """the same B rows on every rank, each rank holding a contiguous slice of the
    vocabulary.  A step = shard candidates -> all-gather -> merged draw (identical tokens on every rank).
    Timed eagerly (no CUDA graph holds the collective); whole-job rows/s, max over ranks."""
    import torch
    import torch.distributed as dist

    import __graft_entry__

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    pkg = __graft_entry__.load_package()
    vs, ths = pkg.vocab_shard, pkg.thinker_sampler
    B, V = w["rows"], w["vocab"]
    bounds = vs.shard_bounds(V, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    full, _ = make_inputs(w, B, 2024)  # the same rows on every rank
    shard_bytes = B * (hi - lo) * 2
    nbuf = max(2, min(4096, math.ceil(max(2 * L2_BYTES, 640 * 2**20) / shard_bytes)))
    g = np.random.default_rng(7)  # the same row permutations on every rank
    base = torch.from_numpy(full[:, lo:hi]).to(dev).to(torch.bfloat16)
    bufs = [base[torch.from_numpy(g.permutation(B)).to(dev)].contiguous() for _ in range(nbuf)]
    del base
    cfg = ths.ThinkerSampling(temperature=w["temperature"], top_k=w["top_k"], top_p=w["top_p"], repetition_penalty=1.0,
                              window=0, rng="philox")
    cap = vs.default_cap(cfg)  # per-shard list: every element above the shard's 64th value, ties up to 64
    steps = torch.ones(B, dtype=torch.int64, device=dev)
    seeds = torch.arange(B, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def one_step(x):
        # stage 1 -> all-gather of [B, 2*cap+1] int32 -> stage 2 -> stage 3 -> max-all-reduce of [B] int64
        v, i, n = vs.shard_candidates(x, lo, None, steps, cfg, cap=cap, status=status)
        if world > 1:
            vv, ii, nn = vs.exchange(v, i, n)
        else:
            vv, ii, nn = v[None], i[None], n[None]
        tok, pend = vs.merge(vv, ii, nn, V, steps, seeds, cfg, rng="philox", status=status)
        out = vs.resolve(x, lo, rank, None, steps, cfg, tok, pend, status=status)
        if world > 1:
            dist.all_reduce(out, op=dist.ReduceOp.MAX)
        return out

    for i in range(args.warmup):
        one_step(bufs[i % nbuf])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local].strip() if vis else local)
    clocks.start()
    time.sleep(0.1)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        one_step(bufs[i % nbuf])
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ck = clocks.stop()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ms_per_step = ms / args.steps
    # end to end: the shard's logits from pinned host memory, the tokens back, every step
    host = torch.from_numpy(full[:, lo:hi]).to(torch.bfloat16).pin_memory()
    dbuf = torch.empty_like(host, device=dev)
    tok_h = torch.empty(B, dtype=torch.int64).pin_memory()
    e2e_steps = max(1, args.e2e_steps)
    for _ in range(2):
        dbuf.copy_(host, non_blocking=True)
        tok_h.copy_(one_step(dbuf), non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record()
    for _ in range(e2e_steps):
        dbuf.copy_(host, non_blocking=True)
        tok_h.copy_(one_step(dbuf), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    et = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    bad = int(status.item())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    per_gpu_bytes = B * ((hi - lo) * 2 + 40)
    peak, peak_kind = measured_peak_gbs()
    achieved = per_gpu_bytes / (ms_per_step / 1e3) / 1e9
    line = {
        "metric": metric_of(w), "value": B * args.steps / (ms / 1e3), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": dtype_of(w), "data": "synthetic",
        "config": {**config_of(args, w, world), "parallelism": f"vocab x{world}", "shard_columns": hi - lo,
                   "shard_list_cap": cap, "cuda_graph_steps": 0, "value_per_gpu": None},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "bytes_per_gpu_step": per_gpu_bytes, "peak_source": peak_kind},
        "e2e": {"value": B * e2e_steps / (float(et.item()) / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": host.numel() * host.element_size(), "d2h_bytes_per_step": B * 8,
                "steps": e2e_steps},
        "gpu_launches": args.steps * 3, "clocks": ck, "status_flags": bad, "cpu_baseline": None,
        "exchange_bytes_per_rank_step": B * (2 * cap + 1) * 4,
    }
    print(json.dumps(line))


def run_reference(args, w, rank: int):
    """The reference's own sampler on the host cores (``reference_cpu``: K timed steps after W warm-up
    steps, each a batch of at most 64 rows); rank 0 only.  The oracle's C restatement is timed beside it
    (``cpu_baseline_port``).  Without the reference bytecode the port is the baseline, and says so."""
    if rank != 0:
        return
    from oracle import ref_build

    if w.get("op") == "lmhead":  # the reference's greedy step from the LM head, CPU torch (no oracle port of a GEMM)
        cb = lmhead_cpu(w, steps=args.steps, warmup=args.warmup)
        print(json.dumps({"impl": "reference", "metric": metric_of(w), "value": cb["value"], "unit": "rows/s",
                          "value_per_gpu": cb["value"], "n_gpus": args.gpus, "steps": args.steps,
                          "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "bf16", "data": "synthetic", "config": config_of(args, w, args.gpus),
                          "cpu_baseline": cb,
                          "e2e": {"value": cb["value"], "unit": "rows/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return
    port = cpu_baseline(w, seconds=min(args.cpu_seconds, 5.0))
    if ref_build.available():
        cb = reference_cpu(w, steps=args.steps, warmup=args.warmup)
    else:
        cb = dict(port, sample=port["sample"] + "; reference bytecode absent (oracle/ref_build.py not run)")
    line = {"impl": "reference", "metric": metric_of(w), "value": cb["value"], "unit": "rows/s",
            "value_per_gpu": cb["value"], "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_of(w),
            "data": "synthetic", "config": config_of(args, w, args.gpus), "cpu_baseline": cb,
            "cpu_baseline_port": port,
            "e2e": {"value": cb["value"], "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_head(args, w, rank: int, world: int, local: int):
    """The codec head and the step in one launch (``CodecHead``): each step reads a whole head -- one of
    ``rotating_buffers`` distinct copies, so that the heads of a sweep exceed the L2 as the Talker's layer weights
    evict it between two head calls in a decode loop -- and advances the state in place."""
    import torch
    import torch.distributed as dist

    import __graft_entry__

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    pkg = __graft_entry__.load_package()
    ts = pkg.talker_sampler
    B, V, W, Hd = w["rows"], w["vocab"], w["window"], w["hidden"]
    eos = w.get("eos", -1)
    nbuf = rotating_buffers(w)
    hid_h, head_h = head_operands(w, B, 1000 + rank)
    _, hist_h = make_inputs(dict(w, vocab=V, dtype="f32"), B, 1000 + rank)
    head0 = torch.from_numpy(head_h).to(dev).to(torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(rank)
    heads, hiddens = [], []
    hid0 = torch.from_numpy(hid_h).to(dev).to(torch.bfloat16)
    for i in range(nbuf):  # distinct heads: a per-copy permutation of the ids (EOS stays in place)
        perm = torch.randperm(V - 1 if eos >= 0 else V, device=dev, generator=g)
        if eos >= 0:
            perm = torch.cat([perm, torch.tensor([V - 1], device=dev)])
        heads.append(head0[perm].contiguous())
        hiddens.append(torch.cat([hid0[:, :1], torch.roll(hid0[:, 1:], i, dims=1)], dim=1).contiguous())
    del head0
    cfg = ts.TalkerSampling(temperature=w["temperature"], top_p=w["top_p"], top_k=w["top_k"],
                            repetition_penalty=w["penalty"], window=W, min_new_tokens=w.get("min_new", 0),
                            max_new_tokens=1 << 62, min_keep=w.get("min_keep", 1), semantics=w.get("order", "omni"),
                            rng="counter")
    state = ts.DecodeState.new(list(range(rank * B, rank * B + B)), cfg, device=dev)
    state.history.copy_(torch.from_numpy(hist_h).to(dev))
    state.steps.fill_(1)
    rp = ts.RowParams(
        temperature=torch.tensor([w["row_temperature"][i % 3] for i in range(B)], dtype=torch.float32, device=dev),
        top_p=torch.tensor([w["row_top_p"][i % 3] for i in range(B)], dtype=torch.float32, device=dev),
        top_k=torch.tensor([w["row_top_k"][i % 3] for i in range(B)], dtype=torch.int32, device=dev),
        max_top_k=max(w["row_top_k"]))
    kw = ts._cfg_kwargs(cfg, state.history, dev, rp)
    ops = pkg._native.ops()
    ch = ts.CodecHead(heads[0], B)

    def one_step(i):
        if args.path == "unfused":  # the same step as two launches: torch's F.linear (cuBLAS), then the sampler
            lg = torch.nn.functional.linear(hiddens[i % nbuf], heads[i % nbuf])
            return ops.sample_state_(lg, state.history, state.steps, state.finished, state.seeds, None, state.active,
                                     kw["alpha"], None, rp.temperature, rp.top_p, rp.top_k, kw["temperature"],
                                     cfg.top_p, cfg.top_k, kw["min_keep"], cfg.min_new_tokens, cfg.max_new_tokens,
                                     eos, kw["semantics"], ts.RNG_PHILOX, kw["max_top_k"], 0, 0)
        return ops.head_sample_state_(hiddens[i % nbuf], heads[i % nbuf], ch.logits, ch.sync, state.history,
                                      state.steps, state.finished, state.seeds, None, state.active, kw["alpha"], None,
                                      rp.temperature, rp.top_p, rp.top_k, kw["temperature"], cfg.top_p, cfg.top_k,
                                      kw["min_keep"], cfg.min_new_tokens, cfg.max_new_tokens, eos, kw["semantics"],
                                      ts.RNG_PHILOX, kw["max_top_k"])

    ms, ck, graphs = time_steps(args, one_step, dev, local, world)
    ms_per_step = ms / args.steps
    value = B * world * args.steps / (ms / 1e3)
    step_bytes = V * Hd * 2 + B * (2 * Hd + 4 * W + 40)
    achieved = step_bytes / (ms_per_step / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()

    # end to end through the public API: pinned host hidden rows -> device, CodecHead.step_, tokens -> host
    e2e_steps = max(1, args.e2e_steps)
    host = torch.from_numpy(hid_h).to(torch.bfloat16).contiguous().pin_memory()
    dbuf = torch.empty_like(host, device=dev)
    tok_h = torch.empty(B, dtype=torch.int64).pin_memory()
    st_e = ts.DecodeState(seeds=state.seeds.clone(), steps=torch.ones(B, dtype=torch.int64, device=dev),
                          history=state.history.clone(), finished=state.finished.clone(), active=state.active.clone())
    ch_e = ts.CodecHead(heads[0], B)

    def api_step():
        dbuf.copy_(host, non_blocking=True)
        tok = ch_e.step_(st_e, dbuf, eos, cfg, row_params=rp, rng="philox")
        tok_h.copy_(tok, non_blocking=True)

    for _ in range(3 if args.e2e_steps else 0):
        api_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        api_step()
    e1.record()
    torch.cuda.synchronize()
    et = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_value = B * world * e2e_steps / (float(et.item()) / 1e3)

    cb = cb_port = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import ref_build

        cb_port = cpu_baseline(w, seconds=min(args.cpu_seconds, 5.0))
        cb = reference_cpu(w, seconds=args.cpu_seconds) if ref_build.available() else cb_port
    for gr, _ in graphs:
        del gr
    graphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": metric_of(w),
        "value": value, "unit": "rows/s", "value_per_gpu": value / world, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (head GEMM, fp32 accumulation) -> f32 (sampling)", "data": "synthetic",
        "config": config_of(args, w, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": profiled_traffic(args.workload, w, args.path), "bytes_per_step": step_bytes,
                     "peak_source": peak_kind},
        "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": host.numel() * host.element_size(),
                "d2h_bytes_per_step": B * 8, "steps": e2e_steps},
        "gpu_launches": args.steps,
        "clocks": ck,
        "cpu_baseline": cb,
        "cpu_baseline_port": cb_port,
    }
    print(json.dumps(line))


def lmhead_cpu(w, *, steps: int = 0, warmup: int = 1, seconds: float = 10.0) -> dict:
    """The reference's greedy step on the host cores: ``F.linear(hidden, lm_head).float().argmax(-1)``
    (``engine/runtime/thinker_decode.py:107``) on CPU torch bf16 tensors of the workload's shape with every host
    thread; ``steps`` > 0 times exactly that many steps, else as many as fit in ``seconds``."""
    import torch

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    B, V, Hd = w["rows"], w["vocab"], w["hidden"]
    hc = torch.randn(B, Hd, generator=g).to(torch.bfloat16)
    wc = (torch.randn(V, Hd, generator=g) * (2.0 / Hd ** 0.5)).to(torch.bfloat16)
    for _ in range(max(1, warmup)):
        torch.nn.functional.linear(hc, wc).float().argmax(-1)
    n, t0 = 0, time.perf_counter()
    while True:
        torch.nn.functional.linear(hc, wc).float().argmax(-1)
        n += 1
        el = time.perf_counter() - t0
        if (steps > 0 and n >= steps) or (steps <= 0 and el >= seconds):
            break
    return {"value": B * n / el, "unit": "rows/s", "cores": threads, "kind": "reference",
            "sample": f"{n} steps x {B} rows: F.linear(hidden, lm_head).float().argmax(-1) (the reference's greedy "
                      f"step, engine/runtime/thinker_decode.py:107) on CPU torch {torch.__version__}, {threads} threads, "
                      f"in {el:.1f} s"}


def run_lmhead(args, w, rank: int, world: int, local: int):
    """The Thinker's greedy step from its LM head (``thinker_sampler.LMHeadArgmax``): each step reads the whole
    1.24 GB head (larger than the L2) and a rotating set of hidden rows."""
    import torch
    import torch.distributed as dist

    import __graft_entry__

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    pkg = __graft_entry__.load_package()
    lm = pkg.thinker_sampler
    B, V, Hd = w["rows"], w["vocab"], w["hidden"]
    g = torch.Generator(device=dev).manual_seed(rank)
    head = (torch.randn(V, Hd, device=dev, generator=g) * (2.0 / Hd ** 0.5)).to(torch.bfloat16)
    hiddens = [torch.randn(B, Hd, device=dev, generator=g).to(torch.bfloat16) for _ in range(16)]
    op = lm.LMHeadArgmax(head, B)
    ops = pkg._native.ops()

    def one_step(i):
        if args.path == "unfused":  # torch's F.linear (cuBLAS, bf16 logits written), then the argmax kernel
            return ops.argmax(torch.nn.functional.linear(hiddens[i % 16], head))
        return ops.lmhead_argmax(hiddens[i % 16], head, op.keys, None)

    ms, ck, graphs = time_steps(args, one_step, dev, local, world)
    ms_per_step = ms / args.steps
    value = B * world * args.steps / (ms / 1e3)
    step_bytes = V * Hd * 2 + B * (2 * Hd + 8)
    achieved = step_bytes / (ms_per_step / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    host = hiddens[0].cpu().contiguous().pin_memory()
    dbuf = torch.empty_like(host, device=dev)
    tok_h = torch.empty(B, dtype=torch.int64).pin_memory()
    e2e_steps = max(1, args.e2e_steps)

    def api_step():
        dbuf.copy_(host, non_blocking=True)
        tok_h.copy_(op(dbuf), non_blocking=True)

    for _ in range(3 if args.e2e_steps else 0):
        api_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        api_step()
    e1.record()
    torch.cuda.synchronize()
    et = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_value = B * world * e2e_steps / (float(et.item()) / 1e3)
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = lmhead_cpu(w, seconds=min(args.cpu_seconds, 10.0))
    for gr, _ in graphs:
        del gr
    graphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": metric_of(w),
        "value": value, "unit": "rows/s", "value_per_gpu": value / world, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (LM-head GEMM, fp32 accumulation, bf16-rounded logits)", "data": "synthetic",
        "config": config_of(args, w, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": profiled_traffic(args.workload, w, args.path), "bytes_per_step": step_bytes,
                     "peak_source": peak_kind},
        "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": host.numel() * host.element_size(),
                "d2h_bytes_per_step": B * 8, "steps": e2e_steps},
        "gpu_launches": 2 * args.steps,
        "clocks": ck,
        "cpu_baseline": cb,
    }
    print(json.dumps(line))


def time_steps(args, one_step, dev, local: int, world: int):
    """W untimed steps, then exactly K steps (CUDA graphs of up to 1000 steps, each replayed once untimed before
    the timed replays) between CUDA events on the launching stream, with nvidia-smi clocks sampled meanwhile;
    the max over ranks.  Returns (ms over the K steps, clocks, graphs -- released by the caller)."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            one_step(i)
    torch.cuda.synchronize()
    # the K timed steps as CUDA graphs (G steps per graph): no host launch cost between steps
    G = min(args.steps, 1000)
    reps, rem = divmod(args.steps, G)
    graphs = []
    for n in ([] if args.eager else ([G] if reps else []) + ([rem] if rem else [])):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(n):
                one_step(i)
        graphs.append((gr, n))
    # one untimed replay of each graph: its upload and the first replay's cold start stay out of the timed region
    with torch.cuda.stream(stream):
        for gr, _ in graphs:
            gr.replay()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local].strip() if vis else local)
    clocks.start()
    time.sleep(0.1)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # a graph replays on the current stream: time that stream
        # a bounded spin (about 0.1 ms, torch's own) holds the stream while the host enqueues the start event and the
        # replays, so the start event fires when the first step can start: the host's launch latency stays out of
        # the K steps' device time, as it does in a decode loop that launches ahead of the GPU
        torch.cuda._sleep(200_000)
        ev0.record(stream)
        if args.eager:
            for i in range(args.steps):
                one_step(i)
        else:
            for r in range(reps):
                graphs[0][0].replay()
            if rem:
                graphs[-1][0].replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ck = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return ms, ck, graphs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="thinker", choices=sorted(WORKLOADS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--eager", action="store_true", help="time plain launches instead of CUDA graphs (profiling)")
    ap.add_argument("--path", default="auto", choices=["auto", "stream", "resident", "unfused"],
                    help="sampling kernel: the launcher's choice (short-row kernel for rows of <= 8192 elements, "
                         "else row-resident), the streaming kernel, or the row-resident kernel; talker_head: "
                         "'unfused' times torch's F.linear followed by the sampler (two launches per step); greedy_head: F.linear "
                         "followed by the argmax kernel")
    ap.add_argument("--cluster", type=int, default=0, help="CTAs per row of the row-resident kernel (0: auto)")
    ap.add_argument("--strong", action="store_true",
                    help="split the workload's batch over the ranks (strong scaling) instead of B rows per rank")
    args = ap.parse_args()
    w = WORKLOADS[args.workload]
    if args.path == "resident" and args.cluster == 0 and w["vocab"] <= 8192 and w.get("window", 0) <= 255:
        args.cluster = 1  # short rows: the launcher's own choice is the short-row kernel; one CTA per row asks for this one
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, w, rank)
    if w.get("op") == "vocab_shard":
        return run_vocab_shard(args, w, rank, world, local)
    if w.get("op") == "head":
        return run_head(args, w, rank, world, local)
    if w.get("op") == "lmhead":
        return run_lmhead(args, w, rank, world, local)

    import torch
    import torch.distributed as dist

    import __graft_entry__

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    pkg = __graft_entry__.load_package()
    ts = pkg.talker_sampler
    B, V, W = w["rows"], w["vocab"], w["window"]
    if args.strong:  # a fixed global batch split over the ranks (1024 rows over 1/2/4/8 GPUs)
        if B % world:
            raise SystemExit(f"--strong needs the batch ({B}) divisible by the rank count ({world})")
        B //= world
    tdt = torch.bfloat16 if w["dtype"] == "bf16" else torch.float32
    row_bytes = bytes_per_row(w)
    step_bytes = B * row_bytes
    nbuf = rotating_buffers(w)
    logits_h, hist_h = make_inputs(w, B, 1000 + rank)
    base = torch.from_numpy(logits_h).to(dev).to(tdt)
    bufs = []
    g = torch.Generator(device=dev).manual_seed(rank)
    eos = w.get("eos", -1)
    for i in range(nbuf):  # distinct contents: a per-buffer permutation of the columns (EOS stays in place)
        perm = torch.randperm(V - 1 if eos >= 0 else V, device=dev, generator=g)
        if eos >= 0:
            perm = torch.cat([perm, torch.tensor([V - 1], device=dev)])
        bufs.append(base[:, perm].contiguous())
    del base
    greedy = w.get("op") == "argmax"
    cfg = ts.TalkerSampling(temperature=w["temperature"] if not greedy else 1.0, top_p=w["top_p"], top_k=w["top_k"],
                            repetition_penalty=w["penalty"], window=W, min_new_tokens=w.get("min_new", 0),
                            max_new_tokens=1 << 62, min_keep=w.get("min_keep", 1), semantics=w.get("order", "omni"),
                            rng="counter")
    state = ts.DecodeState.new(list(range(rank * B, rank * B + B)), cfg, device=dev)
    state.history.copy_(torch.from_numpy(hist_h).to(dev))
    if w.get("order") == "hf":
        state.steps.fill_(1)  # past frame 0, so the hf filters apply from the first step
    rp = None
    if "row_temperature" in w:
        rp = ts.RowParams(
            temperature=torch.tensor([w["row_temperature"][i % 3] for i in range(B)], dtype=torch.float32, device=dev),
            top_p=torch.tensor([w["row_top_p"][i % 3] for i in range(B)], dtype=torch.float32, device=dev),
            top_k=torch.tensor([w["row_top_k"][i % 3] for i in range(B)], dtype=torch.int32, device=dev),
            max_top_k=max(w["row_top_k"]))
    kw = None if greedy else ts._cfg_kwargs(cfg, state.history, dev, rp)
    ops = pkg._native.ops()

    K = w.get("frames", 1)
    if K > 1:  # [n, B, V] frames: step i decodes frames (i * K) mod n ... + K - 1 in one launch
        frames_all = torch.stack(bufs)
        del bufs[:]
        nfr = frames_all.shape[0] - K

    def one_step(i):
        if greedy:
            return ops.argmax(bufs[i % nbuf])
        if K > 1:
            f0 = (i * K) % nfr
            return ops.sample_frames_(frames_all[f0:f0 + K], state.history, state.steps, state.finished, state.seeds,
                                      None, state.active, kw["alpha"], None, None if rp is None else rp.temperature,
                                      None if rp is None else rp.top_p, None if rp is None else rp.top_k,
                                      kw["temperature"], cfg.top_p, cfg.top_k, kw["min_keep"], cfg.min_new_tokens,
                                      cfg.max_new_tokens, eos, kw["semantics"], ts.RNG_PHILOX, kw["max_top_k"])
        return ops.sample_state_(bufs[i % nbuf], state.history, state.steps, state.finished, state.seeds, None,
                                 state.active, kw["alpha"], None, None if rp is None else rp.temperature,
                                 None if rp is None else rp.top_p, None if rp is None else rp.top_k,
                                 kw["temperature"], cfg.top_p, cfg.top_k, kw["min_keep"], cfg.min_new_tokens,
                                 cfg.max_new_tokens, eos, kw["semantics"], ts.RNG_PHILOX, kw["max_top_k"],
                                 args.cluster, ts.FLAG_STREAM if args.path == "stream" else 0)

    ms, ck, graphs = time_steps(args, one_step, dev, local, world)
    ms_per_step = ms / args.steps
    value = B * K * world * args.steps / (ms / 1e3)  # sampled rows (row-frames) per second
    peak, peak_kind = measured_peak_gbs()
    achieved = K * step_bytes / (ms_per_step / 1e3) / 1e9

    # end to end through the public API: pinned host logits -> device, sample, tokens -> host, every step
    e2e_steps = max(1, args.e2e_steps)
    host = torch.from_numpy(logits_h).to(tdt)
    host = (host[None].expand(K, B, V) if K > 1 else host).contiguous().pin_memory()
    dbuf = torch.empty_like(host, device=dev)
    tok_h = torch.empty((K, B) if K > 1 else (B,), dtype=torch.int64).pin_memory()
    hist_e = state.history.clone()
    steps_e = torch.ones(B, dtype=torch.int64, device=dev)
    seeds_e = state.seeds.clone()
    st_e = ts.DecodeState(seeds=seeds_e, steps=steps_e, history=hist_e, finished=state.finished.clone(),
                          active=state.active.clone())

    def api_step():
        if greedy:
            return pkg.thinker_sampler.argmax(dbuf)
        if K > 1:  # the public K-frame entry (its counter RNG; per-row parameters are the sample-level form)
            return ts.decode_k(st_e, dbuf, eos, cfg)
        return ts.sample(dbuf, hist_e, steps_e, seeds_e, eos, cfg, rng="philox", row_params=rp)

    for i in range(3 if args.e2e_steps else 0):
        dbuf.copy_(host, non_blocking=True)
        tok = api_step()
        tok_h.copy_(tok, non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        dbuf.copy_(host, non_blocking=True)
        tok = api_step()
        tok_h.copy_(tok, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    et = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_value = B * K * world * e2e_steps / (float(et.item()) / 1e3)

    cb = cb_port = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import ref_build

        cb_port = cpu_baseline(w, seconds=min(args.cpu_seconds, 5.0))
        cb = reference_cpu(w, seconds=args.cpu_seconds) if ref_build.available() else cb_port
    for gr, _ in graphs:
        del gr
    graphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    traffic = profiled_traffic(args.workload, w, args.path)
    line = {
        "metric": metric_of(w),
        "value": value, "unit": "rows/s", "value_per_gpu": value / world, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
        "dtype": dtype_of(w), "data": "synthetic",
        "config": config_of(args, w, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "bytes_per_row": row_bytes, "peak_source": peak_kind},
        "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": host.numel() * host.element_size(),
                "d2h_bytes_per_step": B * K * 8, "steps": e2e_steps},
        "gpu_launches": args.steps,
        "clocks": ck,
        "cpu_baseline": cb,
        "cpu_baseline_port": cb_port,
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()
