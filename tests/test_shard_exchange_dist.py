"""Vocabulary-sharded sampling, host side, on two gloo ranks (CPU).

Each rank holds half of the vocabulary.  It builds its shard's candidate list the way
``b2s_shard_candidates`` defines it (omni-processed values: every element above the shard's k-th largest, then
elements equal to it up to ``cap = k``, and the count of every element >= the k-th), packs it and runs
``vocab_shard.exchange`` -- the same single ``all_gather_into_tensor`` the NCCL path uses.  From the gathered lists
and counts alone, the row's value multiset above the threshold (the sent values plus the unsent ties' copies) must
give the oracle's threshold on the unsharded row, and so its kept set and token: the decomposition the sharded
path relies on, with ties heavy enough that shards leave many unsent.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.dist

B, V, W, K, TOP_P, T = 4, 6000, 48, 20, 0.8, 0.7
PEN, PRES, FREQ = 1.1, 0.1, 0.05


def _inputs(seed: int = 11):
    g = np.random.default_rng(seed)
    x = (np.round(g.standard_normal((B, V)) * 2.0 * 16) / 16).astype(np.float32)  # ties at every level
    hist = g.integers(0, V, size=(B, W)).astype(np.int64)
    hist[0, :5] = -1  # PAD
    hist[1, :10] = hist[1, 10:20]  # repeated ids
    u = g.random(B).astype(np.float32)
    return x, hist, u


def omni_processed(x: np.ndarray, hist: np.ndarray) -> np.ndarray:
    """Penalty -> presence / frequency -> /T in fp32 (the omni order of talker_sampler.py:117-122)."""
    alpha = orc.alpha_table(PEN, W + 1)
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        h = hist[r]
        cnt = np.bincount(h[h >= 0], minlength=x.shape[1])
        v = x[r].copy()
        m = cnt > 0
        a = alpha[cnt[m]].astype(np.float32)
        xm = x[r, m]
        pen = np.where(xm < 0, xm * a, xm / a).astype(np.float32)
        pen = (pen - np.float32(PRES)).astype(np.float32)
        pen = (pen - np.float32(FREQ) * cnt[m].astype(np.float32)).astype(np.float32)
        v[m] = pen
        out[r] = (v / np.float32(T)).astype(np.float32)
    return out


def shard_list(p: np.ndarray, lo: int, hi: int, cap: int):
    """(values [B, cap], global ids [B, cap], count [B]) of the shard's candidates."""
    vals = np.full((p.shape[0], cap), -np.inf, np.float32)
    ids = np.zeros((p.shape[0], cap), np.int32)
    cnt = np.zeros(p.shape[0], np.int32)
    for r in range(p.shape[0]):
        s = p[r, lo:hi]
        kth = np.sort(s)[-K]
        sel = np.concatenate([np.nonzero(s > kth)[0], np.nonzero(s == kth)[0]])  # above first, then ties
        m = min(len(sel), cap)
        vals[r, :m] = s[sel[:m]]
        ids[r, :m] = sel[:m] + lo
        cnt[r] = len(sel)
    return vals, ids, cnt


def threshold_from_lists(vv, ii, nn, cap, r):
    """The row's value multiset relevant to top-k (sent values, plus up to K copies of each shard's unsent ties at
    its smallest sent value), placed in an otherwise -inf row, and its omni threshold from the oracle."""
    vals = []
    for s in range(vv.shape[0]):
        c = int(nn[s, r])
        sent = vv[s, r, :min(c, cap)]
        vals.extend(sent.tolist())
        if c > cap:
            vals.extend([float(sent.min())] * min(c - cap, K))
    row = np.full((1, V), -np.inf, np.float32)
    row[0, :len(vals)] = np.array(vals, np.float32)
    cfg = orc.Cfg(temperature=1.0, top_p=TOP_P, top_k=K, repetition_penalty=1.0, window=0, min_new_tokens=0,
                  max_new_tokens=1 << 40, min_keep=1, semantics="omni")
    proc, _, _, _ = orc.sample(row, np.zeros((1, 0), np.int64), np.full(1, 5, np.int64), None, -1, cfg,
                               uniforms=np.zeros(1, np.float32))
    return proc[0][~np.isneginf(proc[0])].min()


def _worker(rank: int, world: int, port: int, cap: int):
    import torch.distributed as dist

    import __graft_entry__

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vs = __graft_entry__.load_package().vocab_shard
        x, hist, u = _inputs()
        p = omni_processed(x, hist)
        bounds = vs.shard_bounds(V, world)
        v, i, n = shard_list(p, bounds[rank], bounds[rank + 1], cap)
        vv, ii, nn = vs.exchange(torch.from_numpy(v), torch.from_numpy(i), torch.from_numpy(n))
        assert tuple(vv.shape) == (world, B, cap) and tuple(nn.shape) == (world, B)
        # every rank sees every shard's list in rank order
        for s in range(world):
            ref = shard_list(p, bounds[s], bounds[s + 1], cap)
            assert np.array_equal(vv[s].numpy().view(np.uint32), ref[0].view(np.uint32))
            assert np.array_equal(ii[s].numpy(), ref[1]) and np.array_equal(nn[s].numpy(), ref[2])
        steps = np.full(B, 5, np.int64)
        seeds = np.arange(B, dtype=np.int64)
        full = orc.Cfg(temperature=T, top_p=TOP_P, top_k=K, repetition_penalty=PEN, window=W, min_new_tokens=0,
                       max_new_tokens=1 << 40, min_keep=1, semantics="omni", presence_penalty=PRES,
                       frequency_penalty=FREQ)
        p_full, want, _, _ = orc.sample(x, hist, steps, seeds, -1, full, uniforms=u)
        kept = ~np.isneginf(p_full)
        # the numpy restatement of the omni processing agrees with the oracle on every kept element
        assert np.array_equal(p_full[kept].view(np.uint32), p[kept].view(np.uint32))
        unsent = 0
        for r in range(B):
            thr = threshold_from_lists(vv.numpy(), ii.numpy(), nn.numpy(), cap, r)
            # the threshold from the capped lists and tie counts is the unsharded row's ...
            assert thr == p_full[r][kept[r]].min(), r
            # ... so the kept set (every element >= it) and the oracle's draw over it are the unsharded row's
            assert np.array_equal(p[r] >= thr, kept[r]), r
            unsent += int(sum(max(0, int(nn[s, r]) - cap) for s in range(world)))
        assert unsent > 0  # the heavy ties left elements unsent
        row = np.where(kept, p, np.float32(-np.inf)).astype(np.float32)
        got, _ = orc.draw(row, u)
        assert np.array_equal(got, want), (got, want)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_two_rank_exchange_matches_unsharded(world):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port(), K), nprocs=world, join=True)
