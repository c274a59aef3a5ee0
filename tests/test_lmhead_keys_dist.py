"""The vocabulary-sharded greedy step's merge, host side, on two gloo ranks (CPU).

Each rank keys its half of every row the way ``b2s_lmhead_argmax_keys`` defines it: the order key of the value
(NaN above every number, -0 as +0) in the high word, the complement of the global id in the low word, the top bit
flipped so that a signed 64-bit maximum keeps the order, INT64_MIN for a shard with nothing to offer.
``vocab_shard.merge_keys`` -- the one max-all-reduce the NCCL path runs -- must give torch's argmax over the whole
row on every rank: the first index among equal maxima, ties across the shard boundary, a NaN, the two zeros and
-inf included.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.dist

B, V = 8, 1000


def _rows() -> np.ndarray:
    g = np.random.default_rng(3)
    x = (np.round(g.standard_normal((B, V)) * 4) / 4).astype(np.float32)  # many equal values
    x[1, 100] = x[1, 700] = 9.0          # a tie across the boundary (500): the first id wins
    x[2, 640] = np.nan                   # NaN wins
    x[2, 900] = np.nan
    x[3, :] = 0.0
    x[3, :300] = -0.0                    # the two zeros tie: id 0
    x[4, :] = -np.inf                    # every value -inf: id 0
    x[5, 499] = x[5, 500] = 9.5          # the tie at the boundary itself
    x[6, 999] = 12.0                     # the last id
    return x


def _okey(v: np.ndarray) -> np.ndarray:
    u = v.view(np.uint32).astype(np.uint64)
    u = np.where((u & 0x7FFFFFFF) == 0, 0, u)
    k = np.where((u & 0x80000000) != 0, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return np.where(np.isnan(v), 0xFFFFFFFF, k).astype(np.uint64)


def shard_words(x: np.ndarray, lo: int, hi: int) -> np.ndarray:
    """One word per row for the ids lo .. hi - 1 (a restatement of the kernel's tile keys and shard output)."""
    out = np.empty(x.shape[0], np.int64)
    for r in range(x.shape[0]):
        if hi <= lo:
            out[r] = np.iinfo(np.int64).min
            continue
        keys = (_okey(x[r, lo:hi]) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.arange(lo, hi, dtype=np.uint64))
        best = int(keys.max()) ^ (1 << 63)
        out[r] = best - (1 << 64) if best >= (1 << 63) else best
    return out


def _worker(rank: int, world: int, port: int):
    import torch.distributed as dist

    import __graft_entry__

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vs = __graft_entry__.load_package().vocab_shard
        x = _rows()
        bounds = [0, 500, V]
        words = torch.from_numpy(shard_words(x, bounds[rank], bounds[rank + 1]))
        if rank == 1:
            words[7] = torch.iinfo(torch.int64).min  # this shard offers nothing for row 7
        got = vs.merge_keys(words, timeout=60)
        want = torch.from_numpy(x).argmax(dim=1)
        want[7] = int(torch.from_numpy(x[7, :500]).argmax())
        assert torch.equal(got, want), (got, want)
        assert got[1].item() == 100 and got[2].item() == 640 and got[3].item() == 0 and got[4].item() == 0
        assert got[5].item() == 499 and got[6].item() == 999
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_key_merge_is_the_argmax():
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)


def test_decode_of_no_candidate_is_pad(pkg):
    vs = pkg.vocab_shard
    assert vs.decode_keys(torch.tensor([torch.iinfo(torch.int64).min])).tolist() == [-1]
