"""Failure detection of the vocabulary-sharded step's collectives, on gloo ranks (CPU): no GPU is faulted, trapped or
hung.  A rank that never joins a step's candidate all-gather, or that leaves the group between steps, must turn
into ``vocab_shard.ShardExchangeError`` on the other ranks within the caller's timeout -- an error the engine
handles by failing the step's rows (the reference fails the requests of a tick that raised,
``engine/runtime/backend.py:197-203``) -- and never into a hang."""

from __future__ import annotations

import os
import socket
import time
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.dist

B, CAP = 4, 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lists(rank: int):
    v = torch.full((B, CAP), float(rank), dtype=torch.float32)
    i = torch.arange(B * CAP, dtype=torch.int32).reshape(B, CAP) + 1000 * rank
    n = torch.full((B,), CAP, dtype=torch.int32)
    return v, i, n


def _init(rank: int, world: int, port: int):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))


def _absent_rank_worker(rank: int, world: int, port: int):
    """Rank 1 never calls the all-gather (it waits, then leaves); rank 0's gather must fail within its timeout."""
    import torch.distributed as dist

    import __graft_entry__

    _init(rank, world, port)
    vs = __graft_entry__.load_package().vocab_shard
    if rank == 1:
        time.sleep(6.0)
        return  # leaves without joining the collective
    t0 = time.monotonic()
    with pytest.raises(vs.ShardExchangeError):
        vs.exchange(*_lists(rank), timeout=2.0)
    assert time.monotonic() - t0 < 15.0


def _leaving_rank_worker(rank: int, world: int, port: int):
    """Three ranks complete a step; rank 2 then leaves; the others' next step fails with ShardExchangeError."""
    import torch.distributed as dist

    import __graft_entry__

    _init(rank, world, port)
    vs = __graft_entry__.load_package().vocab_shard
    vv, ii, nn = vs.exchange(*_lists(rank), timeout=10.0)
    assert tuple(vv.shape) == (world, B, CAP)
    for s in range(world):  # every rank has every shard's lists
        assert torch.equal(vv[s], torch.full((B, CAP), float(s)))
    tok = torch.full((B,), -1, dtype=torch.int64)
    tok[rank] = 100 + rank
    assert vs.publish(tok, timeout=10.0).tolist() == [100, 101, 102, -1]
    dist.barrier()
    if rank == 2:
        dist.destroy_process_group()
        return  # leaves between steps, with nothing in flight
    t0 = time.monotonic()
    with pytest.raises(vs.ShardExchangeError):
        vs.exchange(*_lists(rank), timeout=2.0)
    assert time.monotonic() - t0 < 15.0


@pytest.mark.timeout(120)
def test_gather_fails_when_a_rank_never_joins():
    import torch.multiprocessing as mp

    mp.spawn(_absent_rank_worker, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.timeout(120)
def test_step_fails_after_a_rank_leaves():
    import torch.multiprocessing as mp

    mp.spawn(_leaving_rank_worker, args=(3, _free_port()), nprocs=3, join=True)
