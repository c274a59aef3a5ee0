"""Multi-GPU paths on real devices (skipped with fewer than two GPUs).

* Vocabulary-sharded sampling: each rank holds a contiguous slice of the head's columns; one NCCL
  all-gather of the packed candidate lists, then every rank draws the same token, which equals the unsharded
  kernel's token on the whole row (and the oracle's).
* The greedy step from a vocabulary-sharded LM head: each rank's slice on the tensor cores with the argmax in the
  epilogue, one NCCL max-all-reduce of [B] int64 words; every rank gets the unsharded launch's tokens.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

B, V, K, TOP_P, T = 6, 20000, 32, 0.9, 0.8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = np.random.default_rng(5)
    x = (np.round(g.standard_normal((B, V)) * 2.0 * 16) / 16).astype(np.float32)  # heavy ties
    hist = g.integers(0, V, size=(B, 24)).astype(np.int64)
    return x, hist


def _worker(rank: int, world: int, port: int, out_q):
    import torch.distributed as dist

    import __graft_entry__

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        pkg = __graft_entry__.load_package()
        vs, ts = pkg.vocab_shard, pkg.thinker_sampler
        x, hist = _inputs()
        bounds = vs.shard_bounds(V, world)
        lo, hi = bounds[rank], bounds[rank + 1]
        xs = torch.from_numpy(x[:, lo:hi]).to(dev).to(torch.bfloat16).contiguous()
        h = torch.from_numpy(hist).to(dev)
        steps = torch.full((B,), 3, dtype=torch.int64, device=dev)
        seeds = torch.arange(B, dtype=torch.int64, device=dev)
        cfg = ts.ThinkerSampling(temperature=T, top_k=K, top_p=TOP_P, repetition_penalty=1.1, rng="counter")
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        tok = vs.sample_sharded(xs, lo, V, h, steps, seeds, cfg, rng="counter", status=status)
        # the unsharded kernel on the whole row, on this rank's GPU
        full = torch.from_numpy(x).to(dev).to(torch.bfloat16)
        want = ts.sample(full, h, seeds, steps, cfg)
        # the greedy step from a vocabulary-sharded LM head (hidden 512): the same head on every rank, one slice each
        g = torch.Generator().manual_seed(9)
        hid = torch.randn(B, 512, generator=g).to(torch.bfloat16).to(dev)
        head = (torch.randn(V, 512, generator=g) * (2.0 / 512 ** 0.5)).to(torch.bfloat16).to(dev)
        keys = torch.zeros(B, dtype=torch.int64, device=dev)
        gtok = vs.lmhead_argmax_sharded(hid, head[lo:hi].contiguous(), lo, keys, timeout=60)
        gwant = ts.LMHeadArgmax(head, B)(hid)
        torch.cuda.synchronize()
        out_q.put((rank, tok.cpu().numpy().tolist(), want.cpu().numpy().tolist(), int(status.item()),
                   gtok.cpu().tolist(), gwant.cpu().tolist()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vocab_sharded_two_gpus_matches_unsharded():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p_ in procs:
        p_.join(timeout=120)
        assert p_.exitcode == 0
    res.sort()
    (_, tok0, want0, st0, g0, gw0), (_, tok1, want1, st1, g1, gw1) = res
    assert st0 == 0 and st1 == 0
    assert tok0 == tok1  # every rank draws the same token
    assert tok0 == want0 == want1  # equal to the unsharded kernel's token
    assert g0 == g1 == gw0 == gw1  # the sharded LM-head greedy step == the unsharded launch, on every rank
