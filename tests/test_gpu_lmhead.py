"""The Thinker's greedy step straight from its LM head (``LMHeadArgmax`` / ``b2s_lmhead_argmax``) on the B200.

The launch rounds each fp32 tensor-core sum to bf16 (as F.linear's bf16 output is rounded) and takes the first
index of the row maximum.  Its sums differ from an exact dot product only in the order of the fp32 accumulation,
so the test accepts a token whose exactly computed logit, rounded to bf16, lies within one bf16 ulp of the row's
rounded exact maximum, and requires the exact argmax wherever the maximum is unique by more than two ulps.  Ties
built from identical head rows (the same sums in the same order) must resolve to the first id, and a NaN logit
must win, as torch's argmax does.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _ulp(x: torch.Tensor) -> torch.Tensor:
    return torch.clamp(x.abs(), min=2.0 ** -100).log2().floor().sub(7).exp2()


def _check(tok: torch.Tensor, exact: torch.Tensor, eps: float):
    """exact: [B, V] fp64 or fp32 logits; eps: allowance for the accumulation order beyond one bf16 ulp."""
    rb = exact.to(torch.bfloat16).double()
    m, am = rb.max(dim=1)
    tok = tok.cpu()
    got = rb.gather(1, tok[:, None])[:, 0]
    assert bool((got >= m - _ulp(m) - eps).all()), (tok, am)
    second = rb.clone()
    second[torch.arange(rb.shape[0]), am] = -float("inf")
    clear = (m - second.max(dim=1).values) > 2 * _ulp(m) + eps
    assert bool((tok[clear] == am[clear]).all())
    return clear.float().mean().item()


def _operands(B, V, H, seed):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(B, H, generator=g).to(torch.bfloat16)
    head = (torch.randn(V, H, generator=g) * (2.0 / H ** 0.5)).to(torch.bfloat16)
    return hidden, head


def test_lmhead_argmax_small_vocab_two_calls(pkg):
    """16 rows, 20,000 ids (the last tile partial), hidden 1024: exact fp64 logits on the CPU; two calls in a row
    leave the reduction words zero."""
    lm = pkg.thinker_sampler
    hidden, head = _operands(16, 20_000, 1024, 1)
    op = lm.LMHeadArgmax(head.to(DEV), 16)
    for call in range(2):
        h = hidden if call == 0 else torch.roll(hidden, 3, dims=1)
        tok = op(h.to(DEV))
        torch.cuda.synchronize()
        frac_clear = _check(tok, h.double() @ head.double().T, 1e-4)
        assert frac_clear > 0.5
        assert op.keys.cpu().tolist() == [0] * 16


def test_lmhead_argmax_thinker_shape(pkg):
    """The Thinker's shape: 64 rows, 151,936 ids, hidden 4096 (a 1.24 GB head); exact logits from an fp32 matmul on
    the GPU (TF32 off); and the unfused path (F.linear's bf16 logits, then the argmax kernel) for comparison."""
    lm = pkg.thinker_sampler
    B, V, H = 64, 151_936, 4096
    g = torch.Generator(device=DEV).manual_seed(2)
    hidden = torch.randn(B, H, device=DEV, generator=g).to(torch.bfloat16)
    head = (torch.randn(V, H, device=DEV, generator=g) * (2.0 / H ** 0.5)).to(torch.bfloat16)
    tok = lm.LMHeadArgmax(head, B)(hidden)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        exact = hidden.float() @ head.float().T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    assert _check(tok, exact.cpu(), 1e-3) > 0.5
    unfused = lm.argmax(torch.nn.functional.linear(hidden, head))
    _check(unfused, exact.cpu(), 1e-3)  # the reference form meets the same bar


def test_lmhead_argmax_ties_and_nan(pkg):
    """Identical head rows give identical sums: the first id wins; a NaN logit wins over every number."""
    lm = pkg.thinker_sampler
    B, V, H = 8, 3000, 512
    hidden, head = _operands(B, V, H, 3)
    w = hidden[0].float() * (8.0 / hidden[0].float().norm())  # large logit for row 0
    for j in (2900, 7, 1500):  # ids 7 and 1500 and 2900 share a row of the head: the ties sit in three tiles
        head[j] = w.to(torch.bfloat16)
    head_nan = head.clone()
    head_nan[2000, 5] = float("nan")
    op = lm.LMHeadArgmax(head.to(DEV), B)
    tok = op(hidden.to(DEV)).cpu()
    assert int(tok[0]) == 7
    tok_nan = lm.LMHeadArgmax(head_nan.to(DEV), B)(hidden.to(DEV)).cpu()
    assert tok_nan.tolist() == [2000] * B
    torch.cuda.synchronize()


def test_lmhead_argmax_rejects_more_than_64_rows(pkg):
    lm = pkg.thinker_sampler
    op = lm.LMHeadArgmax(torch.zeros(1000, 128, dtype=torch.bfloat16, device=DEV), 65)
    with pytest.raises(RuntimeError, match="unsupported"):
        op(torch.zeros(65, 128, dtype=torch.bfloat16, device=DEV))
    torch.cuda.synchronize()


def test_lmhead_shards_merge_to_the_unsharded_argmax(pkg):
    """The vocabulary-sharded greedy step with its shards run one after another on one GPU: the signed maximum of
    the shards' words decodes to the unsharded launch's tokens exactly (each id's sum is the same in any tile), ties
    across shard boundaries included."""
    lm, vs = pkg.thinker_sampler, pkg.vocab_shard
    B, V, H = 16, 20_003, 768
    hidden, head = _operands(B, V, H, 4)
    w = hidden[5].float() * (8.0 / hidden[5].float().norm())
    for j in (4999, 15000):  # a tie between shards 0 and 3: the first id must win
        head[j] = w.to(torch.bfloat16)
    head_d, hid_d = head.to(DEV), hidden.to(DEV)
    want = lm.LMHeadArgmax(head_d, B)(hid_d)
    bounds = [0, 5000, 10_003, 15_000, V]
    keys = torch.zeros(B, dtype=torch.int64, device=DEV)
    words = torch.stack([vs.lmhead_keys(hid_d, head_d[a:b].contiguous(), a, keys) for a, b in zip(bounds, bounds[1:])])
    got = vs.decode_keys(words.max(dim=0).values)
    torch.cuda.synchronize()
    assert torch.equal(got, want), (got, want)
    assert int(got[5]) == 4999
    assert keys.cpu().tolist() == [0] * B
