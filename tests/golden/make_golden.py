"""Generate the golden outputs by running the REFERENCE sampler (``engine/talker_sampler.py``) on the
cases of ``cases.py``.

Run it with ``REFERENCE_ROOT`` naming a checkout of the reference source:

    REFERENCE_ROOT=<reference checkout> python -m tests.golden.make_golden

It writes ``tests/golden/{talker,thinker,edge,seq,rng}.npz``.  Each case stores the sha256 of its
regenerated inputs, the reference's ``processed_logits`` output, its ``draw`` tokens with the
case's injected uniforms (``uniform_values=``) and with the reference counter RNG, so the tests need
neither the reference nor its inputs on disk.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def reference_module():
    root = os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit("set REFERENCE_ROOT to a checkout of the reference source")
    if root not in sys.path:
        sys.path.insert(0, root)
    from engine import talker_sampler as ts  # noqa: E402  (reference module, imported unchanged)

    return ts


def run_case(ts, case) -> dict:
    B = case.rows
    x = torch.from_numpy(case.logits.copy())
    if case.dtype == "bf16":
        x = x.to(torch.bfloat16)
    hist = torch.from_numpy(case.history)
    steps = torch.from_numpy(case.steps)
    seeds = torch.from_numpy(case.seeds)
    u = torch.from_numpy(case.uniforms)
    proc = torch.empty(B, case.vocab, dtype=torch.float32)
    for r in range(B):  # rows are independent (talker_sampler.py:92-102 batch independence); cfg may differ per row
        cfg = ts.TalkerSampling(**{k: v for k, v in case.cfgs[r].items() if k in ts.TalkerSampling.__dataclass_fields__})
        proc[r:r + 1] = ts.processed_logits(x[r:r + 1], hist[r:r + 1], steps[r:r + 1], case.eos, cfg)
    tok_u = ts.draw(proc, seeds, steps, uniform_values=u)
    tok_c = ts.draw(proc, seeds, steps)
    return {"processed": proc.numpy(), "tok_u": tok_u.numpy(), "tok_c": tok_c.numpy(),
            "digest": np.array(case.digest())}


def run_sequence(ts, name) -> dict:
    from tests.golden import cases as C

    x, cfgd, seeds, inactive = C.sequence_inputs(name)
    cfg = ts.TalkerSampling(**cfgd)
    state = ts.DecodeState.new(seeds, cfg)
    for r in inactive:
        state.active[r] = False
    toks = ts.decode_k(state, torch.from_numpy(x), C.I.TALKER_EOS, cfg)
    return {"tokens": toks.numpy(), "steps": state.steps.numpy(), "history": state.history.numpy(),
            "finished": state.finished.numpy(), "digest": np.array(C.I.digest(x))}


def multinomial_scenario(mod):
    """The native-RNG block of the reference (``draw_multinomial`` then
    ``restore_multinomial_states_after_block``, ``talker_sampler.py:175-212``) on seeded CPU generators:
    K = 4 draws per row, PAD patterns that end a row's block at every position, then one more draw from
    the restored generators.  ``mod`` is the reference module or the engine's drop-in module."""
    g = torch.Generator().manual_seed(3)
    K, B, V = 4, 6, 6562
    xs = torch.randn(K + 1, B, V, generator=g) * 2.0
    gens = [torch.Generator().manual_seed(100 + r) for r in range(B)]
    toks, states = [], []
    for s in range(K):
        toks.append(mod.draw_multinomial(xs[s], gens))
        states.append([gen.get_state() for gen in gens])
    host = torch.stack(toks).clone()
    # the first PAD of each row's column: none, 0, 1, 3, 2, 1 (then 3)
    for row, cols in ((1, [0, 1, 2, 3]), (2, [1, 2, 3]), (3, [3]), (4, [2, 3]), (5, [1, 3])):
        host[cols, row] = mod.PAD
    mod.restore_multinomial_states_after_block(gens, states, host)
    after = mod.draw_multinomial(xs[K], gens)
    return {"block_tokens": torch.stack(toks).numpy(), "host_tokens": host.numpy(), "after_restore": after.numpy()}


def main() -> None:
    from tests.golden import cases as C

    if sys.argv[1:] == ["request_seed"]:  # only the request-seed fixture (engine/runtime/backend.py:51-54)
        root = os.environ.get("REFERENCE_ROOT")
        if not root:
            raise SystemExit("set REFERENCE_ROOT to a checkout of the reference source")
        sys.path.insert(0, root)
        from types import SimpleNamespace

        from engine.runtime.backend import request_seed  # noqa: E402  (reference function, imported unchanged)

        ids = ["req-0", "abc", "x" * 40, "", "ümlaut-request", "7f3a9c"] + [f"chat-{i}" for i in range(10)]
        explicit = [0, 1, 12345, -5, (1 << 63) - 1, 1 << 63, (1 << 64) + 7, -(1 << 70)]
        np.savez_compressed(HERE / "request_seed.npz", ids=np.array(ids), by_id=np.array(
            [request_seed(SimpleNamespace(request_id=i, seed=None)) for i in ids], np.int64),
            explicit=np.array([str(e) for e in explicit]), by_seed=np.array(
            [request_seed(SimpleNamespace(request_id="r", seed=e)) for e in explicit], np.int64))
        print("request_seed done")
        return
    if sys.argv[1:] == ["multinomial"]:  # only the native-RNG fixture
        ts = reference_module()
        np.savez_compressed(HERE / "multinomial.npz", **multinomial_scenario(ts))
        print("multinomial done")
        return

    ts = reference_module()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    groups = {"talker": C.talker_cases(), "thinker": C.thinker_cases(), "edge": C.edge_cases()}
    for group, cs in groups.items():
        out = {}
        for case in cs:
            for k, v in run_case(ts, case).items():
                out[f"{case.name}.{k}"] = v
        np.savez_compressed(HERE / f"{group}.npz", **out)
        print(group, len(cs), "cases")
    seq = {}
    for name in C.SEQUENCES:
        for k, v in run_sequence(ts, name).items():
            seq[f"{name}.{k}"] = v
    np.savez_compressed(HERE / "seq.npz", **seq)
    # counter uniforms over extreme seeds (test_talker_post_graph_npu.py:12, :84-90 pattern) + argmax
    seeds = torch.tensor(C.SEQ_SEEDS, dtype=torch.int64)
    steps = torch.arange(1024, dtype=torch.int64)[:, None]
    uni = ts.uniform(seeds[None, :], steps)
    g = C.I.rng(9)
    am_f32 = C.I.quantised_rows(g, 6, C.I.THINKER_V, q=4)
    am_f32[3, 1000:1010] = am_f32[3].max() + 1.0  # an explicit tie on the maximum: first index wins
    am_bf16_bits = C.I.to_bf16_bits(C.I.quantised_rows(g, 6, C.I.THINKER_V, q=16))
    am_bf16 = torch.from_numpy(am_bf16_bits.view(np.int16)).view(torch.bfloat16)
    np.savez_compressed(HERE / "rng.npz", uniform=uni.numpy(), seeds=seeds.numpy(),
                        argmax_f32=torch.from_numpy(am_f32).argmax(-1).numpy(),
                        argmax_f32_digest=np.array(C.I.digest(am_f32)),
                        argmax_bf16=am_bf16.float().argmax(-1).numpy(),
                        argmax_bf16_digest=np.array(C.I.digest(am_bf16_bits)))
    print("seq/rng done")


if __name__ == "__main__":
    main()
