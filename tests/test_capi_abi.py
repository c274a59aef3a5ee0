"""The C-ABI boundary without a GPU: ``libb2s.so`` loads, exports every function ``include/b2s_sampler.h``
declares, the ctypes mirror of ``b2s_sample_args`` has the C layout (checked against gcc's own offsets),
and the calls that need no device answer.  The CUDA extension must exist: there is no CPU fallback."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b2s_sampler.h"


def _declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(b2s_\w+)\s*\(", text, flags=re.M)))


def _struct_fields():
    body = re.search(r"typedef struct b2s_sample_args \{(.*?)\} b2s_sample_args;", HEADER.read_text(), re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", re.sub(r"//[^\n]*", "", body), flags=re.S)
    return re.findall(r"([A-Za-z_][A-Za-z0-9_]*)\s*;", body)


def test_header_declares_the_abi():
    names = _declared_functions()
    assert {"b2s_sample", "b2s_argmax", "b2s_uniform", "b2s_shard_candidates", "b2s_shard_merge",
            "b2s_repetition_penalty", "b2s_error_string", "b2s_last_cuda_error", "b2s_abi_version"} <= set(names)


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._native.capi()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    # the ctypes signatures cover exactly the header's functions
    assert sorted(pkg._native.CAPI_SIGNATURES) == _declared_functions()


def test_host_only_calls(pkg):
    lib = pkg._native.capi()
    assert lib.b2s_abi_version() >= 1
    for code in range(0, 6):
        s = lib.b2s_error_string(code)
        assert isinstance(s, bytes) and len(s) > 0
    assert b"unknown" in lib.b2s_error_string(-12345).lower() or len(lib.b2s_error_string(-12345)) > 0


def test_head_entry_points_check_arguments_on_the_host(pkg):
    """The codec-head entry points refuse what they cannot take before touching the device (no GPU needed):
    fake, 16-byte aligned addresses stand in for the buffers."""
    import ctypes

    lib = pkg._native.capi()
    nat = pkg._native
    fake = [ctypes.c_void_p(0x10000 * (i + 1)) for i in range(8)]

    def args(rows=8, vocab=6562, logits=None, dtype=1):
        a = nat.SampleArgs()
        a.logits, a.logits_dtype, a.rows, a.vocab, a.logits_row_stride = logits, dtype, rows, vocab, vocab
        a.steps, a.tokens, a.seeds, a.rng, a.temperature, a.top_k, a.min_keep = fake[4], fake[5], fake[6], 1, 1.0, 1, 1
        return a

    def head(hidden_dim=768, stride=768, hidden=fake[0]):
        return nat.HeadArgs(hidden=hidden.value, hidden_row_stride=stride, head=fake[1].value, hidden_dim=hidden_dim,
                            logits=fake[2].value, sync=fake[3].value)

    call = lambda h, a: lib.b2s_head_sample(ctypes.byref(h), ctypes.byref(a), None)
    assert call(head(), args(rows=17)) == 2            # more rows than one MMA's N: unsupported
    assert call(head(hidden_dim=832, stride=832), args()) == 2  # more K than the tile's shared memory holds
    assert call(head(hidden_dim=100, stride=100), args()) == 1  # K not a multiple of 64
    assert call(head(stride=770), args()) == 1          # hidden rows not 16-byte aligned
    assert call(head(hidden=ctypes.c_void_p(0x10008)), args()) == 1  # hidden not 16-byte aligned
    assert call(head(), args(dtype=0)) == 1             # the head's logits are bf16
    assert call(head(), args(logits=fake[7])) == 1      # args->logits must be NULL or the head's logits
    noalloc = lambda a: lib.b2s_head_sample_noalloc(fake[0], 768, fake[1], 768, ctypes.byref(a), None)
    assert noalloc(args(vocab=8193)) == 2                # beyond the library's scratch
    assert noalloc(args(rows=17)) == 2
    assert noalloc(args(logits=fake[7])) == 1           # the logits live in the library's scratch


def test_sample_args_layout_matches_c(pkg, tmp_path):
    """Offsets of every field of b2s_sample_args as gcc lays them out == the ctypes mirror's."""
    fields = _struct_fields()
    mirror = pkg._native.SampleArgs
    assert [f[0] for f in mirror._fields_] == fields
    src = tmp_path / "layout.c"
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {",
             '  printf("size %zu\\n", sizeof(b2s_sample_args));']
    lines += [f'  printf("{f} %zu\\n", offsetof(b2s_sample_args, {f}));' for f in fields]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-x", "c", str(src), "-o", str(exe)], check=True)
    out = dict(l.split() for l in subprocess.run([str(exe)], check=True, capture_output=True,
                                                 text=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(mirror)
    for f in fields:
        assert int(out[f]) == getattr(mirror, f).offset, f


def test_torch_op_library_registers_ops(pkg):
    import torch

    pkg._native.ops()
    for op in ("sample", "sample_state_", "argmax", "uniform", "repetition_penalty", "shard_candidates",
               "shard_merge", "shard_resolve"):
        assert hasattr(torch.ops.minicpmo_sampler, op), op


def test_product_path_refuses_cpu_tensors(pkg):
    import torch

    x = torch.zeros(2, 16)
    with pytest.raises(ValueError):
        pkg.thinker_sampler.argmax(x)
    head = torch.zeros(1000, 64, dtype=torch.bfloat16)  # the head entry points too: no CPU path
    with pytest.raises(ValueError):
        pkg.talker_sampler.CodecHead(head, 2)
    with pytest.raises(ValueError):
        pkg.thinker_sampler.LMHeadArgmax(head, 2)
    with pytest.raises(ValueError):
        pkg.vocab_shard.lmhead_keys(torch.zeros(2, 64, dtype=torch.bfloat16), head, 0, torch.zeros(2, dtype=torch.int64))


def test_shard_pending_record_layout(tmp_path):
    """b2s_shard_pending is 32 bytes with the double first: the torch layer keeps it as [rows, 4] int64."""
    src = tmp_path / "pend.c"
    src.write_text("\n".join([
        "#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {",
        '  printf("%zu %zu %zu %zu\\n", sizeof(b2s_shard_pending), offsetof(b2s_shard_pending, base),',
        "         offsetof(b2s_shard_pending, thr), offsetof(b2s_shard_pending, shard));",
        "  return 0;", "}"]) + "\n")
    exe = tmp_path / "pend"
    subprocess.run(["gcc", "-std=c11", "-x", "c", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    assert out == ["32", "0", "8", "24"]
