"""Build recipe for ``oracle/_ref/``: the reference sampler compiled to bytecode -- TEST / BASELINE
INFRASTRUCTURE ONLY.

The reference's sampling path is one pure-torch module, ``engine/talker_sampler.py``.  This recipe
compiles that file, where it lies in the reference checkout, with ``py_compile`` into
``oracle/_ref/talker_sampler.refbc`` (CPython bytecode; the suffix keeps tools that skip ``*.pyc`` caches
from dropping it): a build output (git-ignored, like the oracle's ``.so``), not a copy
of the source.  The GPU box has no reference checkout; the bytecode travels with the built files and
``load()`` imports it unchanged, so ``bench.py --impl reference`` times the reference's own torch code
on the host cores.  Nothing in the product package imports this module.

    REFERENCE_ROOT=<reference checkout> python -m oracle.ref_build
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import py_compile
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
PYC = OUT_DIR / "talker_sampler.refbc"
MODULE = Path("engine") / "talker_sampler.py"


def build(reference_root: str | os.PathLike) -> Path | None:
    """Compile the reference module into ``oracle/_ref``; None when the checkout is absent."""
    src = Path(reference_root) / MODULE
    if not src.is_file():
        return None
    OUT_DIR.mkdir(exist_ok=True)
    if not PYC.exists() or PYC.stat().st_mtime < src.stat().st_mtime:
        tmp = PYC.with_suffix(".refbc.tmp")
        py_compile.compile(str(src), cfile=str(tmp), dfile=str(MODULE), doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
        os.replace(tmp, PYC)
    return PYC


def available() -> bool:
    return PYC.is_file()


def load():
    """The reference module from its bytecode (raises if ``build`` has not run)."""
    name = "reference_talker_sampler"
    mod = sys.modules.get(name)
    if mod is not None:
        return mod
    if not PYC.is_file():
        raise FileNotFoundError(f"{PYC} is missing: run oracle/ref_build.py with REFERENCE_ROOT set")
    loader = importlib.machinery.SourcelessFileLoader(name, str(PYC))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses resolve their module while the class body runs
    try:
        loader.exec_module(mod)
    except BaseException:
        sys.modules.pop(name, None)
        raise
    return mod


if __name__ == "__main__":
    root = os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit("set REFERENCE_ROOT to the reference checkout")
    out = build(root)
    if out is None:
        raise SystemExit(f"{Path(root) / MODULE} not found")
    print("built", out)
