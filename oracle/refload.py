"""TEST INFRASTRUCTURE ONLY -- loads the reference implementation (KAVYANSHTYAGI/x, package ``atl``).

Two consumers:
* ``tests/golden/gen_golden.py`` (run in the build container, where the reference tree exists) to
  produce the committed golden fixtures;
* ``bench.py --impl reference`` / the cpu_baseline leg, which time the reference's own CPU path.

The Python package comes from ``baseline/_ref`` (an unmodified ``pip install --target`` of the
reference) or, failing that, from the reference tree itself.  The reference builds its OpenMP
extension by JIT (atl/ops/_ext.py:16-42) from ``csrc/``, which a pip install does not ship; the same
unmodified sources are compiled by ``oracle/Makefile`` (target ``ref``) into ``oracle/_ref/`` and
registered as the module ``get_ext()`` returns, which is what its loader would have produced.
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
REF_TREE = Path(os.environ.get("ATL_REFERENCE_TREE", "/root/reference"))


def ref_extension_path() -> Path | None:
    hits = sorted(glob.glob(str(REPO / "oracle" / "_ref" / "atl_ops_cpu*.so")))
    return Path(hits[0]) if hits else None


def load_reference():
    """Import ``atl`` and install its CPU extension.  Returns the ``atl`` module or raises."""
    base = REPO / "baseline" / "_ref"
    if (base / "atl").is_dir():
        sys.path.insert(0, str(base))
    elif (REF_TREE / "atl").is_dir():
        sys.path.insert(0, str(REF_TREE))
    else:
        raise ImportError("reference package not found (baseline/_ref or the reference tree)")
    import atl  # noqa: F401
    import atl.ops._ext as ext_mod

    so = ref_extension_path()
    if so is None:
        raise ImportError("oracle/_ref/atl_ops_cpu*.so not built (make -C oracle ref)")
    spec = importlib.util.spec_from_file_location("atl_ops_cpu", str(so))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    ext_mod._EXT, ext_mod._TRIED = mod, True
    return sys.modules["atl"]
