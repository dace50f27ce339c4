"""The C-ABI library loads and exports every entry point include/atl_b200.h declares (no GPU needed)."""
import re
from pathlib import Path

import pytest

from x_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "atl_b200.h"


def declared():
    src = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(atlb_\w+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = declared()
    for must in ("atlb_ats_pair_fwd", "atlb_ats_pair_bwd", "atlb_plan_count", "atlb_plan_fill", "atlb_splat_gauss_fwd",
                 "atlb_gather_bilinear_bwd", "atlb_window_counts", "atlb_visible_fraction"):
        assert must in names


def test_library_exports_every_declared_symbol():
    L = _lib.load_library()
    for name in declared():
        assert hasattr(L, name), name


def test_binding_covers_header_exactly():
    assert set(_lib.exported_symbols()) == set(declared())


def test_abi_version_and_counter():
    L = _lib.load_library()
    assert L.atlb_abi_version() == 12
    assert L.atlb_kernel_launches() >= 0


def test_argument_validation_needs_no_device():
    """Invalid arguments are rejected before any CUDA call, with a message."""
    L = _lib.load_library()
    st = L.atlb_splat_gauss_fwd(None, None, None, 10, 1, 4, 4, 1.0, 3, None, None, 0, None)
    assert st == _lib.ATLB_ERR_ARG
    assert b"NULL" in L.atlb_last_error()
    st = L.atlb_velocity(7, None, 1, 1, 1, 4, 4, None, None, 0, None, None)
    assert st == _lib.ATLB_ERR_ARG and b"kind" in L.atlb_last_error()
    st = L.atlb_plan_geometry(None, None, 0, None, None, 0, 4, 4, 1.0, 3.0, 0, None, None, None)
    assert st == _lib.ATLB_ERR_ARG


def test_compute_entry_requires_cuda_tensors():
    import torch
    from x_b200 import functional as F
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    with pytest.raises(RuntimeError):
        F.splat(torch.zeros(3, 2), torch.ones(3), torch.zeros(3, dtype=torch.long), 1, 4, 4)
