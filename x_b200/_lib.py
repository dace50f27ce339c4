"""ctypes binding of libatlb200.so (C ABI declared in include/atl_b200.h).

Torch is only plumbing here: tensors provide device memory and the current CUDA stream.  There is
no CPU path -- every call requires CUDA tensors and raises if the library or a device is missing.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libatlb200.so"

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_dbl = ctypes.c_double
_int = ctypes.c_int
_size = ctypes.c_size_t

ATLB_OK, ATLB_ERR_ARG, ATLB_ERR_CUDA, ATLB_ERR_WORKSPACE, ATLB_ERR_UNSORTED, ATLB_ERR_OVERFLOW = range(6)
MOTION_TRANSLATION, MOTION_AFFINE, MOTION_DENSE = 0, 1, 2


class PlanGeom(ctypes.Structure):
    _fields_ = [("cell", ctypes.c_double), ("ox", ctypes.c_double), ("oy", ctypes.c_double),
                ("GW", ctypes.c_int64), ("GH", ctypes.c_int64), ("vmax", ctypes.c_float), ("S", ctypes.c_int32),
                ("t_lo", ctypes.c_float), ("t_hi", ctypes.c_float)]


class ExactCfg(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("theta", ctypes.c_void_p), ("Bt", ctypes.c_int64), ("Hg", ctypes.c_int64),
                ("Wg", ctypes.c_int64), ("B", ctypes.c_int64), ("H", ctypes.c_int64), ("W", ctypes.c_int64),
                ("h", ctypes.c_double), ("tau", ctypes.c_double), ("cut", ctypes.c_double),
                ("eps_frac", ctypes.c_double), ("S", ctypes.c_int64), ("visibility", ctypes.c_int32),
                ("n_check", ctypes.c_int64), ("src_begin", ctypes.c_int64), ("src_end", ctypes.c_int64),
                ("rng", ctypes.c_int32), ("rng_seed", ctypes.c_uint64), ("rng_call", ctypes.c_uint64)]


class UnitRates(ctypes.Structure):
    _fields_ = [("fp32_lane_ops", ctypes.c_double), ("fp32x2_lane_ops", ctypes.c_double), ("ex2", ctypes.c_double),
                ("red_f32", ctypes.c_double), ("red_v4", ctypes.c_double), ("smem_atomic", ctypes.c_double)]


# name -> (restype, argtypes)
_SIGS = {
    "atlb_last_error": (ctypes.c_char_p, []),
    "atlb_abi_version": (_int, []),
    "atlb_tile_ops_workspace_bytes": (_size, [_i64, _i64, _i64, _i64]),
    "atlb_blur": (_int, [_vp, _i64, _i64, _i64, _dbl, _vp, _vp]),
    "atlb_count_keys": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "atlb_sliced_score": (_int, [_i64, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _dbl, _dbl, _dbl, _i64, _i64,
                                 _vp, _vp]),
    "atlb_sliced_score_bwd": (_int, [_i64, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _dbl, _dbl, _dbl,
                                     _i64, _i64, _vp, _vp, _vp]),
    "atlb_flow_exact": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _dbl, _vp, _i64, _vp, _vp]),
    "atlb_flow_exact_bwd": (_int, [_int, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _dbl, _vp, _i64, _vp, _vp, _vp]),
    "atlb_flow_rk4": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _dbl, _vp, _i64, _int, _vp, _vp]),
    "atlb_flow_rk4_bwd": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _dbl, _vp, _i64, _int, _vp,
                                 _vp]),
    "atlb_rng_uniform2": (_int, [ctypes.c_uint64, ctypes.c_uint64, _i64, _vp, _vp]),
    "atlb_rng_normal2": (_int, [ctypes.c_uint64, ctypes.c_uint64, _i64, _vp, _vp]),
    "atlb_kernel_launches": (ctypes.c_uint64, []),
    "atlb_timing_enable": (_int, [_int]),
    "atlb_timing_read": (_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64),
                                _int]),
    "atlb_unit_rates_scratch_bytes": (_size, []),
    "atlb_measure_unit_rates": (_int, [ctypes.POINTER(UnitRates), _vp, _size, _vp]),
    "atlb_splat_bilinear_fwd": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _size, _vp]),
    "atlb_splat_bilinear_bwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _size, _vp]),
    "atlb_splat_gauss_workspace_bytes": (_size, [_i64, _i64, _i64, _i64]),
    "atlb_splat_gauss_fwd": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _dbl, _i64, _vp, _vp, _size, _vp]),
    "atlb_splat_gauss_bwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _dbl, _i64, _vp, _vp, _vp, _size, _vp]),
    "atlb_splat_gauss_bwd_pos": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _dbl, _i64, _vp, _vp, _size, _vp]),
    "atlb_gather_bilinear_fwd": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _size, _vp]),
    "atlb_gather_bilinear_bwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _size, _vp]),
    "atlb_voxel_grid": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _size, _vp]),
    "atlb_plan_geometry": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _dbl, _dbl, _i64, _vp,
                                  ctypes.POINTER(PlanGeom), _vp]),
    "atlb_plan_workspace_bytes": (_size, [_i64]),
    "atlb_plan_count": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _dbl, ctypes.POINTER(PlanGeom), _vp, _vp, _size,
                               ctypes.POINTER(ctypes.c_int64), _vp]),
    "atlb_plan_fill": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _dbl, ctypes.POINTER(PlanGeom), _vp, _vp, _i64, _vp,
                              _vp, _size, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "atlb_pair_workspace_bytes": (_size, [_i64, _i64]),
    "atlb_ats_pair_fwd": (_int, [_vp] * 10 + [_i64] * 6 + [_dbl] * 3 + [_vp, _vp, _size, _vp]),
    "atlb_ats_pair_fwd_noalloc": (_int, [_vp] * 10 + [_i64] * 6 + [_dbl] * 3 + [_vp, _vp]),
    "atlb_ats_pair_bwd": (_int, [_vp] * 11 + [_i64] * 6 + [_dbl] * 3 + [_i64, _vp, _vp, _size, _vp]),
    "atlb_window_counts": (_int, [_vp, _vp, _i64, _vp, _i64, _dbl, _vp, _vp, _vp]),
    "atlb_window_counts_keys": (_int, [_vp, _i64, _vp, _vp, _vp, _i64, _dbl, _vp, _vp]),
    "atlb_velocity": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp]),
    "atlb_velocity_bwd": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp]),
    "atlb_visible_fraction": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _i64,
                                     _dbl, _i64, _vp, _vp, _vp]),
    "atlb_traj_transport": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _int, _vp, _dbl, _dbl, _i64, _vp, _vp, _vp,
                                   _dbl, _vp, _i64, _vp, _vp]),
    "atlb_traj_transport_bwd": (_int, [_int, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _dbl, _dbl, _i64, _vp, _vp,
                                       _vp, _dbl, _vp, _i64, _vp, _vp, _vp]),
    "atlb_traj_records": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _vp, _dbl, _dbl, _i64, _vp, _i64, _vp, _vp, _dbl,
                                 _vp, _i64, _vp, _vp, _vp]),
    "atlb_traj_records_bwd": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _dbl, _dbl, _i64, _vp, _i64, _vp,
                                     _vp, _dbl, _vp, _i64, _vp, _vp, _vp]),
    "atlb_traj_targets": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _vp, _dbl, _dbl, _i64, _vp, _vp, _vp, _i64, _vp,
                                 _i64, _vp, _vp]),
    "atlb_traj_targets_bwd": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _dbl, _dbl, _i64, _vp, _vp, _vp,
                                     _i64, _vp, _i64, _vp, _vp]),
    "atlb_traj_visible_fraction": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _vp, _dbl, _dbl, _i64, _vp, _vp, _vp,
                                          _i64, _vp, _vp, _i64, _dbl, _i64, _i64, _vp, _vp]),
    "atlb_exact_prepare": (_int, [ctypes.POINTER(ExactCfg), _vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp,
                                  _vp, ctypes.POINTER(PlanGeom), _vp]),
    "atlb_exact_workspace_bytes": (_size, [ctypes.POINTER(ExactCfg), _i64, _i64, ctypes.POINTER(PlanGeom)]),
    "atlb_exact_forward": (_int, [ctypes.POINTER(ExactCfg), _vp, _vp, _i64, _i64, _vp, _vp, _vp,
                                  ctypes.POINTER(PlanGeom), _vp, _size, _vp, _vp, _vp, _vp]),
    "atlb_exact_backward": (_int, [ctypes.POINTER(ExactCfg), _vp, _vp, _i64, _i64, _vp, ctypes.POINTER(PlanGeom), _vp,
                                   _size, _vp, _vp, _vp, _vp, _vp]),
    "atlb_exact_prepare_forward": (_int, [ctypes.POINTER(ExactCfg), _vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _vp,
                                          _vp, _vp, _vp, ctypes.POINTER(PlanGeom), _vp, _size, _vp, _vp, _vp, _vp]),
}

_LIB = None


def exported_symbols():
    """Names of the entry points this binding expects (the declarations of include/atl_b200.h)."""
    return sorted(_SIGS)


def load_library():
    """Load libatlb200.so and bind every entry point (no device needed)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"x_b200: {LIB_PATH.name} is not built (python -m x_b200.build)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def lib():
    """The bound library, for compute calls: requires a CUDA device."""
    if not torch.cuda.is_available():
        raise RuntimeError("x_b200: no CUDA device; the anchored-score kernels have no CPU path")
    return load_library()


def check(status: int, what: str):
    if status != ATLB_OK:
        msg = load_library().atlb_last_error().decode(errors="replace")
        raise RuntimeError(f"x_b200.{what} failed (status {status}): {msg}")


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t):
    """Device address of a tensor (None for None)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def require_cuda(name: str, t: torch.Tensor, dtype=None):
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (x_b200 has no CPU path)")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def unit_rates(device=None) -> dict:
    """Execution-unit rates of the current (or given) CUDA device, operations per second (atlb_measure_unit_rates):
    fp32_lane_ops, fp32x2_lane_ops, ex2, red_f32, red_v4, smem_atomic.  Blocks for about 10 ms."""
    L = lib()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        nb = L.atlb_unit_rates_scratch_bytes()
        scratch = workspace(nb, dev)
        r = UnitRates()
        check(L.atlb_measure_unit_rates(ctypes.byref(r), ptr(scratch), nb, stream()), "measure_unit_rates")
    return {name: float(getattr(r, name)) for name, _ in UnitRates._fields_}


def timing_read(name: str, reset: bool = True):
    """(total milliseconds, launches) of a timed kernel since the last reset (see atlb_timing_enable)."""
    ms, n = ctypes.c_double(0), ctypes.c_int64(0)
    check(load_library().atlb_timing_read(name.encode(), ctypes.byref(ms), ctypes.byref(n), int(reset)), "timing_read")
    return float(ms.value), int(n.value)
