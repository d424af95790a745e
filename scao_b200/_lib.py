"""ctypes binding of ``libscao_b200.so`` (the C ABI in include/scao_b200.h).

The table layouts below mirror the C structs byte for byte; ``check_layout``
asserts the sizes at import.  Loading fails loudly: there is no CPU fallback
anywhere in the product path.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libscao_b200.so")

F32, BF16, F16 = 0, 1, 2

PARAM_DT = np.dtype([
    ("offset", "<i8"), ("numel", "<i8"), ("rows", "<i4"), ("cols", "<i4"),
    ("mode", "<i4"), ("dtype", "<i4"), ("leaf_begin", "<i4"), ("leaf_end", "<i4"),
    ("tile_begin", "<i4"), ("tile_end", "<i4"), ("chunk_begin", "<i4"),
    ("chunk_end", "<i4")], align=True)

STEP_DT = np.dtype([
    ("p_ptr", "<u8"), ("g_ptr", "<u8"), ("phase", "<i4"), ("clip", "<i4"),
    ("lr", "<f8"), ("alpha1", "<f8"),
    ("wd_mult", "<f4"), ("wd", "<f4"), ("beta1", "<f4"), ("beta2", "<f4"),
    ("beta3", "<f4"), ("c1", "<f4"), ("c2", "<f4"), ("c3", "<f4"),
    ("bc1", "<f4"), ("bc2", "<f4"), ("bc3", "<f4"), ("sqrt_bc2", "<f4"),
    ("eps", "<f4"), ("blend", "<f4"), ("one_minus_blend", "<f4"), ("tau", "<f4"),
    ("lars", "<f4"), ("diag_bias", "<f4"), ("rbc1", "<f4"), ("rbc2", "<f4"),
    ("rbc3", "<f4")], align=True)

LEAF_DT = np.dtype([
    ("param", "<i4"), ("row0", "<i4"), ("col0", "<i4"), ("a", "<i4"), ("b", "<i4"),
    ("ld", "<i4"), ("kmin", "<i4"), ("kmax", "<i4"), ("kpad", "<i4"), ("sl", "<i4"),
    ("sr", "<i4"), ("tile_begin", "<i4"), ("tile_end", "<i4"), ("panel_begin", "<i4"),
    ("panel_end", "<i4"), ("pad0", "<i4"),
    ("lq_off", "<i8"), ("rq_off", "<i8"), ("ul_off", "<i8"), ("ur_off", "<i8"),
    ("hl_off", "<i8"), ("hr_off", "<i8"), ("evl_off", "<i8"), ("evr_off", "<i8"),
    ("w_off", "<i8"), ("ua_off", "<i8"), ("ut_off", "<i8"), ("wa_off", "<i8")], align=True)

TILE_DT = np.dtype([("leaf", "<i4"), ("row0", "<i4"), ("col0", "<i4"), ("pad0", "<i4")])
PANEL_DT = np.dtype([("leaf", "<i4"), ("row0", "<i4"), ("nrows", "<i4"), ("pad0", "<i4")])
CHUNK_DT = np.dtype([("param", "<i4"), ("pad0", "<i4"), ("begin", "<i8"), ("end", "<i8")],
                    align=True)
STRIP_DT = np.dtype([("param", "<i4"), ("count", "<i4"), ("stride", "<i4"), ("pad0", "<i4"),
                     ("begin", "<i8")], align=True)

_P = C.c_void_p


class FilterDev(C.Structure):
    _fields_ = [
        ("mode", C.c_int32), ("n_sel", C.c_int32), ("sel", _P), ("mag_ema", _P),
        ("fp", _P), ("hist", _P), ("sel_part", _P),
        ("base", C.c_double), ("min_s", C.c_double), ("max_s", C.c_double),
        ("norm_coeff", C.c_double), ("ema", C.c_float), ("ema_c", C.c_float),
        ("noise_on", C.c_int32), ("noise_std", C.c_float),
        ("noise_seed", C.c_uint64), ("noise_step", C.c_uint64),
        ("gsnr_on", C.c_int32), ("gsnr_thr", C.c_float),
    ]


FILTER_PARAM_DT = np.dtype([
    ("norm_ema", "<f8"), ("global_ref", "<f8"), ("sparsity", "<f8"),
    ("rem_lo", "<i8"), ("rem_hi", "<i8"), ("pre_lo", "<u4"), ("pre_hi", "<u4"),
    ("w", "<f4"), ("thr", "<f4"), ("gsq", "<f4"), ("first", "<i4"), ("nan", "<i4"),
    ("sel_begin", "<i4"), ("sel_end", "<i4"), ("pad0", "<i4")])


class PlanDev(C.Structure):
    _fields_ = [
        ("n_params", C.c_int32), ("n_leaves", C.c_int32), ("n_tiles", C.c_int32),
        ("n_panels", C.c_int32), ("n_chunks", C.c_int32), ("int8_ema", C.c_int32),
        ("kpad_max", C.c_int32), ("p_stride", C.c_int32),
        ("kron_dtypes", C.c_int32), ("max_leaf_rows_tiles", C.c_int32),
        ("params", _P), ("leaves", _P), ("tiles", _P), ("panels", _P), ("chunks", _P),
        ("step", _P),
        ("exp_avg", _P), ("exp_avg_sq", _P), ("exp_avg_diff", _P), ("prev_grad", _P),
        ("diag_ema", _P), ("fac", _P), ("absmax", _P), ("u", _P), ("ev", _P), ("k", _P),
        ("eig_y", _P), ("eig_x", _P), ("eig_ax", _P), ("eig_h", _P), ("eig_v", _P),
        ("eig_aux", _P), ("w", _P), ("p_part", _P), ("tile_part", _P), ("chunk_part", _P),
        ("upd", _P), ("upd32", _P), ("leaf_nat2", _P), ("param_scalars", _P),
        ("global_norm_ema", _P), ("slow", _P), ("slow32", _P), ("ua", _P), ("ut", _P), ("wa", _P), ("counters", _P),
        ("diag_list", _P), ("flat_list", _P), ("p_list", _P),
        ("n_diag", C.c_int32), ("n_flat", C.c_int32), ("n_p", C.c_int32), ("proj_fallback", C.c_int32),
        ("apply_fallback", C.c_int32), ("sm_reserve", C.c_int32),
        ("la_fused", C.c_int32), ("la_init", C.c_int32), ("la_alpha", C.c_float),
        ("pad5_", C.c_int32),
        ("err", _P),
        ("tmaps", _P), ("tmaps_ok", C.c_int32), ("gnorm_host", C.c_int32),
        ("filt", FilterDev),
        ("strips", _P), ("strip_part", _P), ("n_strips", C.c_int32), ("pad6_", C.c_int32),
        ("eig_img", _P), ("eig_img_stride", C.c_int64),
    ]


def check_layout():
    assert PARAM_DT.itemsize == 56, PARAM_DT.itemsize
    assert STEP_DT.itemsize == 128, STEP_DT.itemsize
    assert LEAF_DT.itemsize == 160, LEAF_DT.itemsize
    assert CHUNK_DT.itemsize == 24, CHUNK_DT.itemsize
    assert STRIP_DT.itemsize == 24, STRIP_DT.itemsize
    assert FILTER_PARAM_DT.itemsize == 80, FILTER_PARAM_DT.itemsize
    assert C.sizeof(FilterDev) == 120, C.sizeof(FilterDev)


check_layout()

# name -> (restype, argtypes); every symbol declared in include/scao_b200.h
SIGNATURES = {
    "scao_fused_kronecker_precond": (C.c_int, [_P, _P, _P, _P, _P, _P, C.c_int, C.c_int,
                                               C.c_int, C.c_int, _P, _P]),
    "scao_fused_precond_scratch_bytes": (C.c_int64, [C.c_int, C.c_int, C.c_int]),
    "scao_low_rank_precond_mm": (C.c_int, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int,
                                           C.c_int, _P, _P]),
    "scao_low_rank_precond_mm_scratch_bytes": (C.c_int64, [C.c_int, C.c_int, C.c_int,
                                                           C.c_int]),
    "scao_int8_ema_update": (C.c_int, [_P, C.c_double, _P, C.c_double, C.c_int64, _P, _P,
                                       _P, _P]),
    "scao_int8_ema_scratch_bytes": (C.c_int64, [C.c_int64]),
    "scao_int8_ema_update_noalloc": (C.c_int, [_P, C.c_double, _P, C.c_double, C.c_int64, _P,
                                               _P, _P]),
    "scao_int8_ema_update_noalloc_max_n": (C.c_int64, []),
    "scao_quantize_sym_int8": (C.c_int, [_P, C.c_int64, _P, _P, _P, _P]),
    "scao_dequantize_sym_int8": (C.c_int, [_P, C.c_double, C.c_int64, _P, _P]),
    "scao_plan_curvature": (C.c_int, [C.POINTER(PlanDev), _P, C.c_int, C.c_int, C.c_int,
                                      C.c_double, _P, C.c_int64, _P, _P, _P, _P, _P]),
    "scao_ema_scratch_bytes": (C.c_int64, [C.c_int, C.c_int, C.c_int]),
    "scao_plan_tensor_maps": (C.c_int, [C.POINTER(PlanDev), _P, _P, _P]),
    "scao_wait_timeout_check": (C.c_int, [_P, C.c_uint, _P]),
    "scao_plan_grad_norms": (C.c_int, [C.POINTER(PlanDev), _P, _P]),
    "scao_plan_curvature_diag": (C.c_int, [C.POINTER(PlanDev), _P, C.c_int, C.c_double, _P]),
    "scao_plan_eigen": (C.c_int, [C.POINTER(PlanDev), _P, C.c_int, _P, _P, C.c_int,
                                  C.c_float, _P, C.c_int, C.c_int, _P]),
    "scao_plan_step": (C.c_int, [C.POINTER(PlanDev), _P]),
    "scao_plan_prep_factors": (C.c_int, [C.POINTER(PlanDev), _P, C.c_int, _P]),
    "scao_plan_lookahead": (C.c_int, [C.POINTER(PlanDev), C.c_float, C.c_int, _P]),
    "scao_version": (C.c_char_p, []),
    "scao_divc_check": (C.c_int, [_P, _P, C.c_int, _P, _P]),
    "scao_tc_selftest": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, _P, C.c_int, _P]),
    "scao_launch_count": (C.c_int64, []),
    "scao_prof_enable": (None, [C.c_int]),
    "scao_prof_read": (C.c_int, [_P, _P, C.c_int]),
    "scao_prof_reset": (None, []),
    "scao_prof_name": (C.c_char_p, [C.c_int]),
    "scao_prof_slots": (C.c_int, []),
}

_lib = None


class ScaoError(RuntimeError):
    pass


def lib():
    """Load the CUDA library (raises if it is missing -- no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        try:
            from . import build as _build
            _build.build()
        except Exception as e:  # noqa: BLE001
            raise ScaoError(
                f"scao_b200 CUDA library not built ({LIB_PATH}) and building it failed: {e}; "
                "run `python -m scao_b200.build` (needs nvcc, sm_100a).") from e
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(rc, what):
    if rc != 0:
        raise ScaoError(f"{what} failed with status {rc}")


def prof_read():
    """{kernel slot name: (total ms, launches)} accumulated since the last reset."""
    L = lib()
    n = L.scao_prof_slots()
    ms = (C.c_double * n)()
    cnt = (C.c_int64 * n)()
    check(L.scao_prof_read(C.cast(ms, _P), C.cast(cnt, _P), n), "scao_prof_read")
    return {L.scao_prof_name(i).decode(): (ms[i], cnt[i]) for i in range(n) if cnt[i]}
