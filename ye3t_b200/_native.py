"""ctypes binding of the C-ABI library ``ye3t_b200/lib/libye3t_b200.so``.

The declarations mirror ``include/ye3t_b200.h``.  There is no fallback: if the
library is missing or fails to load, every native operation raises
:class:`NativeUnavailable` naming the build command.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libye3t_b200.so")

ABI_VERSION = 8
F32, F64, C64, C128 = 0, 1, 2, 3
STATUS_INDEX_RANGE = 1
STATUS_CAPACITY = 2
STATUS_TABLE = 4
STATUS_TIMEOUT = 8

_DTYPE_CODE = {torch.float32: F32, torch.float64: F64, torch.complex64: C64, torch.complex128: C128}

I64 = ctypes.c_int64
I32 = ctypes.c_int32
VP = ctypes.c_void_p
P64 = ctypes.POINTER(ctypes.c_int64)
DBL = ctypes.c_double


class NativeUnavailable(RuntimeError):
    pass


class NativeError(RuntimeError):
    pass


class AceTables(ctypes.Structure):
    """``y3b_ace_tables`` (include/ye3t_b200.h)."""

    _fields_ = [
        ("nmax", I64), ("lmax", I64), ("smem_entries", I64), ("feature_count", I64), ("item_count", I64),
        ("phase_count", I64), ("sym_output_count", I64), ("items", VP), ("item_coef", VP), ("phases", VP),
        ("sym_outputs", VP), ("sym_term_factors", VP), ("sym_term_coeff", VP),
        ("group_count", I64), ("groups", VP), ("group_offsets", VP),
        ("sym_grad_count", I64), ("sym_grad_offsets", VP), ("sym_grad_index", VP), ("sym_grad_coeff", VP),
        ("sym_term_count", I64),
    ]


class RecoupledTables(ctypes.Structure):
    """``y3b_recoupled_tables`` (include/ye3t_b200.h)."""

    _fields_ = [
        ("pass_count", I32), ("max_pass_components", I32), ("row_width", I32), ("dot_count", I32),
        ("component_count", I64), ("cg_count", I64), ("own_count", I64), ("bp_count", I64),
        ("pass_begin", VP), ("comp", VP), ("cg_index", VP), ("cg_value", VP), ("own", VP),
        ("bp_begin", VP), ("bp_gi", VP), ("bp_other", VP), ("bp_value", VP),
        ("feature_count", I64), ("feat_count", I64), ("dot_begin", VP), ("dot", VP), ("feat_index", VP),
        ("feat_weight", VP), ("atoms_per_cta", I32), ("threads_per_cta", I32),
    ]


class RecoupledSymTables(ctypes.Structure):
    """``y3b_recoupled_sym_tables`` (include/ye3t_b200.h)."""

    _fields_ = [
        ("pass_count", I32), ("max_pass_components", I32), ("row_width", I32), ("dot_count", I32),
        ("component_count", I64), ("cg_count", I64), ("own_count", I64), ("bp_count", I64),
        ("pass_begin", VP), ("comp", VP), ("cg_index", VP), ("cg_value", VP), ("own", VP),
        ("bp_begin", VP), ("bp_gi", VP), ("bp_other", VP), ("bp_value", VP), ("mirror", VP),
        ("dot_begin", VP), ("dot", VP), ("atoms_per_cta", I32), ("threads_per_cta", I32),
    ]


class RecoupledTileTables(ctypes.Structure):
    """``y3b_recoupled_tile_tables`` (include/ye3t_b200.h)."""

    _fields_ = [
        ("rows", I32), ("pass_count", I32), ("tile_count", I64), ("step_count", I64), ("item_count", I64),
        ("group_count", I64), ("pack_count", I64),
        ("tile_begin", VP), ("tile_row", VP), ("tile_col_begin", VP), ("col_comp", VP),
        ("bp_item_begin", VP), ("t_item_begin", VP), ("t_item", VP), ("bp_group_begin", VP), ("bp_group_off", VP),
        ("bp_pack", VP), ("unit_count", I64), ("fix_count", I64), ("scratch_slots", I32), ("unit_begin", VP),
        ("unit", VP), ("fix_begin", VP), ("fix", VP), ("kval", VP),
    ]


_SIGS = {
    "y3b_abi_version": (I32, []),
    "y3b_last_error": (ctypes.c_char_p, []),
    "y3b_factorized_schedule_evaluate": (ctypes.c_int, [ctypes.c_int, VP, I64, I64, I64, I64, VP, VP, VP, VP,
                                                        I64, I64, VP, VP, VP]),
    "y3b_factorized_schedule_adjoint": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, I64, I64, I64, VP, VP, I64, I64,
                                                       VP, VP, VP, VP, VP, VP]),
    "y3b_symmetric_power_monomial": (ctypes.c_int, [ctypes.c_int, VP, I64, I64, VP, VP, VP, I64, I64, VP, VP]),
    "y3b_symmetric_power_shared_monomial": (ctypes.c_int, [ctypes.c_int, VP, I64, I64, VP, I64, VP, I64, VP, VP, I64,
                                                           VP, VP, VP]),
    "y3b_scheduled_radial_angular_channels": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, VP, VP, I64, VP, VP, I64, VP,
                                                             VP, VP, VP, I64, VP, VP, VP, VP]),
    "y3b_symmetric_power_monomial_adjoint": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, I64, VP, VP, VP, I64, I64, VP,
                                                            VP, VP]),
    "y3b_plain_site_basis_product_adjoint": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, VP, VP, I64, VP, VP, VP, VP, VP,
                                                            VP, I64, VP, VP, I64, VP, VP, VP, VP, VP, VP]),
    "y3b_plain_site_basis_product": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, VP, VP, I64, VP, VP, VP, VP, I64, VP,
                                                    VP, I64, VP, VP, VP, VP, VP, VP]),
    "y3b_cheb_exp_cos_radial_table": (ctypes.c_int, [ctypes.c_int, VP, VP, VP, I64, I64, VP, VP, VP]),
    "y3b_spherical_harmonics_table": (ctypes.c_int, [ctypes.c_int, VP, I64, I64, ctypes.c_int, DBL, VP, VP,
                                                     VP]),
    "y3b_density_accumulate_workspace_bytes": (I64, [I64, I64]),
    "y3b_density_accumulate": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, I64, I64, VP, I64, VP, VP, VP]),
    "y3b_density_accumulate_noalloc": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, I64, I64, VP, VP, VP]),
    "y3b_density_accumulate_csr": (ctypes.c_int, [ctypes.c_int, VP, VP, VP, I64, I64, VP, VP]),
    "y3b_density_accumulate_adjoint": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, I64, I64, VP, VP, VP]),
    "y3b_neighbor_workspace_bytes": (I64, [I64, DBL, DBL]),
    "y3b_neighbor_count": (ctypes.c_int, [VP, I64, I64, I64, DBL, DBL, VP, I64, VP, VP]),
    "y3b_neighbor_fill": (ctypes.c_int, [VP, I64, I64, I64, DBL, DBL, VP, I64, VP, VP, VP]),
    "y3b_neighbor_cells_per_side": (I64, [DBL, DBL]),
    "y3b_neighbor_count_window": (ctypes.c_int, [VP, I64, I64, I64, DBL, DBL, I64, I64, VP, I64, VP, VP, VP]),
    "y3b_neighbor_fill_window": (ctypes.c_int, [VP, I64, I64, I64, DBL, DBL, I64, I64, VP, I64, VP, I64, VP, VP,
                                                VP]),
    "y3b_ace_density": (ctypes.c_int, [VP, VP, I64, I64, I64, DBL, VP, VP, VP, I64, I64, I64, DBL, DBL, VP, VP,
                                       VP]),
    "y3b_ace_features": (ctypes.c_int, [ctypes.POINTER(AceTables), VP, I64, VP, VP]),
    "y3b_ace_features_typed": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(AceTables), VP, I64, VP, VP]),
    "y3b_ace_energy": (ctypes.c_int, [ctypes.POINTER(AceTables), VP, I64, VP, VP, I64, VP, VP]),
    "y3b_radial_channel_contraction": (ctypes.c_int, [ctypes.c_int, VP, VP, VP, I64, I64, I64, VP, VP, VP]),
    "y3b_ace_density_mixed": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, I64, I64, DBL, VP, VP, VP, I64, I64, I64,
                                             I64, DBL, DBL, VP, VP, VP]),
    "y3b_ace_density_mixed_split_workspace_bytes": (I64, [ctypes.c_int, I64, I64, I64, I64, I64]),
    "y3b_ace_density_mixed_split": (ctypes.c_int, [ctypes.c_int, VP, VP, I64, I64, I64, DBL, VP, VP, VP, I64, I64,
                                                   I64, I64, DBL, DBL, VP, I64, VP, VP, VP]),
    "y3b_ace_energy_grad": (ctypes.c_int, [ctypes.POINTER(AceTables), VP, I64, VP, VP, I64, VP, VP, VP, VP]),
    "y3b_ace_recoupled_energy_grad": (ctypes.c_int, [ctypes.POINTER(RecoupledTables), VP, I64, VP, VP, I64, VP,
                                                     VP, VP, VP]),
    "y3b_ace_recoupled_energy": (ctypes.c_int, [ctypes.POINTER(RecoupledTables), VP, I64, VP, VP, I64, VP, VP,
                                                VP]),
    "y3b_ace_recoupled_features": (ctypes.c_int, [ctypes.POINTER(RecoupledTables), VP, I64, VP, VP, VP]),
    "y3b_ace_recoupled_energy_grad_symmetric": (ctypes.c_int, [ctypes.POINTER(RecoupledSymTables), VP, I64, VP,
                                                               VP, I64, VP, VP, VP, VP]),
    "y3b_ace_recoupled_energy_symmetric": (ctypes.c_int, [ctypes.POINTER(RecoupledSymTables), VP, I64, VP, VP,
                                                          I64, VP, VP, VP]),
    "y3b_ace_recoupled_energy_grad_tiled": (ctypes.c_int, [ctypes.POINTER(RecoupledSymTables),
                                                           ctypes.POINTER(RecoupledTileTables), VP, I64, VP, VP,
                                                           I64, VP, VP, VP, VP]),
    "y3b_ace_edge_grad": (ctypes.c_int, [VP, VP, I64, I64, I64, DBL, VP, VP, VP, I64, I64, I64, DBL, DBL, VP, VP,
                                         VP, VP]),
    "y3b_forces_gather": (ctypes.c_int, [VP, VP, I64, VP, VP, VP, VP]),
    "y3b_forces_scatter": (ctypes.c_int, [VP, VP, I64, I64, I64, VP, VP, VP]),
    "y3b_fma_peak_launch": (ctypes.c_int, [ctypes.c_int, I32, I32, I32, VP, ctypes.POINTER(DBL), VP]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load the library once; raise NativeUnavailable when it cannot be used."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeUnavailable(
                f"{LIB_PATH} is missing; build it with `make -C ye3t_b200/csrc` "
                "(or __graft_entry__.build()). ye3t_b200 has no CPU fallback.")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        abi = handle.y3b_abi_version()
        if abi != ABI_VERSION:
            raise NativeUnavailable(f"{LIB_PATH}: ABI {abi}, expected {ABI_VERSION}; rebuild the library")
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().y3b_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed ({rc}): {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors, what: str) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"{what}: ye3t_b200 evaluates on CUDA devices only (got a {t.device} tensor); "
                             "there is no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{what}: tensors are on different devices ({dev}, {t.device})")
    if dev is None:
        raise ValueError(f"{what}: no tensor argument")
    return dev


def exported_symbols():
    return sorted(_SIGS)
