"""ctypes binding of ``libngdn2.so`` (the C ABI declared in include/ngdn2.h).

The structs below mirror ``ngdn2_fwd_args``, ``ngdn2_update_args``,
``ngdn2_step_args``, ``ngdn2_bwd_args`` and ``ngdn2_update_bwd_args`` field
for field; ``check_layout()`` compares their sizes with the library's own
``sizeof``. Loading fails loudly: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libngdn2.so"

ABI_VERSION = 2
MAX_LEVELS = 8
CHUNK = 64

F32, BF16, F16 = 0, 1, 2
PROMOTION = {"learned": 0, "merge": 1}
PATHS = {"auto": 0, "simt": 1, "tc": 2, "tc_seg": 3}
PATH_NAMES = {1: "simt", 2: "tc", 3: "tc_seg"}

ERR_CHUNK_SIZE = -1
ERR_N_POW2 = -2
ERR_BLOCK_V = -3
ERR_DIVISIBLE = -4
ERR_UNIT_STRIDE = -5
ERR_INCONSISTENT = -6

STATUS_WAIT_TIMEOUT = 1
STATUS_GATE_TIMEOUT = 2

c_i32, c_i64, c_ptr = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p


def _tok(name, rank):
    return [(name, c_ptr), (f"{name}_dtype", c_i32), (f"{name}_stride", c_i64 * rank)]


class FwdArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32), ("path", c_i32),
        ("B", c_i32), ("T", c_i32), ("H", c_i32), ("K", c_i32), ("V", c_i32), ("L", c_i32),
        ("chunk_size", c_i32), ("promotion", c_i32), ("dtype", c_i32), ("param_dtype", c_i32),
        ("scale", ctypes.c_float), ("n_max", c_i32),
        ("n_queries", c_i32 * MAX_LEVELS), ("firing", c_i32 * MAX_LEVELS),
        *_tok("q", 5), *_tok("k", 4), *_tok("v", 4), *_tok("g", 4), *_tok("b", 4),
        *_tok("w", 4), *_tok("mix", 4),
        ("query_banks", c_ptr), ("key_projections", c_ptr), ("b_projections", c_ptr),
        ("w_projections", c_ptr), ("g_projections", c_ptr),
        ("initial_state", c_ptr), ("o", c_ptr), ("final_state", c_ptr),
        ("workspace", c_ptr), ("workspace_bytes", ctypes.c_size_t), ("status", c_ptr),
        ("gate", c_ptr), ("gate_polls", ctypes.c_uint32),
    ]


class UpdateArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32),
        ("B", c_i32), ("NF", c_i32), ("NG", c_i32), ("H", c_i32), ("K", c_i32),
        ("V", c_i32), ("N", c_i32), ("block_v", c_i32), ("dtype", c_i32), ("g_dtype", c_i32),
        ("keys", c_ptr), ("keys_stride", c_i64 * 5),
        ("values", c_ptr), ("g", c_ptr), ("b", c_ptr), ("w", c_ptr),
        ("initial_state", c_ptr), ("states", c_ptr), ("final_state", c_ptr),
    ]


class StepArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32),
        ("B", c_i32), ("H", c_i32), ("K", c_i32), ("V", c_i32), ("L", c_i32),
        ("chunk_size", c_i32), ("promotion", c_i32), ("dtype", c_i32), ("param_dtype", c_i32),
        ("scale", ctypes.c_float), ("n_max", c_i32),
        ("n_queries", c_i32 * MAX_LEVELS), ("firing", c_i32 * MAX_LEVELS),
        *_tok("q", 4), *_tok("k", 3), *_tok("v", 3), *_tok("g", 3), *_tok("b", 3),
        *_tok("w", 3), *_tok("mix", 3),
        ("query_banks", c_ptr), ("key_projections", c_ptr), ("b_projections", c_ptr),
        ("w_projections", c_ptr), ("g_projections", c_ptr),
        ("positions", c_ptr), ("position", c_i64),
        ("state_in", c_ptr), ("state_out", c_ptr), ("o", c_ptr),
        ("workspace", c_ptr), ("workspace_bytes", ctypes.c_size_t), ("status", c_ptr),
    ]


class UpdateBwdArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32),
        ("B", c_i32), ("NF", c_i32), ("NG", c_i32), ("H", c_i32), ("K", c_i32),
        ("V", c_i32), ("N", c_i32), ("block_v", c_i32), ("dtype", c_i32), ("g_dtype", c_i32),
        ("has_init", c_i32),
        ("states", c_ptr), ("keys", c_ptr), ("keys_stride", c_i64 * 5),
        ("values", c_ptr), ("g", c_ptr), ("b", c_ptr), ("w", c_ptr),
        ("d_states", c_ptr), ("d_final", c_ptr),
        ("dkeys", c_ptr), ("dvalues", c_ptr), ("dg", c_ptr), ("db", c_ptr), ("dw", c_ptr),
        ("dinit", c_ptr), ("workspace", c_ptr), ("workspace_bytes", ctypes.c_size_t),
    ]


class BwdArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32), ("fwd", FwdArgs), *_tok("d_o", 4), ("d_final", c_ptr),
        ("dq", c_ptr), ("dk", c_ptr), ("dv", c_ptr), ("dg", c_ptr), ("db", c_ptr),
        ("dw", c_ptr), ("dmix", c_ptr),
        ("dquery_banks", c_ptr), ("dkey_projections", c_ptr), ("db_projections", c_ptr),
        ("dw_projections", c_ptr), ("dg_projections", c_ptr), ("dinitial_state", c_ptr),
        ("workspace", c_ptr), ("workspace_bytes", ctypes.c_size_t),
    ]


EXPORTS = (
    "ngdn2_abi_version", "ngdn2_sizeof_fwd_args", "ngdn2_sizeof_update_args",
    "ngdn2_error_string", "ngdn2_fwd_workspace_size", "ngdn2_fwd_select_path",
    "ngdn2_fwd", "ngdn2_fwd_stage", "ngdn2_fwd_num_launches", "ngdn2_update_state",
    "ngdn2_fwd_noalloc", "ngdn2_sizeof_step_args", "ngdn2_step_workspace_size", "ngdn2_step",
    "ngdn2_sizeof_bwd_args", "ngdn2_bwd_workspace_size", "ngdn2_bwd", "ngdn2_bwd_num_launches",
    "ngdn2_sizeof_update_bwd_args", "ngdn2_update_bwd_workspace_size", "ngdn2_update_state_bwd",
)

_LIB = None


def load(path: str | os.PathLike | None = None):
    """Load the library (once) and declare its signatures."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = pathlib.Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python -m nested_recurrent_memory_b200.build`"
            " (there is no fallback implementation)")
    lib = ctypes.CDLL(str(p))
    lib.ngdn2_abi_version.restype = ctypes.c_int
    lib.ngdn2_sizeof_fwd_args.restype = ctypes.c_size_t
    lib.ngdn2_sizeof_update_args.restype = ctypes.c_size_t
    lib.ngdn2_error_string.restype = ctypes.c_char_p
    lib.ngdn2_error_string.argtypes = [ctypes.c_int]
    lib.ngdn2_fwd_workspace_size.argtypes = [ctypes.POINTER(FwdArgs), ctypes.POINTER(ctypes.c_size_t)]
    lib.ngdn2_fwd_workspace_size.restype = ctypes.c_int
    lib.ngdn2_fwd_select_path.argtypes = [ctypes.POINTER(FwdArgs)]
    lib.ngdn2_fwd_select_path.restype = ctypes.c_int
    lib.ngdn2_fwd.argtypes = [ctypes.POINTER(FwdArgs), c_ptr]
    lib.ngdn2_fwd.restype = ctypes.c_int
    lib.ngdn2_fwd_stage.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_int, c_ptr]
    lib.ngdn2_fwd_stage.restype = ctypes.c_int
    lib.ngdn2_fwd_num_launches.argtypes = [ctypes.POINTER(FwdArgs)]
    lib.ngdn2_fwd_num_launches.restype = ctypes.c_int
    lib.ngdn2_update_state.argtypes = [ctypes.POINTER(UpdateArgs), c_ptr]
    lib.ngdn2_update_state.restype = ctypes.c_int
    lib.ngdn2_fwd_noalloc.argtypes = [ctypes.POINTER(FwdArgs), c_ptr]
    lib.ngdn2_fwd_noalloc.restype = ctypes.c_int
    lib.ngdn2_sizeof_step_args.restype = ctypes.c_size_t
    lib.ngdn2_step_workspace_size.argtypes = [ctypes.POINTER(StepArgs), ctypes.POINTER(ctypes.c_size_t)]
    lib.ngdn2_step_workspace_size.restype = ctypes.c_int
    lib.ngdn2_step.argtypes = [ctypes.POINTER(StepArgs), c_ptr]
    lib.ngdn2_step.restype = ctypes.c_int
    lib.ngdn2_sizeof_bwd_args.restype = ctypes.c_size_t
    lib.ngdn2_bwd_workspace_size.argtypes = [ctypes.POINTER(BwdArgs), ctypes.POINTER(ctypes.c_size_t)]
    lib.ngdn2_bwd_workspace_size.restype = ctypes.c_int
    lib.ngdn2_bwd.argtypes = [ctypes.POINTER(BwdArgs), c_ptr]
    lib.ngdn2_bwd.restype = ctypes.c_int
    lib.ngdn2_bwd_num_launches.argtypes = [ctypes.POINTER(BwdArgs)]
    lib.ngdn2_bwd_num_launches.restype = ctypes.c_int
    lib.ngdn2_sizeof_update_bwd_args.restype = ctypes.c_size_t
    lib.ngdn2_update_bwd_workspace_size.argtypes = [ctypes.POINTER(UpdateBwdArgs),
                                                    ctypes.POINTER(ctypes.c_size_t)]
    lib.ngdn2_update_bwd_workspace_size.restype = ctypes.c_int
    lib.ngdn2_update_state_bwd.argtypes = [ctypes.POINTER(UpdateBwdArgs), c_ptr]
    lib.ngdn2_update_state_bwd.restype = ctypes.c_int
    if path is None:
        _LIB = lib
    return lib


def check_layout(lib=None) -> None:
    lib = lib or load()
    if lib.ngdn2_abi_version() != ABI_VERSION:
        raise RuntimeError("libngdn2 ABI version mismatch")
    if lib.ngdn2_sizeof_fwd_args() != ctypes.sizeof(FwdArgs):
        raise RuntimeError("ngdn2_fwd_args layout mismatch")
    if lib.ngdn2_sizeof_update_args() != ctypes.sizeof(UpdateArgs):
        raise RuntimeError("ngdn2_update_args layout mismatch")
    if lib.ngdn2_sizeof_step_args() != ctypes.sizeof(StepArgs):
        raise RuntimeError("ngdn2_step_args layout mismatch")
    if lib.ngdn2_sizeof_bwd_args() != ctypes.sizeof(BwdArgs):
        raise RuntimeError("ngdn2_bwd_args layout mismatch")
    if lib.ngdn2_sizeof_update_bwd_args() != ctypes.sizeof(UpdateBwdArgs):
        raise RuntimeError("ngdn2_update_bwd_args layout mismatch")


def error_string(code: int) -> str:
    return load().ngdn2_error_string(code).decode()
