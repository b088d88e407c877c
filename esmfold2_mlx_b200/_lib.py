"""ctypes binding of ``libtmu.so`` (the C ABI in ``include/tmu.h``).

The shared library is built in-tree (``python -m esmfold2_mlx_b200.build``) and loaded from
``esmfold2_mlx_b200/lib/``.  There is no fallback: if it is missing, every CUDA entry point
raises ``TmuError`` naming the build command.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
LIB_PATH = os.path.join(LIB_DIR, "libtmu.so")

TMU_STATUS_BYTES = 256
TMU_IPC_HANDLE_BYTES = 64

STATUS_NAMES = {
    0: "TMU_OK",
    1: "TMU_ERR_INVALID_ARGUMENT",
    2: "TMU_ERR_MISALIGNED",
    3: "TMU_ERR_WORKSPACE_TOO_SMALL",
    4: "TMU_ERR_UNSUPPORTED",
    5: "TMU_ERR_CUDA",
    6: "TMU_ERR_DEVICE_TIMEOUT",
    7: "TMU_ERR_ARCH",
    8: "TMU_ERR_DRIVER",
    9: "TMU_ERR_SMEM_LAYOUT",
}

# Every symbol include/tmu.h declares, with its ctypes signature.
_vp, _i, _f, _sz, _ull = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_ulonglong


class TmuTrimulWeights(ctypes.Structure):
    """Mirror of ``tmu_trimul_weights``."""

    _fields_ = [
        ("ln_in_w", _vp), ("ln_in_b", _vp), ("w_proj", _vp), ("b_proj", _vp),
        ("ln_mix_w", _vp), ("ln_mix_b", _vp), ("w_emit", _vp), ("b_emit", _vp),
        ("w_gate", _vp), ("b_gate", _vp),
    ]


class TmuPairLayout(ctypes.Structure):
    """Mirror of ``tmu_pair_layout``."""

    _fields_ = [
        ("B", ctypes.c_int), ("rows", ctypes.c_int), ("cols", ctypes.c_int),
        ("stride_b", ctypes.c_longlong), ("stride_row", ctypes.c_longlong), ("stride_col", ctypes.c_longlong),
        ("mask_stride_b", ctypes.c_longlong), ("mask_stride_row", ctypes.c_longlong),
        ("mask_stride_col", ctypes.c_longlong),
    ]


class TmuTransitionWeights(ctypes.Structure):
    """Mirror of ``tmu_transition_weights``."""

    _fields_ = [("ln_w", _vp), ("ln_b", _vp), ("w12", _vp), ("w3", _vp)]


TMU_ACT_SWIGLU, TMU_ACT_RELU = 0, 1


class TmuCondTransitionWeights(ctypes.Structure):
    """Mirror of ``tmu_cond_transition_weights``."""

    _fields_ = [("ln_w", _vp), ("ln_b", _vp), ("w12", _vp), ("w3", _vp)]


class TmuParcaeWeights(ctypes.Structure):
    """Mirror of ``tmu_parcae_weights``."""

    _fields_ = [("ln_w", _vp), ("ln_b", _vp), ("a", _vp), ("b_split", _vp)]


class TmuPairCondWeights(ctypes.Structure):
    """Mirror of ``tmu_pair_cond_weights``."""

    _fields_ = [("ln_w", _vp), ("ln_b", _vp), ("proj", _vp), ("n_transitions", _i),
                ("transitions", ctypes.POINTER(TmuCondTransitionWeights)), ("bias_w", _vp), ("bias_b", _vp)]

_W = ctypes.POINTER(TmuTrimulWeights)
_G = ctypes.POINTER(TmuPairLayout)
_TW = ctypes.POINTER(TmuTransitionWeights)
SIGNATURES = {
    "tmu_version": (ctypes.c_char_p, []),
    "tmu_status_name": (ctypes.c_char_p, [_i]),
    "tmu_last_error": (ctypes.c_char_p, []),
    "tmu_device_check": (_i, []),
    "tmu_row_pitch": (_i, [_i]),
    "tmu_proj_row_order": (_i, [_i, ctypes.POINTER(_i)]),
    "tmu_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "tmu_set_wait_timeout_ns": (_ull, [_ull]),
    "tmu_reset_status": (_i, [_vp, _vp]),
    "tmu_read_status": (_i, [_vp, _vp, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "tmu_read_first_error": (_i, [_vp, _vp, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "tmu_trace_arm": (_i, [_vp, _vp]),
    "tmu_trace_read": (_i, [_vp, _vp, ctypes.POINTER(_ull), ctypes.POINTER(_ull)]),
    "tmu_project_gate": (_i, [_vp, _vp, _W, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "tmu_contract": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "tmu_emit_residual": (_i, [_vp, _vp, _vp, _W, _i, _i, _i, _i, _f, _vp, _vp]),
    "tmu_project_gate_ex": (_i, [_vp, _vp, _G, _W, _i, _i, _vp, _vp, _vp, _vp]),
    "tmu_contract_ex": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp]),
    "tmu_emit_residual_ex": (_i, [_vp, _vp, _vp, _i, _i, _i, _W, _i, _i, _f, _vp, _vp]),
    "tmu_trimul": (_i, [_vp, _vp, _vp, _W, _i, _i, _i, _i, _i, _f, _vp, _sz, _vp]),
    "tmu_trimul_noalloc": (_i, [_vp, _vp, _vp, _W, _i, _i, _i, _i, _i, _f, _vp, _vp]),
    "tmu_transition": (_i, [_vp, _vp, _TW, _i, _i, _i, _i, _i, _vp, _vp]),
    "tmu_pair_block_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "tmu_pair_block": (_i, [_vp, _vp, _vp, _W, _W, _TW, _i, _i, _i, _i, _i, _i, _f, _vp, _sz, _vp]),
    "tmu_disto_expected": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "tmu_pair_cond_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "tmu_pair_cond": (_i, [_vp, _vp, ctypes.POINTER(TmuPairCondWeights), _i, _i, _i, _i, _i, _i, _i, _i, _vp, _vp,
                           _sz, _vp, _vp]),
    "tmu_parcae_workspace_bytes": (_sz, [_i, _i, _i]),
    "tmu_parcae_step": (_i, [_vp, _vp, _vp, ctypes.POINTER(TmuParcaeWeights), _vp, _i, _i, _i, _vp, _sz, _vp, _vp]),
    "tmu_ipc_export": (_i, [_vp, _vp, ctypes.POINTER(_ull)]),
    "tmu_ipc_import": (_i, [_vp, _ull, ctypes.POINTER(_vp)]),
    "tmu_ipc_close": (_i, [_vp]),
    "tmu_copy_async": (_i, [_vp, _vp, _sz, _vp]),
    "tmu_copy2d_async": (_i, [_vp, _sz, _vp, _sz, _sz, _sz, _vp]),
    "tmu_selftest_wait_timeout": (_i, [_vp, _ull, _vp]),
}


class TmuError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, where: str, detail: str = ""):
        self.code = code
        self.name = STATUS_NAMES.get(code, f"TMU_ERR_{code}")
        super().__init__(f"{where}: {self.name}" + (f" ({detail})" if detail else ""))


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load ``libtmu.so`` once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise TmuError(5, "load", f"{LIB_PATH} not built; run `python -m esmfold2_mlx_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(code: int, where: str) -> None:
    if code != 0:
        detail = load().tmu_last_error().decode(errors="replace")
        raise TmuError(code, where, detail)
