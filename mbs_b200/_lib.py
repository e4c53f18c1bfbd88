"""ctypes binding of libmbs_gemm_kernel.so (declared in include/mbs_gemm_a4w4.h).

The library is the product's compute path; there is no fallback.  If it is
missing, every operator raises instead of computing anything elsewhere.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

_c_int, _c_void_p, _c_size_t, _c_char_p = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p

# name -> (restype, argtypes); must match include/mbs_gemm_a4w4.h
SIGNATURES = {
    "mbs_status_string": (_c_char_p, [_c_int]),
    "mbs_last_error_message": (_c_char_p, []),
    "gemm_a4w4_mxfp4_launch": (_c_int, [_c_void_p] * 7 + [_c_int] * 5 + [_c_void_p]),
    "mbs_gemm_a4w4_workspace_size": (_c_size_t, [_c_int] * 3),
    "mbs_gemm_a4w4_kernels_per_call": (_c_int, [_c_int] * 3),
    "mbs_gemm_a4w4_launch_ws": (_c_int, [_c_void_p] * 7 + [_c_int] * 5 + [_c_void_p, _c_size_t,
                                                                           _c_void_p]),
    "mbs_gemm_a4w4_launch_noalloc": (_c_int, [_c_void_p] * 7 + [_c_int] * 5 + [_c_void_p]),
    "mbs_gemm_a4w4_launch_ex": (_c_int, [_c_void_p] * 7 + [_c_int] * 5 + [ctypes.c_float, _c_void_p,
                                                                           _c_void_p, _c_size_t, _c_void_p]),
    "mbs_gemm_a4w4_launch_multi": (_c_int, [_c_void_p] * 6 + [_c_void_p, _c_int, ctypes.c_longlong]
                                   + [_c_int] * 5 + [ctypes.c_float, _c_void_p, _c_void_p, _c_size_t,
                                                     _c_void_p]),
    "mbs_quant_gemm_a4w4_workspace_size": (_c_size_t, [_c_int] * 3),
    "mbs_quant_gemm_a4w4_packed_workspace_size": (_c_size_t, [_c_int] * 3),
    "mbs_quant_gemm_a4w4_packed_launch": (_c_int, [_c_void_p, _c_int] + [_c_void_p] * 4 + [_c_int] * 3
                                          + [_c_void_p, _c_size_t, _c_void_p]),
    "mbs_quant_gemm_a4w4_launch": (_c_int, [_c_void_p, _c_int] + [_c_void_p] * 5 + [_c_int] * 4
                                   + [_c_void_p, _c_size_t, _c_void_p]),
    "mbs_gemm_a4w4_macro_launch_ws": (_c_int, [_c_void_p] * 7 + [_c_int] * 6
                                      + [_c_void_p, _c_size_t, _c_void_p]),
    "mbs_quantize_mxfp4": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_int,
                                    _c_void_p]),
    "mbs_quantize_mxfp4_mbs": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p,
                                        _c_int, _c_void_p]),
    "mbs_quantize_mxfp4_macro": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                          _c_void_p]),
    "mbs_shuffle_weight": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p]),
    "mbs_shuffle_scales": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p]),
    "mbs_device_error": (_c_int, [ctypes.POINTER(_c_int), _c_int]),
    "mbs_set_profile_events": (_c_int, [_c_void_p, _c_void_p]),
    "mbs_set_grid_limit": (_c_int, [_c_int]),
    "mbs_set_plan_override": (_c_int, [_c_void_p]),
    "mbs_set_withhold_release": (_c_int, [_c_int]),
    "mbs_ipc_alloc": (_c_int, [_c_size_t, ctypes.POINTER(_c_void_p), _c_void_p]),
    "mbs_ipc_open": (_c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "mbs_ipc_close": (_c_int, [_c_void_p]),
    "mbs_ipc_free": (_c_int, [_c_void_p]),
    "mbs_copy_async": (_c_int, [_c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "mbs_packed_weight_bytes": (_c_size_t, [_c_int, _c_int]),
    "mbs_pack_weight": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mbs_gemm_a4w4_packed_workspace_size": (_c_size_t, [_c_int] * 3),
    "mbs_gemm_a4w4_packed_launch_ws": (_c_int, [_c_void_p] * 6 + [_c_int] * 5 + [_c_void_p, _c_size_t,
                                                                                _c_void_p]),
    "mbs_mxf4_peak_probe": (_c_int, [_c_int] + [ctypes.POINTER(ctypes.c_double)] * 3 + [_c_void_p]),
}



class PlanOverride(ctypes.Structure):
    """mbs_plan_override of include/mbs_gemm_a4w4.h (field defaults = "auto")."""
    _fields_ = [(name, _c_int) for name in ("schedule", "grid", "pair", "swap", "pair_bn", "pair_wide",
                                            "ksplit", "split_bn")]
    AUTO = dict(schedule=0, grid=0, pair=-1, swap=-1, pair_bn=0, pair_wide=0, ksplit=-1, split_bn=0)

    def __init__(self, **kw):
        unknown = set(kw) - set(self.AUTO)
        if unknown:
            raise ValueError(f"unknown plan override fields: {sorted(unknown)}")
        super().__init__(**{**self.AUTO, **{k: int(v) for k, v in kw.items()}})


_lock = threading.Lock()
_lib = None


class MbsError(RuntimeError):
    """A non-zero status from the kernel library."""

    def __init__(self, func: str, status: int, name: str, detail: str):
        super().__init__(f"{func}: {name}: {detail}" if detail else f"{func}: {name}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load (once) and return the kernel library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            # MBS_LIB selects another build of the same library (e.g. the
            # MBS_TIMING debug build); it never selects a non-CUDA path.
            path = os.environ.get("MBS_LIB") or LIB_PATH
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m mbs_b200.build` "
                    "(the MXFP4 operators have no non-CUDA fallback)")
            handle = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(func: str, status: int) -> None:
    if status != 0:
        L = lib()
        name = L.mbs_status_string(status).decode()
        detail = L.mbs_last_error_message().decode()
        raise MbsError(func, status, name, detail)


def call(func: str, *args) -> None:
    check(func, getattr(lib(), func)(*args))
