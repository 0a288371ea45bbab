"""Loader and thin typed wrapper of the C-ABI library libtrnfft_b200.so.

The library is the only compute path of this package: there is no CPU
fallback.  If it is missing (not built) or no CUDA device is visible, every
transform raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libtrnfft_b200.so")
ABI_VERSION = 1

# Status codes (include/trnfft_b200.h)
SUCCESS = 0
INVALID_VALUE = 1
UNSUPPORTED = 2
CUDA_ERROR = 3
ALLOC_FAILED = 4

ALG_COPY, ALG_STOCKHAM, ALG_MULTIPASS, ALG_BLUESTEIN, ALG_MIXED = 0, 1, 2, 3, 4

_lib = None
_lib_lock = threading.Lock()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int

# name -> (restype, argtypes); every symbol include/trnfft_b200.h declares
SIGNATURES = {
    "trnfft_abi_version": (_INT, []),
    "trnfft_last_error": (ctypes.c_char_p, []),
    "trnfft_plan_create": (_INT, [ctypes.POINTER(_P), _I64, _INT]),
    "trnfft_plan_destroy": (_INT, [_P]),
    "trnfft_device_status": (_INT, [_INT, ctypes.POINTER(_INT), _INT]),
    "trnfft_plan_query": (_INT, [_P, ctypes.POINTER(_INT), ctypes.POINTER(_I64), _I64, ctypes.POINTER(_I64)]),
    "trnfft_exec_c2c": (_INT, [_P, _P, _P, _P, _P, _I64, _INT, _P, _P]),
    "trnfft_exec_c2c_axis": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _INT, _P, _P]),
    "trnfft_exec_c2c_inplace_noalloc": (_INT, [_P, _P, _P, _I64, _INT, _P]),
    "trnfft_exec_stft": (_INT, [_P, _P, _I64, _I64, _I64, _P, _INT, _INT, _INT, _INT, _I64, _P, _P, _P]),
    "trnfft_complex_linear_work_bytes": (_I64, [_I64, _I64, _I64]),
    "trnfft_complex_linear": (_INT, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _INT, _P]),
    "trnfft_split_tf32": (_INT, [_P, _P, _P, _I64, _INT, _P]),
    "trnfft_split_tf32_sum": (_INT, [_P, _P, _P, _P, _I64, _INT, _P]),
    "trnfft_complex_linear_presplit": (_INT, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _INT, _P]),
    "trnfft_exec_c2c_axis_tw": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _INT, _I64, _P]),
    "trnfft_ipc_handle_bytes": (_INT, []),
    "trnfft_xbuf_alloc": (_INT, [_INT, _I64, ctypes.POINTER(_P), _P]),
    "trnfft_xbuf_free": (_INT, [_INT, _P]),
    "trnfft_ipc_open": (_INT, [_INT, _P, ctypes.POINTER(_P)]),
    "trnfft_ipc_close": (_INT, [_INT, _P]),
    "trnfft_exec_fourstep_scatter": (_INT, [_P, _P, _P, _P, _I64, _I64, _INT, _I64, _INT,
                                            ctypes.POINTER(_P), ctypes.POINTER(_P), _I64, _I64, _I64, _P, _P]),
    "trnfft_exec_r2c": (_INT, [_P, _P, _P, _P, _I64, _P, _P]),
    "trnfft_copy2d": (_INT, [_P, _I64, _P, _I64, _I64, _I64, _INT, _P]),
    "trnfft_plan_enable_f64": (_INT, [_P]),
    "trnfft_plan_query_f64": (_INT, [_P, _I64, ctypes.POINTER(_I64)]),
    "trnfft_exec_c2c_f64": (_INT, [_P, _P, _P, _P, _P, _I64, _INT, _P, _P]),
    "trnfft_exec_c2c_f64_f32io": (_INT, [_P, _P, _P, _P, _P, _I64, _INT, _P, _P]),
    "trnfft_convert_f32_f64": (_INT, [_P, _P, _I64, _INT, _INT, _P]),
    "trnfft_exec_istft": (_INT, [_P, _P, _P, _I64, _I64, _I64, _P, _INT, _INT, _INT, _I64, _P, _P]),
    "trnfft_complex_mask_apply": (_INT, [_P, _P, _I64, _P, _P, _P, _P, _I64, _INT, _P]),
    "trnfft_exec_c2r": (_INT, [_P, _P, _P, _P, _I64, _P, _P]),
}


class TrnfftError(RuntimeError):
    """A C-ABI call returned a non-zero trnfft_status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


def load(path: str = LIB_PATH):
    """Load the library (once) and bind every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"trnfft_b200 CUDA library not found at {path}; build it with "
                "`python -m trnfft_b200.build` (there is no CPU fallback)"
            )
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        v = lib.trnfft_abi_version()
        if v != ABI_VERSION:
            raise RuntimeError(f"trnfft_b200 ABI mismatch: library {v}, package {ABI_VERSION}")
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != SUCCESS:
        msg = lib.trnfft_last_error().decode(errors="replace")
        if rc == UNSUPPORTED:
            raise NotImplementedError(f"{name}: {msg}")
        if rc == INVALID_VALUE:
            raise ValueError(f"{name}: {msg}")
        raise TrnfftError(name, rc, msg)


def device_status(device_index: int, clear: bool = True) -> int:
    """Read (and by default clear) the kernels' device status word (0 = ok)."""
    v = ctypes.c_int()
    call("trnfft_device_status", int(device_index), ctypes.byref(v), int(bool(clear)))
    return v.value


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError(
            "trnfft_b200 runs its transforms on CUDA (sm_100a) only and no CUDA device is "
            "visible; there is no CPU fallback"
        )


class DevicePlan:
    """Owner of one C plan (one length on one device)."""

    def __init__(self, n: int, device_index: int):
        h = ctypes.c_void_p()
        call("trnfft_plan_create", ctypes.byref(h), int(n), int(device_index))
        self.handle = h
        self.n = n
        self.device_index = device_index
        alg = ctypes.c_int()
        pn = ctypes.c_int64()
        call("trnfft_plan_query", h, ctypes.byref(alg), ctypes.byref(pn), 0, None)
        self.algorithm = alg.value
        self.padded_n = pn.value

    def enable_f64(self) -> None:
        """Build the plan's fp64 tables (once)."""
        if not getattr(self, "_f64", False):
            call("trnfft_plan_enable_f64", self.handle)
            self._f64 = True

    def work_bytes_f64(self, batch: int) -> int:
        wb = ctypes.c_int64()
        call("trnfft_plan_query_f64", self.handle, int(batch), ctypes.byref(wb))
        return wb.value

    def work_bytes(self, batch: int) -> int:
        wb = ctypes.c_int64()
        call("trnfft_plan_query", self.handle, None, None, int(batch), ctypes.byref(wb))
        return wb.value

    def __del__(self):
        try:
            if _lib is not None and self.handle:
                _lib.trnfft_plan_destroy(self.handle)
        except Exception:
            pass


_device_plans: dict[tuple[int, int], DevicePlan] = {}
_plans_lock = threading.Lock()


def device_plan(n: int, device: torch.device) -> DevicePlan:
    """Cached C plan keyed by (n, device index)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (int(n), idx)
    p = _device_plans.get(key)
    if p is None:
        with _plans_lock:
            p = _device_plans.get(key)
            if p is None:
                p = DevicePlan(n, idx)
                _device_plans[key] = p
    return p


def clear_device_plans() -> None:
    with _plans_lock:
        _device_plans.clear()
