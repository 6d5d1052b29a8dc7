"""ctypes binding of ``libddpm_b200.so`` (the C ABI in ``include/ddpm_b200.h``).

The library is loaded from this package directory only. There is no fallback:
if the shared object is missing or does not load, every GPU entry point raises
``RuntimeError`` — the CUDA path never silently degrades to a CPU or PyTorch
implementation. Build it with ``python -m dynamicconvolutionoperator_b200._build``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libddpm_b200.so")

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_c_int = ctypes.c_int
_c_ptr = ctypes.c_void_p
_c_size = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/ddpm_b200.h
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ddpm_version": (_c_int, []),
    "ddpm_last_error": (ctypes.c_char_p, []),
    "ddpm_launch_count": (ctypes.c_ulonglong, []),
    "ddpm_device_status": (_c_int, [_c_int, ctypes.POINTER(ctypes.c_int)]),
    "ddpm_dyncat_fwd": (
        _c_int,
        [_c_ptr, _c_int, _c_ptr, _c_int, _c_ptr] + [_c_int] * 4 + [_c_int] * 4 + [_c_ptr],
    ),
    "ddpm_dyncat_bwd": (
        _c_int,
        [_c_ptr, _c_int, _c_ptr, _c_ptr, _c_int, _c_ptr, _c_ptr]
        + [_c_int] * 4
        + [_c_int] * 4
        + [_c_ptr],
    ),
    "ddpm_gencat_pack_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "ddpm_gencat_pack": (
        _c_int, [_c_ptr, _c_ptr, _c_int, _c_int, _c_int, _c_ptr, _c_size, _c_ptr]
    ),
    "ddpm_gencat_fwd": (
        _c_int,
        [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_fwd_staged": (
        _c_int,
        [_c_ptr, _c_size, _c_ptr, _c_ptr, _c_ptr] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_fwd_staged_planes": (
        _c_int,
        [_c_ptr, _c_size] + [_c_ptr] * 4 + [_c_size] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_bwd_x": (
        _c_int,
        [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_stage_bytes": (_c_size, [_c_int] * 9),
    "ddpm_gencat_stage": (
        _c_int,
        [_c_ptr, _c_ptr, _c_ptr, _c_size] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_bwd_x_staged": (
        _c_int,
        [_c_ptr, _c_size, _c_ptr, _c_ptr, _c_ptr, _c_ptr] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_bwd_x_staged_nhwc": (
        _c_int,
        [_c_ptr, _c_size, _c_ptr, _c_ptr, _c_ptr, _c_ptr] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_bwd_yw_staged_nhwc": (
        _c_int,
        [_c_ptr, _c_size] + [_c_ptr] * 6 + [_c_size] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_bwd_workspace_bytes": (_c_size, [_c_int] * 5),
    "ddpm_gencat_bwd_yw": (
        _c_int,
        [_c_ptr] * 8 + [_c_size] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_bwd_yw_staged": (
        _c_int,
        [_c_ptr, _c_size] + [_c_ptr] * 6 + [_c_size] + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_gencat_bwd_yw_static": (
        _c_int,
        [_c_ptr] * 7 + [_c_int] * 4 + [_c_int] * 5 + [_c_ptr],
    ),
    "ddpm_fuseconv_pack_bytes": (_c_size, [_c_int] * 3),
    "ddpm_fuseconv_pack": (_c_int, [_c_ptr, _c_int, _c_int, _c_int, _c_ptr, _c_size, _c_ptr]),
    "ddpm_fuseconv_fwd": (_c_int, [_c_ptr] * 4 + [_c_int] * 6 + [_c_ptr]),
    "ddpm_fuseconv_bwd_data": (_c_int, [_c_ptr] * 3 + [_c_int] * 6 + [_c_ptr]),
    "ddpm_fuseconv_stage_bytes": (_c_size, [_c_int] * 5),
    "ddpm_fuseconv_stage": (_c_int, [_c_ptr, _c_ptr, _c_size] + [_c_int] * 5 + [_c_ptr]),
    "ddpm_fuseconv_fwd_staged": (
        _c_int, [_c_ptr, _c_size] + [_c_ptr] * 3 + [_c_int] * 6 + [_c_ptr]
    ),
    "ddpm_fuseconv_bwd_data_staged": (
        _c_int, [_c_ptr, _c_size] + [_c_ptr] * 2 + [_c_int] * 6 + [_c_ptr]
    ),
    "ddpm_fuseconv_bwd": (
        _c_int, [_c_ptr] * 7 + [_c_size] + [_c_int] * 6 + [_c_ptr]
    ),
    "ddpm_fuseconv_bwd_nhwc": (
        _c_int, [_c_ptr] * 7 + [_c_size] + [_c_int] * 6 + [_c_ptr]
    ),
    "ddpm_fuseconv_bwd_weight_workspace_bytes": (_c_size, [_c_int] * 5),
    "ddpm_fuseconv_bwd_weight": (
        _c_int, [_c_ptr] * 5 + [_c_size] + [_c_int] * 6 + [_c_ptr]
    ),
    "ddpm_test_skip_arrive": (_c_int, [_c_int]),
    "ddpm_test_disable_tma": (_c_int, [_c_int]),
    "ddpm_umma_selftest": (
        _c_int, [_c_int, _c_ptr, _c_ptr, _c_ptr, _c_int, _c_int, _c_int, _c_ptr]
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def exported_symbols() -> list[str]:
    """Names of every entry point this binding expects the library to export."""
    return list(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load (once) and return the shared library, with argtypes configured."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built (expected at {LIB_PATH}); run "
                "`python -m dynamicconvolutionoperator_b200._build`"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Invoke an entry point; a non-zero return raises RuntimeError with its message."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.ddpm_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (code {rc}): {msg}")


def device_status(reset: bool = True) -> int:
    """Failure code recorded by a bounded wait inside a kernel (0 = none) on
    the current device; synchronises. With ``reset`` the code is cleared."""
    code = ctypes.c_int(0)
    call("ddpm_device_status", 1 if reset else 0, ctypes.byref(code))
    return code.value


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(load().ddpm_launch_count())


def stream_handle(device: torch.device) -> int:
    """Raw cudaStream_t of torch's current stream on ``device``."""
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise RuntimeError(
            f"dtype {dtype} is not supported by the CUDA path (float32, bfloat16, float16)"
        ) from None
