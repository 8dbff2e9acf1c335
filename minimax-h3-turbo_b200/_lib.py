"""ctypes binding of libh3b.so (include/h3b.h).

The library is loaded lazily on first use.  There is no fallback: if libh3b.so is missing or cannot be loaded, every
entry point raises RuntimeError naming the problem.  Status codes map to exceptions the way the reference's qlinear
raises them: H3B_ERR_ARG -> ValueError, anything else -> RuntimeError.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path
from typing import Optional

import torch

LIB_PATH = Path(__file__).resolve().parent / "libh3b.so"
ABI_VERSION = 1
NOALLOC_SCRATCH_BYTES = 16 << 20  # H3B_NOALLOC_SCRATCH_BYTES

# enum h3b_status / h3b_dtype / h3b_quant_mode
OK, ERR_ARG, ERR_CUDA, ERR_UNSUPPORTED, ERR_DEVICE = 0, 1, 2, 3, 4
BF16, FP16, FP32, FP8_E4M3, INT32 = 0, 1, 2, 3, 4
QMODE = {"ck": 0, "eager": 1}
COPY_DIRECT, COPY_STAGED, COPY_PAGEABLE = 0, 1, 2

_ACT_CODES = {torch.bfloat16: BF16, torch.float16: FP16, torch.float32: FP32}
_SCALE_CODES = {torch.float8_e4m3fn: FP8_E4M3, torch.uint8: FP8_E4M3, torch.float16: FP16, torch.bfloat16: BF16,
                torch.float32: FP32}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None

_c_void_p, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
_SIGNATURES = {
    "h3b_version": ([], _int),
    "h3b_last_error": ([], ctypes.c_char_p),
    "h3b_rotq": ([_c_void_p, _int, _i64, _i64, _i64, _int, _int, _int, _c_void_p, _i64, _c_void_p, _c_void_p], _int),
    "h3b_rotq_rms_modulate": ([_c_void_p, _i64, _i64, _i64, _c_void_p, ctypes.c_float, _c_void_p, _c_void_p, _i64, _i64,
                               _c_void_p, _int, _c_void_p, _int, _int, _c_void_p, _i64, _c_void_p, _c_void_p], _int),
    "h3b_rotate": ([_c_void_p, _int, _i64, _i64, _i64, _int, _c_void_p, _int, _i64, _c_void_p], _int),
    "h3b_qk_norm_rope": ([_c_void_p, _i64, _c_void_p, _i64, _int, _i64, _int, _int, _c_void_p, _c_void_p, _int,
                          ctypes.c_float, _c_void_p, _c_void_p, _i64, _int, _int, _c_void_p], _int),
    "h3b_rms_modulate": ([_c_void_p, _int, _i64, _i64, _int, _c_void_p, _int, ctypes.c_float, _c_void_p, _c_void_p, _i64,
                          _i64, _int, _c_void_p, _int, _c_void_p, _c_void_p, _i64, _c_void_p], _int),
    "h3b_gate_residual": ([_c_void_p, _int, _i64, _c_void_p, _i64, _i64, _int, _c_void_p, _i64, _i64, _int, _c_void_p, _int,
                           _c_void_p, _c_void_p], _int),
    "h3b_attn_merge": ([_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _int, _c_void_p, _i64, _i64, _int, _int, _c_void_p, _i64,
                        _c_void_p], _int),
    "h3b_w4a8_gemm_decodes_in_kernel": ([_i64, _i64, _i64, _c_void_p, _i64, _int, _int], _int),
    "h3b_decode_grid": ([_c_void_p, _i64, _i64, _i64, _c_void_p, _int, _i64, _c_void_p, _int, _c_void_p, _i64, _c_void_p], _int),
    "h3b_int8_gemm_s32": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p], _int),
    "h3b_gemm_workspace_bytes": ([_i64, _i64, _i64], _sz),
    "h3b_linear_workspace_bytes": ([_i64, _i64, _i64], _sz),
    "h3b_w4a8_gemm": ([_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _int, _i64, _c_void_p, _c_void_p, _int,
                       _c_void_p, _c_void_p, _int, _i64, _i64, _i64, _int, _c_void_p, _sz, _c_void_p], _int),
    "h3b_int8_gemm_epilogue": ([_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _int,
                                _i64, _i64, _i64, _int, _c_void_p], _int),
    "h3b_w4a8_linear": ([_c_void_p, _int, _i64, _i64, _i64, _int, _c_void_p, _i64, _c_void_p, _int, _i64, _c_void_p,
                         _c_void_p, _int, _int, _c_void_p, _c_void_p, _int, _i64, _i64, _int, _c_void_p, _sz, _c_void_p], _int),
    "h3b_w4a8_gemm_noalloc": ([_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _int, _i64, _c_void_p,
                               _c_void_p, _int, _c_void_p, _c_void_p, _int, _i64, _i64, _i64, _int, _c_void_p], _int),
    "h3b_streamer_create": ([_int, _int, _int, _sz, _int, ctypes.POINTER(ctypes.c_void_p)], _int),
    "h3b_streamer_destroy": ([_c_void_p], _int),
    "h3b_streamer_copy": ([_c_void_p, _int, _c_void_p, _c_void_p, _sz, _int], _int),
    "h3b_streamer_begin": ([_c_void_p, _int], _int),
    "h3b_streamer_end": ([_c_void_p, _int, _sz], _int),
    "h3b_streamer_stream": ([_c_void_p], _c_void_p),
    "h3b_streamer_acquire": ([_c_void_p, _int, _c_void_p], _int),
    "h3b_streamer_release": ([_c_void_p, _int, _c_void_p], _int),
    "h3b_streamer_wait": ([_c_void_p, _int, ctypes.c_double], _int),
    "h3b_streamer_stats": ([_c_void_p, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                            ctypes.POINTER(ctypes.c_double)], _int),
    "h3b_host_register": ([_c_void_p, _sz, _int], _int),
    "h3b_host_unregister": ([_c_void_p], _int),
    "h3b_device_error": ([_int], _int),
    "h3b_selftest_wait_timeout": ([ctypes.c_double, _c_void_p, _c_void_p], _int),
}


def exported_symbols():
    """Every entry point include/h3b.h declares (the loader binds exactly these)."""
    return tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """The loaded library (RuntimeError if it is missing or broken -- there is no fallback)."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"libh3b.so is not built ({LIB_PATH}); run `python minimax-h3-turbo_b200/build.py`")
            try:
                handle = ctypes.CDLL(str(LIB_PATH))
            except OSError as e:
                _load_error = str(e)
                raise RuntimeError(f"cannot load {LIB_PATH}: {e}") from None
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes, fn.restype = args, res
            if handle.h3b_version() != ABI_VERSION:
                raise RuntimeError(f"libh3b.so ABI {handle.h3b_version()} != expected {ABI_VERSION}; rebuild it")
            _lib = handle
    return _lib


def available() -> bool:
    try:
        lib()
        return True
    except RuntimeError:
        return False


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    msg = lib().h3b_last_error().decode(errors="replace")
    if rc == ERR_ARG:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed (h3b status {rc}): {msg}")


def act_code(dt: torch.dtype) -> int:
    try:
        return _ACT_CODES[dt]
    except KeyError:
        raise ValueError(f"the b200 backend takes bf16, fp16 or fp32 activations, got {dt}") from None


def scale_code(dt: torch.dtype) -> int:
    try:
        return _SCALE_CODES[dt]
    except KeyError:
        raise ValueError(f"group scales must be float8_e4m3fn (or its raw uint8 bytes), fp16, bf16 or fp32, got {dt}") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()
