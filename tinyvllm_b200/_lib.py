"""ctypes binding of ``libtvk.so`` (the C ABI declared in ``include/tvk.h``).

The library is loaded from this package directory.  There is no fallback: if
the library is missing, or a tensor is not on a CUDA device, calls raise.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libtvk.so"

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
_TORCH_TO_CODE = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}

_c_int, _c_size, _c_void = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p
_c_float, _c_int64 = ctypes.c_float, ctypes.c_int64

# name -> (restype, argtypes); every symbol declared in include/tvk.h
SIGNATURES = {
    "tvk_abi_version": (_c_int, []),
    "tvk_last_error": (ctypes.c_char_p, []),
    "tvk_paged_decode_workspace_size": (_c_size, [_c_int] * 7),
    "tvk_paged_decode_plan": (_c_int, [_c_int] * 8 + [_c_void]),
    "tvk_paged_decode_attention": (
        _c_int,
        [_c_void] * 6 + [_c_int] * 9 + [_c_void, _c_size, _c_void],
    ),
    "tvk_selftest_umma_gemm": (_c_int, [_c_void] * 3 + [_c_int] * 5 + [_c_void, _c_void]),
    "tvk_paged_decode_attention_noalloc": (_c_int, [_c_void] * 6 + [_c_int] * 9 + [_c_void]),
    "tvk_paged_decode_noalloc_status": (_c_int, [_c_void, _c_void]),
    "tvk_debug_arm_wait_timeout": (_c_int, [ctypes.c_longlong]),
    "tvk_rms_norm": (_c_int, [_c_void] * 5 + [_c_int, _c_int, _c_float, _c_int, _c_void]),
    "tvk_rms_norm_write_kv": (_c_int, [_c_void] * 5 + [_c_int, _c_int, _c_float] + [_c_void] * 5 +
                              [_c_int] * 5 + [_c_void]),
    "tvk_rope": (_c_int, [_c_void] * 5 + [_c_int] * 6 + [_c_void]),
    "tvk_rope_write_kv": (_c_int, [_c_void] * 9 + [_c_int] * 8 + [_c_void]),
    "tvk_write_kv_slots": (_c_int, [_c_void] * 5 + [_c_int] * 6 + [_c_void]),
    "tvk_qkv_rope": (_c_int, [_c_void, _c_int64] + [_c_void] * 9 + [_c_int] * 8 + [_c_void]),
    "tvk_silu_mul": (_c_int, [_c_void] * 3 + [_c_int, _c_int, _c_int64, _c_int64, _c_int64, _c_int, _c_void]),
    "tvk_embedding": (_c_int, [_c_void] * 3 + [_c_int] * 4 + [_c_void, _c_void]),
    "tvk_argmax": (_c_int, [_c_void] * 2 + [_c_int, _c_int, _c_int64, _c_int, _c_void]),
    "tvk_flash_prefill_workspace_size": (_c_size, [_c_int] * 2),
    "tvk_prefill_select_kernel": (_c_int, [_c_int]),
    "tvk_flash_prefill_attention": (
        _c_int,
        [_c_void] * 5 + [_c_int] * 8 + [_c_void] * 3 + [_c_int] * 2 + [_c_void, _c_size, _c_void],
    ),
    "tvk_probe_mma_issue": (_c_int, [_c_int, _c_int, _c_void, _c_int, _c_void]),
    "tvk_probe_exp_unit": (_c_int, [_c_int, _c_int, _c_void, _c_int, _c_void, _c_void]),
}

_lib = None
_lock = threading.Lock()


class TvkError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def lib() -> ctypes.CDLL:
    """Load (once) and return the library, declaring every prototype."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m tinyvllm_b200.build` "
                    "(the CUDA path has no fallback)")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().tvk_last_error().decode(errors="replace")
        raise TvkError(f"{what} failed with status {rc}: {msg}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _TORCH_TO_CODE[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype} (float32, float16 or bfloat16)") from None


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError("tinyvllm_b200 kernels need CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev
