"""ctypes binding of libctfa_b200.so (the C ABI declared in include/ctfa.h).

The shared library is built in-tree (``cudatransformer_b200/libctfa_b200.so``,
see ``cudatransformer_b200/build.py``).  There is no fallback: if the library
is missing or fails to load, every call raises, so a GPU run can never
silently take another code path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libctfa_b200.so"
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "ctfa.h"

CTFA_OK = 0
CTFA_ERR_INVALID_ARGUMENT = 1
CTFA_ERR_UNSUPPORTED = 2
CTFA_ERR_MISALIGNED = 3
CTFA_ERR_CUDA = 4
CTFA_ERR_DEVICE_TIMEOUT = 5
CTFA_ERR_WORKSPACE = 6

CTFA_DTYPE_F32 = 0
CTFA_DTYPE_BF16 = 1
CTFA_DTYPE_F16 = 2
CTFA_DTYPE_F64 = 3
CTFA_DTYPE_TF32 = 4

CTFA_NOALLOC_SCRATCH_BYTES = 32 << 20

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_size_t = ctypes.c_size_t
_c_ull = ctypes.c_ulonglong

# name -> (restype, argtypes); mirrors include/ctfa.h one to one.
SIGNATURES = {
    "ctfa_version": (_c_int, []),
    "ctfa_status_string": (ctypes.c_char_p, [_c_int]),
    "ctfa_last_error_message": (ctypes.c_char_p, []),
    "ctfa_forward": (
        _c_int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_void_p, _c_size_t, _c_void_p],
    ),
    "ctfa_forward_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "ctfa_backward_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "ctfa_backward": (
        _c_int,
        [_c_void_p] * 10 + [_c_size_t] + [_c_int] * 6 + [_c_void_p],
    ),
    "ctfa_backward_with_events": (
        _c_int,
        [_c_void_p] * 10 + [_c_size_t] + [_c_int] * 6 + [_c_void_p, _c_void_p],
    ),
    "ctfa_backward_noalloc": (
        _c_int,
        [_c_void_p] * 9 + [_c_int] * 6 + [_c_void_p],
    ),
    "ctfa_forward_block": (_c_int, [_c_void_p] * 5 + [_c_int] * 12 + [_c_void_p]),
    "ctfa_forward_block_merge": (_c_int, [_c_void_p] * 5 + [_c_int] * 13 + [_c_void_p]),
    "ctfa_merge_blocks": (_c_int, [_c_void_p] * 4 + [_c_int] * 7 + [_c_void_p]),
    "ctfa_convert_f32": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_size_t, _c_void_p]),
    "ctfa_backward_block_workspace_bytes": (_c_size_t, [_c_int] * 5),
    "ctfa_backward_block": (_c_int, [_c_void_p] * 10 + [_c_size_t] + [_c_int] * 12 + [_c_void_p]),
    "ctfa_set_wait_limit_ns": (_c_int, [_c_ull]),
    "ctfa_check_device_error": (_c_int, [_c_void_p]),
    "ctfa_selftest_wait_timeout": (_c_int, [_c_ull, _c_void_p]),
    "ctfa_qkv_forward": (_c_int, [_c_void_p] * 10 + [_c_int] * 6 + [_c_void_p]),
    "ctfa_qkv_backward": (_c_int, [_c_void_p] * 14 + [_c_int] * 6 + [_c_void_p]),
    "ctfa_out_proj_forward": (_c_int, [_c_void_p] * 4 + [_c_int] * 6 + [_c_void_p]),
    "ctfa_out_proj_backward": (_c_int, [_c_void_p] * 6 + [_c_int] * 6 + [_c_void_p]),
    "ctfa_linear_forward": (_c_int, [_c_void_p] * 4 + [_c_int] * 5 + [_c_void_p]),
    "ctfa_linear_backward": (_c_int, [_c_void_p] * 7 + [_c_int] * 4 + [_c_void_p]),
    "ctfa_layernorm_forward": (_c_int, [_c_void_p] * 6 + [_c_int] * 2 + [ctypes.c_float, _c_int, _c_void_p]),
    "ctfa_layernorm_backward": (_c_int, [_c_void_p] * 8 + [_c_int] * 2 + [ctypes.c_float, _c_int, _c_void_p]),
}

_lib = None


class CtfaError(RuntimeError):
    """Non-zero status from the C ABI (std::runtime_error in the C++ layer)."""

    def __init__(self, status: int, where: str, detail: str):
        self.status = status
        super().__init__(f"{where}: {status_name(status)}: {detail}")


def load() -> ctypes.CDLL:
    """Load the in-tree library once; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m cudatransformer_b200.build` "
            "(the attention path has no fallback implementation)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_name(status: int) -> str:
    return load().ctfa_status_string(status).decode()


def last_error() -> str:
    return load().ctfa_last_error_message().decode()


def check(status: int, where: str) -> None:
    if status != CTFA_OK:
        raise CtfaError(status, where, last_error())


def rounded_copies(ws, B: int, H: int, T: int, D: int):
    """Byte offsets of the tf32-rounded q, k, v that an fp32 ctfa_forward
    leaves in its workspace (include/ctfa.h)."""
    a = (B * H * T * D * 4 + 255) // 256 * 256
    return [ws.data_ptr() + i * a for i in range(3)]


def sync_check_enabled() -> bool:
    """When CTFA_SYNC_CHECK=1, every layer call synchronises and reads the
    device error word (kernels that gave up on a bounded wait)."""
    return os.environ.get("CTFA_SYNC_CHECK", "0") == "1"
