"""ctypes binding of ``libb200paged.so`` (the C ABI declared in ``include/b200_paged.h``).

The library is built in-tree by ``build.py``. Loading fails loudly when it is missing:
there is no CPU or library fallback for any entry point.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200paged.so"

B2P_BF16 = 0
B2P_F16 = 1
B2P_F32 = 2

B2P_OK = 0
B2P_EINVAL = -1
B2P_EUNSUPPORTED = -2
B2P_ERANGE = -3
B2P_EWORKSPACE = -4
B2P_ELAUNCH = -5
B2P_EDRIVER = -6

DEV_SLOT_RANGE = 1
DEV_BLOCK_RANGE = 2
DEV_WAIT_TIMEOUT = 4
DEV_LENGTH = 8

EXPORTED_SYMBOLS = (
    "b2p_version",
    "b2p_last_cuda_error",
    "b2p_status_string",
    "b2p_cuda_core_fallbacks",
    "b2p_reset_scratch",
    "b2p_kv_write",
    "b2p_paged_decode_workspace_size",
    "b2p_paged_decode",
    "b2p_paged_decode_noalloc",
    "b2p_paged_decode_append",
    "b2p_paged_prefill",
    "b2p_build_metadata",
    "b2p_lm_head_argmax_workspace_size",
    "b2p_lm_head_argmax",
)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "b2p_version": (_i32, []),
    "b2p_last_cuda_error": (_i32, []),
    "b2p_status_string": (ctypes.c_char_p, [_i32]),
    "b2p_cuda_core_fallbacks": (_i64, [_i32]),
    "b2p_reset_scratch": (_i32, [_p]),
    "b2p_kv_write": (
        _i32,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _i32, _i32,
         _p, _p],
    ),
    "b2p_paged_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32]),
    "b2p_paged_decode": (
        _i32,
        [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _i32, _i32, _i32, _i32, _i32,
         _f32, _p, _i64, _i64, _p, _sz, _i32, _p, _p],
    ),
    "b2p_paged_decode_noalloc": (
        _i32,
        [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _i32, _i32, _i32, _i32, _i32,
         _f32, _p, _i64, _i64, _i32, _p, _p],
    ),
    "b2p_paged_decode_append": (
        _i32,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p,
         _i32, _i32, _i32, _i32, _i32, _f32, _p, _i64, _i64, _p, _sz, _i32, _p, _p],
    ),
    "b2p_paged_prefill": (
        _i32,
        [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _p, _i32, _i64, _i32, _i32,
         _i32, _i32, _i32, _f32, _p, _i64, _i64, _i32, _p, _p],
    ),
    "b2p_build_metadata": (
        _i32,
        [_p, _p, _p, _i32, _p, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _i32, _i64, _p, _p],
    ),
    "b2p_lm_head_argmax_workspace_size": (_sz, [_i32]),
    "b2p_lm_head_argmax": (
        _i32,
        [_p, _i64, _p, _i64, _i32, _i64, _i32, _i32, _p, _p, _p, _sz, _p, _p],
    ),
}


class KernelLibraryMissing(RuntimeError):
    """Raised when the compiled CUDA library is not present next to the package."""


def load() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise KernelLibraryMissing(
                f"{LIB_PATH.name} is not built; run `python -c 'import __graft_entry__ as g; "
                "g.build()'` (nvcc for sm_100a) before using the paged-attention kernels."
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def status_text(code: int) -> str:
    return load().b2p_status_string(code).decode()


def check(code: int, what: str) -> None:
    """Turn a C-ABI status into the exception type the reference uses for that case."""
    if code == B2P_OK:
        return
    text = status_text(code)
    if code in (B2P_EINVAL, B2P_ERANGE, B2P_EUNSUPPORTED, B2P_EWORKSPACE):
        raise ValueError(f"{what}: {text} (status {code})")
    cuda = load().b2p_last_cuda_error()
    raise RuntimeError(f"{what}: {text} (status {code}, cudaError {cuda})")
