"""ctypes binding of the C ABI in ``include/dominus_ultra_b200.h``.

The library is loaded lazily from the package directory. There is no fallback: if the shared
object is missing or fails to load, every kernel call raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path
from typing import Optional

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libdominus_b200.so"

DU_OK = 0
DU_ERR_INVALID = 1
DU_ERR_UNSUPPORTED = 2
DU_ERR_CUDA = 3
DU_ERR_WORKSPACE = 4
DU_ERR_TIMEOUT = 5

DU_DTYPE_F16 = 0
DU_DTYPE_BF16 = 1
DU_DTYPE_F32 = 2

DU_NOALLOC_SCRATCH_BYTES = 4 << 20  # scratch held by du_decode_noalloc (see the header)

_vp = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/dominus_ultra_b200.h one to one.
SIGNATURES = {
    "du_version": (_i, []),
    "du_last_error": (ctypes.c_char_p, []),
    "du_prefill_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "du_prefill": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _ll, _vp, _sz, _vp],
    ),
    "du_rope": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _ll, _ll, _i, _vp]),
    "du_rope_segments": (
        _i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _ll, _ll, _ll, _ll, _i, _vp]
    ),
    "du_prefill_block": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
         _ll, _ll, _ll, _i, _i, _f, _ll, _vp],
    ),
    "du_decode_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "du_decode": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _ll, _vp, _sz, _vp],
    ),
    "du_decode_kvcache_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "du_decode_kvcache": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _ll, _vp, _sz, _vp],
    ),
    "du_decode_partial": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _ll, _ll, _ll, _vp, _sz, _vp],
    ),
    "du_merge_partials": (
        _i,
        [_vp, _vp, _i, _i, _i, _ll, _ll, _ll, _ll, _vp, _i, _vp, _vp],
    ),
    "du_exchange_buffer_bytes": (_sz, [_i, _i, _i]),
    "du_exchange_buffer_alloc": (_i, [_sz, ctypes.POINTER(_vp)]),
    "du_exchange_buffer_free": (_i, [_vp]),
    "du_ipc_get_handle": (_i, [_vp, _vp]),
    "du_ipc_open_handle": (_i, [_vp, ctypes.POINTER(_vp)]),
    "du_ipc_close_handle": (_i, [_vp]),
    "du_exchange_merge": (
        _i, [_vp, _vp, ctypes.POINTER(_vp), _i, _i, _i, _i, _vp, _i, _vp, _vp]
    ),
    "du_decode_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _ll, _vp]),
    "du_selftest_wait_timeout": (_i, [_i, _vp]),
    "du_read_status": (_i, [ctypes.POINTER(ctypes.c_uint), _i]),
}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library, with argument types set."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built: run `python -m dominusultra_b200.build` "
                "(the CUDA extension is required; there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().du_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != DU_OK:
        raise RuntimeError(f"{what} failed (status {rc}): {last_error()}")


def read_status(reset: bool = True):
    """Return the 4 device status words (synchronises the device)."""
    words = (ctypes.c_uint * 4)()
    check(load().du_read_status(words, 1 if reset else 0), "du_read_status")
    return list(words)
