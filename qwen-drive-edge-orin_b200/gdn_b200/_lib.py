"""Loader for the C-ABI shared library ``libgdn_b200.so`` (declared in include/gdn_prefill.h).

The library is built in-tree by ``build.py`` (nvcc, sm_100a). Loading fails
with :class:`GdnLibraryError` when it is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_HERE = Path(__file__).resolve().parent
_LIB_NAME = "libgdn_b200.so"
_lock = threading.Lock()
_lib = None

c_void_p, c_int, c_float, c_size_t, c_int64 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_float,
                                               ctypes.c_size_t, ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/gdn_prefill.h
SIGNATURES = {
    "deltanet_prefill_workspace_size": (c_size_t, [c_int] * 6),
    "deltanet_prefill_debug_workspace_size": (c_size_t, [c_int] * 6),
    "deltanet_tcop_prefill_workspace_size": (c_size_t, [c_int] * 6),
    "deltanet_chunk_prefill": (c_int, [c_void_p] * 8 + [c_int] * 7 + [c_void_p, c_size_t, c_void_p, c_int]),
    "deltanet_tcop_chunk_prefill": (c_int, [c_void_p] * 8 + [c_int] * 7 + [c_void_p, c_size_t, c_void_p, c_int]),
    "deltanet_chunk_prefill_gated": (c_int, [c_void_p] * 7 + [c_float, c_void_p, c_void_p, c_void_p]
                                     + [c_int] * 7 + [c_void_p, c_size_t, c_void_p]),
    "deltanet_chunk_prefill_varlen": (c_int, [c_void_p] * 7 + [c_float, c_void_p, c_void_p, c_void_p,
                                                               c_void_p, c_int] + [c_int] * 6
                                      + [c_void_p, c_size_t, c_void_p]),
    "deltanet_segmented_workspace_size": (c_size_t, [c_int] * 7),
    "deltanet_segmented_plan": (c_int, [c_int] * 4 + [ctypes.POINTER(c_int)] * 3),
    "deltanet_chunk_prefill_segmented": (c_int, [c_void_p] * 7 + [c_float, c_void_p, c_void_p, c_void_p]
                                         + [c_int] * 8 + [c_void_p, c_size_t, c_void_p]),
    "deltanet_chunk_prefill_gated_noalloc": (c_int, [c_void_p] * 7 + [c_float, c_void_p, c_void_p, c_void_p]
                                             + [c_int] * 7 + [c_void_p]),
    "deltanet_test_withheld_load": (c_int, [c_void_p] * 7 + [c_float, c_void_p, c_void_p, c_void_p]
                                    + [c_int] * 7 + [c_void_p, c_size_t, c_void_p, c_int, c_int]),
    "gdn_run_chunk_prefill": (c_int, [c_void_p, c_void_p]),
    "deltanet_recurrent_decode": (c_int, [c_void_p] * 7 + [c_float, c_void_p, c_void_p] + [c_int] * 6 + [c_void_p]),
    "gated_rmsnorm_forward": (c_int, [c_void_p] * 4 + [c_int64, c_int, c_float, c_int, c_void_p]),
    "deltanet_read_status": (c_int, [c_void_p, ctypes.POINTER(c_int), c_int, c_void_p]),
    "deltanet_noalloc_read_status": (c_int, [ctypes.POINTER(c_int), c_int, c_void_p]),
    "gdn_b200_version": (ctypes.c_char_p, []),
}


class GdnPrefillParams(ctypes.Structure):
    """Mirror of ``gdn_prefill_params`` (include/gdn_prefill.h)."""
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("a", c_void_p), ("b", c_void_p),
                ("A_log", c_void_p), ("dt_bias", c_void_p), ("h0_source", c_void_p), ("o", c_void_p),
                ("z", c_void_p), ("norm_w", c_void_p), ("eps", c_float),
                ("n", c_int), ("seq_len", c_int), ("h", c_int), ("hv", c_int), ("k_dim", c_int), ("v_dim", c_int),
                ("workspace", c_void_p), ("workspace_bytes", c_size_t)]


class GdnLibraryError(RuntimeError):
    """The CUDA library is missing or does not export the expected symbols."""


def library_path() -> Path:
    return _HERE / _LIB_NAME


def load_library():
    """Load (once) and return the ctypes handle with typed signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise GdnLibraryError(f"{path} is not built; run qwen-drive-edge-orin_b200/build.py "
                                  "(there is no CPU fallback for this path)")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError as e:  # pragma: no cover - build mismatch
                raise GdnLibraryError(f"{path} does not export {name}") from e
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def cuda_error_string(code: int) -> str:
    try:
        import torch  # noqa: F401
        rt = ctypes.CDLL("libcudart.so.12")
        rt.cudaGetErrorString.restype = ctypes.c_char_p
        rt.cudaGetErrorString.argtypes = [ctypes.c_int]
        return rt.cudaGetErrorString(code).decode()
    except OSError:
        return f"cudaError {code}"
