"""ctypes binding of ``libbsattn.so`` (the C ABI in ``include/bsattn.h``).

The library is loaded lazily from this package directory.  There is no
fallback: if the shared object is missing or cannot be loaded, ``lib()``
raises ``RuntimeError`` naming the variant, like the reference's GPU variant
does when its backend is unavailable (block_indexer_triton.py:100-105).
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbsattn.so")

BSA_OK = 0
BSA_ERR_INVALID = 1
BSA_ERR_UNSUPPORTED = 2
BSA_ERR_ALIGNMENT = 3
BSA_ERR_WORKSPACE = 4
BSA_ERR_CUDA = 5

BSA_FLAG_SIMT_SELECT = 1
BSA_FLAG_SIMT_FINE = 2
BSA_FLAG_QBLOCK = 4
BSA_FLAG_TEST_TIMEOUT = 8
BSA_FLAG_FINE_KEY_STATIONARY = 16
BSA_FLAG_FINE_QUERY_STATIONARY = 32

# Every function include/bsattn.h declares, with its ctypes signature.
_c = ctypes
_P = _c.c_void_p


class Problem(ctypes.Structure):
    """Mirror of ``struct bsa_problem``."""

    _fields_ = [
        ("batch", _c.c_int32),
        ("heads", _c.c_int32),
        ("seq_len", _c.c_int32),
        ("head_dim", _c.c_int32),
        ("block_size", _c.c_int32),
        ("top_k", _c.c_int32),
        ("causal", _c.c_int32),
        ("scale", _c.c_float),
        ("flags", _c.c_uint32),
    ]


_PP = _c.POINTER(Problem)

SIGNATURES = {
    "bsa_abi_version": (_c.c_int, []),
    "bsa_status_string": (_c.c_char_p, [_c.c_int]),
    "bsa_last_error": (_c.c_char_p, []),
    "bsa_check_problem": (_c.c_int, [_PP]),
    "bsa_workspace_bytes": (_c.c_size_t, [_PP, _c.c_int64]),
    "bsa_forward": (_c.c_int, [_PP, _P, _P, _P, _P, _P, _c.c_size_t, _P]),
    "bsa_forward_ex": (_c.c_int, [_PP, _P, _P, _P, _P, _P, _c.c_size_t, _P,
                                  _c.POINTER(_P), _c.c_int, _c.POINTER(_c.c_int)]),
    "bsa_pool_k": (_c.c_int, [_PP, _P, _P, _P, _P]),
    "bsa_select_blocks": (_c.c_int, [_PP, _P, _P, _P, _P, _P]),
    "bsa_forward_heads": (_c.c_int, [_PP, _P, _P, _P, _P, _P, _P, _c.c_size_t, _P]),
    "bsa_select_blocks_heads": (_c.c_int, [_PP, _P, _P, _P, _P, _P, _P]),
    "bsa_fine": (_c.c_int, [_PP, _P, _P, _P, _P, _P, _P, _c.c_size_t, _P]),
    "bsa_fine_workspace_bytes": (_c.c_size_t, [_PP]),
    "bsa_backward_workspace_bytes": (_c.c_size_t, [_PP]),
    "bsa_backward": (_c.c_int, [_PP, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _c.c_size_t, _P]),
    "bsa_workspace_error": (_c.c_int, [_PP, _P, _c.c_size_t, _c.c_int, _c.POINTER(_c.c_uint32)]),
    "bsa_forward_noalloc": (_c.c_int, [_PP, _P, _P, _P, _P, _P]),
    "bsa_noalloc_error": (_c.c_int, [_PP, _c.POINTER(_c.c_uint32)]),
    "bsa_workspace_error_offset": (_c.c_int, [_PP, _c.c_size_t, _c.c_int, _c.POINTER(_c.c_size_t)]),
    "bsa_host_workspace_bytes": (_c.c_size_t, [_PP, _c.c_int64]),
    "bsa_forward_host": (_c.c_int, [_PP, _P, _P, _P, _P, _c.c_int64, _P, _c.c_size_t, _P]),
    "bsa_pool_k_blocks": (_c.c_int, [_PP, _P, _P, _P, _c.c_int, _c.c_int, _c.c_int, _P]),
    "bsa_decode_workspace_bytes": (_c.c_size_t, [_PP, _c.c_int]),
    "bsa_decode": (_c.c_int, [_PP, _P, _c.c_int, _c.c_int, _P, _P, _P, _P, _P, _c.c_size_t, _P]),
    "bsa_decode_step": (_c.c_int, [_PP, _P, _P, _P, _c.c_int, _P, _P, _P, _P, _P]),
}

ABI_VERSION = 1
_lib = None


def lib(variant: str = "block_indexer_b200"):
    """Load (once) and return the library with typed entry points."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{variant} requires libbsattn.so, which is not built. Build it with "
            "`python -m flash_vs_sparse_attention_b200.build` (nvcc 12.9, sm_100a).")
    try:
        h = ctypes.CDLL(LIB_PATH)
    except OSError as e:  # pragma: no cover - depends on the host
        raise RuntimeError(f"{variant}: cannot load {LIB_PATH}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
        f = getattr(h, name)
        f.restype = res
        f.argtypes = args
    if h.bsa_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{variant}: libbsattn.so ABI {h.bsa_abi_version()} != {ABI_VERSION}")
    _lib = h
    return h


class BsaError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, where: str):
        L = lib()
        detail = L.bsa_last_error().decode()
        msg = L.bsa_status_string(status).decode()
        super().__init__(f"{where}: {msg} ({status}): {detail}")
        self.status = status


def check(status: int, where: str):
    if status != BSA_OK:
        raise BsaError(status, where)
