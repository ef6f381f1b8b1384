"""ctypes binding of the engine's C ABI (``include/gmmxx_b200.h``).

The shared library ``gmmxx_b200/_lib/libgmmxx_b200.so`` is built in-tree by
``python -m gmmxx_b200.build``.  There is no fallback: if the library is
missing every CUDA entry point raises :class:`CudaBackendUnavailable`, and a
failing call raises :class:`GmmxxError` carrying the library's message.

This module replaces the reference's lazy ``gmmxx._C`` import and its
``require_cuda`` / ``CudaBackendUnavailable`` plumbing (gmmxx/_cuda.py:25-64).
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "_lib", "libgmmxx_b200.so")

SPHERICAL, DIAG, TIED, FULL = 0, 1, 2, 3
COV_TYPES = {"spherical": SPHERICAL, "diag": DIAG, "tied": TIED, "full": FULL}
FLOAT32, BFLOAT16, FLOAT16 = 0, 1, 2

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_NOT_PD = 4
ERR_WORKSPACE = 5
ERR_TIMEOUT = 6

# Windows of the compiled kernels (mirrors gmm_common.cuh).
MAX_D = 128
MAX_D_FULL = 26


class CudaBackendUnavailable(RuntimeError):
    """The CUDA engine library is not built or cannot be loaded
    (reference: gmmxx/_cuda.py:37-38)."""


class GmmxxError(RuntimeError):
    """A C ABI call returned an error status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[gmmxx status {status}] {message}")
        self.status = status


class UnsupportedShape(GmmxxError, ValueError):
    """Shape outside the compiled kernel windows (GMMXX_ERR_UNSUPPORTED)."""


_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[BaseException] = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

_SIGNATURES = {
    "gmmxx_abi_version": (_I32, []),
    "gmmxx_last_error": (ctypes.c_char_p, []),
    "gmmxx_canary_add_offset": (_I32, [_P, _P, _I64, ctypes.c_int32, _P]),
    "gmmxx_stat_width": (_I64, [_I32, _I64]),
    "gmmxx_workspace_bytes": (_SZ, [_I32, _I64, _I64, _I64, _I64]),
    "gmmxx_workspace_status": (_I32, [_P, _P, _P]),
    "gmmxx_accumulate_path": (_I32, [_I32, _I32, _I64, _I64, _I64, _I64, _P]),
    "gmmxx_last_accumulate_path": (_I32, []),
    "gmmxx_em_prepare": (_I32, [_I32, _I64, _I64, _I64, _P, _P, _P, _F, _F, _P, _SZ, _P]),
    "gmmxx_em_accumulate": (_I32, [_I32, _I32, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P, _P, _P]),
    "gmmxx_topk_scratch_bytes": (_SZ, [_I64, _I64, _I64]),
    "gmmxx_em_accumulate_topk": (_I32, [_I32, _I32, _P, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P, _SZ, _P, _P,
                                        _P]),
    "gmmxx_em_finalize": (_I32, [_I32, _I64, _I64, _I64, _I64, _P, _P, _P, _F, _F, _P, _P, _P, _P, _P]),
    "gmmxx_xx_total": (_I32, [_I32, _P, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "gmmxx_assign": (_I32, [_I32, _I32, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _SZ, _P]),
    "gmmxx_logsumexp": (_I32, [_I32, _I32, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _SZ, _P]),
    "gmmxx_resp": (_I32, [_I32, _I32, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "gmmxx_predict_proba": (_I32, [_I32, _I32, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _SZ, _P]),
    "gmmxx_logsumexp_noalloc": (_I32, [_I32, _I32, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P]),
    "gmmxx_kmeans_pp_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "gmmxx_kmeans_pp": (_I32, [_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _SZ, _P]),
    "gmmxx_label_stats_width": (_I64, [_I32, _I64]),
    "gmmxx_label_stats_workspace_bytes": (_SZ, [_I32, _I64, _I64, _I64, _I64]),
    "gmmxx_label_stats": (_I32, [_I32, _P, _I64, _I64, _I64, _I64, _P, _P, _I32, _P, _P, _SZ, _P]),
}


def exported_symbols():
    """Names of every C ABI function this binding requires."""
    return sorted(_SIGNATURES)


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the shared library; raise if it is absent."""
    global _lib, _load_error
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            _load_error = FileNotFoundError(path)
            raise CudaBackendUnavailable(
                f"gmmxx_b200 CUDA library not built ({path} missing); run `python -m gmmxx_b200.build`"
            )
        try:
            lib = ctypes.CDLL(path)
        except OSError as exc:  # pragma: no cover - depends on the host
            _load_error = exc
            raise CudaBackendUnavailable(f"cannot load {path}: {exc}") from exc
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.gmmxx_abi_version() != 1:
            raise CudaBackendUnavailable("gmmxx_b200 library ABI version mismatch")
        _lib = lib
        return lib


def available() -> bool:
    try:
        load()
        return True
    except CudaBackendUnavailable:
        return False


def call(name: str, *args) -> None:
    """Invoke a C ABI function and raise on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.gmmxx_last_error().decode("utf-8", "replace")
        if rc == ERR_UNSUPPORTED:
            raise UnsupportedShape(rc, f"{name}: {msg}")
        raise GmmxxError(rc, f"{name}: {msg}")


def stat_width(cov: int, d: int) -> int:
    return int(load().gmmxx_stat_width(cov, d))


def accumulate_path(cov: int, xdt: int, b: int, n: int, d: int, k: int) -> int:
    """1 when gmmxx_em_accumulate runs the tensor-core kernel for this shape, else 0."""
    out = ctypes.c_int(0)
    call("gmmxx_accumulate_path", cov, xdt, b, n, d, k, ctypes.addressof(out))
    return out.value


# gmmxx_last_accumulate_path values
PATH_NAMES = {-1: None, 0: "cuda-core", 1: "tensor-core", 2: "cuda-core (tensor-core launch had no co-resident cluster)"}


def last_accumulate_path() -> int:
    """Statistics path of the last successful gmmxx_em_accumulate on this host
    thread: 1 tensor cores, 0 CUDA cores, 2 CUDA cores after the tensor-core
    launch found no co-resident cluster, -1 none yet."""
    return int(load().gmmxx_last_accumulate_path())


def workspace_bytes(cov: int, b: int, n: int, d: int, k: int) -> int:
    return int(load().gmmxx_workspace_bytes(cov, b, n, d, k))


def topk_scratch_bytes(b: int, n: int, top_k: int) -> int:
    return int(load().gmmxx_topk_scratch_bytes(b, n, top_k))


def kmeans_pp_workspace_bytes(b: int, s: int, trials: int) -> int:
    return int(load().gmmxx_kmeans_pp_workspace_bytes(b, s, trials))


def label_stats_width(mode: int, d: int) -> int:
    return int(load().gmmxx_label_stats_width(mode, d))


def label_stats_workspace_bytes(mode: int, b: int, n: int, d: int, k: int) -> int:
    return int(load().gmmxx_label_stats_workspace_bytes(mode, b, n, d, k))
