"""ctypes binding of libkf_attn.so (the C ABI declared in include/kf_attn.h,
include/kf_pointwise.h and include/kf_synth.h).

There is no fallback: if the library is missing this module raises, and every
compute entry point goes through the CUDA kernels in the library.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH

KF_OK = 0
KF_ERR_INVALID_ARG = 1
KF_ERR_UNSUPPORTED_HEAD_DIM = 2
KF_ERR_MISALIGNED = 3
KF_ERR_CUDA = 4
KF_ERR_DEVICE_TIMEOUT = 5
KF_ERR_UNSUPPORTED_DEVICE = 6
KF_ERR_WORKSPACE = 7

KF_FLAG_CAUSAL = 1
KF_FLAG_OUT_F16 = 2
KF_FLAG_OUT_BF16 = 4

KF_PW_BF16 = 1
KF_ROPE_GPTJ = 2

# Every symbol include/kf_attn.h, include/kf_pointwise.h and include/kf_synth.h declare.
EXPORTED = [
    "kf_strerror", "kf_last_cuda_error", "kf_version",
    "kf_attn_fwd", "kf_attn_fwd_lse", "kf_attn_fwd_ex", "kf_attn_fwd_paged", "kf_attn_paged_workspace_bytes", "kf_attn_fwd_partial", "kf_attn_combine", "kf_attn_combine_packed",
    "kf_attn_workspace_bytes", "kf_attn_workspace_init", "kf_attn_plan",
    "kf_launch_flash_attn", "kf_attn_fwd_noalloc", "kf_device_error", "kf_set_wait_timeout_ns",
    "kf_selftest_wait_timeout",
    "kf_rmsnorm", "kf_rope", "kf_swiglu",
    "kf_peer_window_bytes", "kf_peer_window_alloc", "kf_peer_window_open", "kf_peer_window_close",
    "kf_peer_window_free", "kf_attn_exchange_combine", "kf_attn_fwd_exchange", "kf_attn_exchange_workspace_bytes",
    "kf_fill_normal_f16",
]

KF_PEER_HANDLE_BYTES = 64
KF_MAX_PEERS = 8


class KFError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = lib().kf_strerror(code).decode()
        if code == KF_ERR_CUDA:
            msg += f" (cudaError {lib().kf_last_cuda_error()})"
        super().__init__(f"{what}: {msg}" if what else msg)


_lib = None


def lib():
    """Load libkf_attn.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python -m kernelfoundry_b200.build` "
                          "(the package has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, I, Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    FP = ctypes.POINTER(ctypes.c_float)
    L.kf_strerror.argtypes = [I]
    L.kf_strerror.restype = ctypes.c_char_p
    L.kf_last_cuda_error.argtypes = []
    L.kf_last_cuda_error.restype = I
    L.kf_version.argtypes = []
    L.kf_version.restype = ctypes.c_char_p
    L.kf_attn_fwd.argtypes = [P, P, P, P, I, I, I, I, I, I, P, Z, P]
    L.kf_attn_fwd.restype = I
    L.kf_attn_fwd_lse.argtypes = [P, P, P, P, P, P, I, I, I, I, I, I, P, Z, P]
    L.kf_attn_fwd_lse.restype = I
    L.kf_attn_fwd_ex.argtypes = [P, P, P, P, P, P, I, I, I, I, I, I, ctypes.c_uint, P, Z, P]
    L.kf_attn_fwd_ex.restype = I
    L.kf_attn_fwd_paged.argtypes = [P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P, Z, P]
    L.kf_attn_fwd_paged.restype = I
    L.kf_attn_paged_workspace_bytes.argtypes = [I, I, I, I, I, I, I]
    L.kf_attn_paged_workspace_bytes.restype = Z
    L.kf_attn_fwd_partial.argtypes = [P, P, P, P, P, P, I, I, I, I, I, I, P, Z, P]
    L.kf_attn_fwd_partial.restype = I
    L.kf_attn_combine.argtypes = [P, P, P, I, P, P, P, I, I, I, I, P]
    L.kf_attn_combine.restype = I
    L.kf_attn_combine_packed.argtypes = [P, ctypes.c_longlong, I, P, P, P, I, I, I, I, P]
    L.kf_attn_combine_packed.restype = I
    L.kf_attn_workspace_bytes.argtypes = [I, I, I, I, I, I]
    L.kf_attn_workspace_bytes.restype = Z
    L.kf_attn_workspace_init.argtypes = [P, Z, P]
    L.kf_attn_workspace_init.restype = I
    L.kf_attn_plan.argtypes = [I, I, I, I, I, I, Z, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(I)]
    L.kf_attn_plan.restype = I
    L.kf_launch_flash_attn.argtypes = [P, P, P, P, I, I, I, I, I, P]
    L.kf_launch_flash_attn.restype = I
    L.kf_attn_fwd_noalloc.argtypes = [P, P, P, P, I, I, I, I, I, I, P]
    L.kf_attn_fwd_noalloc.restype = I
    L.kf_device_error.argtypes = [I, ctypes.POINTER(ctypes.c_uint)]
    L.kf_device_error.restype = I
    L.kf_set_wait_timeout_ns.argtypes = [ctypes.c_ulonglong]
    L.kf_set_wait_timeout_ns.restype = None
    L.kf_selftest_wait_timeout.argtypes = [ctypes.c_ulonglong, P]
    L.kf_selftest_wait_timeout.restype = I
    LL, U, F = ctypes.c_longlong, ctypes.c_uint, ctypes.c_float
    L.kf_peer_window_bytes.argtypes = [I, LL, I]
    L.kf_peer_window_bytes.restype = Z
    L.kf_peer_window_alloc.argtypes = [Z, ctypes.POINTER(P), P]
    L.kf_peer_window_alloc.restype = I
    L.kf_peer_window_open.argtypes = [P, ctypes.POINTER(P)]
    L.kf_peer_window_open.restype = I
    L.kf_peer_window_close.argtypes = [P]
    L.kf_peer_window_close.restype = I
    L.kf_peer_window_free.argtypes = [P]
    L.kf_peer_window_free.restype = I
    L.kf_attn_exchange_combine.argtypes = [ctypes.POINTER(P), I, I, LL, I, P, P, P, I, I, I, I, P]
    L.kf_attn_exchange_combine.restype = I
    L.kf_attn_fwd_exchange.argtypes = [P, P, P, ctypes.POINTER(P), I, I, LL, P, P, P, I, I, I, I, I, I, P, Z, P]
    L.kf_attn_fwd_exchange.restype = I
    L.kf_attn_exchange_workspace_bytes.argtypes = [I, I, I, I, I, I]
    L.kf_attn_exchange_workspace_bytes.restype = Z
    L.kf_rmsnorm.argtypes = [P, P, P, P, LL, I, F, U, P]
    L.kf_rmsnorm.restype = I
    L.kf_rope.argtypes = [P, P, P, P, I, I, I, I, I, I, F, LL, LL, LL, LL, LL, LL, U, P]
    L.kf_rope.restype = I
    L.kf_swiglu.argtypes = [P, P, LL, I, U, P]
    L.kf_swiglu.restype = I
    L.kf_fill_normal_f16.argtypes = [P, LL, ctypes.c_ulonglong, LL, P]
    L.kf_fill_normal_f16.restype = I
    del FP
    _lib = L
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != KF_OK:
        raise KFError(rc, what)
