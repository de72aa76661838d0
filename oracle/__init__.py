"""CPU oracle for the attention forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker (or as the timed
CPU baseline).  The product (``kernelfoundry_b200``) never imports it.

Contents:
  attn_oracle.py  NumPy restatement of kernel_models/flash_attn.py
                  (reference_attn, tile model) plus Mi/Li and split-KV
                  partial/combine identities.
  cpu_attn.c      C restatement of tests/test_flash_attn.cu:cpu_attn and
                  tests/test_utils.h:fill_random_f32 (mt19937 uniform).
  ref_wrap.cu     Wrapper that compiles the unmodified reference sources into
                  oracle/_ref/libkfref.so (reference CPU code and CUDA kernel).
  Makefile        Builds lib/libkforacle.so and _ref/libkfref.so.
  pointwise_oracle.py  RMSNorm / RoPE / SwiGLU in fp64 with explicit fp16 /
                  bf16 rounding.  The reference has no code for these
                  (README.md:16-18): parity against it is unpinned; the
                  functions are pinned to transformers' Llama modules
                  instead (tests/golden/make_pointwise_golden.py).

Parity is pinned: tests/test_oracle.py checks these against golden vectors
produced by the reference itself (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
C_ORACLE_PATH = os.path.join(_HERE, "lib", "libkforacle.so")
REF_LIB_PATH = os.path.join(_HERE, "_ref", "libkfref.so")

_c_lib = None
_ref_lib = None


def build_c_oracle() -> str:
    """Compile cpu_attn.c into lib/libkforacle.so (gcc, no FMA contraction)."""
    subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)
    return C_ORACLE_PATH


def load_c_oracle():
    global _c_lib
    if _c_lib is None:
        if not os.path.exists(C_ORACLE_PATH):
            build_c_oracle()
        lib = ctypes.CDLL(C_ORACLE_PATH)
        P = ctypes.c_void_p
        lib.kfo_mt19937_uniform_f32.argtypes = [P, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_uint32]
        lib.kfo_mt19937_uniform_f32.restype = None
        lib.kfo_mt19937_raw.argtypes = [P, ctypes.c_size_t, ctypes.c_uint32]
        lib.kfo_mt19937_raw.restype = None
        lib.kfo_cpu_attn.argtypes = [P, P, P, P] + [ctypes.c_int] * 6 + [P]
        lib.kfo_cpu_attn.restype = ctypes.c_int
        _c_lib = lib
    return _c_lib


def mt19937_uniform_f32(n: int, lo: float, hi: float, seed: int) -> np.ndarray:
    """tests/test_utils.h:fill_random_f32 restated (std::mt19937 + uniform<float>)."""
    out = np.empty(int(n), dtype=np.float32)
    load_c_oracle().kfo_mt19937_uniform_f32(out.ctypes.data_as(ctypes.c_void_p), out.size,
                                            float(lo), float(hi), int(seed) & 0xFFFFFFFF)
    return out


def cpu_attn_f32(Q, K, V) -> np.ndarray:
    """tests/test_flash_attn.cu:cpu_attn restated (fp32 loops), S_q may differ from S_kv."""
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    B, H_q, S_q, D = Q.shape
    H_kv, S_kv = K.shape[1], K.shape[2]
    O = np.empty_like(Q)
    scratch = np.empty(max(S_kv, 1), dtype=np.float32)
    P = ctypes.c_void_p
    rc = load_c_oracle().kfo_cpu_attn(Q.ctypes.data_as(P), K.ctypes.data_as(P), V.ctypes.data_as(P),
                                      O.ctypes.data_as(P), B, S_q, S_kv, H_q, H_kv, D,
                                      scratch.ctypes.data_as(P))
    if rc != 0:
        raise ValueError("cpu_attn_f32: bad shapes")
    return O


def legacy_case_inputs(B, S, H_q, H_kv, D, seed):
    """Inputs of one reference harness case (tests/test_flash_attn.cu:237-251).

    Q/K/V are mt19937 uniform[-1,1] fp32 with seeds seed, seed+1, seed+2; the
    GPU receives their fp16 round-to-nearest copies.  Returns the fp32 arrays
    and their fp16 copies.
    """
    qn = B * H_q * S * D
    kn = B * H_kv * S * D
    q = mt19937_uniform_f32(qn, -1.0, 1.0, seed).reshape(B, H_q, S, D)
    k = mt19937_uniform_f32(kn, -1.0, 1.0, seed + 1).reshape(B, H_kv, S, D)
    v = mt19937_uniform_f32(kn, -1.0, 1.0, seed + 2).reshape(B, H_kv, S, D)
    return (q, k, v), (q.astype(np.float16), k.astype(np.float16), v.astype(np.float16))


# The reference harness's 18 cases, verbatim: (B, S, H_q, H_kv, D, seed)
# (tests/test_flash_attn.cu:295-318) and its tolerance (:22).
LEGACY_CASES = [
    (1, 16, 1, 1, 16, 100), (1, 16, 1, 1, 64, 101), (1, 64, 1, 1, 128, 102), (1, 17, 1, 1, 128, 103),
    (1, 129, 1, 1, 128, 202), (1, 255, 1, 1, 128, 203), (1, 256, 1, 1, 64, 200), (1, 256, 1, 1, 128, 201),
    (1, 64, 4, 2, 64, 300), (1, 64, 8, 2, 64, 301), (1, 64, 32, 8, 128, 302), (1, 64, 40, 8, 128, 303),
    (1, 64, 8, 1, 128, 304), (1, 16, 1, 1, 256, 305),
    (2, 64, 4, 4, 64, 400), (2, 128, 4, 2, 128, 401), (3, 33, 4, 4, 128, 402), (2, 129, 32, 8, 128, 403),
]
LEGACY_TOL = 5e-2


def load_ref_lib():
    """oracle/_ref/libkfref.so: the unmodified reference compiled from its sources."""
    global _ref_lib
    if _ref_lib is None:
        if not os.path.exists(REF_LIB_PATH):
            raise FileNotFoundError(f"{REF_LIB_PATH} not built (make -C oracle ref)")
        lib = ctypes.CDLL(REF_LIB_PATH)
        P = ctypes.c_void_p
        lib.kfref_fill_random_f32.argtypes = [P, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_uint32]
        lib.kfref_fill_random_f32.restype = None
        lib.kfref_cpu_attn.argtypes = [P, P, P, P] + [ctypes.c_int] * 5
        lib.kfref_cpu_attn.restype = ctypes.c_int
        lib.kfref_launch_flash_attn.argtypes = [P, P, P, P] + [ctypes.c_int] * 5 + [P]
        lib.kfref_launch_flash_attn.restype = ctypes.c_int
        lib.kfref_launch_general.argtypes = [P, P, P, P, P, P] + [ctypes.c_int] * 6 + [P]
        lib.kfref_launch_general.restype = ctypes.c_int
        _ref_lib = lib
    return _ref_lib
