"""The C-ABI library loads, exports what include/kf_attn.h,
include/kf_pointwise.h and include/kf_synth.h declare, and validates arguments
before touching a GPU (no compute calls here)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO

HEADERS = [os.path.join(REPO, "include", h) for h in ("kf_attn.h", "kf_pointwise.h", "kf_synth.h")]


def _declared():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names.update(re.findall(r"\b(kf_[a-z_0-9]+)\s*\(", text))
    return sorted(names)


def test_header_symbols_exported(kf_lib):
    from kernelfoundry_b200 import _lib
    from kernelfoundry_b200.build import LIB_PATH

    declared = _declared()
    assert len(declared) >= 17
    assert {"kf_rmsnorm", "kf_rope", "kf_swiglu", "kf_fill_normal_f16"} <= set(declared)
    assert sorted(declared) == sorted(_lib.EXPORTED)
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (kf_\w+)", out))
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(kf_lib, s)


def test_library_is_product_only(kf_lib):
    """The product library contains no oracle / reference code."""
    from kernelfoundry_b200.build import LIB_PATH

    out = subprocess.run(["nm", "-D", LIB_PATH], capture_output=True, text=True, check=True).stdout
    assert "kfo_" not in out and "kfref" not in out
    pkg = os.path.join(REPO, "kernelfoundry_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(root, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f


def test_no_gpu_dependency_at_load():
    """libkf_attn.so needs no libcuda / libcudart at load time (static runtime, driver via entry point)."""
    from kernelfoundry_b200.build import LIB_PATH

    out = subprocess.run(["readelf", "-d", LIB_PATH], capture_output=True, text=True, check=True).stdout
    needed = re.findall(r"Shared library: \[(.*?)\]", out)
    assert not any(n.startswith("libcuda.so") or n.startswith("libcudart") for n in needed), needed


def test_strerror_covers_codes(kf_lib):
    texts = {kf_lib.kf_strerror(c).decode() for c in range(0, 8)}
    assert len(texts) == 8
    assert kf_lib.kf_strerror(12345).decode() == "unknown status"
    assert b"sm_100a" in kf_lib.kf_version()


FAKE = ctypes.c_void_p(0x10000)          # 16-byte aligned, never dereferenced
MISALIGNED = ctypes.c_void_p(0x10008)


def _fwd(lib, B=1, Hq=4, Hkv=2, Sq=8, Skv=8, D=64, q=FAKE, k=FAKE, v=FAKE, o=FAKE):
    return lib.kf_attn_fwd(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, None, 0, None)


def test_argument_validation_without_gpu(kf_lib):
    from kernelfoundry_b200 import _lib as L

    assert _fwd(kf_lib, D=32) == L.KF_ERR_UNSUPPORTED_HEAD_DIM
    assert _fwd(kf_lib, D=96) == L.KF_ERR_UNSUPPORTED_HEAD_DIM
    assert _fwd(kf_lib, Hq=6, Hkv=4) == L.KF_ERR_INVALID_ARG        # H_q % H_kv != 0
    assert _fwd(kf_lib, Hkv=0) == L.KF_ERR_INVALID_ARG
    assert _fwd(kf_lib, B=-1) == L.KF_ERR_INVALID_ARG
    assert _fwd(kf_lib, Skv=0) == L.KF_ERR_INVALID_ARG              # softmax over no keys
    assert _fwd(kf_lib, q=ctypes.c_void_p(0)) == L.KF_ERR_INVALID_ARG
    assert _fwd(kf_lib, k=MISALIGNED) == L.KF_ERR_MISALIGNED
    assert _fwd(kf_lib, o=MISALIGNED) == L.KF_ERR_MISALIGNED
    # Empty problems are a successful no-op and never reach the GPU.
    assert _fwd(kf_lib, B=0) == L.KF_OK
    assert _fwd(kf_lib, Sq=0) == L.KF_OK
    assert kf_lib.kf_attn_fwd_partial(FAKE, FAKE, FAKE, FAKE, None, None, 1, 4, 2, 8, 8, 64, None, 0, None) \
        == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_attn_combine(FAKE, FAKE, FAKE, 0, FAKE, None, None, 1, 4, 8, 64, None) == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_attn_combine(FAKE, FAKE, FAKE, 2, FAKE, None, None, 1, 4, 8, 48, None) \
        == L.KF_ERR_UNSUPPORTED_HEAD_DIM
    assert kf_lib.kf_attn_combine(FAKE, FAKE, FAKE, 2, FAKE, None, None, 0, 4, 8, 64, None) == L.KF_OK
    # kf_attn_fwd_ex: unknown flag bits and causal with S_q > S_kv are rejected before any launch.
    assert kf_lib.kf_attn_fwd_ex(FAKE, FAKE, FAKE, FAKE, None, None, 1, 4, 2, 8, 8, 64, 8, None, 0, None) \
        == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_attn_fwd_ex(FAKE, FAKE, FAKE, FAKE, None, None, 1, 4, 2, 9, 8, 64, L.KF_FLAG_CAUSAL, None, 0,
                                 None) == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_attn_fwd_ex(FAKE, FAKE, FAKE, FAKE, None, None, 0, 4, 2, 9, 8, 64, 0, None, 0, None) == L.KF_OK
    assert kf_lib.kf_attn_fwd_ex(FAKE, FAKE, FAKE, FAKE, None, None, 1, 4, 2, 8, 8, 64,
                                 L.KF_FLAG_OUT_F16 | L.KF_FLAG_OUT_BF16, None, 0, None) == L.KF_ERR_INVALID_ARG
    # Paged decode: bad block sizes, non-decode shapes and a zero pool are rejected before any launch.
    def _paged(B=2, Hq=8, Hkv=2, Sq=1, D=128, nb=64, bs=16, mb=8):
        return kf_lib.kf_attn_fwd_paged(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, B, Hq, Hkv, Sq, D, nb, bs, mb,
                                        None, 0, None)
    assert _paged(bs=24) == L.KF_ERR_INVALID_ARG
    assert _paged(bs=8) == L.KF_ERR_INVALID_ARG
    assert _paged(bs=512) == L.KF_ERR_INVALID_ARG
    assert _paged(nb=0) == L.KF_ERR_INVALID_ARG
    assert _paged(Sq=64) == L.KF_ERR_INVALID_ARG            # 4 x 64 rows: not a decode shape
    assert _paged(D=48) == L.KF_ERR_UNSUPPORTED_HEAD_DIM
    assert _paged(B=0) == L.KF_OK
    assert kf_lib.kf_attn_paged_workspace_bytes(1, 8, 2, 64, 128, 16, 8) == 0
    # Packed combine: part stride below rows*(D+2) or not a multiple of 4 is rejected before any launch.
    assert kf_lib.kf_attn_combine_packed(FAKE, 4 * 8 * 66 - 4, 2, FAKE, None, None, 1, 4, 8, 64, None) \
        == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_attn_combine_packed(FAKE, 4 * 8 * 66 + 2, 2, FAKE, None, None, 1, 4, 8, 64, None) \
        == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_attn_combine_packed(FAKE, 4 * 8 * 66, 0, FAKE, None, None, 1, 4, 8, 64, None) \
        == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_attn_combine_packed(FAKE, 4 * 8 * 50, 2, FAKE, None, None, 1, 4, 8, 48, None) \
        == L.KF_ERR_UNSUPPORTED_HEAD_DIM
    assert kf_lib.kf_attn_combine_packed(FAKE, 4 * 8 * 66, 2, FAKE, None, None, 0, 4, 8, 64, None) == L.KF_OK
    assert kf_lib.kf_attn_workspace_bytes(1, 6, 4, 1, 100, 128) == 0
    assert kf_lib.kf_launch_flash_attn(FAKE, FAKE, FAKE, FAKE, 1, 16, 1, 1, 48, None) \
        == L.KF_ERR_UNSUPPORTED_HEAD_DIM


def test_peer_exchange_argument_validation_without_gpu(kf_lib):
    from kernelfoundry_b200 import _lib as L

    # window size: staging part + 2 parities x world slots of 8-byte words + n_chunks counters
    # staging + 2 x 2 slots of 8-byte words + per-unit counters (part / 16) + 4 chunk counters
    assert kf_lib.kf_peer_window_bytes(2, 4160, 4) == (4160 * (1 + 4 * 2) + 4160 // 16 + 4) * 4
    assert kf_lib.kf_peer_window_bytes(0, 4160, 4) == 0
    assert kf_lib.kf_peer_window_bytes(9, 4160, 4) == 0          # more than KF_MAX_PEERS
    assert kf_lib.kf_peer_window_bytes(2, 4162, 4) == 0          # part stride not a multiple of 4
    assert kf_lib.kf_peer_window_bytes(2, 4160, 0) == 0
    wins = (ctypes.c_void_p * 2)(FAKE, FAKE)

    def ex(world=2, rank=0, ps=32 * 130, nch=4, B=1, Hq=32, Sq=1, D=128, w=wins, o=FAKE):
        return kf_lib.kf_attn_exchange_combine(w, world, rank, ps, nch, o, None, None, B, Hq, Sq, D, None)

    assert ex(rank=2) == L.KF_ERR_INVALID_ARG
    assert ex(world=0) == L.KF_ERR_INVALID_ARG
    assert ex(ps=32 * 130 - 4) == L.KF_ERR_INVALID_ARG           # part smaller than rows*(D+2)
    assert ex(ps=32 * 130 + 2) == L.KF_ERR_INVALID_ARG
    assert ex(nch=0) == L.KF_ERR_INVALID_ARG
    assert ex(D=96) == L.KF_ERR_UNSUPPORTED_HEAD_DIM
    assert ex(o=ctypes.c_void_p(0)) == L.KF_ERR_INVALID_ARG
    assert ex(w=(ctypes.c_void_p * 2)(FAKE, ctypes.c_void_p(0))) == L.KF_ERR_INVALID_ARG
    assert ex(w=(ctypes.c_void_p * 2)(FAKE, MISALIGNED)) == L.KF_ERR_MISALIGNED
    assert ex(B=0) == L.KF_OK
    assert kf_lib.kf_peer_window_alloc(0, ctypes.byref(ctypes.c_void_p()), FAKE) == L.KF_ERR_INVALID_ARG
    assert kf_lib.kf_peer_window_open(None, ctypes.byref(ctypes.c_void_p())) == L.KF_ERR_INVALID_ARG


def test_pointwise_argument_validation_without_gpu(kf_lib):
    from kernelfoundry_b200 import _lib as L

    def rms(x=FAKE, w=FAKE, o=FAKE, r=None, rows=4, hidden=256, eps=1e-6, flags=0):
        return kf_lib.kf_rmsnorm(x, w, o, r, rows, hidden, eps, flags, None)

    assert rms(hidden=12) == L.KF_ERR_INVALID_ARG              # not a multiple of 8
    assert rms(hidden=0) == L.KF_ERR_INVALID_ARG
    assert rms(hidden=32776) == L.KF_ERR_INVALID_ARG           # above 32768
    assert rms(rows=-1) == L.KF_ERR_INVALID_ARG
    assert rms(eps=-1.0) == L.KF_ERR_INVALID_ARG
    assert rms(eps=float("nan")) == L.KF_ERR_INVALID_ARG
    assert rms(flags=4) == L.KF_ERR_INVALID_ARG
    assert rms(w=ctypes.c_void_p(0)) == L.KF_ERR_INVALID_ARG
    assert rms(x=MISALIGNED) == L.KF_ERR_MISALIGNED
    assert rms(r=MISALIGNED) == L.KF_ERR_MISALIGNED
    assert rms(rows=0) == L.KF_OK

    def rope(q=FAKE, k=FAKE, B=1, S=8, Hq=4, Hkv=2, D=128, rot=128, theta=1e4, qs=(4096, 1024, 128),
             ks=(2048, 1024, 128), flags=0, inv=None):
        return kf_lib.kf_rope(q, k, None, inv, B, S, Hq, Hkv, D, rot, theta, *qs, *ks, flags, None)

    assert rope(rot=136) == L.KF_ERR_INVALID_ARG               # rot_dim > D
    assert rope(rot=40) == L.KF_ERR_INVALID_ARG                # NeoX needs a multiple of 16
    # Accepted argument sets are checked on empty problems (S = 0): they pass validation and
    # return before any launch, so no kernel ever runs on these placeholder pointers.
    assert rope(rot=40, flags=L.KF_ROPE_GPTJ, S=0) == L.KF_OK
    assert rope(rot=36, flags=L.KF_ROPE_GPTJ) == L.KF_ERR_INVALID_ARG
    assert rope(D=1032, rot=64) == L.KF_ERR_INVALID_ARG
    assert rope(theta=0.0) == L.KF_ERR_INVALID_ARG
    assert rope(theta=0.0, inv=FAKE, S=0) == L.KF_OK            # a frequency table replaces theta
    assert rope(qs=(4096, 1024, 130)) == L.KF_ERR_INVALID_ARG  # stride not a multiple of 8
    assert rope(ks=(-2048, 1024, 128)) == L.KF_ERR_INVALID_ARG
    assert rope(k=ctypes.c_void_p(0)) == L.KF_ERR_INVALID_ARG
    assert rope(k=ctypes.c_void_p(0), Hkv=0, S=0) == L.KF_OK
    assert rope(Hq=0, Hkv=0) == L.KF_ERR_INVALID_ARG
    assert rope(flags=8) == L.KF_ERR_INVALID_ARG
    assert rope(q=MISALIGNED) == L.KF_ERR_MISALIGNED
    assert rope(B=0) == L.KF_OK
    assert rope(S=0) == L.KF_OK

    def swiglu(g=FAKE, o=FAKE, rows=4, inter=256, flags=0):
        return kf_lib.kf_swiglu(g, o, rows, inter, flags, None)

    assert swiglu(inter=12) == L.KF_ERR_INVALID_ARG
    assert swiglu(rows=-3) == L.KF_ERR_INVALID_ARG
    assert swiglu(flags=2) == L.KF_ERR_INVALID_ARG
    assert swiglu(o=ctypes.c_void_p(0)) == L.KF_ERR_INVALID_ARG
    assert swiglu(o=MISALIGNED) == L.KF_ERR_MISALIGNED
    assert swiglu(rows=0) == L.KF_OK


def test_fill_normal_argument_validation_without_gpu(kf_lib):
    from kernelfoundry_b200 import _lib as L

    fill = kf_lib.kf_fill_normal_f16
    assert fill(None, 0, 1, 0, None) == L.KF_OK               # empty fill: no CUDA call
    assert fill(FAKE, 0, 1, 7, None) == L.KF_OK
    assert fill(FAKE, -1, 1, 0, None) == L.KF_ERR_INVALID_ARG
    assert fill(FAKE, 8, 1, -2, None) == L.KF_ERR_INVALID_ARG
    assert fill(None, 8, 1, 0, None) == L.KF_ERR_INVALID_ARG
    assert fill(FAKE, 1 << 62, 1, 1, None) == L.KF_ERR_INVALID_ARG
    assert fill(ctypes.c_void_p(FAKE.value + 1), 8, 1, 0, None) == L.KF_ERR_MISALIGNED


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="checks the no-driver path")
def test_pointwise_compute_call_without_driver_reports_cuda_error(kf_lib):
    from kernelfoundry_b200 import _lib as L

    assert kf_lib.kf_rmsnorm(FAKE, FAKE, FAKE, None, 4, 256, 1e-6, 0, None) in (L.KF_ERR_CUDA,
                                                                              L.KF_ERR_UNSUPPORTED_DEVICE)
    assert kf_lib.kf_swiglu(FAKE, FAKE, 4, 256, 0, None) in (L.KF_ERR_CUDA, L.KF_ERR_UNSUPPORTED_DEVICE)
    assert kf_lib.kf_fill_normal_f16(FAKE, 8, 1, 0, None) in (L.KF_ERR_CUDA, L.KF_ERR_UNSUPPORTED_DEVICE)


def test_pointwise_python_api_refuses_cpu_tensors(kf_lib):
    import torch

    from kernelfoundry_b200 import rms_norm, rope_, swiglu

    x = torch.zeros(4, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        rms_norm(x, torch.ones(64, dtype=torch.float16))
    with pytest.raises(ValueError, match="CUDA"):
        swiglu(x)
    with pytest.raises(ValueError, match="CUDA"):
        rope_(x.view(1, 1, 4, 64), None)


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="checks the no-driver path")
def test_compute_call_without_driver_reports_cuda_error(kf_lib):
    """Without a GPU a valid call fails with a status code (never a crash or a CPU fallback)."""
    from kernelfoundry_b200 import _lib as L

    rc = _fwd(kf_lib)
    assert rc in (L.KF_ERR_CUDA, L.KF_ERR_UNSUPPORTED_DEVICE)
    assert kf_lib.kf_last_cuda_error() != 0


def test_python_api_refuses_cpu_tensors(kf_lib):
    import torch

    from kernelfoundry_b200 import flash_attn_fwd

    q = torch.zeros(1, 2, 4, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        flash_attn_fwd(q, q[:, :1], q[:, :1])


def test_fused_exchange_argument_checks_without_gpu(kf_lib):
    """kf_attn_fwd_exchange rejects bad world sizes, ranks, windows and part strides
    before any CUDA call."""
    from kernelfoundry_b200 import _lib as L

    wins = (ctypes.c_void_p * 2)(FAKE, FAKE)

    def _x(world=2, rank=0, ps=8 * 132, windows=wins, B=1, D=128):
        return kf_lib.kf_attn_fwd_exchange(FAKE, FAKE, FAKE, windows, world, rank, ps, FAKE, None, None,
                                           B, 8, 2, 1, 4096, D, None, 0, None)
    assert _x(world=3) == L.KF_ERR_INVALID_ARG
    assert _x(world=0) == L.KF_ERR_INVALID_ARG
    assert _x(rank=2) == L.KF_ERR_INVALID_ARG
    assert _x(windows=None) == L.KF_ERR_INVALID_ARG
    assert _x(ps=8 * 129) == L.KF_ERR_INVALID_ARG                      # part smaller than rows * (D + 2)
    assert _x(ps=8 * 130 + 2) == L.KF_ERR_INVALID_ARG                  # not a multiple of 4
    assert _x(windows=(ctypes.c_void_p * 2)(FAKE, MISALIGNED)) == L.KF_ERR_MISALIGNED
    assert _x(D=96) == L.KF_ERR_UNSUPPORTED_HEAD_DIM
    assert _x(B=0) == L.KF_OK                                          # empty problem: no launch
