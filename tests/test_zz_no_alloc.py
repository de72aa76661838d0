"""kf_attn_fwd_noalloc: the decode entry point that allocates nothing.

Some callers cannot allocate device memory when they call attention: a serving
loop that handed all free memory to its KV-cache pool at start-up, or a
latency-bound decode loop that must not call cudaMalloc because it can
synchronize the device.  kf_attn_fwd_noalloc takes its split-KV scratch from a
fixed array inside the library instead of a workspace.  These checks call it
through the C ABI, twice in a row (every call reuses the same array), and
compare each result with the fp64 oracle (reference_attn on the fp16 inputs)
at the north-star tolerance and with kf_attn_fwd given a workspace.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes when run alone in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle.attn_oracle import error_stats, normal_qkv

from gpu_util import MAX_ABS_TOL, REL_L2_TOL, assert_close, oracle64, to_dev

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 2 << 20
P = ctypes.c_void_p


def _call_noalloc(lib, q, k, v, out, stream):
    B, H_q, S_q, D = q.shape
    H_kv, S_kv = k.shape[1], k.shape[2]
    return lib.kf_attn_fwd_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(out.data_ptr()),
                                   B, H_q, H_kv, S_q, S_kv, D, P(stream))


def _call_with_workspace(lib, q, k, v, out, ws, stream):
    B, H_q, S_q, D = q.shape
    H_kv, S_kv = k.shape[1], k.shape[2]
    return lib.kf_attn_fwd(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(out.data_ptr()),
                           B, H_q, H_kv, S_q, S_kv, D, P(ws.data_ptr()), ws.numel(), P(stream))


SHAPES = [
    (1, 32, 8, 1, 4096, 128),     # decode KV=4096, 16 splits
    (1, 32, 8, 1, 65536, 128),    # long decode
    (2, 32, 1, 1, 1000, 64),      # MQA, D=64
    (3, 8, 8, 1, 777, 256),       # D=256
    (2, 32, 8, 2, 2048, 128),     # two query positions
    (8, 32, 1, 1, 32768, 128),    # full plan needs more than the scratch: fewer splits
]


def _split_count(lib, shape, ws_bytes):
    path, ns, ctas = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    assert lib.kf_attn_plan(*shape, ws_bytes, ctypes.byref(path), ctypes.byref(ns), ctypes.byref(ctas)) == 0
    assert path.value == 1
    return ns.value


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_noalloc_matches_oracle_and_workspace_entry_point(cuda, shape):
    import torch

    from kernelfoundry_b200._lib import KF_OK, lib

    L = lib()
    B, H_q, H_kv, S_q, S_kv, D = shape
    need = L.kf_attn_workspace_bytes(*shape)
    Q, K, V = normal_qkv(*shape, seed=11 * sum(shape))
    O64 = oracle64(Q, K, V)[0]
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    stream = torch.cuda.current_stream(cuda).cuda_stream
    # kf_attn_fwd with the workspace the same plan gets inside the fixed scratch.
    ws_bytes = min(need, SCRATCH_BYTES)
    ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=cuda)
    ref = torch.empty((B, H_q, S_q, D), dtype=torch.float32, device=cuda)
    assert _call_with_workspace(L, q, k, v, ref, ws, stream) == KF_OK
    torch.cuda.synchronize()
    ref_np = ref.cpu().numpy()
    assert_close(ref_np, O64, f"kf_attn_fwd {shape}")
    if need > SCRATCH_BYTES:
        assert _split_count(L, shape, SCRATCH_BYTES) < _split_count(L, shape, need)
    for call in range(2):
        out = torch.full((B, H_q, S_q, D), float("nan"), dtype=torch.float32, device=cuda)
        assert _call_noalloc(L, q, k, v, out, stream) == KF_OK
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert_close(got, O64, f"noalloc call {call} {shape}")
        max_abs, rel_l2 = error_stats(got, ref_np)
        assert max_abs <= MAX_ABS_TOL and rel_l2 <= REL_L2_TOL, (call, max_abs, rel_l2)


def test_noalloc_rejects_prefill_shapes(cuda):
    import torch

    from kernelfoundry_b200._lib import KF_ERR_INVALID_ARG, KF_OK, lib

    L = lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    # Prefill shapes use no split scratch and belong to kf_attn_fwd.
    q = torch.zeros((1, 8, 512, 128), dtype=torch.float16, device=cuda)
    kv = torch.zeros((1, 2, 512, 128), dtype=torch.float16, device=cuda)
    out = torch.zeros((1, 8, 512, 128), dtype=torch.float32, device=cuda)
    assert _call_noalloc(L, q, kv, kv, out, stream) == KF_ERR_INVALID_ARG
    # Empty problems are a no-op.
    assert L.kf_attn_fwd_noalloc(None, None, None, None, 0, 32, 8, 1, 128, 128, None) == KF_OK
