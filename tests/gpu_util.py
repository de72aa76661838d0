"""Helpers for the GPU parity tests: run the kernels through the C ABI on
numpy inputs and compare with the oracle."""
from __future__ import annotations

import numpy as np

from oracle.attn_oracle import error_stats, reference_attn_lse

# North-star tolerance vs the fp64 oracle (reference_attn on fp16-rounded inputs).
MAX_ABS_TOL = 2e-3
REL_L2_TOL = 1e-3


def to_dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def run_fwd(Q, K, V, device, return_lse=False, workspace=None):
    from kernelfoundry_b200 import flash_attn_fwd

    q, k, v = (to_dev(x, device) for x in (Q, K, V))
    res = flash_attn_fwd(q, k, v, return_lse=return_lse, workspace=workspace)
    if return_lse:
        return tuple(r.cpu().numpy() for r in res)
    return res.cpu().numpy()


def oracle64(Q, K, V):
    return reference_attn_lse(Q.astype(np.float64), K.astype(np.float64), V.astype(np.float64))


def assert_close(got, ref, what="", max_abs=MAX_ABS_TOL, rel_l2=REL_L2_TOL):
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    ma, rl = error_stats(got, ref)
    assert ma <= max_abs and rl <= rel_l2, f"{what}: max_abs={ma:.3e} rel_l2={rl:.3e}"
    return ma, rl
