"""Failure detection on the GPU without a GPU fault.

The only induced failure is a bounded wait on a barrier that nothing
signals (kf_selftest_wait_timeout): the kernel gives up after its limit,
records KF_ERR_DEVICE_TIMEOUT in the device error word and returns, and the
context stays usable.  No test traps, faults or hangs the GPU.
"""
from __future__ import annotations

import pytest

from oracle.attn_oracle import normal_qkv

from gpu_util import assert_close, oracle64, run_fwd

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    from kernelfoundry_b200 import _lib
    from kernelfoundry_b200.attention import device_error, selftest_wait_timeout

    assert device_error()[0] == _lib.KF_OK
    assert selftest_wait_timeout(20_000_000) == _lib.KF_ERR_DEVICE_TIMEOUT   # 20 ms limit, expired as designed
    assert device_error() == (_lib.KF_OK, 0)                                # cleared by the self-test
    Q, K, V = normal_qkv(1, 8, 2, 300, 300, 128, seed=1)
    assert_close(run_fwd(Q, K, V, cuda), oracle64(Q, K, V)[0], "after timeout")
    assert device_error()[0] == _lib.KF_OK


def test_normal_runs_leave_error_word_clear(cuda):
    from kernelfoundry_b200 import _lib
    from kernelfoundry_b200.attention import device_error

    for shape in [(1, 32, 8, 1, 4096, 128), (1, 32, 8, 512, 512, 128)]:
        Q, K, V = normal_qkv(*shape, seed=2)
        run_fwd(Q, K, V, cuda)
    assert device_error() == (_lib.KF_OK, 0)


def test_python_errors_raise(cuda):
    import torch

    from kernelfoundry_b200 import KFError, flash_attn_fwd

    q = torch.zeros(1, 6, 4, 64, dtype=torch.float16, device=cuda)
    k = torch.zeros(1, 4, 4, 64, dtype=torch.float16, device=cuda)
    with pytest.raises(KFError, match="invalid argument"):
        flash_attn_fwd(q, k, k)
    q = torch.zeros(1, 2, 4, 48, dtype=torch.float16, device=cuda)
    with pytest.raises(KFError, match="head dimension"):
        flash_attn_fwd(q, q, q)
