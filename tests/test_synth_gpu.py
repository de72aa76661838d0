"""Device generator kf_fill_normal_f16 (include/kf_synth.h) vs its NumPy restatement.

Both evaluate the same binary64 formula and round once to fp16; their log,
cos and sin may differ by an ulp or two of binary64, which changes the fp16
result only for a value within a few 2^-53 of an fp16 rounding boundary
(about 1e-12 per element), so the outputs are compared bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.synth_oracle import normal_f16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,seed,offset", [(1, 5, 0), (2, 5, 1), (1_000_003, 0x5EED, 0),
                                           (654_321, 2**64 - 1, 12_345), (4096, 42, (1 << 40) + 7)])
def test_device_matches_numpy(cuda, n, seed, offset):
    import torch

    from kernelfoundry_b200 import fill_normal_f16

    t = torch.full((n,), float("nan"), dtype=torch.float16, device=cuda)
    fill_normal_f16(t, seed, offset)
    got = t.cpu().numpy()
    want = normal_f16(n, seed, offset)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


def test_writes_only_its_range(cuda):
    import torch

    from kernelfoundry_b200 import fill_normal_f16

    buf = torch.full((1000,), 7.0, dtype=torch.float16, device=cuda)
    fill_normal_f16(buf[101:900], 9, 3)                    # odd start, odd length
    host = buf.cpu().numpy()
    assert (host[:101] == 7.0).all() and (host[900:] == 7.0).all()
    assert np.array_equal(host[101:900].view(np.uint16), normal_f16(799, 9, 3).view(np.uint16))


def test_stream_draws_are_consecutive(cuda):
    from kernelfoundry_b200 import NormalStream

    s = NormalStream(1002)
    q = s.f16((2, 3, 5, 8), cuda)
    k = s.f16((2, 1, 5, 8), cuda)
    assert s.offset == q.numel() + k.numel()
    both = normal_f16(q.numel() + k.numel(), 1002)
    assert np.array_equal(q.cpu().numpy().reshape(-1).view(np.uint16), both[:q.numel()].view(np.uint16))
    assert np.array_equal(k.cpu().numpy().reshape(-1).view(np.uint16), both[q.numel():].view(np.uint16))


def test_large_fill_moments(cuda):
    """A 1 GiB-scale fill (256 Mi elements) stays N(0,1) and matches NumPy on sampled slices."""
    import torch

    from kernelfoundry_b200 import fill_normal_f16

    n = 1 << 28
    t = torch.empty(n, dtype=torch.float16, device=cuda)
    fill_normal_f16(t, 31337)
    x = t.float()
    assert abs(x.mean().item()) < 1e-3 and abs(x.std().item() - 1.0) < 1e-3
    assert torch.isfinite(x).all().item()
    for off in (0, n // 3 + 1, n - 4096):
        assert np.array_equal(t[off:off + 4096].cpu().numpy().view(np.uint16),
                              normal_f16(4096, 31337, off).view(np.uint16)), off
