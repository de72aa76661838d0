"""RMSNorm / RoPE / SwiGLU kernels (include/kf_pointwise.h) vs the fp64 oracle.

Tolerances, in units of the storage type's spacing (ulp) at the oracle's value:
* RMSNorm and SwiGLU: the kernels round at the same points as the oracle but
  carry fp32 intermediates (sum of squares, rsqrtf, exp), so a value can land
  on the other side of a rounding boundary: at most 2 ulp, and at least 99 %
  (RMSNorm) / 98 % (SwiGLU) of outputs bit-identical.  The fused residual sum
  is exact.
* RoPE: one rounding of a rotation whose fp32 cos/sin carry ~2^-23 relative
  error: at most 1 ulp plus 2^-20 of the pair's magnitude |x0| + |x1| (the
  second term covers outputs that cancel to near zero), at any position up to
  2^31 - 1.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import pointwise_oracle as po

pytestmark = pytest.mark.gpu


def _dev(a, dt, device):
    import torch

    a = np.ascontiguousarray(a)
    if dt == "f16":
        return torch.from_numpy(a.astype(np.float16)).to(device)
    return torch.from_numpy(a.astype(np.float32)).to(device).to(torch.bfloat16)


def _host(t):
    return t.float().cpu().numpy().astype(np.float64)


def _rand(rng, shape, dt, scale=1.0):
    return po.round_to(rng.standard_normal(shape) * scale, dt)


def _assert_ulps(got, ref, dt, max_ulps, min_exact, what, extra=None):
    assert np.isfinite(got).all() == np.isfinite(ref).all(), f"{what}: non-finite mismatch"
    fin = np.isfinite(ref)
    np.testing.assert_array_equal(got[~fin], ref[~fin])
    g, r = got[fin], ref[fin]
    d = np.abs(g - r)
    tol = max_ulps * po.ulp(r, dt)
    if extra is not None:
        tol = tol + extra[fin]
    bad = d > tol
    assert not bad.any(), f"{what}: {bad.sum()} outside tolerance, worst {(d / tol).max():.2f}x"
    exact = (d == 0).mean() if d.size else 1.0
    assert exact >= min_exact, f"{what}: only {exact:.4f} bit-identical"


# ---------------------------------------------------------------- RMSNorm
RMS_SHAPES = [(1, 8), (3, 24), (7, 128), (5, 1000), (33, 1032), (64, 4096), (3, 5120), (2, 8192), (4, 16384),
              (2, 32768)]


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("rows,hidden", RMS_SHAPES)
def test_rmsnorm(cuda, dt, rows, hidden):
    from kernelfoundry_b200 import fused_add_rms_norm, rms_norm

    rng = np.random.default_rng(rows * 100003 + hidden)
    x = _rand(rng, (rows, hidden), dt, 2.0)
    w = po.round_to(1.0 + 0.3 * rng.standard_normal(hidden), dt)
    res = _rand(rng, (rows, hidden), dt)
    eps = 1e-5
    y_ref, _ = po.rms_norm(x, w, eps, dt)
    xt, wt = _dev(x, dt, cuda), _dev(w, dt, cuda)
    _assert_ulps(_host(rms_norm(xt, wt, eps)), y_ref, dt, 2, 0.99, f"rmsnorm {rows}x{hidden}")
    y2_ref, s_ref = po.rms_norm(x, w, eps, dt, residual=res)
    rt = _dev(res, dt, cuda)
    y2 = fused_add_rms_norm(xt, rt, wt, eps)
    np.testing.assert_array_equal(_host(rt), s_ref)
    _assert_ulps(_host(y2), y2_ref, dt, 2, 0.99, f"fused add rmsnorm {rows}x{hidden}")


def test_rmsnorm_in_place_and_batched_shape(cuda):
    """out may alias x; leading dimensions flatten into rows."""
    from kernelfoundry_b200 import fused_add_rms_norm, rms_norm

    rng = np.random.default_rng(11)
    x = _rand(rng, (2, 3, 5, 256), "f16")
    w = po.round_to(1.0 + 0.3 * rng.standard_normal(256), "f16")
    res = _rand(rng, (2, 3, 5, 256), "f16")
    y_ref, _ = po.rms_norm(x.reshape(-1, 256), w, 1e-6, "f16")
    xt = _dev(x, "f16", cuda)
    rms_norm(xt, _dev(w, "f16", cuda), 1e-6, out=xt)
    _assert_ulps(_host(xt).reshape(-1, 256), y_ref, "f16", 2, 0.99, "in place")
    y2_ref, s_ref = po.rms_norm(x.reshape(-1, 256), w, 1e-6, "f16", residual=res.reshape(-1, 256))
    xt, rt = _dev(x, "f16", cuda), _dev(res, "f16", cuda)
    fused_add_rms_norm(xt, rt, _dev(w, "f16", cuda), 1e-6, out=xt)
    np.testing.assert_array_equal(_host(rt).reshape(-1, 256), s_ref)
    _assert_ulps(_host(xt).reshape(-1, 256), y2_ref, "f16", 2, 0.99, "fused in place")


def test_rmsnorm_full_size_rows(cuda):
    """The benchmark shape [16384, 4096]: the residual update is exact everywhere and a
    sample of rows matches the oracle."""
    import torch

    from kernelfoundry_b200 import fused_add_rms_norm

    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(16384, 4096, generator=g, device=cuda).half()
    res = torch.randn(16384, 4096, generator=g, device=cuda).half()
    w = (1 + 0.2 * torch.randn(4096, generator=g, device=cuda)).half()
    s_expect = (x.float() + res.float()).half()
    x_h, res_h, w_h = _host(x), _host(res), _host(w)
    y = fused_add_rms_norm(x, res, w, 1e-5)
    assert torch.equal(res, s_expect)
    rows = np.random.default_rng(0).choice(16384, 96, replace=False)
    y_ref, _ = po.rms_norm(x_h[rows], w_h, 1e-5, "f16", residual=res_h[rows])
    _assert_ulps(_host(y)[rows], y_ref, "f16", 2, 0.99, "full-size sample")


# ---------------------------------------------------------------- RoPE
def _pair_mag(x, rot, interleaved):
    mag = np.zeros_like(x)
    if interleaved:
        m = np.abs(x[..., 0:rot:2]) + np.abs(x[..., 1:rot:2])
        mag[..., 0:rot:2] = m
        mag[..., 1:rot:2] = m
    else:
        h = rot // 2
        m = np.abs(x[..., :h]) + np.abs(x[..., h:rot])
        mag[..., :h] = m
        mag[..., h:rot] = m
    return mag


def _check_rope(got, x, pos, dt, theta, rot, interleaved, what, inv_freq=None):
    ref = po.rope(x, pos, dt, theta=theta, rot_dim=rot, interleaved=interleaved, inv_freq=inv_freq)
    extra = 2.0 ** -20 * _pair_mag(x, rot, interleaved)
    _assert_ulps(got, ref, dt, 1, 0.9, what, extra=extra)
    np.testing.assert_array_equal(got[..., rot:], x[..., rot:])


ROPE_CASES = [
    # B, H_q, H_kv, S, D, rot, interleaved, dt
    (1, 4, 2, 16, 64, 64, False, "f16"),
    (2, 32, 8, 33, 128, 128, False, "f16"),
    (2, 32, 8, 33, 128, 128, True, "f16"),
    (1, 8, 1, 7, 128, 64, False, "f16"),         # partial rotary
    (1, 8, 1, 7, 128, 40, True, "f16"),          # partial rotary, GPT-J, rot % 16 != 0
    (3, 5, 5, 9, 256, 256, False, "bf16"),
    (2, 12, 4, 5, 80, 80, False, "bf16"),        # D = 80 (5 NeoX units)
    (1, 1, 0, 300, 16, 16, False, "f16"),        # Q only, smallest NeoX head
    (1, 2, 1, 3, 1024, 1024, True, "f16"),       # largest head_dim
]


@pytest.mark.parametrize("B,Hq,Hkv,S,D,rot,inter,dt", ROPE_CASES)
def test_rope(cuda, B, Hq, Hkv, S, D, rot, inter, dt):
    import torch

    from kernelfoundry_b200 import rope_

    rng = np.random.default_rng(B * 7 + Hq * 13 + S * 17 + D + rot)
    q = _rand(rng, (B, Hq, S, D), dt)
    k = _rand(rng, (B, Hkv, S, D), dt)
    pos = rng.integers(0, 131072, size=(B, S)).astype(np.int32)
    for theta in (10000.0, 500000.0):
        qt, kt = _dev(q, dt, cuda), (_dev(k, dt, cuda) if Hkv else None)
        rope_(qt, kt, torch.from_numpy(pos).to(cuda), theta=theta, rot_dim=rot, interleaved=inter)
        _check_rope(_host(qt), q, pos, dt, theta, rot, inter, f"q theta={theta}")
        if Hkv:
            _check_rope(_host(kt), k, pos, dt, theta, rot, inter, f"k theta={theta}")


def test_rope_default_positions_and_extremes(cuda):
    import torch

    from kernelfoundry_b200 import rope_

    rng = np.random.default_rng(2)
    q = _rand(rng, (2, 4, 64, 128), "f16")
    qt = _dev(q, "f16", cuda)
    rope_(qt, None)                                          # positions 0..S-1
    _check_rope(_host(qt), q, None, "f16", 10000.0, 128, False, "default positions")
    pos = np.array([[0, 1, 2 ** 31 - 1, 2 ** 30 + 12345] * 16, [131071, 65536, 4095, 7] * 16], dtype=np.int32)
    qt = _dev(q, "f16", cuda)
    rope_(qt, None, torch.from_numpy(pos).to(cuda))
    _check_rope(_host(qt), q, pos, "f16", 10000.0, 128, False, "extreme positions")


def test_rope_bshd_views_and_inv_freq_table(cuda):
    """[B, S, H, D] storage, q/k as strided views of one fused QKV buffer, and a
    caller frequency table (a scaled variant) in place of theta."""
    import torch

    from kernelfoundry_b200 import rope_

    rng = np.random.default_rng(9)
    B, S, Hq, Hkv, D = 2, 40, 8, 2, 128
    qkv = _rand(rng, (B, S, Hq + 2 * Hkv, D), "bf16")
    inv = po.rope_inv_freq(D, 500000.0)
    inv = np.where(np.arange(D // 2) >= 40, inv / 8.0, inv).astype(np.float32)
    pos = rng.integers(0, 8192, size=(B, S)).astype(np.int32)
    t = _dev(qkv, "bf16", cuda)
    q, k = t[:, :, :Hq], t[:, :, Hq:Hq + Hkv]
    rope_(q, k, torch.from_numpy(pos).to(cuda), layout="bshd", inv_freq=torch.from_numpy(inv).to(cuda))
    got = _host(t)
    for sl, what in ((slice(0, Hq), "q"), (slice(Hq, Hq + Hkv), "k")):
        x = qkv[:, :, sl].transpose(0, 2, 1, 3)
        _check_rope(got[:, :, sl].transpose(0, 2, 1, 3), x, pos, "bf16", 0.0, D, False, what, inv_freq=inv)
    np.testing.assert_array_equal(got[:, :, Hq + Hkv:], qkv[:, :, Hq + Hkv:])   # V untouched


# ---------------------------------------------------------------- SwiGLU
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("rows,inter", [(1, 8), (3, 264), (5, 1000), (64, 14336), (2, 2056)])
def test_swiglu(cuda, dt, rows, inter):
    from kernelfoundry_b200 import swiglu

    rng = np.random.default_rng(rows * 31 + inter)
    gu = _rand(rng, (rows, 2 * inter), dt, 3.0)
    ref = po.swiglu(gu, dt)
    _assert_ulps(_host(swiglu(_dev(gu, dt, cuda))), ref, dt, 2, 0.98, f"swiglu {rows}x{inter}")


def test_swiglu_special_values(cuda):
    """Zero, tiny, saturated and the largest finite gates."""
    from kernelfoundry_b200 import swiglu

    g = np.array([0.0, -0.0, 1e-3, -1e-3, 30.0, -30.0, 65504.0, -65504.0, 11.0, -17.5, 0.5, -0.5, 2.0, -2.0,
                  6e-5, -6e-5])
    u = np.array([1.0, -1.0, 2.0, 3.0, 0.5, 0.25, 0.5, 4.0, -1.0, 1.0, 0.0, 100.0, -3.0, 7.0, 1.0, 1.0])
    gu = po.round_to(np.concatenate([g, u])[None, :], "f16")
    ref = po.swiglu(gu, "f16")
    _assert_ulps(_host(swiglu(_dev(gu, "f16", cuda))), ref, "f16", 2, 0.8, "special values")


def test_swiglu_full_size_rows(cuda):
    """The benchmark shape [8192, 2 x 14336]: a sample of rows matches the oracle."""
    import torch

    from kernelfoundry_b200 import swiglu

    g = torch.Generator(device=cuda).manual_seed(8)
    gu = (3 * torch.randn(8192, 2 * 14336, generator=g, device=cuda)).half()
    y = swiglu(gu)
    rows = np.random.default_rng(1).choice(8192, 64, replace=False)
    ref = po.swiglu(_host(gu[torch.from_numpy(rows).to(cuda)]), "f16")
    _assert_ulps(_host(y)[rows], ref, "f16", 2, 0.98, "full-size sample")
