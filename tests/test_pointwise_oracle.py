"""Pin the RMSNorm / RoPE / SwiGLU oracle (no GPU).

The reference ships no code for these kernels (README.md:16-18), so the pin
is tests/golden/pointwise_golden.npz: outputs of transformers' Llama modules
(LlamaRMSNorm, LlamaRotaryEmbedding + apply_rotary_pos_emb, LlamaMLP's
act_fn(gate) * up) made by tests/golden/make_pointwise_golden.py.
RMSNorm and SwiGLU share transformers' rounding points and must match it bit
for bit.  RoPE rounds once where transformers rounds cos/sin and each product
to fp16 first, so its fp16 comparison allows 2^-9 of the pair's magnitude
|x0| + |x1| (transformers' own error is up to ~2^-10 of it); the float32
variant pins the unrounded rotation to 2e-4 of that magnitude (the fp32
angle pos * inv_freq carries ~1e-4 rad at positions < 2048).
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import pointwise_oracle as po


@pytest.fixture(scope="module")
def z():
    return np.load(os.path.join(GOLDEN, "pointwise_golden.npz"))


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_rmsnorm_matches_transformers(z, dt):
    x, w, eps = z[f"rms_{dt}_x"], z[f"rms_{dt}_w"], float(z[f"rms_{dt}_eps"])
    y, none = po.rms_norm(x, w, eps, dt)
    assert none is None
    np.testing.assert_array_equal(y, z[f"rms_{dt}_y"].astype(np.float64))
    y2, s = po.rms_norm(x, w, eps, dt, residual=z[f"rms_{dt}_res"])
    np.testing.assert_array_equal(s, z[f"rms_{dt}_s"].astype(np.float64))
    np.testing.assert_array_equal(y2, z[f"rms_{dt}_yres"].astype(np.float64))


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_swiglu_matches_transformers(z, dt):
    y = po.swiglu(z[f"swiglu_{dt}_gu"], dt)
    np.testing.assert_array_equal(y, z[f"swiglu_{dt}_y"].astype(np.float64))


def _pair_mag(x):
    h = x.shape[-1] // 2
    m = np.abs(x[..., :h]) + np.abs(x[..., h:])
    return np.concatenate([m, m], axis=-1)


@pytest.mark.parametrize("tag", ["t1e4", "t5e5"])
def test_rope_matches_transformers(z, tag):
    theta = float(z[f"rope_{tag}_theta"])
    D = z[f"rope_{tag}_q"].shape[-1]
    np.testing.assert_allclose(po.rope_inv_freq(D, theta), z[f"rope_{tag}_inv_freq"], rtol=1e-7)
    for nm in ("q", "k"):
        x = z[f"rope_{tag}_{nm}"].astype(np.float64)
        pos = z[f"rope_{tag}_pos"]
        mag = _pair_mag(x)
        y16 = po.rope(x, pos, "f16", theta=theta)
        d = np.abs(y16 - z[f"rope_{tag}_{nm}o"])
        assert (d <= 2.0 ** -9 * mag).all(), (d / mag).max()
        assert (d == 0).mean() > 0.5                 # same pairing, signs and frequencies
        y = po.rope(x, pos, None, theta=theta)
        d32 = np.abs(y - z[f"rope_{tag}_{nm}o32"])
        assert (d32 <= 2e-4 * mag).all(), (d32 / mag).max()


def test_rope_pairings_and_pass_through():
    """GPT-J pairs (2i, 2i+1); partial rotary leaves dims >= rot_dim; position 0 is the identity."""
    rng = np.random.default_rng(3)
    x = po.round_to(rng.standard_normal((1, 2, 5, 32)), "f16")
    pos = np.array([[0, 1, 7, 100, 4095]])
    np.testing.assert_array_equal(po.rope(x, pos, "f16")[:, :, 0], x[:, :, 0])
    y = po.rope(x, pos, "f16", rot_dim=16)
    np.testing.assert_array_equal(y[..., 16:], x[..., 16:])
    # GPT-J on x equals NeoX on the de-interleaved x, re-interleaved.
    perm = np.concatenate([np.arange(0, 32, 2), np.arange(1, 32, 2)])
    gj = po.rope(x, pos, None, interleaved=True)
    nx = po.rope(x[..., perm], pos, None)
    np.testing.assert_allclose(gj[..., perm], nx, rtol=0, atol=1e-12)


def test_bf16_rounding_matches_torch():
    import torch

    rng = np.random.default_rng(0)
    x = rng.standard_normal(50000) * 10.0 ** rng.integers(-40, 38, 50000)
    x = np.concatenate([x, [1e-39, -3e-40, 3.39e38, 3.4e38, 0.0, 1.00390625, 1.01171875]])
    ref = torch.from_numpy(x).to(torch.bfloat16).double().numpy()
    np.testing.assert_array_equal(po.round_bf16(x), ref)
