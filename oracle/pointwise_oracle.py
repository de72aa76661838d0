"""NumPy oracle for the RMSNorm, RoPE and SwiGLU kernels.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this module, and only as the
checker (or, for the baseline, as the timed CPU path).

Parity against the reference is unpinned: sviraaj/kernelfoundry lists the
three kernels as planned and ships no code for them (``README.md:16-18``).
The definitions restated here are the published ones as the Llama-family
modules of ``transformers`` (5.5, in this image) compute them:

* RMSNorm (Zhang & Sennrich, 2019) as ``LlamaRMSNorm.forward``: fp32 mean of
  squares, ``x * rsqrt(mean + eps)`` rounded to the storage dtype, then the
  product with the weight rounded again.  The fused residual form first
  rounds ``x + residual`` to the storage dtype.
* RoPE (Su et al., RoFormer, 2021) as ``rotate_half`` / ``apply_rotary_pos_emb``
  with ``inv_freq[i] = theta^(-2i/rot_dim)``: pair ``(i, i + rot_dim/2)``
  (NeoX) or ``(2i, 2i+1)`` (GPT-J) turns by ``pos * inv_freq[i]``.  Here the
  rotation is exact and rounded once; transformers rounds cos/sin to the
  storage dtype first, which is why the golden comparison for RoPE carries a
  few-ulp tolerance.
* SwiGLU (Shazeer, 2020) as ``LlamaMLP``: ``act_fn(gate) * up`` with SiLU,
  i.e. ``rnd(rnd(silu(g)) * u)``.

``tests/test_oracle.py`` pins these functions against
``tests/golden/pointwise_golden.npz``, which ``tests/golden/make_pointwise_golden.py``
produced by running those transformers modules on CPU.

Arithmetic is fp64 with explicit rounding to fp16 (NumPy's correctly rounded
float64 -> float16 conversion) or bf16 (:func:`round_bf16`, round to nearest
even on 8 significant bits).  Values travel as float64 arrays holding exactly
representable 16-bit numbers.
"""
from __future__ import annotations

import numpy as np

__all__ = ["round_to", "round_bf16", "ulp", "rms_norm", "rope", "rope_inv_freq", "swiglu"]


def round_bf16(x) -> np.ndarray:
    """float64 -> nearest bfloat16 value (ties to even), returned as float64."""
    x = np.asarray(x, dtype=np.float64)
    out = np.array(x, copy=True)
    fin = np.isfinite(x) & (x != 0)
    _, e = np.frexp(x[fin])                      # x = m 2^e, |m| in [0.5, 1)
    qe = np.maximum(e - 8, -133)                 # quantum: 8 significant bits, subnormals 2^-133
    out[fin] = np.ldexp(np.rint(np.ldexp(x[fin], -qe)), qe)
    big = np.abs(out) > 3.3895313892515355e38    # largest finite bfloat16
    out[big] = np.copysign(np.inf, out[big])
    return out


def round_to(x, dtype: str | None) -> np.ndarray:
    """Round float64 values to ``dtype`` ("f16" or "bf16"; None: no rounding), returned as float64."""
    if dtype is None:
        return np.asarray(x, dtype=np.float64)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float64).astype(np.float16).astype(np.float64)
    if dtype == "bf16":
        return round_bf16(x)
    raise ValueError(dtype)


def ulp(x, dtype: str) -> np.ndarray:
    """Spacing of ``dtype`` values at |x| (the subnormal spacing below the normal range)."""
    x = np.abs(np.asarray(x, dtype=np.float64))
    mant, emin = (10, -14) if dtype == "f16" else (7, -126)
    e = np.floor(np.log2(np.maximum(x, 2.0 ** emin)))
    return np.ldexp(1.0, (e - mant).astype(np.int64))


def rms_norm(x, w, eps: float, dtype: str, residual=None):
    """Returns ``(out, new_residual)``; ``new_residual`` is None without a residual.

    ``x`` ``[rows, hidden]`` and ``w`` ``[hidden]`` hold ``dtype`` values.
    """
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    new_res = None
    if residual is not None:
        x = round_to(x + np.asarray(residual, dtype=np.float64), dtype)
        new_res = x
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return round_to(round_to(x * r, dtype) * w, dtype), new_res


def rope_inv_freq(rot_dim: int, theta: float) -> np.ndarray:
    return float(theta) ** (-(2.0 * np.arange(rot_dim // 2)) / rot_dim)


def rope(x, positions, dtype: str, theta: float = 10000.0, rot_dim: int | None = None,
         interleaved: bool = False, inv_freq=None) -> np.ndarray:
    """Rotate ``x`` ``[B, H, S, D]`` by ``positions`` ``[B, S]`` (None: 0..S-1)."""
    x = np.asarray(x, dtype=np.float64)
    B, H, S, D = x.shape
    rot = D if rot_dim is None else rot_dim
    f = rope_inv_freq(rot, theta) if inv_freq is None else np.asarray(inv_freq, dtype=np.float64)
    pos = np.broadcast_to(np.arange(S), (B, S)) if positions is None else np.asarray(positions)
    ang = pos.astype(np.float64)[:, None, :, None] * f[None, None, None, :]    # [B, 1, S, rot/2]
    c, s = np.cos(ang), np.sin(ang)
    out = np.array(x, copy=True)
    if interleaved:
        x0, x1 = x[..., 0:rot:2], x[..., 1:rot:2]
        out[..., 0:rot:2] = x0 * c - x1 * s
        out[..., 1:rot:2] = x1 * c + x0 * s
    else:
        h = rot // 2
        x0, x1 = x[..., :h], x[..., h:rot]
        out[..., :h] = x0 * c - x1 * s
        out[..., h:rot] = x1 * c + x0 * s
    return round_to(out, dtype)


def swiglu(gate_up, dtype: str) -> np.ndarray:
    """``gate_up`` ``[rows, 2 * inter]`` (gate first) -> ``[rows, inter]``."""
    gu = np.asarray(gate_up, dtype=np.float64)
    inter = gu.shape[-1] // 2
    g, u = gu[..., :inter], gu[..., inter:]
    with np.errstate(over="ignore"):
        h = round_to(g / (1.0 + np.exp(-g)), dtype)
    return round_to(h * u, dtype)
