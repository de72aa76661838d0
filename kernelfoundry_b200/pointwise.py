"""Host API of the RMSNorm, RoPE and SwiGLU kernels (include/kf_pointwise.h).

The reference lists these kernels as planned and has no code for them
(sviraaj/kernelfoundry, README.md:16-18); the conventions are those of the
Llama-family modules in transformers (rounding points in kf_pointwise.h).
Tensors are CUDA fp16 or bf16; calls are asynchronous on the current stream
and run in libkf_attn.so.  There is no CPU path.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import KF_PW_BF16, KF_ROPE_GPTJ, check, lib

__all__ = ["rms_norm", "fused_add_rms_norm", "rope_", "swiglu"]

_DT_FLAGS = {torch.float16: 0, torch.bfloat16: KF_PW_BF16}


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _flags(*ts) -> int:
    dt = ts[0].dtype
    for t in ts:
        if not t.is_cuda:
            raise ValueError("tensors must be CUDA tensors (no CPU path)")
        if t.dtype != dt or dt not in _DT_FLAGS:
            raise ValueError("tensors must all be float16 or all bfloat16")
        if t.device != ts[0].device:
            raise ValueError("tensors must be on one device")
    return _DT_FLAGS[dt]


def _rows(x: torch.Tensor, hidden: int, name: str) -> int:
    if not x.is_contiguous() or x.shape[-1] != hidden:
        raise ValueError(f"{name} must be contiguous with last dimension {hidden}")
    return x.numel() // hidden if hidden else 0


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """``weight * rnd(x / sqrt(mean(x^2, -1) + eps))`` over the last dimension."""
    hidden = x.shape[-1]
    if weight.dim() != 1 or weight.shape[0] != hidden or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [hidden] tensor")
    out = torch.empty_like(x) if out is None else out
    flags = _flags(x, weight, out)
    if out.shape != x.shape:
        raise ValueError("out must have x's shape")
    rows = _rows(x, hidden, "x")
    _rows(out, hidden, "out")
    check(lib().kf_rmsnorm(_p(x), _p(weight), _p(out), None, rows, hidden, float(eps), flags, _stream(x)),
          "kf_rmsnorm")
    return out


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual <- rnd(x + residual)`` in place, then returns RMSNorm of it."""
    hidden = x.shape[-1]
    if weight.dim() != 1 or weight.shape[0] != hidden or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [hidden] tensor")
    if residual.shape != x.shape:
        raise ValueError("residual must have x's shape")
    out = torch.empty_like(x) if out is None else out
    flags = _flags(x, residual, weight, out)
    if out.shape != x.shape:
        raise ValueError("out must have x's shape")
    rows = _rows(x, hidden, "x")
    _rows(residual, hidden, "residual")
    _rows(out, hidden, "out")
    check(lib().kf_rmsnorm(_p(x), _p(weight), _p(out), _p(residual), rows, hidden, float(eps), flags,
                           _stream(x)), "kf_rmsnorm")
    return out


def rope_(q: torch.Tensor, k: torch.Tensor | None, positions: torch.Tensor | None = None, *,
          theta: float = 10000.0, rot_dim: int | None = None, interleaved: bool = False,
          inv_freq: torch.Tensor | None = None, layout: str = "bhsd") -> None:
    """Rotary embedding in place on ``q`` and ``k``.

    layout ``"bhsd"``: q ``[B, H_q, S, D]``, k ``[B, H_kv, S, D]`` (the
    attention layout); ``"bshd"``: ``[B, S, H, D]``.  Any strides with a
    contiguous head dimension are accepted.  positions: int32 ``[B, S]``
    (None: 0..S-1).  interleaved selects GPT-J pairs (2i, 2i+1), else NeoX
    pairs (i, i + rot_dim/2).  inv_freq: optional float32 ``[rot_dim/2]``
    table replacing ``theta^(-2i/rot_dim)``.
    """
    ts = [q] + ([k] if k is not None else [])
    flags = _flags(*ts) | (KF_ROPE_GPTJ if interleaved else 0)
    if layout not in ("bhsd", "bshd"):
        raise ValueError("layout must be 'bhsd' or 'bshd'")
    for t in ts:
        if t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError("q/k must be 4-D with a contiguous head dimension")

    def dims(t):
        if layout == "bhsd":
            B, H, S, D = t.shape
            return B, H, S, D, t.stride(0), t.stride(1), t.stride(2)
        B, S, H, D = t.shape
        return B, H, S, D, t.stride(0), t.stride(2), t.stride(1)

    B, H_q, S, D, qsb, qsh, qss = dims(q)
    if k is not None:
        Bk, H_kv, Sk, Dk, ksb, ksh, kss = dims(k)
        if (Bk, Sk, Dk) != (B, S, D):
            raise ValueError("k must match q in B, S and D")
    else:
        H_kv, ksb, ksh, kss = 0, 0, 0, 0
    rot = D if rot_dim is None else int(rot_dim)
    if positions is not None:
        if positions.dtype != torch.int32 or positions.shape != (B, S) or not positions.is_contiguous() \
                or positions.device != q.device:
            raise ValueError("positions must be a contiguous int32 [B, S] tensor on q's device")
    if inv_freq is not None:
        if inv_freq.dtype != torch.float32 or inv_freq.numel() != rot // 2 or not inv_freq.is_contiguous() \
                or inv_freq.device != q.device:
            raise ValueError("inv_freq must be a contiguous float32 [rot_dim/2] tensor on q's device")
    check(lib().kf_rope(_p(q), _p(k), _p(positions), _p(inv_freq), B, S, H_q, H_kv, D, rot, float(theta),
                        qsb, qsh, qss, ksb, ksh, kss, flags, _stream(q)), "kf_rope")


def swiglu(gate_up: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """``rnd(rnd(silu(g)) * u)`` of ``gate_up = [..., 2 * inter]`` (gate first)."""
    two_i = gate_up.shape[-1]
    if two_i % 2:
        raise ValueError("last dimension of gate_up must be even")
    inter = two_i // 2
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], inter, dtype=gate_up.dtype, device=gate_up.device)
    flags = _flags(gate_up, out)
    if out.shape != (*gate_up.shape[:-1], inter):
        raise ValueError("out must be [..., inter]")
    rows = _rows(gate_up, two_i, "gate_up")
    _rows(out, inter, "out")
    check(lib().kf_swiglu(_p(gate_up), _p(out), rows, inter, flags, _stream(gate_up)), "kf_swiglu")
    return out
