"""Seeded N(0,1) fp16 inputs generated on the GPU (include/kf_synth.h).

Element i of the stream with seed s is a pure function of (s, i)
(splitmix64 counter -> Box-Muller in binary64 -> fp16), so the benchmark's
inputs need no files and any slice of them can be rebuilt bit for bit on the
host.  No counterpart in the reference (its harnesses use mt19937
uniform[-1,1], tests/test_utils.h:27-31).  There is no CPU path here.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib

__all__ = ["fill_normal_f16", "NormalStream"]


def fill_normal_f16(t: torch.Tensor, seed: int, offset: int = 0) -> torch.Tensor:
    """Fill the contiguous CUDA fp16 tensor ``t`` with elements ``[offset, offset + t.numel())``
    of the stream with ``seed``; asynchronous on the current stream.  Returns ``t``."""
    if not t.is_cuda:
        raise ValueError("t must be a CUDA tensor (no CPU path)")
    if t.dtype != torch.float16 or not t.is_contiguous():
        raise ValueError("t must be a contiguous float16 tensor")
    if offset < 0:
        raise ValueError("offset must be non-negative")
    stream = ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
    check(lib().kf_fill_normal_f16(ctypes.c_void_p(t.data_ptr()), t.numel(), seed & (2**64 - 1), offset, stream),
          "kf_fill_normal_f16")
    return t


class NormalStream:
    """Consecutive draws from one seeded stream: each ``f16`` call takes the next
    ``prod(shape)`` elements, so a config seeded once yields Q, K, V in draw order."""

    def __init__(self, seed: int, offset: int = 0):
        self.seed = seed & (2**64 - 1)
        self.offset = offset

    def f16(self, shape, device) -> torch.Tensor:
        t = torch.empty(shape, dtype=torch.float16, device=device)
        fill_normal_f16(t, self.seed, self.offset)
        self.offset += t.numel()
        return t

    def skip(self, n: int) -> "NormalStream":
        """Advance past ``n`` elements without generating them."""
        self.offset += n
        return self
