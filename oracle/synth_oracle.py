"""NumPy restatement of the counter-based N(0,1) fp16 generator (include/kf_synth.h).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU legs of ``bench.py`` (``cpu_baseline`` and ``--impl reference``) may import
this module: the tests check the device generator against it, and the CPU legs
use it to rebuild the exact inputs the GPU arm reads.

The reference has no such generator (its harnesses use mt19937 uniform[-1,1],
tests/test_utils.h:27-31).  Definition, identical to the device kernel:

* ``w(c)`` = output ``c`` of splitmix64 seeded with ``s`` (Steele, Lea and
  Flood, OOPSLA 2014; Vigna's splitmix64.c), all arithmetic mod 2^64;
* pair ``k``: ``u1 = ((w(2k) >> 11) + 1) * 2^-53``, ``u2 = (w(2k+1) >> 11) * 2^-53``,
  ``r = sqrt(-2 ln u1)``, ``t = 6.283185307179586 * u2``; element ``2k`` is
  ``r cos t`` and element ``2k+1`` is ``r sin t`` (Box and Muller, 1958), in
  binary64, each rounded once to fp16.
"""
from __future__ import annotations

import numpy as np

__all__ = ["splitmix64", "normal_f16"]

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, counters) -> np.ndarray:
    """Outputs ``counters`` (uint64 array) of splitmix64 seeded with ``seed``."""
    c = np.asarray(counters, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + (c + np.uint64(1)) * _GAMMA
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def normal_f16(n: int, seed: int, offset: int = 0, chunk: int = 1 << 22) -> np.ndarray:
    """Elements ``[offset, offset + n)`` of the stream with ``seed`` as float16."""
    if n < 0 or offset < 0:
        raise ValueError("n and offset must be non-negative")
    out = np.empty(n, dtype=np.float16)
    first = offset >> 1
    end = (offset + n + 1) >> 1
    for k0 in range(first, end, chunk):
        k = np.arange(k0, min(end, k0 + chunk), dtype=np.uint64)
        w0 = splitmix64(seed, np.uint64(2) * k)
        w1 = splitmix64(seed, np.uint64(2) * k + np.uint64(1))
        u1 = ((w0 >> np.uint64(11)) + np.uint64(1)).astype(np.float64) * 2.0 ** -53
        u2 = (w1 >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
        r = np.sqrt(-2.0 * np.log(u1))
        t = 6.283185307179586 * u2
        pair = np.empty((k.size, 2), dtype=np.float64)
        pair[:, 0] = r * np.cos(t)
        pair[:, 1] = r * np.sin(t)
        vals = pair.reshape(-1)
        lo = 2 * k0 - offset                       # index in `out` of element 2*k0
        s = max(0, -lo)
        e = min(vals.size, n - lo)
        out[lo + s:lo + e] = vals[s:e].astype(np.float16)
    return out
