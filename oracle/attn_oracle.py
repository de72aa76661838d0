"""NumPy restatement of the reference's attention oracle.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this module, and only as the
checker (or, for the baseline, as the timed CPU path).  The product library
never calls it; its CUDA entry points fail loudly when the extension is
missing instead of falling back here.

What it restates (sviraaj/kernelfoundry):

* :func:`reference_attn` -- ``kernel_models/flash_attn.py:250-265``: per
  (b, h_q) one GEMM ``Q Kᵀ · 1/sqrt(D)``, max-subtracted softmax, one GEMM with
  V, computed in the input dtype (fp64 inputs give the fp64 oracle the
  north-star tolerance is quoted against).  GQA maps ``h_kv = h // (H_q/H_kv)``
  (``kernel_models/flash_attn.py:254,259``; ``kernels/flash_attn.cu:406``).
  Like the reference it accepts ``S_q != S_kv`` (decode).
* :func:`reference_attn_lse` -- the same plus the softmax state the reference
  kernel writes (``kernels/flash_attn.cu:575-578``): ``Mi`` = row max of the
  scaled scores, ``Li`` = sum of ``exp(score - Mi)`` (natural-log units).
* :func:`attn_partial` / :func:`combine_partials` -- the (m, l, O_unnormalised)
  split-KV form of the same math: partial results over disjoint KV ranges,
  merged by log-sum-exp.  The reference has no split-KV; these are the
  algebraic identity behind its online softmax
  (``kernels/flash_attn.cu:261-294``) applied across ranges.
* :func:`tile_model_attn` -- ``kernel_models/flash_attn.py:184-246``, the
  reference's fp32 tile-for-tile model (prefill only, S_q == S_kv): Q tiles of
  16 rows, KV blocks of ``kv_block_rows`` rows, 8-column online-softmax steps.
  It is the slow single-threaded CPU path the reference ships.

Pinning: ``tests/test_oracle.py`` checks every function against
``tests/golden/*.npz``, which ``tests/golden/make_golden.py`` produced by
importing the reference's own ``kernel_models/flash_attn.py``.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "reference_attn",
    "reference_attn_lse",
    "attn_partial",
    "combine_partials",
    "tile_model_attn",
    "normal_qkv",
    "error_stats",
]


def _check_shapes(Q, K, V):
    if Q.ndim != 4 or K.ndim != 4 or V.ndim != 4:
        raise ValueError("Q, K, V must be [B, H, S, D]")
    B, H_q, _, D = Q.shape
    if K.shape != V.shape or K.shape[0] != B or K.shape[3] != D:
        raise ValueError("K/V shape mismatch")
    H_kv = K.shape[1]
    if H_q % H_kv != 0:
        raise ValueError("H_q must be a multiple of H_kv")
    return B, H_q, H_kv, D


def reference_attn(Q: np.ndarray, K: np.ndarray, V: np.ndarray) -> np.ndarray:
    """SDPA per head in the input dtype (kernel_models/flash_attn.py:250-265)."""
    return reference_attn_lse(Q, K, V)[0]


def reference_attn_lse(Q: np.ndarray, K: np.ndarray, V: np.ndarray):
    """Return (O, Mi, Li): output and the reference kernel's softmax state.

    Mi[b,h,i] = max_j s_ij and Li[b,h,i] = sum_j exp(s_ij - Mi) with
    s_ij = q_i . k_j / sqrt(D)  (kernels/flash_attn.cu:575-578, natural log).
    """
    B, H_q, H_kv, D = _check_shapes(Q, K, V)
    gqa = H_q // H_kv
    scale = 1.0 / np.sqrt(float(D))
    O = np.zeros_like(Q)
    S_q = Q.shape[2]
    Mi = np.zeros((B, H_q, S_q), dtype=Q.dtype)
    Li = np.zeros((B, H_q, S_q), dtype=Q.dtype)
    for b in range(B):
        for h in range(H_q):
            hk = h // gqa
            scores = Q[b, h] @ K[b, hk].T * scale
            m = scores.max(axis=-1, keepdims=True)
            P = np.exp(scores - m)
            l = P.sum(axis=-1, keepdims=True)
            P /= l
            O[b, h] = P @ V[b, hk]
            Mi[b, h] = m[:, 0]
            Li[b, h] = l[:, 0]
    return O, Mi, Li


def causal_attn_lse(Q: np.ndarray, K: np.ndarray, V: np.ndarray):
    """Causal (O, Mi, Li): extension with no reference counterpart -- the reference
    lists the missing causal mask as the gap for decoder use (docs/flash_attn.md:105).

    Bottom-right aligned, as in chunked prefill over a KV cache: query row i of S_q
    sits at absolute position S_kv - S_q + i and attends keys j <= S_kv - S_q + i.
    Every row sees at least key 0 when S_q <= S_kv (required).  Same scores, Mi and
    Li as reference_attn_lse restricted to the visible keys.
    """
    B, H_q, H_kv, D = _check_shapes(Q, K, V)
    S_q, S_kv = Q.shape[2], K.shape[2]
    if S_q > S_kv:
        raise ValueError("causal attention needs S_q <= S_kv")
    gqa = H_q // H_kv
    scale = 1.0 / np.sqrt(float(D))
    visible = np.arange(S_kv)[None, :] <= (S_kv - S_q + np.arange(S_q))[:, None]     # [S_q, S_kv]
    O = np.zeros_like(Q)
    Mi = np.zeros((B, H_q, S_q), dtype=Q.dtype)
    Li = np.zeros((B, H_q, S_q), dtype=Q.dtype)
    for b in range(B):
        for h in range(H_q):
            hk = h // gqa
            scores = np.where(visible, Q[b, h] @ K[b, hk].T * scale, -np.inf)
            m = scores.max(axis=-1, keepdims=True)
            P = np.exp(scores - m)
            l = P.sum(axis=-1, keepdims=True)
            O[b, h] = (P / l) @ V[b, hk]
            Mi[b, h] = m[:, 0]
            Li[b, h] = l[:, 0]
    return O, Mi, Li


def paged_attn_lse(Q, K_pool, V_pool, block_table, seq_lens, block_size):
    """(O, Mi, Li) over a paged KV cache: sequence b's keys are the first seq_lens[b]
    rows of its logical blocks, block j stored at pool block block_table[b, j] of
    K_pool/V_pool [n_blocks, H_kv, block_size, D] (the page layout of the reference's
    paged benchmark, reference_benchmarks/bench_flash_attn2.py:153-215, gathered the
    way its naive path gathers them).  A sequence with no keys gives O = 0,
    Mi = -inf, Li = 0.
    """
    B, H_q, S_q, D = Q.shape
    H_kv = K_pool.shape[1]
    O = np.zeros_like(Q)
    Mi = np.full((B, H_q, S_q), -np.inf, dtype=Q.dtype)
    Li = np.zeros((B, H_q, S_q), dtype=Q.dtype)
    for b in range(B):
        n = int(seq_lens[b])
        if n <= 0:
            continue
        nb = (n + block_size - 1) // block_size
        blocks = [int(x) for x in block_table[b, :nb]]
        Kb = np.concatenate([K_pool[pb] for pb in blocks], axis=1)[:, :n][None]     # [1, H_kv, n, D]
        Vb = np.concatenate([V_pool[pb] for pb in blocks], axis=1)[:, :n][None]
        o, mi, li = reference_attn_lse(Q[b:b + 1], Kb, Vb)
        O[b], Mi[b], Li[b] = o[0], mi[0], li[0]
    return O, Mi, Li


def causal_pairs(S_q: int, S_kv: int) -> int:
    """Number of visible (query, key) pairs under the bottom-right causal mask."""
    off = S_kv - S_q
    return sum(min(S_kv, off + i + 1) for i in range(S_q))


def attn_partial(Q: np.ndarray, K: np.ndarray, V: np.ndarray, kv_lo: int, kv_hi: int):
    """Softmax partials over keys [kv_lo, kv_hi).

    Returns (m, l, O_u): m = row max of scaled scores over the range, l = sum of
    exp(s - m), O_u = sum exp(s - m) v  (un-normalised; O = O_u / l).
    """
    return reference_attn_lse_unnorm(Q, K[:, :, kv_lo:kv_hi], V[:, :, kv_lo:kv_hi])


def reference_attn_lse_unnorm(Q, K, V):
    O, Mi, Li = reference_attn_lse(Q, K, V)
    return Mi, Li, O * Li[..., None]


def combine_partials(ms, ls, Os):
    """Merge per-range partials by log-sum-exp: M = max_g m_g,
    O = sum_g e^{m_g-M} O_g / sum_g e^{m_g-M} l_g."""
    ms = np.stack(ms)
    ls = np.stack(ls)
    Os = np.stack(Os)
    M = ms.max(axis=0)
    w = np.exp(ms - M[None])
    L = (w * ls).sum(axis=0)
    O = (w[..., None] * Os).sum(axis=0) / L[..., None]
    return O, M, L


def tile_model_attn(Q: np.ndarray, K: np.ndarray, V: np.ndarray, kv_block_rows: int = 128):
    """fp32 tile model of the reference kernel (kernel_models/flash_attn.py:184-246).

    Prefill only (S taken from Q for both loops, as in the reference).  Q tiles
    of 16 rows; KV blocks of ``kv_block_rows``; within a block, 8-column steps
    with the online max/sum update and O rescale of
    kernel_models/flash_attn.py:125-180.
    """
    Br, Bc_col = 16, 8
    B, H_q, S, D = Q.shape
    H_kv = K.shape[1]
    gqa = H_q // H_kv
    scale = np.float32(1.0 / np.sqrt(float(D)))
    O = np.zeros((B, H_q, S, D), dtype=np.float32)
    for b in range(B):
        for h in range(H_q):
            hk = h // gqa
            for q0 in range(0, S, Br):
                q_rows = min(Br, S - q0)
                q = Q[b, h, q0:q0 + q_rows].astype(np.float32)
                mi = np.full(q_rows, -np.inf, dtype=np.float32)
                li = np.zeros(q_rows, dtype=np.float32)
                o = np.zeros((q_rows, D), dtype=np.float32)
                for k0 in range(0, S, kv_block_rows):
                    kr = min(kv_block_rows, S - k0)
                    kb = K[b, hk, k0:k0 + kr].astype(np.float32)
                    vb = V[b, hk, k0:k0 + kr].astype(np.float32)
                    for c0 in range(0, kr, Bc_col):
                        n = min(Bc_col, kr - c0)
                        s = (q @ kb[c0:c0 + n].T) * scale
                        m_new = np.maximum(mi, s.max(axis=1))
                        p = np.exp(s - m_new[:, None])
                        resc = np.exp(mi - m_new)
                        li = li * resc + p.sum(axis=1)
                        mi = m_new
                        o = o * resc[:, None] + p @ vb[c0:c0 + n]
                O[b, h, q0:q0 + q_rows] = o / li[:, None]
    return O


def normal_qkv(B, H_q, H_kv, S_q, S_kv, D, seed):
    """Seeded i.i.d. N(0,1) inputs rounded to fp16 (round-to-nearest-even).

    One ``np.random.default_rng(seed)`` stream draws Q, then K, then V in fp32
    and rounds each to fp16, matching the benchmark configurations' "fp16
    N(0,1) from a fixed seed".
    """
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((B, H_q, S_q, D), dtype=np.float32).astype(np.float16)
    K = rng.standard_normal((B, H_kv, S_kv, D), dtype=np.float32).astype(np.float16)
    V = rng.standard_normal((B, H_kv, S_kv, D), dtype=np.float32).astype(np.float16)
    return Q, K, V


def error_stats(got: np.ndarray, ref: np.ndarray):
    """(max-abs error, relative-L2 error) of got vs ref, computed in fp64."""
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    diff = g - r
    max_abs = float(np.abs(diff).max()) if diff.size else 0.0
    denom = float(np.sqrt((r * r).sum()))
    rel_l2 = float(np.sqrt((diff * diff).sum()) / denom) if denom > 0 else 0.0
    return max_abs, rel_l2
