"""Pin the CPU oracle to the reference (no GPU).

The golden vectors in tests/golden/ were produced by the reference itself
(tests/golden/make_golden.py): its NumPy model kernel_models/flash_attn.py
(reference_attn, the tile model, its __main__ smoke test) and its compiled C++
host code (fill_random_f32, cpu_attn).  The oracle restatements must
reproduce them: bit-exactly for the C++ ports, to fp64 round-off for the
NumPy ones.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import oracle
from oracle.attn_oracle import (
    attn_partial,
    combine_partials,
    error_stats,
    normal_qkv,
    reference_attn,
    reference_attn_lse,
    tile_model_attn,
)

from conftest import golden_case, golden_names


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_legacy_inputs_bit_exact(legacy_golden):
    """mt19937 uniform[-1,1] restatement == reference fill_random_f32 (tests/test_utils.h:27-31)."""
    cases = legacy_golden["cases"]
    digests = legacy_golden["digests"]
    heads = legacy_golden["heads"]
    for (B, S, Hq, Hkv, D, seed), dig, head in zip(cases, digests, heads):
        (q, k, v), _ = oracle.legacy_case_inputs(int(B), int(S), int(Hq), int(Hkv), int(D), int(seed))
        assert _sha(q.ravel()) == dig[0]
        assert _sha(k.ravel()) == dig[1]
        assert _sha(v.ravel()) == dig[2]
        np.testing.assert_array_equal(q.ravel()[:8], head[:8])


def test_legacy_cpu_attn_bit_exact(legacy_golden):
    """C restatement of cpu_attn == the reference's own cpu_attn output, bit for bit."""
    for (B, S, Hq, Hkv, D, seed), dig, head in zip(legacy_golden["cases"], legacy_golden["digests"],
                                                  legacy_golden["heads"]):
        (q, k, v), _ = oracle.legacy_case_inputs(int(B), int(S), int(Hq), int(Hkv), int(D), int(seed))
        o = oracle.cpu_attn_f32(q, k, v)
        assert _sha(o.ravel()) == dig[3], f"case {(B, S, Hq, Hkv, D, seed)}"
        np.testing.assert_array_equal(o.ravel()[:8], head[24:32])


def test_reference_attn_matches_golden(sdpa_golden):
    for name in golden_names(sdpa_golden):
        _, Q, K, V = golden_case(sdpa_golden, name)
        O = reference_attn(Q.astype(np.float64), K.astype(np.float64), V.astype(np.float64))
        np.testing.assert_allclose(O, sdpa_golden[f"{name}/O_ref64"], rtol=0, atol=1e-13, err_msg=name)


def test_tile_model_matches_golden(sdpa_golden):
    for name in golden_names(sdpa_golden):
        key = f"{name}/O_tile32"
        if key not in sdpa_golden.files:
            continue
        _, Q, K, V = golden_case(sdpa_golden, name)
        O = tile_model_attn(Q.astype(np.float32), K.astype(np.float32), V.astype(np.float32), kv_block_rows=16)
        np.testing.assert_allclose(O, sdpa_golden[key], rtol=0, atol=2e-6, err_msg=name)


def test_reference_smoke_test_reproduced(sdpa_golden):
    """kernel_models/flash_attn.py:269-281 (np.random.seed(42), D = 16/64/128)."""
    np.random.seed(42)
    for D in (16, 64, 128):
        Q = np.random.randn(1, 2, 16, D).astype(np.float32)
        K = np.random.randn(1, 1, 16, D).astype(np.float32)
        V = np.random.randn(1, 1, 16, D).astype(np.float32)
        np.testing.assert_allclose(reference_attn(Q, K, V), sdpa_golden[f"smoke{D}/ref"], atol=1e-6)
        np.testing.assert_allclose(tile_model_attn(Q, K, V, kv_block_rows=16), sdpa_golden[f"smoke{D}/tile"],
                                   atol=2e-6)


def test_lse_state_consistent():
    """Mi/Li reproduce O: O = sum exp(s - Mi) v / Li."""
    Q, K, V = normal_qkv(1, 4, 2, 9, 70, 64, seed=11)
    Q, K, V = (x.astype(np.float64) for x in (Q, K, V))
    O, Mi, Li = reference_attn_lse(Q, K, V)
    s = np.einsum("bhqd,bhkd->bhqk", Q, np.repeat(K, 2, axis=1)) / np.sqrt(64.0)
    np.testing.assert_allclose(Mi, s.max(-1), atol=1e-12)
    np.testing.assert_allclose(Li, np.exp(s - Mi[..., None]).sum(-1), rtol=1e-12)
    P = np.exp(s - Mi[..., None]) / Li[..., None]
    np.testing.assert_allclose(O, P @ np.repeat(V, 2, axis=1), atol=1e-12)


@pytest.mark.parametrize("cuts", [[0, 1000], [0, 300, 1000], [0, 1, 500, 999, 1000], [0, 250, 500, 750, 1000]])
def test_split_combine_identity(cuts):
    """Partials over disjoint KV ranges merged by log-sum-exp == full attention."""
    Q, K, V = normal_qkv(2, 8, 2, 1, 1000, 128, seed=5)
    Q, K, V = (x.astype(np.float64) for x in (Q, K, V))
    full, Mi, Li = reference_attn_lse(Q, K, V)
    parts = [attn_partial(Q, K, V, lo, hi) for lo, hi in zip(cuts[:-1], cuts[1:])]
    O, M, L = combine_partials(*zip(*parts))
    np.testing.assert_allclose(O, full, atol=1e-12)
    np.testing.assert_allclose(M, Mi, atol=1e-12)
    np.testing.assert_allclose(L, Li, rtol=1e-12)


def test_error_stats():
    a = np.array([1.0, 2.0, 3.0])
    assert error_stats(a, a) == (0.0, 0.0)
    ma, rl = error_stats(a + [0, 0, 0.5], a)
    assert ma == 0.5 and abs(rl - 0.5 / np.sqrt(14)) < 1e-15


def test_planted_mistake_is_caught(sdpa_golden):
    """A deliberately wrong oracle (GQA map h % H_kv instead of h // G) must fail the golden check."""
    name = "prefill_ratio5"
    _, Q, K, V = golden_case(sdpa_golden, name)
    Q, K, V = (x.astype(np.float64) for x in (Q, K, V))
    H_q, H_kv = Q.shape[1], K.shape[1]
    wrong = np.zeros_like(Q)
    for h in range(H_q):
        s = Q[0, h] @ K[0, h % H_kv].T / np.sqrt(Q.shape[3])
        p = np.exp(s - s.max(-1, keepdims=True))
        wrong[0, h] = (p / p.sum(-1, keepdims=True)) @ V[0, h % H_kv]
    max_abs, _ = error_stats(wrong, sdpa_golden[f"{name}/O_ref64"])
    assert max_abs > 1e-2


def test_causal_oracle_against_independent_forms():
    """The causal restatement agrees with (1) torch SDPA is_causal in fp64 for S_q == S_kv
    (an independent implementation) and (2) per-row plain attention over the visible keys
    for S_q < S_kv (bottom-right alignment)."""
    import torch

    from oracle.attn_oracle import causal_attn_lse, causal_pairs, normal_qkv, reference_attn_lse

    Q, K, V = (x.astype(np.float64) for x in normal_qkv(1, 4, 2, 33, 33, 16, seed=5))
    O, Mi, Li = causal_attn_lse(Q, K, V)
    Kr = np.repeat(K, 2, axis=1)
    Vr = np.repeat(V, 2, axis=1)
    ref = torch.nn.functional.scaled_dot_product_attention(
        torch.from_numpy(Q), torch.from_numpy(Kr), torch.from_numpy(Vr), is_causal=True).numpy()
    assert np.abs(O - ref).max() < 1e-12
    Q, K, V = (x.astype(np.float64) for x in normal_qkv(1, 2, 1, 5, 19, 16, seed=6))
    O, Mi, Li = causal_attn_lse(Q, K, V)
    for i in range(5):
        hi = 19 - 5 + i + 1
        o, mi, li = reference_attn_lse(Q[:, :, i:i + 1], K[:, :, :hi], V[:, :, :hi])
        assert np.abs(O[:, :, i:i + 1] - o).max() < 1e-12
        assert np.abs(Mi[:, :, i] - mi[:, :, 0]).max() < 1e-12 and np.abs(Li[:, :, i] - li[:, :, 0]).max() < 1e-12
    assert causal_pairs(4, 4) == 10 and causal_pairs(2, 5) == 4 + 5
    with pytest.raises(ValueError):
        causal_attn_lse(*normal_qkv(1, 1, 1, 5, 4, 16, seed=1))
