"""Decode over a paged KV cache (kf_attn_fwd_paged) vs the fp64 oracle.

Pools [n_blocks, H_kv, block_size, D] with randomly permuted block tables (the
reference benchmark's worst-case fragmentation, bench_flash_attn2.py:170-182),
per-sequence lengths that end inside a block, several block sizes and head
dims, split-KV on and off, and pool memory past each sequence's end holding
non-finite values (stale cache pages) that must not reach the output.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.attn_oracle import paged_attn_lse

from gpu_util import assert_close, to_dev

pytestmark = pytest.mark.gpu


def _paged_case(B, H_q, H_kv, S_q, D, block_size, seq_lens, seed, poison=True):
    rng = np.random.default_rng(seed)
    max_blocks = max((n + block_size - 1) // block_size for n in seq_lens) + 1
    n_blocks = B * max_blocks + 5
    pool_k = rng.standard_normal((n_blocks, H_kv, block_size, D)).astype(np.float16)
    pool_v = rng.standard_normal((n_blocks, H_kv, block_size, D)).astype(np.float16)
    perm = rng.permutation(n_blocks)
    table = perm[:B * max_blocks].reshape(B, max_blocks).astype(np.int32)
    if poison:
        # Rows past each sequence's end inside its last block, and every pool block no
        # sequence uses, hold Inf/NaN: they must be masked, not multiplied by 0.
        used = set()
        for b, n in enumerate(seq_lens):
            nb = (n + block_size - 1) // block_size
            used.update(int(x) for x in table[b, :nb])
            if n % block_size:
                last = int(table[b, nb - 1])
                pool_k[last, :, n % block_size:] = np.inf
                pool_v[last, :, n % block_size:] = np.nan
        for pb in range(n_blocks):
            if pb not in used:
                pool_k[pb] = np.nan
                pool_v[pb] = np.inf
        # Entries past each sequence's last block are garbage (never read).
        for b, n in enumerate(seq_lens):
            nb = (n + block_size - 1) // block_size
            table[b, nb:] = -7
    Q = rng.standard_normal((B, H_q, S_q, D)).astype(np.float16)
    return Q, pool_k, pool_v, table, np.array(seq_lens, dtype=np.int32)


CASES = [
    # B, H_q, H_kv, S_q, D, block_size, seq_lens
    (4, 32, 8, 1, 128, 16, [4096, 1, 1000, 2049]),
    (3, 32, 8, 1, 128, 32, [777, 4096, 64]),
    (2, 8, 2, 1, 64, 64, [130, 5000]),
    (2, 8, 8, 1, 256, 128, [300, 129]),
    (2, 16, 4, 2, 128, 256, [1024, 513]),       # two query positions per sequence
    (1, 32, 8, 1, 128, 16, [131072]),           # long context: split-KV across many CTAs
    (2, 4, 1, 1, 16, 16, [33, 17]),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}_Hq{}_Hkv{}_Sq{}_D{}_bs{}".format(*c[:6]))
def test_paged_matches_oracle(cuda, case):
    import torch

    from kernelfoundry_b200 import flash_attn_paged

    B, H_q, H_kv, S_q, D, bs, lens = case
    Q, pk, pv, table, seq = _paged_case(B, H_q, H_kv, S_q, D, bs, lens, seed=sum(lens) + D)
    got, Mi, Li = (t.cpu().numpy() for t in flash_attn_paged(
        to_dev(Q, cuda), to_dev(pk, cuda), to_dev(pv, cuda), to_dev(table, cuda), to_dev(seq, cuda),
        return_lse=True))
    pk64, pv64 = (np.nan_to_num(x.astype(np.float64), nan=0.0, posinf=0.0) for x in (pk, pv))
    O, rMi, rLi = paged_attn_lse(Q.astype(np.float64), pk64, pv64, table, seq, bs)
    assert_close(got, O, f"paged {case[:6]}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


def test_paged_equals_contiguous_decode(cuda):
    """Pages laid out in order hold the same cache as a contiguous tensor: the same result
    up to the summation order of a different KV split (the planners differ)."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd, flash_attn_paged

    rng = np.random.default_rng(3)
    B, H_q, H_kv, D, S, bs = 2, 32, 8, 128, 4096, 16
    K = rng.standard_normal((B, H_kv, S, D)).astype(np.float16)
    V = rng.standard_normal((B, H_kv, S, D)).astype(np.float16)
    Q = rng.standard_normal((B, H_q, 1, D)).astype(np.float16)
    nb = S // bs
    pool_k = K.reshape(B, H_kv, nb, bs, D).transpose(0, 2, 1, 3, 4).reshape(B * nb, H_kv, bs, D).copy()
    pool_v = V.reshape(B, H_kv, nb, bs, D).transpose(0, 2, 1, 3, 4).reshape(B * nb, H_kv, bs, D).copy()
    table = np.arange(B * nb, dtype=np.int32).reshape(B, nb)
    seq = np.full(B, S, dtype=np.int32)
    got = flash_attn_paged(*(to_dev(x, cuda) for x in (Q, pool_k, pool_v, table, seq)))
    ref = flash_attn_fwd(*(to_dev(x, cuda) for x in (Q, K, V)))
    assert torch.allclose(got, ref, atol=1e-4, rtol=0)


def test_paged_empty_sequence_and_bad_entry(cuda):
    """seq_len 0 gives zeros; a block-table entry outside the pool reads zeros (no fault)."""
    from kernelfoundry_b200 import flash_attn_paged

    Q, pk, pv, table, seq = _paged_case(2, 8, 2, 1, 128, 16, [0, 40], seed=9, poison=False)
    table[1, 1] = 10 ** 6                       # keys 16..31 of sequence 1 -> zeros
    got = flash_attn_paged(*(to_dev(x, cuda) for x in (Q, pk, pv, table, seq))).cpu().numpy()
    assert np.all(got[0] == 0)
    pk2, pv2 = pk.copy(), pv.copy()
    pk2 = np.concatenate([pk2, np.zeros_like(pk2[:1])])
    pv2 = np.concatenate([pv2, np.zeros_like(pv2[:1])])
    t2 = table.copy()
    t2[1, 1] = pk2.shape[0] - 1                 # the same keys as explicit zero pages
    O, _, _ = paged_attn_lse(Q.astype(np.float64), pk2.astype(np.float64), pv2.astype(np.float64), t2, seq, 16)
    assert_close(got[1:], O[1:], "bad entry reads zeros")
