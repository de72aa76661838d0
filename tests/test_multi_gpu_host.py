"""Host logic of the multi-GPU partitioning, on CPU ranks (gloo, world_size 2).

The per-rank attention math is replaced by the oracle (test-only stand-ins
injected through long_decode_forward's partial_fn/combine_fn) so that the
sharding, the packed all-gather and the merge order are checked without a
GPU.  The CUDA version of the same path runs on two GPUs in
tests/test_multi_gpu_nccl.py (NCCL all-gather) and tests/test_multi_gpu_p2p.py
(NVLink peer exchange), and in bench.py for N > 1.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from kernelfoundry_b200.multi_gpu import batch_shard, head_shard, kv_shard, shard_range


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 131072, 4097])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_range_partitions(n, world):
    ranges = [shard_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a, b), (c, d) in zip(ranges[:-1], ranges[1:]):
        assert b == c
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_head_shard_keeps_gqa_groups():
    for H_q, H_kv, world in [(32, 8, 8), (32, 8, 4), (32, 8, 2), (40, 8, 8), (32, 1, 1)]:
        G = H_q // H_kv
        seen = []
        for r in range(world):
            (q0, q1), (k0, k1) = head_shard(H_q, H_kv, world, r)
            for h in range(q0, q1):
                assert k0 <= h // G < k1
            seen.extend(range(q0, q1))
        assert seen == list(range(H_q))
    with pytest.raises(ValueError):
        head_shard(6, 4, 2, 0)


def test_batch_and_kv_shard():
    assert [batch_shard(8, 8, r) for r in range(8)] == [(r, r + 1) for r in range(8)]
    assert kv_shard(131072, 8, 7) == (7 * 16384, 131072)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_partial(q, k, v):
    from oracle.attn_oracle import attn_partial

    m, l, O = attn_partial(q.numpy(), k.numpy(), v.numpy(), 0, k.shape[2])
    return torch.from_numpy(O), torch.from_numpy(m), torch.from_numpy(l)


def _oracle_combine(O_p, m_p, l_p):
    from oracle.attn_oracle import combine_partials

    O, _, _ = combine_partials(list(m_p.numpy()), list(l_p.numpy()), list(O_p.numpy()))
    return torch.from_numpy(O)


def _worker(rank, world, port, result_dir):
    import torch.distributed as dist

    from kernelfoundry_b200.multi_gpu import kv_shard, long_decode_forward
    from oracle.attn_oracle import normal_qkv, reference_attn

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Q, K, V = normal_qkv(1, 8, 2, 1, 1001, 64, seed=42)
        Q, K, V = (x.astype(np.float64) for x in (Q, K, V))
        lo, hi = kv_shard(K.shape[2], world, rank)
        q = torch.from_numpy(Q)
        k = torch.from_numpy(np.ascontiguousarray(K[:, :, lo:hi]))
        v = torch.from_numpy(np.ascontiguousarray(V[:, :, lo:hi]))
        out = long_decode_forward(q, k, v, partial_fn=_oracle_partial, combine_fn=_oracle_combine)
        err = float(np.abs(out.numpy() - reference_attn(Q, K, V)).max())
        np.save(os.path.join(result_dir, f"err{rank}.npy"), np.array(err))
    finally:
        dist.destroy_process_group()


def test_long_decode_split_gloo_world2(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        assert float(np.load(tmp_path / f"err{r}.npy")) < 1e-12
