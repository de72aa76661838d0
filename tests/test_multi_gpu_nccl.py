"""KV-split long decode over 2 GPUs with NCCL (one process per GPU).

Each rank holds a contiguous KV range, writes its partials into its slot of the
gather buffer, all-gathers in place and merges; every rank must get the
attention over the whole cache (fp64 oracle).  Needs two
visible GPUs; skipped otherwise.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from kernelfoundry_b200.multi_gpu import kv_shard, long_decode_forward
    from oracle.attn_oracle import normal_qkv, reference_attn

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        Q, K, V = normal_qkv(1, 32, 8, 1, 50001, 128, seed=77)
        lo, hi = kv_shard(K.shape[2], world, rank)
        q = torch.from_numpy(Q).to(dev)
        k = torch.from_numpy(np.ascontiguousarray(K[:, :, lo:hi])).to(dev)
        v = torch.from_numpy(np.ascontiguousarray(V[:, :, lo:hi])).to(dev)
        buf = None
        outs = []
        for _ in range(2):                           # the gather buffer is reused across steps
            n = (32 * 130 + 3) // 4 * 4
            buf = buf if buf is not None else torch.empty(world * n, dtype=torch.float32, device=dev)
            outs.append(long_decode_forward(q, k, v, gather_buf=buf).cpu().numpy())
        ref = reference_attn(Q.astype(np.float64), K.astype(np.float64), V.astype(np.float64))
        err = max(float(np.abs(o - ref).max()) for o in outs)
        np.save(os.path.join(result_dir, f"err{rank}.npy"), np.array(err))
    finally:
        dist.destroy_process_group()


def test_long_decode_split_nccl_world2(tmp_path):
    import multiprocessing as mp

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        assert float(np.load(tmp_path / f"err{r}.npy")) < 2e-3
